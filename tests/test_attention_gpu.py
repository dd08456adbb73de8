"""Parity of the tcgen05 flash attention (h3_mha through the C-ABI) with fp32
softmax attention.

Tolerances follow the reference's own attention check
(tools/verify_attention.py:60-72): max |err| <= 2e-3 and mean |err| <= 2e-4
against fp32 math on sampled query rows, for sequences >= 1024.  Short
sequences have larger outputs (fewer keys to average), so there the bound is
one BF16 rounding of the output plus 2e-3.
"""
import math

import pytest
import torch

from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def h3():
    import h3b200
    h3b200.load()
    return h3b200


def _check(out, q, k, v, rows=None, max_err=None, mean_err=2e-4):
    """Compare rows of out [B,Sq,H,D] against fp32 attention computed on the GPU
    (torch fp32 matmul: the checker, not the product)."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    qf = q.float() if rows is None else q[:, rows].float()
    logits = torch.einsum("bshd,bthd->bhst", qf, k.float()) * scale
    ref = torch.einsum("bhst,bthd->bshd", torch.softmax(logits, -1), v.float())
    o = (out if rows is None else out[:, rows]).float()
    err = (o - ref).abs()
    bound = 2e-3 + ref.abs() * 2.0 ** -8 if max_err is None else max_err
    assert bool((err <= bound).all()), f"max err {float(err.max()):.3e}"
    assert float(err.mean()) <= mean_err, f"mean err {float(err.mean()):.3e}"
    return float(err.max()), float(err.mean())


@pytest.mark.parametrize("B,Sq,Sk,H", [(1, 128, 128, 1), (1, 200, 136, 3), (2, 333, 333, 2),
                                       (1, 256, 1000, 4), (1, 1000, 777, 2), (1, 600, 129, 1),
                                       (1, 130, 40, 2), (1, 64, 100, 1), (1, 300, 64, 1), (1, 257, 192, 3)])
def test_small_shapes(h3, B, Sq, Sk, H):
    torch.manual_seed(B * 1000 + Sq + Sk + H)
    q = torch.randn(B, Sq, H, 128, dtype=torch.bfloat16, device=DEV)
    k = torch.randn(B, Sk, H, 128, dtype=torch.bfloat16, device=DEV)
    v = torch.randn(B, Sk, H, 128, dtype=torch.bfloat16, device=DEV)
    out = h3.mha(q, k, v)
    _check(out, q, k, v, mean_err=1e-3)


def test_growing_logits_rescale(h3):
    """Keys whose logits grow along the sequence: the running row max rises past
    the lazy-rescale threshold many times, so O is rescaled between key tiles."""
    torch.manual_seed(21)
    Sq, Sk, H = 256, 1100, 2
    q = torch.randn(1, Sq, H, 128, device=DEV).abs()
    ramp = torch.linspace(0.0, 3.0, Sk, device=DEV).view(1, Sk, 1, 1)
    k = (torch.rand(1, Sk, H, 128, device=DEV) * ramp).bfloat16()
    q = q.bfloat16()
    v = torch.randn(1, Sk, H, 128, dtype=torch.bfloat16, device=DEV)
    out = h3.mha(q, k, v)
    _check(out, q, k, v, mean_err=1e-3)


def test_matches_cpu_oracle(h3):
    torch.manual_seed(11)
    q = torch.randn(1, 300, 2, 128, dtype=torch.bfloat16)
    k = torch.randn(1, 260, 2, 128, dtype=torch.bfloat16)
    v = torch.randn(1, 260, 2, 128, dtype=torch.bfloat16)
    out = h3.mha(q.to(DEV), k.to(DEV), v.to(DEV)).cpu().float()
    ref = O.attention_fp32(q, k, v, 128 ** -0.5)
    assert float((out - ref).abs().max()) <= 2e-3 + 2.0 ** -8 * float(ref.abs().max())


def test_packed_qkv_strides_seed2026(h3):
    """The reference's verification layout: q,k,v strided views of one packed
    [1, S, 3, H, 128] tensor (tools/verify_attention.py:41-43), S=8192, 14 heads."""
    torch.manual_seed(2026)
    seq, heads = 8192, 14
    packed = torch.randn(1, seq, 3, heads, 128, dtype=torch.bfloat16, device=DEV)
    q, k, v = (packed[:, :, i] for i in range(3))
    out = torch.empty(1, seq, heads, 128, dtype=torch.bfloat16, device=DEV)
    h3.mha_(out, q, k, v)
    rows = torch.linspace(0, seq - 1, 16, device=DEV).long()
    err_max, err_mean = _check(out, q, k, v, rows=rows, max_err=2e-3, mean_err=2e-4)
    first = out.clone()
    h3.mha_(out, q, k, v)
    assert torch.equal(first, out), "attention is not deterministic"


def test_sequence_parallel_shapes(h3):
    """Queries padded past the key length (Ulysses: Sq = W*T >= Sk), output
    rows independent of the query offset so W-GPU == 1-GPU bitwise."""
    torch.manual_seed(4)
    Sk, Sq, H = 1000, 1024, 5
    q = torch.randn(1, Sq, H, 128, dtype=torch.bfloat16, device=DEV)
    k = torch.randn(1, Sk, H, 128, dtype=torch.bfloat16, device=DEV)
    v = torch.randn(1, Sk, H, 128, dtype=torch.bfloat16, device=DEV)
    full = h3.mha(q, k, v)
    _check(full[:, :Sk], q[:, :Sk], k, v, mean_err=5e-4)
    part = h3.mha(q[:, 300:700], k, v)
    assert torch.equal(part, full[:, 300:700])
    heads = h3.mha(q[:, :, 2:4], k[:, :, 2:4], v[:, :, 2:4])
    assert torch.equal(heads, full[:, :, 2:4])


def test_bench_shape_sampled_rows(h3):
    """Benchmark config 2: [1, 40, 18432, 128] (given here in the [B,S,H,D] mha layout)."""
    torch.manual_seed(0)
    S, H = 18432, 40
    q = torch.randn(1, S, H, 128, dtype=torch.bfloat16, device=DEV)
    k = torch.randn(1, S, H, 128, dtype=torch.bfloat16, device=DEV)
    v = torch.randn(1, S, H, 128, dtype=torch.bfloat16, device=DEV)
    out = h3.mha(q, k, v)
    rows = torch.linspace(0, S - 1, 16, device=DEV).long()
    _check(out, q, k, v, rows=rows, max_err=2e-3, mean_err=2e-4)
    assert h3.load().h3_device_error() == 0


def test_bad_shapes(h3):
    q = torch.zeros(1, 16, 2, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        h3.mha(q, q, q)


def test_one_tile_ctas_equal_pairs(h3):
    """When the grid's last wave would hold at most half as many Q-tile pairs as
    there are SMs, those pairs run as one-tile CTAs.  158 heads of two tiles put
    the last 10 pairs (on a 148-SM B200) in one-tile CTAs, and every single-head
    call of two tiles runs one-tile CTAs; each tile's arithmetic is the same
    either way, so every head agrees bitwise with its single-head call."""
    torch.manual_seed(31)
    Sq, Sk, H = 256, 1000, 158
    q = torch.randn(1, Sq, H, 128, dtype=torch.bfloat16, device=DEV)
    k = torch.randn(1, Sk, H, 128, dtype=torch.bfloat16, device=DEV)
    v = torch.randn(1, Sk, H, 128, dtype=torch.bfloat16, device=DEV)
    out = h3.mha(q, k, v)
    _check(out, q, k, v, mean_err=5e-4)
    for h in range(H):
        one = h3.mha(q[:, :, h:h + 1], k[:, :, h:h + 1], v[:, :, h:h + 1])
        assert torch.equal(one, out[:, :, h:h + 1]), f"head {h}"
    # an odd tile count: the last pair of each head has one tile
    q3 = q[:, :129]
    out3 = h3.mha(q3, k, v)
    assert torch.equal(out3, out[:, :129])
    assert h3.load().h3_device_error() == 0
