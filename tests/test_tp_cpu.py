"""Tensor-parallel block on the CPU (no GPU): the weight slices reproduce the
full projections exactly, and the tensor-parallel composition of the block
(per-rank partial products summed in fp32 in rank order, as the peer all-reduce
does) matches the one-GPU block within the block tolerance."""
import pytest
import torch

from oracle import h3_oracle as O

D, F, N = 128, 512, 40
# (tensor-parallel size, heads): 1 head per rank at 2 and 4 ranks, FFN slices of 256 and 128
SIZES = [(2, 2), (4, 4)]


def _weights(H):
    HD = H * D
    from h3b200.block import BlockWeights
    g = torch.Generator().manual_seed(3)
    r = lambda *s: (torch.randn(*s, generator=g) * 0.05).bfloat16()  # noqa: E731
    ones = lambda n: torch.ones(n, dtype=torch.bfloat16)  # noqa: E731
    return BlockWeights(w_qkv=r(3 * HD, HD), norm_q=ones(D), norm_k=ones(D), w_o=r(HD, HD), w_gate_up=r(2 * F, HD),
                        w_down=r(HD, F), norm1=ones(HD), norm2=ones(HD))


def _cfg(H):
    from h3b200.block import BlockConfig
    return BlockConfig(hidden=H * D, heads=H, ffn=F)


@pytest.mark.parametrize("W,H", SIZES)
def test_slices_reproduce_the_full_projections(W, H):
    from h3b200.tp import shard_block_weights
    HD = H * D
    w = _weights(H)
    x = torch.randn(N, HD).bfloat16()
    full_qkv = O.linear(x, w.w_qkv).view(N, 3, H, D)
    full_up_gate = O.linear(x, w.w_gate_up)
    hidden = torch.randn(N, F).bfloat16()
    down_sum = (hidden.float() @ w.w_down.float().t())
    parts = []
    for r in range(W):
        s = shard_block_weights(w, _cfg(H), W, r, prepare=False)
        hl, fr = H // W, F // W
        assert torch.equal(O.linear(x, s.w_qkv).view(N, 3, hl, D), full_qkv[:, :, r * hl:(r + 1) * hl])
        ug = O.linear(x, s.w_gate_up)
        assert torch.equal(ug[:, :fr], full_up_gate[:, r * fr:(r + 1) * fr])
        assert torch.equal(ug[:, fr:], full_up_gate[:, F + r * fr:F + (r + 1) * fr])
        parts.append(hidden[:, r * fr:(r + 1) * fr].float() @ s.w_down.float().t())
    assert torch.allclose(sum(parts), down_sum, rtol=1e-5, atol=1e-5)


def _tp_block(x, mod, w, cos, sin, W, H):
    """The TP composition with the oracle's ops: each rank's partial BF16 product,
    summed over ranks in fp32 in rank order, rounded once."""
    from h3b200.tp import shard_block_weights
    n = x.shape[0]
    HD = H * D
    sh = [shard_block_weights(w, _cfg(H), W, r, prepare=False) for r in range(W)]
    m = mod.view(6, HD)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (m[i].expand(n, HD) for i in range(6))
    n1 = O.rms_modulate(x, w.norm1, scale_msa, shift_msa, 1e-6)
    o_parts = []
    for s in sh:
        hl = s.w_qkv.shape[0] // (3 * D)
        qkv = O.linear(n1, s.w_qkv).view(n, 3, hl, D)
        q = O.qk_norm_rope(qkv[:, 0], s.norm_q, cos, sin, 1e-6)
        k = O.qk_norm_rope(qkv[:, 1], s.norm_k, cos, sin, 1e-6)
        a = O._r(O.attention_fp32(q[None], k[None], qkv[:, 2][None], D ** -0.5)[0]).reshape(n, hl * D)
        o_parts.append(O.linear(a, s.w_o))
    o = O._r(sum(p.float() for p in o_parts))
    res = O.gated_residual(x, gate_msa, o)
    n2 = O.rms_modulate(res, w.norm2, scale_mlp, shift_mlp, 1e-6)
    m_parts = []
    for s in sh:
        fr = s.w_down.shape[1]
        ug = O.linear(n2, s.w_gate_up)
        m_parts.append(O.linear(O.swiglu(ug[:, :fr], ug[:, fr:]), s.w_down))
    mlp = O._r(sum(p.float() for p in m_parts))
    return O.gated_residual(res, gate_mlp, mlp)


@pytest.mark.parametrize("W,H", SIZES)
def test_tensor_parallel_composition_matches_one_gpu_block(W, H):
    HD = H * D
    w = _weights(H)
    torch.manual_seed(5)
    x = torch.randn(N, HD).bfloat16()
    mod = (torch.randn(6 * HD) * 0.3).bfloat16()
    table = O.rotary_cache(O.grid_positions(1, 5, 8))
    cos, sin = table[:, :48], table[:, 48:]
    ref = O.block_forward(x, mod, {k: getattr(w, k) for k in ("w_qkv", "norm_q", "norm_k", "w_o", "w_gate_up",
                                                             "w_down", "norm1", "norm2")}, cos, sin, H)
    tp = _tp_block(x, mod, w, cos, sin, W, H)
    assert O.max_abs_rel(tp, ref) <= 2e-2
