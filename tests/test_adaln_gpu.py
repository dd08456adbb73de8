"""Parity of the AdaLN projection kernel (h3_adaln_projection, through the C-ABI):
the linear + bias of MiniMaxH3AdaLNProjection::forward (patches/InfiniLM.patch:
1260-1279) for a few conditioning rows.

Checked against an fp64-accumulated reference with the same two BF16 roundings
(the linear's output, then the bias add): max-abs-rel <= 1e-2 and >= 99 % of
outputs exact (the K products are summed in fp32 in the kernel's fixed order, so
a BF16 rounding of the linear's output may differ by one ulp).  A column slice
of the weight gives bitwise the same columns (the column-split all-gather of the
sequence-parallel step relies on it).
"""
import pytest
import torch

from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    import h3b200
    h3b200.load()
    from h3b200 import ops
    return ops


def _ref(x, w, b):
    y = (x.double() @ w.double().t()).to(torch.bfloat16)
    if b is None:
        return y
    return (y.double() + b.double()).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(1, 92160, 5120), (2, 11520, 5120), (3, 1000, 256), (4, 37, 64), (1, 8, 8)])
@pytest.mark.parametrize("bias", [True, False])
def test_adaln_projection_matches_fp64(ops, M, N, K, bias):
    torch.manual_seed(M * 7 + N)
    x = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) * K ** -0.5).bfloat16()
    b = torch.randn(N, device=DEV).bfloat16() if bias else None
    y = ops.adaln_projection(x, w, b)
    ref = _ref(x.cpu(), w.cpu(), None if b is None else b.cpu())
    rel = O.max_abs_rel(y.cpu(), ref)
    exact = float((y.cpu() == ref).float().mean())
    assert rel <= 1e-2 and exact >= 0.99, f"max-abs-rel {rel:.3e}, exact {exact:.5f}"
    import h3b200
    assert h3b200.load().h3_device_error() == 0


def test_adaln_projection_column_slices_bitwise(ops):
    torch.manual_seed(3)
    x = torch.randn(1, 5120, device=DEV).bfloat16()
    w = (torch.randn(8 * 1440, 5120, device=DEV) * 0.02).bfloat16()
    b = torch.randn(8 * 1440, device=DEV).bfloat16()
    full = ops.adaln_projection(x, w, b)
    for r in range(8):
        cols = slice(r * 1440, (r + 1) * 1440)
        part = ops.adaln_projection(x, w[cols].contiguous(), b[cols].contiguous())
        assert torch.equal(part, full[:, cols])


def test_adaln_projection_rejects(ops):
    x = torch.randn(5, 64, device=DEV).bfloat16()
    w = torch.randn(16, 64, device=DEV).bfloat16()
    with pytest.raises((RuntimeError, ValueError)):
        ops.adaln_projection(x, w)          # more rows than the kernel serves
    with pytest.raises((RuntimeError, ValueError)):
        ops.adaln_projection(x[:2, :60], w[:, :60])   # K not a multiple of 8


@pytest.mark.parametrize("rows", [[0, 1], [1], [2], [0, 3, 4]])
def test_modulations_of_used_rows_only(ops, rows):
    """The step's batched AdaLN computes only the modalities its segments read: those
    rows equal the rows of the full computation bit for bit (t = 2 timesteps)."""
    from h3b200.block import BlockConfig
    from h3b200.step import BlockStack
    bc = BlockConfig(hidden=256, heads=2, ffn=512)
    stack = BlockStack(bc, 3, DEV, seed=3)
    temb = torch.randn(2, 256, device=DEV)
    full = stack.modulations(temb)
    part = stack.modulations(temb, rows=rows)
    for f, q in zip(full, part):
        for r in rows:
            m = r % bc.modalities
            for i in range(2):                  # every timestep row of a needed modality
                assert torch.equal(f[i * bc.modalities + m], q[i * bc.modalities + m])
