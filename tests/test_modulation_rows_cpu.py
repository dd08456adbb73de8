"""Host logic of the batched AdaLN's modality skip on CPU: for every rank of a
column-split projection (W = 1, 2, 8), the columns it computes are exactly its share of
the modalities the segments read, and gathering the ranks' shares gives those
modalities' rows of the full projection.  The device kernel is stood in for by a
torch product (its own parity is a GPU test)."""
from types import SimpleNamespace

import pytest
import torch

import h3b200  # noqa: F401  (puts the package on the path)
from h3b200 import ops
from h3b200.block import BlockConfig
from h3b200.step import BlockStack


def _fake_projection(x, weight, bias=None, out=None):
    y = x.float() @ weight.float().t()
    if bias is not None:
        y = y + bias.float()
    out.copy_(y.to(out.dtype))
    return out


def _stack(bc, blocks, world, rank, seed=4):
    """The attributes BlockStack._project_rows reads: the config, this rank's
    column slice of every block's AdaLN weight and bias, world and rank (the
    block's other weights need the device and play no part here)."""
    g = torch.Generator().manual_seed(seed)
    weights = []
    for _ in range(blocks):
        w = (torch.randn(bc.modalities * 6 * bc.hidden, bc.hidden, generator=g) * 0.05).bfloat16()
        b = (torch.randn(bc.modalities * 6 * bc.hidden, generator=g) * 0.05).bfloat16()
        n = w.shape[0] // world
        weights.append(SimpleNamespace(w_adaln=w[rank * n:(rank + 1) * n].contiguous(),
                                       b_adaln=b[rank * n:(rank + 1) * n].contiguous()))
    return SimpleNamespace(cfg=bc, weights=weights, world=world, rank=rank)


@pytest.mark.parametrize("world", [1, 2, 8])
@pytest.mark.parametrize("rows", [[0, 1], [2], [1, 5]])
def test_each_rank_computes_its_share_of_the_used_modalities(monkeypatch, world, rows):
    monkeypatch.setattr(ops, "adaln_projection", _fake_projection)
    bc = BlockConfig(hidden=128, heads=1, ffn=256)            # 3 modalities x 6 x 128 = 2304 columns
    full_stack = _stack(bc, 2, 1, 0)
    temb = torch.randn(2, 128)
    act = torch.nn.functional.silu(temb).bfloat16()
    width, mods = 6 * bc.hidden, bc.modalities
    used = sorted({r % mods for r in rows})
    ref = [_fake_projection(act, w.w_adaln, w.b_adaln, torch.empty(2, w.w_adaln.shape[0], dtype=torch.bfloat16))
           for w in full_stack.weights]
    gathered = [torch.full((2, mods * width), float("nan"), dtype=torch.bfloat16) for _ in ref]
    for rank in range(world):
        local = BlockStack._project_rows(_stack(bc, 2, world, rank), act, rows)
        assert local is not None
        n = local.shape[2]
        for b in range(2):
            for m in range(mods):
                lo, hi = max(m * width, rank * n), min((m + 1) * width, (rank + 1) * n)
                if lo < hi and m in used:
                    gathered[b][:, lo:hi] = local[b, :, lo - rank * n:hi - rank * n]
    for g, r in zip(gathered, ref):
        for m in used:
            assert torch.equal(g[:, m * width:(m + 1) * width], r[:, m * width:(m + 1) * width])


def test_every_modality_used_takes_the_full_path(monkeypatch):
    monkeypatch.setattr(ops, "adaln_projection", _fake_projection)
    stack = _stack(BlockConfig(hidden=128, heads=1, ffn=256), 1, 1, 0)
    act = torch.randn(1, 128).bfloat16()
    assert BlockStack._project_rows(stack, act, [0, 1, 2]) is None
    assert BlockStack._project_rows(stack, act, None) is None
