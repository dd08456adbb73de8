"""Building blocks of the peer-memory Ulysses exchange on one GPU (local
destinations): the multi-destination q/k RMSNorm + RoPE equals one call per
block bit for bit, the block copy equals torch's copy, and the arguments are
checked.  The cross-GPU exchange itself is tested in test_ulysses_gpu.py."""
import ctypes

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


def _descs(tensors):
    from h3b200 import _lib
    return (_lib.H3Tensor * len(tensors))(*[_lib.desc(t) for t in tensors])


@pytest.mark.parametrize("T,W,Hs", [(37, 3, 2), (300, 8, 5), (64, 1, 4)])
def test_qk_norm_rope_multi_equals_per_block(h3, T, W, Hs):
    from h3b200 import _lib
    torch.manual_seed(T + W)
    qkv = torch.randn(T, 3, W, Hs, 128, device=DEV).bfloat16()
    weight = (torch.randn(128, device=DEV) * 0.1 + 1).bfloat16()
    table = O.rotary_cache(O.grid_positions(1, 1, T)).to(DEV)
    cos, sin = table[:, :48], table[:, 48:]
    outs = [torch.empty(T, Hs, 128, dtype=torch.bfloat16, device=DEV) for _ in range(W)]
    _lib.call("h3_qk_norm_rope_multi", _descs(outs), W, _lib.desc(qkv[:, 0]), _lib.desc(weight), _lib.desc(cos),
              _lib.desc(sin), 1e-6, _lib.stream_of(qkv))
    for p in range(W):
        ref = torch.empty(T, 1, Hs, 128, dtype=torch.bfloat16, device=DEV)
        h3.h3_qk_norm_rope_(ref, qkv[:, 0, p].unsqueeze(1), weight, cos, sin, 1e-6)
        assert torch.equal(outs[p], ref[:, 0]), f"block {p}"


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_copy_blocks_equals_torch(h3, dt):
    from h3b200 import _lib
    W, T, C = 5, 41, 640
    src_full = torch.randn(T, 3, W, C, device=DEV).to(dt)
    src = src_full[:, 2].permute(1, 0, 2)            # [W, T, C], strided
    dsts = [torch.zeros(T, C, dtype=dt, device=DEV) for _ in range(W)]
    _lib.call("h3_copy_blocks", _descs(dsts), W, _lib.desc(src), _lib.stream_of(src))
    for b in range(W):
        assert torch.equal(dsts[b], src[b])


def test_exchange_kernels_check_arguments(h3):
    from h3b200 import _lib
    lib = h3.load()
    src = torch.zeros(9, 4, 128, dtype=torch.bfloat16, device=DEV)
    dsts = _descs([torch.zeros(4, 128, dtype=torch.bfloat16, device=DEV) for _ in range(9)])
    s = _lib.stream_of(src)
    assert lib.h3_copy_blocks(dsts, 9, ctypes.byref(_lib.desc(src)), s) == 2        # more than 8 blocks
    bad = _descs([torch.zeros(5, 128, dtype=torch.bfloat16, device=DEV) for _ in range(2)])
    assert lib.h3_copy_blocks(bad, 2, ctypes.byref(_lib.desc(src[:2])), s) == 2     # row count mismatch
    x = torch.zeros(10, 2, 3, 128, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(128, dtype=torch.bfloat16, device=DEV)
    cs = torch.zeros(10, 48, dtype=torch.bfloat16, device=DEV)
    outs = _descs([torch.zeros(10, 3, 128, dtype=torch.bfloat16, device=DEV) for _ in range(3)])
    args = [ctypes.byref(_lib.desc(t)) for t in (x, w, cs, cs)]
    assert lib.h3_qk_norm_rope_multi(outs, 3, *args, 1e-6, s) == 2                  # n != x.shape[1]
