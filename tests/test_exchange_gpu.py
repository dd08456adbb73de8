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


@pytest.mark.parametrize("W,T,Hl,valid", [(4, 300, 5, 1190), (8, 2368, 5, 18944), (2, 181, 2, 361), (1, 257, 3, 257)])
def test_mha_scatter_equals_mha_then_permute(h3, W, T, Hl, valid):
    """The scatter epilogue stores row g of head h at row g % T of destination g // T,
    head slot h: the same bits as h3_mha followed by the heads -> tokens permute
    (destinations are slices of token-major return buffers [T, W, Hl, 128], this
    rank's slot 1 of W)."""
    from h3b200 import _lib
    torch.manual_seed(W * 1000 + T)
    q = torch.randn(1, W * T, Hl, 128, device=DEV).bfloat16()
    k = torch.randn(1, valid, Hl, 128, device=DEV).bfloat16()
    v = torch.randn(1, valid, Hl, 128, device=DEV).bfloat16()
    ref = h3.mha(q, k, v)
    slot = min(1, W - 1)
    backs = [torch.full((T, W, Hl, 128), 7.0, dtype=torch.bfloat16, device=DEV) for _ in range(W)]
    dsts = (_lib.H3Tensor * W)(*[_lib.desc(b[:, slot]) for b in backs])
    _lib.call("h3_mha_scatter", dsts, W, _lib.desc(q), _lib.desc(k), _lib.desc(v), 128 ** -0.5, _lib.stream_of(q))
    for p in range(W):
        assert torch.equal(backs[p][:, slot], ref[0, p * T:(p + 1) * T]), f"destination {p}"
        others = [s for s in range(W) if s != slot]
        assert all(bool((backs[p][:, s] == 7.0).all()) for s in others), "stores outside the head slot"
    assert h3.load().h3_device_error() == 0


def test_mha_scatter_checks_arguments(h3):
    from h3b200 import _lib
    lib = h3.load()
    q = torch.zeros(1, 100, 2, 128, dtype=torch.bfloat16, device=DEV)
    s = _lib.stream_of(q)
    few = (_lib.H3Tensor * 2)(*[_lib.desc(torch.zeros(40, 2, 128, dtype=torch.bfloat16, device=DEV))
                                for _ in range(2)])
    args = [ctypes.byref(_lib.desc(t)) for t in (q, q, q)]
    assert lib.h3_mha_scatter(few, 2, *args, 0.1, s) == 2          # 2 x 40 rows < 100 queries
    heads = (_lib.H3Tensor * 3)(*[_lib.desc(torch.zeros(40, 3, 128, dtype=torch.bfloat16, device=DEV))
                                  for _ in range(3)])
    assert lib.h3_mha_scatter(heads, 3, *args, 0.1, s) == 2        # head count differs from q's
    assert lib.h3_mha_scatter(heads, 9, *args, 0.1, s) == 2        # more than 8 destinations
