"""Parity of the tcgen05 projections (h3_linear*, through the C-ABI).

The plain GEMM is compared with an fp32-accumulated reference rounded to BF16
(the GEMM accumulation order is not pinned by the reference, which only checks
its BLAS for determinism): max-abs-rel <= 1e-2 and >= 95% of outputs within 1
BF16 ulp.  The fused epilogues must equal the unfused composition (same GEMM,
then the pointwise op) bit for bit.
"""
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


def _ref(x, w):
    return (x.float() @ w.float().t()).bfloat16()


def _assert_gemm_close(y, ref):
    rel = O.max_abs_rel(y.cpu(), ref.cpu())
    within = float((O.bf16_ulp_distance(y.cpu(), ref.cpu()) <= 1).float().mean())
    assert rel <= 1e-2 and within >= 0.95, f"max-abs-rel {rel:.3e}, within-1-ulp {within:.4f}"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1, 32, 64), (300, 384, 128), (1000, 1024, 512),
                                   (257, 5120, 1024), (4096, 768, 5120)])
def test_linear_shapes(h3, M, N, K):
    torch.manual_seed(M + N + K)
    x = torch.randn(M, K, dtype=torch.bfloat16, device=DEV)
    w = (torch.randn(N, K, device=DEV) * 0.02).bfloat16()
    y = h3.linear(x, w)
    _assert_gemm_close(y, _ref(x, w))


def test_linear_empty_rows(h3):
    """M = 0: every projection entry point returns success and launches nothing,
    as the attention entry point does for an empty query sequence."""
    w = (torch.randn(512, 256, device=DEV) * 0.02).bfloat16()
    x = torch.empty(0, 256, dtype=torch.bfloat16, device=DEV)
    assert h3.linear(x, w).shape == (0, 512)
    res = torch.empty(0, 512, dtype=torch.bfloat16, device=DEV)
    assert h3.linear_gated_residual(x, w, res, torch.ones(512, dtype=torch.bfloat16, device=DEV)).shape == (0, 512)
    packed = h3.pack_gate_up((torch.randn(512, 256, device=DEV) * 0.02).bfloat16())
    assert h3.linear_swiglu(x, packed).shape == (0, 256)
    torch.cuda.synchronize()


def test_linear_strided_rows(h3):
    torch.manual_seed(9)
    big = torch.randn(500, 1024 + 64, dtype=torch.bfloat16, device=DEV)
    x = big[:, 64:]                                  # row stride 1088, 16-B aligned
    w = (torch.randn(512, 1024, device=DEV) * 0.02).bfloat16()
    out = torch.zeros(500, 512 + 32, dtype=torch.bfloat16, device=DEV)[:, :512]
    h3.linear_(out, x, w)
    _assert_gemm_close(out, _ref(x, w))


def test_linear_deterministic(h3):
    torch.manual_seed(10)
    x = torch.randn(2048, 2048, dtype=torch.bfloat16, device=DEV)
    w = (torch.randn(2048, 2048, device=DEV) * 0.02).bfloat16()
    a = h3.linear(x, w)
    b = h3.linear(x, w)
    assert torch.equal(a, b)


def test_pack_gate_up(h3):
    torch.manual_seed(2)
    F, K = 384, 128
    w = torch.randn(2 * F, K, dtype=torch.bfloat16, device=DEV)
    packed = h3.pack_gate_up(w)
    order = []
    for blk in range(F // 128):
        order += list(range(blk * 128, blk * 128 + 128)) + list(range(F + blk * 128, F + blk * 128 + 128))
    assert torch.equal(packed, w[torch.tensor(order, device=DEV)])


@pytest.mark.parametrize("M,F,K", [(300, 384, 256), (1024, 1536, 1024)])
def test_linear_swiglu_fused_equals_unfused(h3, M, F, K):
    torch.manual_seed(M + F)
    x = torch.randn(M, K, dtype=torch.bfloat16, device=DEV)
    w = (torch.randn(2 * F, K, device=DEV) * 0.05).bfloat16()   # [up; gate]
    fused = h3.linear_swiglu(x, h3.pack_gate_up(w))
    gate_up = h3.linear(x, w)
    unfused = h3.h3_swiglu(gate_up[:, :F], gate_up[:, F:])
    assert torch.equal(fused, unfused)
    ref = O.swiglu(_ref(x, w)[:, :F].cpu(), _ref(x, w)[:, F:].cpu())
    assert O.max_abs_rel(fused.cpu(), ref) <= 2e-2


@pytest.mark.parametrize("broadcast_gate", [True, False])
def test_linear_gated_residual_fused_equals_unfused(h3, broadcast_gate):
    torch.manual_seed(12)
    M, N, K = 777, 1024, 512
    x = torch.randn(M, K, dtype=torch.bfloat16, device=DEV)
    w = (torch.randn(N, K, device=DEV) * 0.05).bfloat16()
    res = torch.randn(M, N, dtype=torch.bfloat16, device=DEV) * 4
    gate = (torch.randn(N, device=DEV) * 0.3).bfloat16() if broadcast_gate else \
        (torch.randn(M, N, device=DEV) * 0.3).bfloat16()
    fused = h3.linear_gated_residual(x, w, res, gate)
    unfused = h3.h3_gated_residual(res, gate, h3.linear(x, w))
    assert torch.equal(fused, unfused)


def test_qkv_projection_shape_sampled(h3):
    """The config-3 QKV projection shape, 18432 x 15360 x 5120, on sampled rows."""
    torch.manual_seed(0)
    M, N, K = 18432, 15360, 5120
    x = torch.randn(M, K, dtype=torch.bfloat16, device=DEV)
    w = (torch.randn(N, K, device=DEV) * 0.02).bfloat16()
    y = h3.linear(x, w)
    rows = torch.linspace(0, M - 1, 64, device=DEV).long()
    _assert_gemm_close(y[rows], _ref(x[rows], w))
    assert h3.load().h3_device_error() == 0


def test_bad_k_rejected(h3):
    x = torch.zeros(4, 96, dtype=torch.bfloat16, device=DEV)      # K not a multiple of 64
    w = torch.zeros(32, 96, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError):
        h3.linear(x, w)
    with pytest.raises(ValueError):                               # K mismatch
        h3.linear(x, torch.zeros(32, 64, dtype=torch.bfloat16, device=DEV))


@pytest.mark.parametrize("sections", [(16, 16, 16), (22, 21, 21)], ids=["half48", "half64"])
@pytest.mark.parametrize("T,H,K,ndst", [(300, 4, 512, 1), (1000, 40, 5120, 1), (257, 8, 256, 2), (130, 10, 640, 5)])
def test_qkv_norm_rope_epilogue_equals_unfused(T, H, K, ndst, sections):
    """The QKV GEMM with q/k RMSNorm + RoPE in its epilogue, each head stored to its
    destination, equals h3_linear followed by h3_qk_norm_rope bit for bit, for the
    reference's 48 rotated pairs and the 64 of the full-D layout."""
    import h3b200
    from h3b200 import ops
    from oracle import h3_oracle as O
    torch.manual_seed(T + H)
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(3 * H * 128, K, device="cuda") * K ** -0.5).bfloat16()
    nq = (torch.randn(128, device="cuda") * 0.1 + 1).bfloat16()
    nk = (torch.randn(128, device="cuda") * 0.1 + 1).bfloat16()
    table = O.rotary_cache(O.grid_positions(1, 1, T), sections).cuda()
    half = table.shape[1] // 2
    cos, sin = table[:, :half], table[:, half:]
    hpd = H // ndst
    outs = [[torch.empty(T, hpd, 128, dtype=torch.bfloat16, device="cuda") for _ in range(ndst)] for _ in range(3)]
    ops.linear_qkv_norm_rope_(outs[0], outs[1], outs[2], x, w, nq, nk, cos, sin, 1e-6)
    qkv = ops.linear(x, w).view(T, 3, H, 128)
    ref_q = torch.empty(T, 1, H, 128, dtype=torch.bfloat16, device="cuda")
    ref_k = torch.empty_like(ref_q)
    h3b200.h3_qk_norm_rope_(ref_q, qkv[:, 0].unsqueeze(1), nq, cos, sin, 1e-6)
    h3b200.h3_qk_norm_rope_(ref_k, qkv[:, 1].unsqueeze(1), nk, cos, sin, 1e-6)
    for p in range(ndst):
        hs = slice(p * hpd, (p + 1) * hpd)
        assert torch.equal(outs[0][p], ref_q[:, 0, hs]), f"q block {p}"
        assert torch.equal(outs[1][p], ref_k[:, 0, hs]), f"k block {p}"
        assert torch.equal(outs[2][p], qkv[:, 2, hs]), f"v block {p}"
    assert h3b200.load().h3_device_error() == 0


def _with_variant(h3, variant, fn):
    lib = h3.load()
    prev = lib.h3_gemm_variant(variant)
    assert prev in (0, 1, 2)
    try:
        out = fn()
        torch.cuda.synchronize()
        return out
    finally:
        lib.h3_gemm_variant(prev)


@pytest.mark.parametrize("M", [1, 100, 128, 129, 256, 300, 1000, 2368, 4736, 18944])
@pytest.mark.parametrize("epi", ["linear", "swiglu", "gated_sq", "segmented", "qkv"])
def test_pair_tiles_equal_single_tiles(h3, M, epi):
    """The CTA-pair form (256-row tiles over two SMs, cta_group::2) gives the same
    bits as single-CTA 128-row tiles, for every epilogue, M not a multiple of 256
    included (rows of the peer CTA past M, a tile whose peer rows are all past M)."""
    from h3b200 import ops
    torch.manual_seed(M)
    K = 5120 if M >= 4736 else 512
    x = torch.randn(M, K, device=DEV).bfloat16()
    if epi == "linear":
        w = (torch.randn(768, K, device=DEV) * K ** -0.5).bfloat16()
        run = lambda: ops.linear(x, w)
    elif epi == "swiglu":
        w = ops.pack_gate_up((torch.randn(1024, K, device=DEV) * K ** -0.5).bfloat16())
        run = lambda: ops.linear_swiglu(x, w)
    elif epi in ("gated_sq", "segmented"):
        N = 1280
        w = (torch.randn(N, K, device=DEV) * K ** -0.5).bfloat16()
        res = torch.randn(M, N, device=DEV).bfloat16()
        if epi == "gated_sq":
            gate = torch.randn(M, N, device=DEV).bfloat16()
            run = lambda: ops.linear_gated_residual_sq(x, w, res, gate)
        else:
            gates = [torch.randn(N, device=DEV).bfloat16() for _ in range(2)]
            lengths = [M // 3, M - M // 3]

            def run():
                sq = torch.empty(ops.sq_partials_shape(M, N), dtype=torch.float32, device=DEV)
                return ops.linear_gated_residual_segmented(x, w, res, gates, lengths, sq=sq), sq
    else:
        H = 4
        w = (torch.randn(3 * H * 128, K, device=DEV) * K ** -0.5).bfloat16()
        nq = (torch.randn(128, device=DEV) * 0.1 + 1).bfloat16()
        nk = (torch.randn(128, device=DEV) * 0.1 + 1).bfloat16()
        table = O.rotary_cache(O.grid_positions(1, 1, M)).to(DEV)
        cos, sin = table[:, :48], table[:, 48:]

        def run():
            outs = [[torch.empty(M, H, 128, dtype=torch.bfloat16, device=DEV)] for _ in range(3)]
            ops.linear_qkv_norm_rope_(outs[0], outs[1], outs[2], x, w, nq, nk, cos, sin, 1e-6)
            return tuple(o[0] for o in outs)
    single = _with_variant(h3, 1, run)
    pair = _with_variant(h3, 2, run)
    flat = lambda r: r if isinstance(r, tuple) else (r,)
    for a, b in zip(flat(single), flat(pair)):
        if isinstance(a, tuple):
            for u, v in zip(a, b):
                assert torch.equal(u, v)
        else:
            assert torch.equal(a, b)
    assert h3.load().h3_device_error() == 0


def test_gemm_variant_rejects_bad_value(h3):
    lib = h3.load()
    prev = lib.h3_gemm_variant(0)
    try:
        assert lib.h3_gemm_variant(3) == -1
        assert lib.h3_gemm_variant(-1) == -1
        assert lib.h3_gemm_variant(0) == 0
    finally:
        lib.h3_gemm_variant(prev)
