"""Bit-exact parity of the normalising kernels with the CPU oracle summed in the
kernel's own order, and the fused out-projection + gated residual + RMSNorm +
AdaLN path.

The reference's RMSNorm sums bf16(x^2) in fp32 in its device's order; the
torch oracle sums in the host CPU's vector order, the CUDA kernels in a fixed
order of their own.  ``oracle.sum_squares_in_kernel_order`` restates each
kernel's order; with it every other step of the op is a correctly rounded fp32
or BF16 operation on both sides, so the kernels must match it bit for bit
(tolerance: 0 ulp).  Against the reference-order oracle the same outputs differ
only where the two sums round to different BF16 means; those differences are
reported (max ulp and exact-match fraction, one ``PARITY`` line per case, shown
with ``pytest -s``) and bounded by the tolerance of the pointwise tests.
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


def _report(op, shape, out, kernel_ref, reference):
    out = out.detach().cpu()
    d_ref = O.bf16_ulp_distance(out, reference)
    exact_kernel = float((O.bf16_ulp_distance(out, kernel_ref) == 0).float().mean())
    print(f"PARITY op={op} shape={list(shape)} max_ulp_vs_reference={int(d_ref.max())} "
          f"exact_vs_reference={float((d_ref == 0).float().mean()):.6f} "
          f"exact_vs_kernel_order={exact_kernel:.6f}")
    assert torch.equal(out, kernel_ref), f"{op}: {1 - exact_kernel:.2e} of elements differ from the kernel-order oracle"


def _rows(rows, width, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, width, generator=g).bfloat16()
    w = (torch.randn(width, generator=g) * 0.1 + 1).bfloat16()
    scale = (torch.randn(width, generator=g) * 0.1).bfloat16()
    shift = (torch.randn(width, generator=g) * 0.1).bfloat16()
    return x, w, scale, shift


SHAPES = [(8192, 1792), (18944, 5120)]   # benchmark config 1, the step's token rows


@pytest.mark.parametrize("rows,width", SHAPES)
def test_rms_norm_and_modulate_in_kernel_order(h3, rows, width):
    x, w, scale, shift = _rows(rows, width, 0)
    gx, gw = x.to(DEV), w.to(DEV)
    out = h3.h3_rms_norm(gx, gw, 1e-6)
    _report("rms_norm", x.shape, out, O.rms_norm_in_kernel_order(x, w, 1e-6, "row"), O.rms_norm(x, w, 1e-6))
    out = h3.h3_rms_modulate(gx, gw, scale.to(DEV), shift.to(DEV), 1e-6)
    _report("rms_modulate", x.shape, out, O.rms_modulate_in_kernel_order(x, w, scale, shift, 1e-6, "row"),
            O.rms_modulate(x, w, scale, shift, 1e-6))


@pytest.mark.parametrize("rows,width", SHAPES)
def test_gated_residual_rms_modulate_in_kernel_order(h3, rows, width):
    x, w, scale, shift = _rows(rows, width, 1)
    y, _, gate, _ = _rows(rows, width, 2)
    res, out = h3.h3_gated_residual_rms_modulate(x.to(DEV), gate.to(DEV), y.to(DEV), w.to(DEV), scale.to(DEV),
                                                 shift.to(DEV), 1e-6)
    rref = O.gated_residual(x, gate, y)
    assert torch.equal(res.cpu(), rref)
    _report("gated_residual_rms_modulate", x.shape, out,
            O.rms_modulate_in_kernel_order(rref, w, scale, shift, 1e-6, "row"),
            O.rms_modulate(rref, w, scale, shift, 1e-6))


@pytest.mark.parametrize("tokens,heads", [(8192, 14), (18944, 40)])
def test_qk_norm_rope_in_kernel_order(h3, tokens, heads):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(tokens, heads, 128, generator=g).bfloat16()
    w = (torch.randn(128, generator=g) * 0.1 + 1).bfloat16()
    side = 1
    while side * side * 8 < tokens:
        side += 1
    table = O.rotary_cache(O.grid_positions(8, side, side)[:tokens])
    cos, sin = table[:, :48], table[:, 48:]
    out = torch.empty(tokens, heads, 128, dtype=torch.bfloat16, device=DEV)
    h3.h3_qk_norm_rope_(out.unsqueeze(1), x.to(DEV).unsqueeze(1), w.to(DEV), cos.to(DEV), sin.to(DEV), 1e-6)
    _report("qk_norm_rope", x.shape, out, O.qk_norm_rope_in_kernel_order(x, w, cos, sin, 1e-6),
            O.qk_norm_rope(x, w, cos, sin, 1e-6))


def test_rope_cache_integer_grid_bit_exact(h3):
    """Config-1 grid (8,32,32) and the step's (32,24,24): integer positions; the
    table equals the oracle with cos/sin evaluated in float64 and rounded once,
    as the kernel evaluates them (no BF16 difference at all)."""
    for grid in ((8, 32, 32), (32, 24, 24)):
        pos = O.grid_positions(*grid)
        out = h3.h3_rope_cache(pos.to(DEV), h3.rope_powers()[:16].contiguous())
        assert torch.equal(out.cpu(), O.rotary_cache_correctly_rounded(pos))


# ---------------------------------------------------------------------------
# out-projection + gated residual + per-tile sums of squares, then the norm pass
# ---------------------------------------------------------------------------
def _proj_case(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).bfloat16()
    wt = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
    res = torch.randn(m, n, generator=g).bfloat16()
    gate = (torch.randn(n, generator=g) * 0.5).bfloat16()
    nw = (torch.randn(n, generator=g) * 0.1 + 1).bfloat16()
    sc = (torch.randn(n, generator=g) * 0.1).bfloat16()
    sh = (torch.randn(n, generator=g) * 0.1).bfloat16()
    return a, wt, res, gate, nw, sc, sh


@pytest.mark.parametrize("m,n,k", [(18944, 5120, 5120), (1000, 1792, 512), (300, 640, 256)])
def test_linear_gated_residual_sq(h3, m, n, k):
    """Output bitwise the unfused projection epilogue's; the partial sums equal the
    oracle's per-tile column-order sums of the same output bit for bit."""
    a, wt, res, gate, *_ = _proj_case(m, n, k, 4)
    ga, gw, gr, gg = a.to(DEV), wt.to(DEV), res.to(DEV), gate.to(DEV)
    plain = h3.linear_gated_residual(ga, gw, gr, gg)
    out, sq = h3.linear_gated_residual_sq(ga, gw, gr, gg)
    assert torch.equal(out, plain)
    assert sq.shape == (m, (n + 255) // 256)
    assert torch.equal(sq.cpu(), O.tile_square_partials(out.cpu()))


@pytest.mark.parametrize("rows,width", SHAPES + [(77, 640)])
def test_rms_modulate_sq_in_kernel_order(h3, rows, width):
    x, w, scale, shift = _rows(rows, width, 5)
    sq = O.tile_square_partials(x)
    out = torch.empty_like(x, device=DEV)
    h3.h3_rms_modulate_sq_(out, x.to(DEV), sq.to(DEV), w.to(DEV), scale.to(DEV), shift.to(DEV), 1e-6)
    _report("rms_modulate_sq", x.shape, out, O.rms_modulate_in_kernel_order(x, w, scale, shift, 1e-6, "tiles"),
            O.rms_modulate(x, w, scale, shift, 1e-6))


def test_fused_out_projection_norm_equals_two_steps(h3):
    """The composite entry point (caller-owned workspace) equals its two launches,
    and its residual equals the unfused projection + K8 residual bit for bit."""
    a, wt, res, gate, nw, sc, sh = [t.to(DEV) for t in _proj_case(2048, 5120, 1024, 6)]
    r1, o1 = h3.linear_gated_residual_rms_modulate(a, wt, res, gate, nw, sc, sh, 1e-6)
    r2, sq = h3.linear_gated_residual_sq(a, wt, res, gate)
    o2 = h3.h3_rms_modulate_sq_(torch.empty_like(r2), r2, sq, nw, sc, sh, 1e-6)
    assert torch.equal(r1, r2) and torch.equal(o1, o2)
    proj = h3.linear(a, wt)
    r3, o3 = h3.h3_gated_residual_rms_modulate(res, gate, proj, nw, sc, sh, 1e-6)
    assert torch.equal(r1, r3)
    # the norm halves differ only by the sum order (tile partials vs one warp per row)
    d = O.bf16_ulp_distance(o1.cpu(), o3.cpu())
    assert float((d == 0).float().mean()) > 0.999


def test_sq_entry_points_reject_bad_partials(h3):
    x = torch.zeros(16, 512, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(512, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):   # wrong tile count
        h3.h3_rms_modulate_sq_(x.clone(), x, torch.zeros(16, 3, device=DEV), w, w, w, 1e-6)
    with pytest.raises(ValueError):   # wrong dtype
        h3.h3_rms_modulate_sq_(x.clone(), x, torch.zeros(16, 2, dtype=torch.float64, device=DEV), w, w, w, 1e-6)
    assert h3.load().h3_device_error() == 0


# ---------------------------------------------------------------------------
# one launch over all modulation segments == one launch per segment
# ---------------------------------------------------------------------------
def test_segmented_launches_equal_per_segment(h3):
    m, n, k = 1000, 1280, 512
    a, wt, res, _, nw, _, _ = [t.to(DEV) for t in _proj_case(m, n, k, 8)]
    g = torch.Generator().manual_seed(9)
    table = (torch.randn(3, 6 * n, generator=g) * 0.3).bfloat16().to(DEV)
    lengths = [600, 13, 387]
    starts = [0, 600, 613]
    row = lambda s, i: table[s, i * n:(i + 1) * n]  # noqa: E731
    # projection + gated residual (+ sums of squares)
    seg_out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    seg_sq = torch.empty(m, (n + 255) // 256, dtype=torch.float32, device=DEV)
    h3.linear_gated_residual_segmented(a, wt, res, [row(s, 2) for s in range(3)], lengths, out=seg_out, sq=seg_sq)
    plain = torch.empty_like(seg_out)
    h3.linear_gated_residual_segmented(a, wt, res, [row(s, 2) for s in range(3)], lengths, out=plain)
    ref_out, ref_sq = torch.empty_like(seg_out), torch.empty_like(seg_sq)
    for s, (st, ln) in enumerate(zip(starts, lengths)):
        r = slice(st, st + ln)
        h3.linear_gated_residual_sq(a[r], wt, res[r], row(s, 2), out=ref_out[r], sq=ref_sq[r])
    assert torch.equal(seg_out, ref_out) and torch.equal(seg_sq, ref_sq) and torch.equal(plain, ref_out)
    # norm pass, from the partials and with its own reduction
    for sq in (seg_sq, None):
        seg = h3.h3_rms_modulate_segmented_(torch.empty_like(seg_out), seg_out, sq, nw,
                                            [row(s, 1) for s in range(3)], [row(s, 0) for s in range(3)], lengths,
                                            1e-6)
        ref = torch.empty_like(seg_out)
        for s, (st, ln) in enumerate(zip(starts, lengths)):
            r = slice(st, st + ln)
            if sq is None:
                h3.h3_rms_modulate_(ref[r], seg_out[r], nw, row(s, 1), row(s, 0), 1e-6)
            else:
                h3.h3_rms_modulate_sq_(ref[r], seg_out[r], sq[r], nw, row(s, 1), row(s, 0), 1e-6)
        assert torch.equal(seg, ref)
    with pytest.raises(ValueError):   # the lengths must cover every row
        h3.linear_gated_residual_segmented(a, wt, res, [row(0, 2)], [999], out=torch.empty_like(seg_out))
    assert h3.load().h3_device_error() == 0
