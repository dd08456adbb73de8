"""Parity of the fused pointwise kernels (through the C-ABI) with the CPU oracle
and with the reference's golden outputs.

Tolerance: the reference's golden fixtures are matched bit for bit (0 ulp).
Against the CPU oracle at benchmark sizes: <= 1 BF16 ulp per element for the
element-wise ops (gated residual and RoPE are bit-exact), and for the
normalising ops (RMS/LN + AdaLN, q/k norm + RoPE) every element within 3 ulps
at the magnitude of its last add's operands with >= 99.99 % within 1 ulp of
the output (see ``assert_close_ulp``); the same ops are bit-exact against the
oracle summed in the kernels' order (test_parity_order_gpu.py).  The reference reaches 0 ulp against
itself on one device; between CPU and GPU the fp32 sum order of the
normalisation and fp32 exp differ, which flips single BF16 roundings.  The
exact-match fraction is also checked so a systematic drift cannot pass.
"""
import os

import pytest
import torch

from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = torch.load(os.path.join(os.path.dirname(__file__), "golden", "reference_golden.pt"))
DEV = "cuda"


@pytest.fixture(scope="module")
def h3():
    import h3b200
    h3b200.load()
    return h3b200


def _ulps(out, ref):
    return O.bf16_ulp_distance(out.detach().cpu(), ref.detach().cpu())


def _bf16_ulp(mag):
    """BF16 ulp at magnitude |mag| (8 significant bits)."""
    m = mag.float().abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(m)) - 7)


def assert_close_ulp(out, ref, max_ulp=1, min_exact=0.999, mag=None):
    """<= max_ulp BF16 ulps of the output.

    With ``mag`` (the magnitude of the operands of the op's last rounded add,
    e.g. |bf16(n*(1+scale))| + |shift| for AdaLN, |a c| + |b s| for RoPE), for
    ops that normalise first: a 1-ulp difference in the normalisation's
    reciprocal (the fp32 sum of squares is reduced in a different order on the
    CPU and on the GPU) moves each rounded product feeding the last add by at
    most one ulp and the add by one more, which can exceed one ulp of the output
    where the add cancels.  The bound there is: every element within 3 ulps at
    the operands' magnitude, >= 99.99 % of elements within ``max_ulp`` ulps of
    the output."""
    out, ref = out.detach().cpu(), ref.detach().cpu()
    d = _ulps(out, ref)
    exact = float((d == 0).float().mean())
    if mag is None:
        assert int(d.max()) <= max_ulp, f"max ulp {int(d.max())}, exact {exact:.6f}"
    else:
        mag = torch.maximum(mag.detach().cpu().float(), ref.float().abs())
        err = (out.float() - ref.float()).abs()
        worst = float((err / (3 * _bf16_ulp(mag))).max())
        assert worst <= 1.0, f"error {3 * worst:.2f} ulps at operand magnitude"
        within = float((d <= max_ulp).float().mean())
        assert within >= 0.9999, f"only {within:.6f} of elements within {max_ulp} ulp"
    assert exact >= min_exact, f"exact-match fraction {exact:.6f}"


def modulate_mag(normalized, scale, shift):
    """|bf16(n * bf16(1 + scale))| + |shift|: operands of the final add of AdaLN."""
    factor = (scale.float() + 1.0).bfloat16().float()
    return (normalized.float() * factor).abs() + shift.float().abs()


def rope_mag(normalized, cos, sin):
    """|a c| + |b s| (and |b c| + |a s|) per output channel of the NeoX rotation."""
    half = cos.shape[-1]
    n = normalized.float()
    extra = n.dim() - 2
    c, s = cos.float(), sin.float()
    for _ in range(extra):
        c, s = c.unsqueeze(-2), s.unsqueeze(-2)
    a, b = n[..., :half], n[..., half:2 * half]
    return torch.cat([(a * c).abs() + (b * s).abs(), (b * c).abs() + (a * s).abs(), n[..., 2 * half:].abs()], -1)


def g(t):
    return t.to(DEV)


# ---------------------------------------------------------------------------
# golden fixtures from the reference harness
# ---------------------------------------------------------------------------
def test_golden_rms(h3):
    x, w, eps, _ = GOLDEN["op_rms"]["args"]
    assert torch.equal(h3.h3_rms_norm(g(x), g(w), eps).cpu(), GOLDEN["op_rms"]["reference"])


def test_golden_rms_modulate(h3):
    x, w, eps, scale, shift, _ = GOLDEN["op_rms_modulate"]["args"]
    out = h3.h3_rms_modulate(g(x), g(w), g(scale), g(shift), eps)
    assert torch.equal(out.cpu(), GOLDEN["op_rms_modulate"]["reference"])


def test_golden_gated_residual(h3):
    x, gate, y, _ = GOLDEN["op_gated_residual"]["args"]
    out = h3.h3_gated_residual(g(x), g(gate), g(y))
    assert torch.equal(out.cpu(), GOLDEN["op_gated_residual"]["reference"])


def test_golden_gated_residual_rms_modulate(h3):
    x, gate, y, w, eps, scale, shift, _, _ = GOLDEN["op_gated_residual_rms_modulate"]["args"]
    res, out = h3.h3_gated_residual_rms_modulate(g(x), g(gate), g(y), g(w), g(scale), g(shift), eps)
    assert torch.equal(res.cpu(), GOLDEN["op_gated_residual_rms_modulate"]["residual"])
    assert torch.equal(out.cpu(), GOLDEN["op_gated_residual_rms_modulate"]["reference"])


def test_golden_swiglu(h3):
    up, gate, _ = GOLDEN["op_swiglu"]["args"]
    assert_close_ulp(h3.h3_swiglu(g(up), g(gate)), GOLDEN["op_swiglu"]["reference"])


def test_golden_rope(h3):
    x, cos, sin = GOLDEN["op_rope"]["args"]
    assert torch.equal(h3.h3_rope(g(x), g(cos), g(sin)).cpu(), GOLDEN["op_rope"]["reference"])


def test_golden_qk_norm_rope_send_layout(h3):
    a = GOLDEN["op_qk_norm_rope"]["args"]
    x, w, eps, cos, sin = a[0], a[3], a[6], a[7], a[8]
    t, p, hs, d = x.shape
    send = torch.empty(p, t, hs, d, dtype=torch.bfloat16, device=DEV)
    h3.h3_qk_norm_rope_(send.permute(1, 0, 2, 3), g(x), g(w), g(cos), g(sin), eps)
    assert torch.equal(send.cpu(), GOLDEN["op_qk_norm_rope"]["reference"])


@pytest.mark.parametrize("family", ["grid_8_32_32", "integer", "uniform", "fine", "fine64"])
def test_golden_rope_cache(h3, family):
    e = GOLDEN["rotary_cache"][family]
    out = h3.h3_rope_cache(g(e["positions"]), g(GOLDEN["rotary_cache"]["power"]))
    assert torch.equal(out.cpu(), e["table"])


def test_rope_cache_config1_grid_vs_host_fp32_table(h3):
    """Config-1 grid (8,32,32) against the oracle table built with the host's fp32
    cos/sin (which can differ from the correctly rounded values by an fp32 ulp):
    within 1 BF16 ulp.  The bit-exact check is test_parity_order_gpu's."""
    pos = O.grid_positions(8, 32, 32)
    out = h3.h3_rope_cache(g(pos), h3.rope_powers()[:16].contiguous())
    assert_close_ulp(out, O.rotary_cache(pos), min_exact=0.9995)


def test_timestep_embedding_golden(h3):
    e = GOLDEN["timestep_embedding"]
    out = h3.timestep_embedding(g(e["t"]), e["dim"])
    torch.testing.assert_close(out.cpu(), e["out"], atol=2e-5, rtol=2e-5)


# ---------------------------------------------------------------------------
# benchmark config-1 shapes, seed 0, vs the CPU oracle
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def cfg1():
    torch.manual_seed(0)
    S, H, D, C, F = 8192, 14, 128, 1792, 4864
    c = {
        "q": torch.randn(S, H, D).bfloat16(), "k": torch.randn(S, H, D).bfloat16(),
        "qk_w": (torch.randn(D) * 0.1 + 1).bfloat16(),
        "x": torch.randn(S, C).bfloat16(), "scale": (torch.randn(C) * 0.1).bfloat16(),
        "shift": (torch.randn(C) * 0.1).bfloat16(), "norm_w": (torch.randn(C) * 0.1 + 1).bfloat16(),
        "a": torch.randn(S, F).bfloat16(), "b": torch.randn(S, F).bfloat16(),
        "y": torch.randn(S, C).bfloat16(), "gate": (torch.randn(C) * 0.1).bfloat16(),
        "pos": O.grid_positions(8, 32, 32),
    }
    return c


def test_cfg1_gated_residual(h3, cfg1):
    c = cfg1
    out = h3.h3_gated_residual(g(c["x"]), g(c["gate"]), g(c["y"]))
    ref = O.gated_residual(c["x"], c["gate"].expand_as(c["x"]), c["y"])
    assert torch.equal(out.cpu(), ref)


def test_cfg1_swiglu(h3, cfg1):
    out = h3.h3_swiglu(g(cfg1["a"]), g(cfg1["b"]))
    assert_close_ulp(out, O.swiglu(cfg1["a"], cfg1["b"]))


def test_cfg1_rms_modulate(h3, cfg1):
    c = cfg1
    out = h3.h3_rms_modulate(g(c["x"]), g(c["norm_w"]), g(c["scale"]), g(c["shift"]), 1e-6)
    assert_close_ulp(out, O.rms_modulate(c["x"], c["norm_w"], c["scale"], c["shift"], 1e-6),
                     mag=modulate_mag(O.rms_norm(c["x"], c["norm_w"], 1e-6), c["scale"], c["shift"]))


def test_cfg1_ln_modulate(h3, cfg1):
    c = cfg1
    out = h3.h3_ln_modulate(g(c["x"]), g(c["scale"]), g(c["shift"]), 1e-6)
    n = torch.nn.functional.layer_norm(c["x"].float(), (c["x"].shape[-1],), eps=1e-6).bfloat16()
    assert_close_ulp(out, O.ln_modulate(c["x"], c["scale"], c["shift"], 1e-6), min_exact=0.995,
                     mag=modulate_mag(n, c["scale"], c["shift"]))


def test_cfg1_gated_residual_rms_modulate(h3, cfg1):
    c = cfg1
    res, out = h3.h3_gated_residual_rms_modulate(g(c["x"]), g(c["gate"]), g(c["y"]), g(c["norm_w"]),
                                                 g(c["scale"]), g(c["shift"]), 1e-6)
    rref, oref = O.gated_residual_rms_modulate(c["x"], c["gate"], c["y"], c["norm_w"], c["scale"],
                                               c["shift"], 1e-6)
    assert torch.equal(res.cpu(), rref)
    assert_close_ulp(out, oref, mag=modulate_mag(O.rms_norm(rref, c["norm_w"], 1e-6), c["scale"], c["shift"]))


@pytest.mark.parametrize("sections", [(16, 16, 16), (22, 21, 21)])
def test_cfg1_qk_norm_rope(h3, cfg1, sections):
    """Reference layout (48 pairs) and the full-D 44/42/42 layout (64 pairs)."""
    c = cfg1
    powers = O.rope_powers(sections)
    if sections == (16, 16, 16):
        table = h3.h3_rope_cache(g(c["pos"]), g(powers[0]))
    else:
        table = h3.h3_rope_cache_sectioned(g(c["pos"]), g(torch.cat(powers)), sections)
    ref_table = O.rotary_cache(c["pos"], sections)
    assert_close_ulp(table, ref_table, min_exact=0.999)
    half = sum(sections)
    cos, sin = ref_table[:, :half], ref_table[:, half:]
    for name in ("q", "k"):
        x = c[name]
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=DEV)
        h3.h3_qk_norm_rope_(out.unsqueeze(1), g(x).unsqueeze(1), g(c["qk_w"]), g(cos), g(sin), 1e-6)
        assert_close_ulp(out, O.qk_norm_rope(x, c["qk_w"], cos, sin, 1e-6),
                         mag=rope_mag(O.rms_norm(x, c["qk_w"], 1e-6), cos, sin))


# ---------------------------------------------------------------------------
# layouts and edge cases (after tools/verify_h3_pointwise_native.py:26-77)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("width", [128, 1792, 5120, 5376, 7168])
@pytest.mark.parametrize("scale", [0.01, 1.0, 100.0])
def test_rms_family_odd_strides(h3, width, scale):
    torch.manual_seed(42)
    packed = torch.randn(2, 129, width * 2 + 1, dtype=torch.bfloat16) * scale
    x = packed[..., 1:width + 1]                       # misaligned, strided rows
    weight_full = torch.randn(width * 2, dtype=torch.bfloat16)
    weight = weight_full[::2]                          # strided weight
    table = torch.randn(2, 129, width * 6, dtype=torch.bfloat16)
    shift, mscale = table[..., :width], table[..., width:2 * width]
    mscale[:, :3] = -1.0                               # scale == -1 edge case
    gx, gt = g(packed)[..., 1:width + 1], g(table)
    gweight = g(weight_full)[::2]
    gshift, gscale = gt[..., :width], gt[..., width:2 * width]
    assert_close_ulp(h3.h3_rms_norm(gx, gweight, 1e-5), O.rms_norm(x, weight, 1e-5))
    assert_close_ulp(h3.h3_rms_modulate(gx, gweight, gscale, gshift, 1e-5),
                     O.rms_modulate(x, weight, mscale, shift, 1e-5),
                     mag=modulate_mag(O.rms_norm(x, weight, 1e-5), mscale, shift))


@pytest.mark.parametrize("width", [7168, 4864, 13824])
def test_swiglu_strided_halves(h3, width):
    torch.manual_seed(1)
    packed = torch.randn(2, 129, width * 2 + 1, dtype=torch.bfloat16) * 2
    up, gate = packed[..., 1:width + 1], packed[..., width + 1:]
    gp = g(packed)
    out = h3.h3_swiglu(gp[..., 1:width + 1], gp[..., width + 1:])
    assert_close_ulp(out, O.swiglu(up, gate))
    # aligned halves take the vectorised path; same bits as the strided path
    packed2 = torch.randn(257, 2 * width, dtype=torch.bfloat16) * 2
    gp2 = g(packed2)
    fast = h3.h3_swiglu(gp2[:, :width], gp2[:, width:])
    slow = h3.h3_swiglu(gp2[:, :width].t().contiguous().t(), gp2[:, width:].t().contiguous().t())
    assert torch.equal(fast, slow)
    assert_close_ulp(fast, O.swiglu(packed2[:, :width], packed2[:, width:]))


def test_vectorised_and_strided_paths_identical(h3):
    torch.manual_seed(3)
    x = torch.randn(300, 5120, dtype=torch.bfloat16, device=DEV) * 4
    w = torch.randn(5120, dtype=torch.bfloat16, device=DEV)
    sc = torch.randn(5120, dtype=torch.bfloat16, device=DEV) * 0.5
    sh = torch.randn(5120, dtype=torch.bfloat16, device=DEV) * 0.5
    fast = h3.h3_rms_modulate(x, w, sc, sh, 1e-6)
    xs = x.t().contiguous().t()                       # column-major: strided path
    slow = h3.h3_rms_modulate(xs, w, sc, sh, 1e-6)
    assert torch.equal(fast, slow)


def test_rope_seq_heads_shapes(h3):
    """tools/verify_h3_pointwise_native.py:50-62 shapes, strided x."""
    for seq, heads in ((17, 28), (257, 56), (2304, 28)):
        torch.manual_seed(seq)
        x = torch.randn(seq, heads, 385, dtype=torch.bfloat16)[..., 1:129]
        angles = torch.randn(seq, 97, dtype=torch.bfloat16)
        c, s = angles[:, 1:49], angles[:, 49:97]
        gx = g(x)
        out = h3.h3_rope(gx, g(angles)[:, 1:49], g(angles)[:, 49:97])
        assert torch.equal(out.cpu(), O.rope(x, c, s))


def test_qk_norm_rope_fused_qkv_views(h3):
    """x is the q slice of a fused [T, 3, P*Hs, 128] projection viewed [T, P, Hs, 128];
    out is the permuted view of the all-to-all send buffer [P, T, Hs, 128]
    (patches/InfiniLM.patch:1092-1103)."""
    torch.manual_seed(7)
    T, P, Hs = 1000, 4, 5
    projected = torch.randn(T, 3, P * Hs, 128, dtype=torch.bfloat16)
    w = (torch.rand(128) + 0.5).bfloat16()
    tbl = O.rotary_cache(O.grid_positions(10, 10, 10))
    cos, sin = tbl[:, :48], tbl[:, 48:]
    gp = g(projected)
    for i in (0, 1):
        src = gp[:, i].view(T, P, Hs, 128)
        send = torch.empty(P, T, Hs, 128, dtype=torch.bfloat16, device=DEV)
        h3.h3_qk_norm_rope_(send.permute(1, 0, 2, 3), src, g(w), g(cos), g(sin), 1e-6)
        xi = projected[:, i].view(T, P, Hs, 128)
        ref = O.qk_norm_rope(xi, w, cos, sin, 1e-6).permute(1, 0, 2, 3)
        mag = rope_mag(O.rms_norm(xi, w, 1e-6), cos, sin).permute(1, 0, 2, 3)
        assert_close_ulp(send, ref, mag=mag)


def test_broadcast_modulation_rows_stride0(h3):
    torch.manual_seed(5)
    x = torch.randn(1, 777, 1792, dtype=torch.bfloat16)
    table = torch.randn(3, 6 * 1792, dtype=torch.bfloat16) * 0.2
    row = 1
    gtab = g(table)
    col = lambda i: gtab[row, i * 1792:(i + 1) * 1792].as_strided((1, 777, 1792), (0, 0, 1))
    w = torch.ones(1792, dtype=torch.bfloat16)
    out = h3.h3_rms_modulate(g(x), g(w), col(1), col(0), 1e-6)
    ref = O.rms_modulate(x, w, table[row, 1792:2 * 1792], table[row, :1792], 1e-6)
    assert_close_ulp(out, ref)


def test_bad_inputs_raise(h3):
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        h3.h3_gated_residual(x, x.float(), x)
    with pytest.raises(ValueError):
        h3.h3_gated_residual(x, torch.zeros(4, 32, dtype=torch.bfloat16, device=DEV), x)
    with pytest.raises(ValueError):
        h3.h3_rms_norm(x, torch.zeros(63, dtype=torch.bfloat16, device=DEV), 1e-6)


def test_empty_inputs(h3):
    x = torch.zeros(0, 1792, dtype=torch.bfloat16, device=DEV)
    w = torch.ones(1792, dtype=torch.bfloat16, device=DEV)
    assert h3.h3_rms_norm(x, w, 1e-6).shape == (0, 1792)
    assert h3.h3_swiglu(x, x).shape == (0, 1792)


def test_no_device_wait_expired(h3):
    assert h3.load().h3_device_error() == 0
