"""The CPU oracle against fixtures generated from the reference's own torch code
(tests/golden/make_golden.py).  Everything here is bit-exact."""
import os

import pytest
import torch

from oracle import h3_oracle as O

GOLDEN = torch.load(os.path.join(os.path.dirname(__file__), "golden", "reference_golden.pt"))


def _args(name):
    return GOLDEN[name]["args"]


def test_rms_norm_golden():
    x, w, eps, _ = _args("op_rms")
    assert torch.equal(O.rms_norm(x, w, eps), GOLDEN["op_rms"]["reference"])


def test_rms_modulate_golden():
    x, w, eps, scale, shift, _ = _args("op_rms_modulate")
    assert torch.equal(O.rms_modulate(x, w, scale, shift, eps), GOLDEN["op_rms_modulate"]["reference"])


def test_gated_residual_golden():
    x, gate, y, _ = _args("op_gated_residual")
    assert torch.equal(O.gated_residual(x, gate, y), GOLDEN["op_gated_residual"]["reference"])


def test_gated_residual_rms_modulate_golden():
    x, gate, y, w, eps, scale, shift, _, _ = _args("op_gated_residual_rms_modulate")
    res, out = O.gated_residual_rms_modulate(x, gate, y, w, scale, shift, eps)
    assert torch.equal(res, GOLDEN["op_gated_residual_rms_modulate"]["residual"])
    assert torch.equal(out, GOLDEN["op_gated_residual_rms_modulate"]["reference"])


def test_swiglu_golden():
    up, gate, _ = _args("op_swiglu")
    assert torch.equal(O.swiglu(up, gate), GOLDEN["op_swiglu"]["reference"])


def test_rope_golden():
    x, cos, sin = _args("op_rope")
    assert torch.equal(O.rope(x, cos, sin), GOLDEN["op_rope"]["reference"])


def test_qk_norm_rope_golden():
    a = _args("op_qk_norm_rope")
    x, w, eps, cos, sin = a[0], a[3], a[6], a[7], a[8]
    ref = GOLDEN["op_qk_norm_rope"]["reference"]           # [P, T, Hs, D] send layout
    out = O.qk_norm_rope(x, w, cos, sin, eps)              # [T, P, Hs, D]
    assert torch.equal(out.permute(1, 0, 2, 3).contiguous(), ref)


def test_rope_cache_harness_golden():
    positions, power, _, _ = _args("op_rope_cache")
    assert torch.equal(O.rotary_cache(positions), GOLDEN["op_rope_cache"]["reference"])
    assert torch.equal(O.rope_powers()[0], power)


@pytest.mark.parametrize("family", ["grid_8_32_32", "integer", "uniform", "fine", "fine64"])
def test_rotary_cache_golden(family):
    entry = GOLDEN["rotary_cache"][family]
    assert torch.equal(O.rotary_cache(entry["positions"]), entry["table"])


def test_grid_positions_bit_exact():
    assert torch.equal(O.grid_positions(8, 32, 32), GOLDEN["rotary_cache"]["grid_8_32_32"]["positions"])


def test_attention_golden():
    g = GOLDEN["attention"]
    q, k, v = (g[n].permute(0, 2, 1, 3) for n in ("q", "k", "v"))   # -> [B, S, H, D]
    out = O.attention_fp32(q, k, v, 128 ** -0.5, chunk=50).permute(0, 2, 1, 3)
    assert torch.allclose(out, g["fp32"], atol=1e-5, rtol=1e-5)
    # SDPA's own output is BF16 (|o| < 0.6 here, so one BF16 ulp <= 2^-9)
    assert (out - g["sdpa"].float()).abs().max() <= 2 * 2.0 ** -9


def test_timestep_embedding_golden():
    g = GOLDEN["timestep_embedding"]
    assert torch.allclose(O.timestep_embedding(g["t"], g["dim"]), g["out"], atol=2e-5, rtol=2e-5)


def test_ulp_metric():
    a = torch.tensor([1.0, -1.0, 0.0, 2.0], dtype=torch.bfloat16)
    b = torch.tensor([1.0078125, -1.0078125, -0.0, 2.0], dtype=torch.bfloat16)
    assert O.bf16_ulp_distance(a, b).tolist() == [1, 1, 0, 0]


def test_ulysses_permutation_roundtrip():
    """Tokens->heads->tokens with uneven head groups is the identity (integer layout)."""
    world, tokens, heads, d = 4, 3, 8, 2
    locals_ = [torch.arange(r * 1000, r * 1000 + tokens * heads * d).view(tokens, heads, d)
               for r in range(world)]
    groups = [1, 1]
    returned = [[] for _ in range(world)]
    off = 0
    for hs in groups:
        send = [O.ulysses_send_blocks(l, world, off, hs) for l in locals_]
        recv = O.ulysses_all_to_all(send)
        for r in range(world):
            glob = O.ulysses_gather(recv[r])              # [W*T, hs, d], global token order
            assert torch.equal(glob[:tokens], send[0][r]) # rank 0's tokens first
        back = O.ulysses_all_to_all(recv)                 # attention = identity here
        for r in range(world):
            returned[r].append(back[r])
        off += hs
    for r in range(world):
        out = O.ulysses_scatter_back(returned[r], groups)  # [T, W, Hl, D]
        assert torch.equal(out.reshape(tokens, heads, d), locals_[r])


def test_kernel_order_sums_match_hand_computation():
    """The kernel-order restatements on a case small enough to add by hand."""
    torch.manual_seed(0)
    sq = O._r(torch.randn(3, 16) ** 2).float()
    # row kernel: two vectors (lanes 0 and 1), each summed left to right, then the tree
    lane0 = torch.zeros(3)
    lane1 = torch.zeros(3)
    for j in range(8):
        lane0 = lane0 + sq[:, j]
        lane1 = lane1 + sq[:, 8 + j]
    assert torch.equal(O.sum_squares_in_kernel_order(sq, "row"), lane0 + lane1)
    # tiles: one partial per 256 columns, here one tile
    assert torch.equal(O.sum_squares_in_kernel_order(sq, "tiles"), O._serial_sum(sq))
    assert O.tile_square_partials(torch.randn(2, 600).bfloat16()).shape == (2, 3)   # ragged last tile


def test_kernel_order_sums_close_to_exact():
    torch.manual_seed(1)
    for width, order in ((1792, "row"), (5120, "row"), (5120, "tiles"), (128, "head")):
        sq = O._r(torch.randn(64, width) ** 2).float()
        exact = sq.double().sum(-1)
        got = O.sum_squares_in_kernel_order(sq, order).double()
        assert float(((got - exact) / exact).abs().max()) < 1e-5


def test_tile_partials_feed_the_tile_order():
    torch.manual_seed(2)
    x = torch.randn(5, 5120).bfloat16()
    partials = O.tile_square_partials(x)
    assert partials.shape == (5, 20)
    sq = O._r(x.float() * x.float()).float()
    lanes = torch.zeros(5, 32)
    lanes[:, :20] = partials
    assert torch.equal(O._xor_tree(lanes), O.sum_squares_in_kernel_order(sq, "tiles"))


def test_kernel_order_norm_equals_reference_on_most_rows():
    """Only the fp32 sum order differs from the reference restatement: the BF16
    outputs agree on nearly every element."""
    torch.manual_seed(3)
    x = torch.randn(512, 5120).bfloat16()
    w = (torch.randn(5120) * 0.1 + 1).bfloat16()
    for order in ("row", "tiles"):
        d = O.bf16_ulp_distance(O.rms_norm_in_kernel_order(x, w, 1e-6, order), O.rms_norm(x, w, 1e-6))
        assert int(d.max()) <= 1 and float((d == 0).float().mean()) > 0.99


def test_correctly_rounded_rope_table_close_to_reference():
    pos = O.grid_positions(8, 32, 32)
    d = O.bf16_ulp_distance(O.rotary_cache_correctly_rounded(pos), O.rotary_cache(pos))
    assert int(d.max()) <= 1
