"""CPU oracle for the MiniMax-H3 DiT-block hot path.  TEST INFRASTRUCTURE ONLY.

This module restates, in eager PyTorch on the CPU, the arithmetic of the
reference's torch compositions for every op on the path, with each BF16
rounding step where the reference places it.  It is the checker for the CUDA
kernels: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg use it.  The product path never imports it.

Parity is pinned: ``tests/test_oracle_golden.py`` checks these functions
bit-for-bit against fixtures generated from the reference's own code
(``tests/golden/make_golden.py`` imports ``tools/bench_h3_ops.py``).

Reference anchors (file:line inside the reference tree; patches are cited by
line number inside the patch file):

* RMSNorm, staged BF16:        tools/bench_h3_ops.py:81-88, kernel tools/h3_pointwise.py:46-57
* AdaLN modulate:              tools/bench_h3_ops.py:91-93, tools/h3_pointwise.py:83-97
* RoPE (NeoX, 3 axes):         tools/bench_h3_ops.py:96-106, tools/h3_pointwise.py:199-214
* RoPE table:                  tools/bench_h3_ops.py:109-113, patches/InfiniLM.patch:6605-6634
* q/k norm + RoPE:             tools/bench_h3_ops.py:129-153, tools/h3_pointwise.py:262-294
* gated residual:              tools/bench_h3_ops.py:208-218, tools/h3_pointwise.py:121-124
* gated residual + RMS/AdaLN:  tools/bench_h3_ops.py:221-241, tools/h3_pointwise.py:150-168
* SwiGLU:                      tools/bench_h3_ops.py:244-258, tools/h3_pointwise.py:18-22
* attention (fp32 math):       tools/verify_attention.py:60-64, tools/h3_attention.py:25-41
* block composition:           patches/InfiniLM.patch:1303-1397 (forward, forward_segmented)
* MLP:                         patches/InfiniLM.patch:1172-1179 ([up; gate] rows, :5775-5784)
* Ulysses permutations:        patches/InfiniLM.patch:895-1137
* timestep embedding:          patches/InfiniCore.patch:2115-2137 (kernel), :2834-2845 (test formula)
* model forward around blocks: patches/InfiniLM.patch:1626-1826 (packing, output norm/projections),
                               :1198-1241 (token refiner), :1494-1538 (time embedder, output norm)
"""
from __future__ import annotations

import math
from typing import Sequence

import torch

BF16 = torch.bfloat16


def _r(t: torch.Tensor) -> torch.Tensor:
    """Round an fp32 tensor to BF16 (round-to-nearest-even), as ``.to(bf16)``."""
    return t.to(BF16)


# --------------------------------------------------------------------------
# RMSNorm / AdaLN (tools/bench_h3_ops.py:81-93)
# --------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Staged BF16 RMSNorm over the last axis: sq=bf16(x*x); mean=bf16(sum/D);
    var=bf16(mean+eps); r=bf16(1/sqrt(var)); out=bf16(bf16(x*r)*w)."""
    xf = x.float()
    squared = _r(xf * xf)
    mean = _r(squared.float().sum(-1, keepdim=True) / x.shape[-1])
    variance = _r(mean.float() + torch.tensor(eps, dtype=torch.float32))
    reciprocal = _r(torch.rsqrt(variance.float()))
    return _r(_r(xf * reciprocal.float()).float() * weight.float())


# --------------------------------------------------------------------------
# The CUDA kernels' fixed summation orders for the RMSNorm sum of squares.
# The reference sums in its device's order (the torch oracle above in the host
# CPU's vector order); the sum is fp32 and the mean is rounded to BF16, so a
# different order can move the mean by one BF16 ulp on rare rows.  These
# restatements sum in exactly the order each CUDA kernel uses, so a kernel can be
# checked bit for bit: with the same order every other step is a correctly
# rounded fp32 or BF16 operation on both sides.
# --------------------------------------------------------------------------
def _serial_sum(cols: torch.Tensor) -> torch.Tensor:
    """fp32 sum over the last axis, one rounding per addition, left to right."""
    acc = torch.zeros(cols.shape[:-1], dtype=torch.float32)
    for j in range(cols.shape[-1]):
        acc = acc + cols[..., j]
    return acc


def _xor_tree(lanes: torch.Tensor) -> torch.Tensor:
    """An xor-shuffle butterfly over the last axis (a power of two, largest stride
    first): lane l adds lane l ^ o; every lane ends with the same value."""
    n = lanes.shape[-1]
    idx = torch.arange(n)
    o = n // 2
    while o >= 1:
        lanes = lanes + lanes[..., idx ^ o]
        o //= 2
    return lanes[..., 0]


def sum_squares_in_kernel_order(squared: torch.Tensor, order: str) -> torch.Tensor:
    """Row sums [R] of the fp32 values bf16(x^2) [R, C] in a kernel's order.

    ``"row"``  -- the row kernels (one warp per row): lane l adds, in column order,
                  the 8 columns of each of its vectors l, l+32, l+64, ...; then
                  the 32-lane xor tree.
    ``"head"`` -- the q/k head kernel and the QKV epilogue (C = 128): 16 lanes,
                  lane l adds columns 8l..8l+7 in order; then the 16-lane tree.
    ``"tiles"``-- a projection epilogue's per-256-column partials (each summed in
                  column order) combined by ``h3_rms_modulate_sq``: lane l adds
                  partials l, l+32, ... in order; then the 32-lane tree."""
    r, c = squared.shape
    sq = squared.float()
    if order == "head":
        lanes = _serial_sum(sq.view(r, 16, 8))
        return _xor_tree(lanes)
    if order == "row":
        nvec = (c + 7) // 8
        vpt = (nvec + 31) // 32
        padded = torch.zeros(r, vpt * 32 * 8)
        padded[:, :c] = sq
        # element (k, lane, e) = column (lane + 32 k) * 8 + e; lane order: k major, then e
        per_lane = padded.view(r, vpt, 32, 8).permute(0, 2, 1, 3).reshape(r, 32, vpt * 8)
        return _xor_tree(_serial_sum(per_lane))
    if order == "tiles":
        nt = (c + 255) // 256
        padded = torch.zeros(r, nt * 256)
        padded[:, :c] = sq
        partials = _serial_sum(padded.view(r, nt, 256))
        k = (nt + 31) // 32
        lanes = torch.zeros(r, k * 32)
        lanes[:, :nt] = partials
        return _xor_tree(_serial_sum(lanes.view(r, k, 32).transpose(1, 2)))
    raise ValueError(f"unknown order {order!r}")


def tile_square_partials(x: torch.Tensor) -> torch.Tensor:
    """[R, ceil(C/256)] fp32: per 256-column tile, the column-order sum of
    bf16(x^2) (what h3_linear_gated_residual_sq writes beside its output)."""
    r, c = x.shape
    nt = (c + 255) // 256
    padded = torch.zeros(r, nt * 256)
    padded[:, :c] = _r(x.float() * x.float()).float()
    return _serial_sum(padded.view(r, nt, 256))


def rms_norm_in_kernel_order(x: torch.Tensor, weight: torch.Tensor, eps: float, order: str) -> torch.Tensor:
    """``rms_norm`` with the sum of squares taken in a CUDA kernel's order (see
    ``sum_squares_in_kernel_order``); every other step as the reference stages it."""
    lead = x.shape[:-1]
    xf = x.float().reshape(-1, x.shape[-1])
    squared = _r(xf * xf)
    total = sum_squares_in_kernel_order(squared, order).unsqueeze(-1)
    mean = _r(total / x.shape[-1])
    variance = _r(mean.float() + torch.tensor(eps, dtype=torch.float32))
    reciprocal = _r(1.0 / torch.sqrt(variance.float()))
    out = _r(_r(xf * reciprocal.float()).float() * weight.float())
    return out.view(*lead, x.shape[-1])


def rms_modulate_in_kernel_order(x, weight, scale, shift, eps, order: str):
    return modulate(rms_norm_in_kernel_order(x, weight, eps, order), scale, shift)


def qk_norm_rope_in_kernel_order(x, weight, cos, sin, eps):
    """``qk_norm_rope`` with the head kernel's sum order."""
    normalized = rms_norm_in_kernel_order(x, weight, eps, "head")
    extra = normalized.dim() - 2
    c, s = cos, sin
    for _ in range(extra - 1):
        c, s = c.unsqueeze(1), s.unsqueeze(1)
    return rope(normalized, c, s)


def modulate(normalized: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor) -> torch.Tensor:
    """bf16(bf16(n * bf16(1 + scale)) + shift)."""
    factor = _r(scale.float() + 1.0)
    return _r(_r(normalized.float() * factor.float()).float() + shift.float())


def rms_modulate(x, weight, scale, shift, eps):
    return modulate(rms_norm(x, weight, eps), scale, shift)


def ln_modulate(x, scale, shift, eps):
    """LayerNorm variant of AdaLN (mean-subtracted, no affine), the form the
    benchmark configs describe.  Not in the reference; defined here as torch's
    fp32 layer_norm rounded once to BF16, then the reference's staged modulate."""
    normalized = _r(torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), eps=eps))
    return modulate(normalized, scale, shift)


# --------------------------------------------------------------------------
# Residuals and SwiGLU
# --------------------------------------------------------------------------
def gated_residual(x, gate, y):
    """bf16(x + bf16(gate * y)) -- torch.add(x, torch.mul(gate, y)) in BF16."""
    return _r(x.float() + _r(gate.float() * y.float()).float())


def gated_residual_rms_modulate(x, gate, y, weight, scale, shift, eps):
    residual = gated_residual(x, gate, y)
    return residual, rms_modulate(residual, weight, scale, shift, eps)


def swiglu(up, gate):
    """bf16(up * bf16(g / (1 + exp(-g))))."""
    g = gate.float()
    activated = _r(g / (1.0 + torch.exp(-g)))
    return _r(up.float() * activated.float())


# --------------------------------------------------------------------------
# RoPE
# --------------------------------------------------------------------------
def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """NeoX half rotation over the first 2*half channels of [T, H, D], angles
    [T, half] in token order; the rest passes through.  Reference layout
    half=48, D=128; the 44/42/42 extension uses half=64."""
    half = cos.shape[-1]
    a, b, rest = x[..., :half].float(), x[..., half:2 * half].float(), x[..., 2 * half:]
    c = cos.float().unsqueeze(-2)
    s = sin.float().unsqueeze(-2)
    y0 = _r(_r(a * c).float() + _r(-b * s).float())
    y1 = _r(_r(b * c).float() + _r(a * s).float())
    return torch.cat([y0, y1, rest], dim=-1)


def qk_norm_rope(x, weight, cos, sin, eps):
    """Per-head staged RMSNorm over D then RoPE.  x [T, ..., D]; cos/sin [T, half]
    broadcast over every middle axis."""
    normalized = rms_norm(x, weight, eps)
    extra = normalized.dim() - 2
    c, s = cos, sin
    for _ in range(extra - 1):
        c, s = c.unsqueeze(1), s.unsqueeze(1)
    return rope(normalized, c, s)


def rope_powers(sections: Sequence[int] = (16, 16, 16), theta: float = 10000.0) -> list[torch.Tensor]:
    """Per-axis fp32 powers theta ** (2k / (2 f)), k < f (torch float pow), as the
    pipeline computes them (patches/InfiniLM.patch:7014-7025)."""
    out = []
    for f in sections:
        exponent = torch.arange(0, 2 * f, 2, dtype=torch.float32) / (2 * f)
        out.append(torch.full_like(exponent, theta) ** exponent)
    return out


def rotary_cache(positions: torch.Tensor, sections: Sequence[int] = (16, 16, 16),
                 theta: float = 10000.0) -> torch.Tensor:
    """[T, 3] positions -> [T, 2*half] BF16 = cat(cos, sin), axis-major angles
    angle[t, off_a + k] = f32(pos[t, a]) * (1 / theta**(2k/(2 f_a))).
    sections=(16,16,16) is the reference table (bench_h3_ops.py:109-113);
    (22,21,21) is the full-D 44/42/42 extension."""
    cols = []
    for axis, power in enumerate(rope_powers(sections, theta)):
        inverse = 1.0 / power
        cols.append(positions[:, axis].float().unsqueeze(-1) * inverse.view(1, -1))
    angles = torch.cat(cols, dim=-1)
    return torch.cat((angles.cos(), angles.sin()), dim=-1).to(BF16)


def rotary_cache_correctly_rounded(positions: torch.Tensor, sections: Sequence[int] = (16, 16, 16),
                                   theta: float = 10000.0) -> torch.Tensor:
    """``rotary_cache`` with cos/sin evaluated in float64 and rounded to fp32 once
    (then to BF16), the way the CUDA table kernel evaluates them; the fp32 angles
    are the reference's.  Host fp32 cos/sin are within an ulp of these values, so
    the two tables differ in rare BF16 roundings only."""
    cols = []
    for axis, power in enumerate(rope_powers(sections, theta)):
        inverse = 1.0 / power
        cols.append(positions[:, axis].float().unsqueeze(-1) * inverse.view(1, -1))
    angles = torch.cat(cols, dim=-1).double()
    return torch.cat((angles.cos().float(), angles.sin().float()), dim=-1).to(BF16)


def grid_positions(t: int, h: int, w: int) -> torch.Tensor:
    """Integer (t, h, w) latent grid enumerated t-major, as fp64 [t*h*w, 3]."""
    tt, hh, ww = torch.meshgrid(torch.arange(t), torch.arange(h), torch.arange(w), indexing="ij")
    return torch.stack((tt, hh, ww), -1).reshape(-1, 3).double()


# --------------------------------------------------------------------------
# Attention
# --------------------------------------------------------------------------
def attention_fp32(q, k, v, scale, chunk: int = 1024) -> torch.Tensor:
    """softmax(q k^T * scale) v in fp32 for [B, S, H, D] inputs (the mha
    layout); K/V length may be shorter than Q's.  Returns fp32 [B, Sq, H, D]."""
    qf = q.float().permute(0, 2, 1, 3)
    kf = k.float().permute(0, 2, 1, 3)
    vf = v.float().permute(0, 2, 1, 3)
    out = torch.empty(qf.shape, dtype=torch.float32)
    for s in range(0, qf.shape[2], chunk):
        logits = (qf[:, :, s:s + chunk] @ kf.transpose(-2, -1)) * scale
        out[:, :, s:s + chunk] = torch.softmax(logits, -1) @ vf
    return out.permute(0, 2, 1, 3)


# --------------------------------------------------------------------------
# Timestep embedding (patches/InfiniCore.patch:2115-2137, test :2834-2845)
# --------------------------------------------------------------------------
def timestep_embedding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    """Sinusoidal embedding [N, dim] = cat(cos(t f_k), sin(t f_k)), f_k =
    exp(-ln(max_period) k / half), with the reference's fp32 exponent and angle.
    exp, cos and sin are evaluated in float64 and rounded once: the correctly
    rounded fp32 values, so the result does not depend on which vectorised fp32
    exp the host CPU's torch build picks (a 1-ulp frequency difference moves
    t = 999's angle by ~6e-5 rad, more than the reference's 2e-5 tolerance)."""
    half = dim // 2
    exponent = -math.log(max_period) * torch.arange(half, dtype=torch.float32) / half
    freqs = exponent.double().exp().float()
    angles = t.float().unsqueeze(1) * freqs.unsqueeze(0)
    return torch.cat((angles.double().cos(), angles.double().sin()), dim=1).float()


# --------------------------------------------------------------------------
# Ulysses permutations (patches/InfiniLM.patch:895-1137), integer layout only
# --------------------------------------------------------------------------
def ulysses_send_blocks(local: torch.Tensor, world: int, group_start: int = 0,
                        group_heads: int | None = None) -> torch.Tensor:
    """[T, H, D] local tokens -> [W, T, Hs, D]: block p holds heads
    p*Hl + group_start + j (j < Hs) of the local tokens (gather_sequence :895-910,
    overlapped send_blocks :926-934)."""
    tokens, heads, d = local.shape
    hl = heads // world
    hs = hl if group_heads is None else group_heads
    idx = torch.tensor([p * hl + group_start + j for p in range(world) for j in range(hs)])
    return local[:, idx].view(tokens, world, hs, d).permute(1, 0, 2, 3).contiguous()


def ulysses_all_to_all(send: Sequence[torch.Tensor]) -> list[torch.Tensor]:
    """Equal-split all-to-all over W ranks: recv[r][q] = send[q][r]."""
    world = len(send)
    return [torch.stack([send[q][r] for q in range(world)]) for r in range(world)]


def ulysses_gather(recv: torch.Tensor) -> torch.Tensor:
    """[W, T, Hs, D] received blocks -> [W*T, Hs, D], token axis in global order."""
    w, t, hs, d = recv.shape
    return recv.reshape(w * t, hs, d)


def ulysses_scatter_back(returned: Sequence[torch.Tensor], group_heads: Sequence[int]) -> torch.Tensor:
    """Per group g: returned[g] [W, T, Hs_g, D] (block q = heads q*Hl + off_g + h
    of the local tokens) -> output [T, W, Hl, D] (attend_exchanged_groups :1006-1014)."""
    w, t, _, d = returned[0].shape
    hl = sum(group_heads)
    out = torch.empty(t, w, hl, d, dtype=returned[0].dtype)
    off = 0
    for r, hs in zip(returned, group_heads):
        out[:, :, off:off + hs] = r.permute(1, 0, 2, 3)
        off += hs
    return out


# --------------------------------------------------------------------------
# DiT block (patches/InfiniLM.patch:1303-1397)
# --------------------------------------------------------------------------
def linear(x: torch.Tensor, weight: torch.Tensor, row_exact: bool = True) -> torch.Tensor:
    """y = x W^T, BF16 in/out, fp32 accumulation (no bias on the block linears,
    patches/InfiniLM.patch:734-741, 1163-1169).  With ``row_exact`` the dot
    products are summed in float64 and rounded to fp32 once, so a row's result
    does not depend on how many rows the host BLAS is given (its fp32 kernels
    change the summation order with the matrix shape) and equals a fp32
    accumulation up to its rounding; without it, the reference's own CPU
    composition (an fp32 BLAS product), which the CPU baseline times."""
    if not row_exact:
        return _r(x.float() @ weight.float().t())
    return _r((x.double() @ weight.double().t()).float())


def token_modulation(modulation: torch.Tensor, segments, n: int) -> torch.Tensor:
    """Per-token modulation [n, 6*Hd] from a table [rows, 6*Hd] and run-length
    segments (start, length, row) (the gather_rows path, patches/InfiniLM.patch:1306-1318)."""
    if modulation.dim() == 1:
        return modulation.unsqueeze(0).expand(n, -1)
    rows = torch.empty(n, dtype=torch.long)
    for start, length, row in segments:
        rows[start:start + length] = row
    return modulation[rows]


def block_forward(x: torch.Tensor, modulation: torch.Tensor, weights: dict, cos: torch.Tensor,
                  sin: torch.Tensor, heads: int, eps: float = 1e-6, qk_eps: float = 1e-6,
                  valid_tokens: int | None = None, norm: str = "rms", segments=None) -> torch.Tensor:
    """One DiT block on [N, Hd] tokens.  ``modulation`` is one row [6*Hd] or a
    table [rows, 6*Hd] addressed by ``segments`` [(start, length, row)]; columns
    are shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp (:1313-1318).

    weights: w_qkv [3*Hd, Hd] rows [q|k|v] head-major; norm_q, norm_k [D];
    w_o [Hd, Hd]; w_gate_up [2F, Hd] rows [up; gate]; w_down [Hd, F];
    norm1, norm2 [Hd].  cos/sin [N, half] token-ordered.  norm="ln" uses the
    LayerNorm AdaLN variant for both norms."""
    n, hd = x.shape
    d = hd // heads
    mod = token_modulation(modulation, segments, n).reshape(n, 6, hd)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (mod[:, i] for i in range(6))
    if norm == "ln":
        normalized = ln_modulate(x, scale_msa, shift_msa, eps)
    else:
        normalized = rms_modulate(x, weights["norm1"], scale_msa, shift_msa, eps)
    qkv = linear(normalized, weights["w_qkv"]).view(n, 3, heads, d)
    q = qk_norm_rope(qkv[:, 0], weights["norm_q"], cos, sin, qk_eps)
    k = qk_norm_rope(qkv[:, 1], weights["norm_k"], cos, sin, qk_eps)
    v = qkv[:, 2]
    kv = n if valid_tokens is None else valid_tokens
    attn = _r(attention_fp32(q[None], k[None, :kv], v[None, :kv], d ** -0.5)[0]).reshape(n, hd)
    attn_out = linear(attn, weights["w_o"])
    residual = gated_residual(x, gate_msa, attn_out)
    if norm == "ln":
        normalized2 = ln_modulate(residual, scale_mlp, shift_mlp, eps)
    else:
        normalized2 = rms_modulate(residual, weights["norm2"], scale_mlp, shift_mlp, eps)
    gate_up = linear(normalized2, weights["w_gate_up"])
    f = gate_up.shape[1] // 2
    hidden = swiglu(gate_up[:, :f], gate_up[:, f:])
    mlp = linear(hidden, weights["w_down"])
    return gated_residual(residual, gate_mlp, mlp)


def block_forward_rows(x: torch.Tensor, modulation: torch.Tensor, weights: dict, cos: torch.Tensor,
                       sin: torch.Tensor, heads: int, rows: torch.Tensor, eps: float = 1e-6,
                       qk_eps: float = 1e-6, segments=None) -> torch.Tensor:
    """``block_forward`` evaluated for the token rows ``rows`` only, at any
    sequence length: every op of the block is row-local except attention, whose
    keys and values need all tokens -- so k and v are projected for every token
    (one fp32-accumulated GEMM over all rows, the only all-token work), the
    queries and everything after attention only for the requested rows.
    Returns [len(rows), Hd]; equals ``block_forward(...)[rows]`` up to the GEMM
    accumulation order of the all-token k/v product."""
    n, hd = x.shape
    d = hd // heads
    mod = token_modulation(modulation, segments, n).reshape(n, 6, hd)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = (mod[:, i] for i in range(6))
    normalized = rms_modulate(x, weights["norm1"], scale_msa, shift_msa, eps)
    w_qkv = weights["w_qkv"]
    kv = _r(normalized.float() @ w_qkv[hd:].float().t()).view(n, 2, heads, d)
    k = qk_norm_rope(kv[:, 0], weights["norm_k"], cos, sin, qk_eps)
    v = kv[:, 1]
    q = qk_norm_rope(linear(normalized[rows], w_qkv[:hd]).view(-1, heads, d), weights["norm_q"], cos[rows],
                     sin[rows], qk_eps)
    attn = _r(attention_fp32(q[None], k[None], v[None], d ** -0.5)[0]).reshape(-1, hd)
    residual = gated_residual(x[rows], gate_msa[rows], linear(attn, weights["w_o"]))
    normalized2 = rms_modulate(residual, weights["norm2"], scale_mlp[rows], shift_mlp[rows], eps)
    gate_up = linear(normalized2, weights["w_gate_up"])
    f = gate_up.shape[1] // 2
    hidden = swiglu(gate_up[:, :f], gate_up[:, f:])
    return gated_residual(residual, gate_mlp[rows], linear(hidden, weights["w_down"]))


# --------------------------------------------------------------------------
# Model forward around the block stack (patches/InfiniLM.patch:1626-1826)
# --------------------------------------------------------------------------
def linear_f32(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 linear of the F32 modules (proj_in/out, audio, time MLP), x widened to fp32."""
    y = x.float() @ weight.float().t()
    return y if bias is None else y + bias.float()


def silu(x: torch.Tensor) -> torch.Tensor:
    """op::silu in fp32."""
    return torch.nn.functional.silu(x.float())


def add_bias(y: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """bias of a BF16 linear: bf16(y + b) after the BF16 GEMM output."""
    return _r(y.float() + bias.float())


def time_embedder(t: torch.Tensor, w1, b1, w2, b2, in_dim: int = 256) -> torch.Tensor:
    """MiniMaxH3TimeEmbedder::forward (:1494-1517): sinusoid -> linear_1 -> silu -> linear_2, fp32."""
    return linear_f32(silu(linear_f32(timestep_embedding(t, in_dim), w1, b1)), w2, b2)


def adaln_rows(temb: torch.Tensor, w: torch.Tensor, b: torch.Tensor, hidden: int, modalities: int = 3):
    """MiniMaxH3AdaLNProjection::forward (:1260-1279): [timesteps*modalities, 6*Hd]."""
    mod = add_bias(linear(_r(silu(temb)), w), b)
    return mod.view(temb.shape[0] * modalities, 6 * hidden)


def refiner_block_forward(x: torch.Tensor, w: dict, heads: int, eps: float, qk_eps: float) -> torch.Tensor:
    """MiniMaxH3TokenRefinerBlock::forward (:1210-1216): plain RMSNorm, attention with
    q/k RMSNorm over the head dim and no RoPE, residual adds; SwiGLU MLP."""
    n, hd = x.shape
    d = hd // heads
    qkv = linear(rms_norm(x, w["norm1"], eps), w["w_qkv"]).view(n, 3, heads, d)
    q = rms_norm(qkv[:, 0], w["norm_q"], qk_eps)
    k = rms_norm(qkv[:, 1], w["norm_k"], qk_eps)
    attn = _r(attention_fp32(q[None], k[None], qkv[:, 2][None], d ** -0.5)[0]).reshape(n, hd)
    out = _r(x.float() + linear(attn, w["w_o"]).float())
    gate_up = linear(rms_norm(out, w["norm2"], eps), w["w_gate_up"])
    f = gate_up.shape[1] // 2
    mlp = linear(swiglu(gate_up[:, :f], gate_up[:, f:]), w["w_down"])
    return _r(out.float() + mlp.float())


def model_forward(inputs: dict, weights: dict, blocks: Sequence[dict], heads: int, eps: float = 1e-6,
                  qk_eps: float = 1e-6, final_eps: float = 1e-6, sections: Sequence[int] = (16, 16, 16),
                  time_in: int = 256):
    """The whole transformer forward on one device (:1626-1826); returns
    (video [1, Nv, patch], audio [1, Na, audio]) in fp32.  ``weights`` holds the
    non-block modules, ``blocks`` the per-block dicts of ``block_forward`` plus
    ``w_adaln`` / ``b_adaln``."""
    w = weights
    hd = w["ctx_w"].shape[0]
    video_embeds = _r(linear_f32(inputs["video"][0], w["proj_in_w"], w["proj_in_b"]))
    audio_embeds = _r(linear_f32(inputs["audio"][0], w["audio_in_w"], w["audio_in_b"]))
    x = add_bias(linear(inputs["text"][0].to(BF16), w["ctx_w"]), w["ctx_b"])
    for rb in w["refiner"]:
        x = refiner_block_forward(x, rb, heads, eps, qk_eps)
    text_embeds = rms_norm(x, w["refiner_norm"], final_eps)
    seq = inputs["position_ids"].shape[0]
    hidden = torch.zeros(seq, hd, dtype=BF16)
    hidden[inputs["text_indices"]] = text_embeds
    hidden[inputs["video_indices"]] = video_embeds
    hidden[inputs["audio_indices"]] = audio_embeds
    temb = time_embedder(inputs["timestep"].float(), w["time_w1"], w["time_b1"], w["time_w2"], w["time_b2"],
                         time_in)
    adaln_idx = (3 * inputs["timestep_indices"] + inputs["token_tags"]).tolist()
    segments = []
    for i, row in enumerate(adaln_idx):
        if segments and segments[-1][2] == row:
            segments[-1][1] += 1
        else:
            segments.append([i, 1, row])
    table = rotary_cache(inputs["position_ids"], sections)
    half = table.shape[1] // 2
    cos, sin = table[:, :half], table[:, half:]
    h = hidden
    for bw in blocks:
        mod = adaln_rows(temb, bw["w_adaln"], bw["b_adaln"], hd)
        h = block_forward(h, mod, bw, cos, sin, heads, eps, qk_eps, segments=segments)
    out_mod = add_bias(linear(_r(silu(temb)), w["norm_out_w"]), w["norm_out_b"])
    tok = out_mod[inputs["timestep_indices"]]
    normalized = rms_modulate(h, w["norm_out"], tok[:, hd:], tok[:, :hd], final_eps)
    video_all = linear_f32(normalized, w["proj_out_w"], w["proj_out_b"])
    audio_all = linear_f32(normalized, w["audio_out_w"], w["audio_out_b"])
    return video_all[inputs["video_indices"]][None], audio_all[inputs["audio_indices"]][None]


# --------------------------------------------------------------------------
# Tolerance metrics
# --------------------------------------------------------------------------
def bf16_ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in BF16 units-in-the-last-place between two BF16 tensors
    (monotone integer mapping of the bit patterns; +0 and -0 coincide)."""
    def key(t):
        i = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -(i & 0x7FFF), i)
    return (key(a) - key(b)).abs()


def max_abs_rel(out: torch.Tensor, ref: torch.Tensor) -> float:
    """max |out - ref| / max |ref| (the block tolerance metric)."""
    o, r = out.float(), ref.float()
    return float((o - r).abs().max() / r.abs().max().clamp_min(1e-30))
