"""Reference-named H3 operators on the sm_100a C-ABI library.

Names, argument order and meaning follow the reference op API
(``include/infinicore/ops/h3_numerics.hpp``, patches/InfiniCore.patch:142-185;
``mha`` :1333-1426).  Out-of-place forms allocate their outputs with torch (the
reference's ``Tensor::empty``); the ``*_`` forms write into caller tensors, like
the reference's ``H3*::execute(out, ...)``.  Shape/dtype errors raise
ValueError (the reference throws std::invalid_argument), launch failures raise
RuntimeError.  Unlike the reference, widths are not pinned to 128/5376.

Modulation tensors may be given as a single row ``[C]``; they are broadcast
over tokens with stride 0, which is how the reference's segmented block passes
them (patches/InfiniLM.patch:1360-1364).
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import call, desc, require_cuda, stream_of

__all__ = [
    "h3_rms_norm", "h3_rms_norm_", "h3_swiglu", "h3_swiglu_", "h3_rms_modulate", "h3_rms_modulate_",
    "h3_ln_modulate", "h3_ln_modulate_", "h3_rope", "h3_rope_", "h3_gated_residual", "h3_gated_residual_",
    "h3_gated_residual_rms_modulate", "h3_gated_residual_rms_modulate_", "h3_qk_norm_rope_",
    "h3_rope_cache", "h3_rope_cache_sectioned", "rope_powers", "timestep_embedding", "mha", "mha_",
    "linear", "linear_", "linear_swiglu", "linear_gated_residual", "pack_gate_up",
    "linear_f32", "linear_f32_", "gather_rows", "gather_rows_", "index_copy_rows_", "silu", "silu_",
    "linear_qkv_norm_rope_", "linear_gated_residual_sq", "h3_rms_modulate_sq_",
    "linear_gated_residual_rms_modulate", "sq_partials_shape", "linear_gated_residual_segmented",
    "h3_rms_modulate_segmented_", "adaln_projection", "ADALN_MAX_ROWS",
]


def _rowlike(t: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """Broadcast a [C] modulation row to ``like``'s shape (stride 0 over tokens)."""
    if t.dim() == 1 and like.dim() > 1:
        return t.expand(like.shape)
    return t


# ---------------------------------------------------------------------------
# RMSNorm / AdaLN
# ---------------------------------------------------------------------------
def h3_rms_norm_(out, x, weight, eps):
    require_cuda(out, x, weight)
    call("h3_rms_norm", desc(out), desc(x), desc(weight), float(eps), stream_of(x))
    return out


def h3_rms_norm(x, weight, eps):
    return h3_rms_norm_(torch.empty_like(x), x, weight, eps)


def h3_rms_modulate_(out, x, weight, scale, shift, eps):
    scale, shift = _rowlike(scale, x), _rowlike(shift, x)
    require_cuda(out, x, weight, scale, shift)
    call("h3_rms_modulate", desc(out), desc(x), desc(weight), desc(scale), desc(shift), float(eps),
         stream_of(x))
    return out


def h3_rms_modulate(x, weight, scale, shift, eps):
    return h3_rms_modulate_(torch.empty_like(x), x, weight, scale, shift, eps)


def h3_ln_modulate_(out, x, scale, shift, eps):
    scale, shift = _rowlike(scale, x), _rowlike(shift, x)
    require_cuda(out, x, scale, shift)
    call("h3_ln_modulate", desc(out), desc(x), desc(scale), desc(shift), float(eps), stream_of(x))
    return out


def h3_ln_modulate(x, scale, shift, eps):
    return h3_ln_modulate_(torch.empty_like(x), x, scale, shift, eps)


# ---------------------------------------------------------------------------
# residuals, SwiGLU
# ---------------------------------------------------------------------------
def h3_gated_residual_(out, x, gate, y):
    gate = _rowlike(gate, x)
    require_cuda(out, x, gate, y)
    call("h3_gated_residual", desc(out), desc(x), desc(gate), desc(y), stream_of(x))
    return out


def h3_gated_residual(x, gate, y):
    return h3_gated_residual_(torch.empty_like(x), x, gate, y)


def h3_gated_residual_rms_modulate_(residual, out, x, gate, y, weight, scale, shift, eps):
    gate, scale, shift = _rowlike(gate, x), _rowlike(scale, x), _rowlike(shift, x)
    require_cuda(residual, out, x, gate, y, weight, scale, shift)
    call("h3_gated_residual_rms_modulate", desc(residual), desc(out), desc(x), desc(gate), desc(y),
         desc(weight), desc(scale), desc(shift), float(eps), stream_of(x))
    return residual, out


def h3_gated_residual_rms_modulate(x, gate, y, weight, scale, shift, eps):
    """Returns (residual, modulated), as the reference's pair."""
    return h3_gated_residual_rms_modulate_(torch.empty_like(x), torch.empty_like(x), x, gate, y, weight,
                                           scale, shift, eps)


def h3_swiglu_(out, up, gate):
    require_cuda(out, up, gate)
    call("h3_swiglu", desc(out), desc(up), desc(gate), stream_of(up))
    return out


def h3_swiglu(up, gate):
    return h3_swiglu_(torch.empty(up.shape, dtype=up.dtype, device=up.device), up, gate)


# ---------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------
def h3_rope_(out, x, cos, sin):
    require_cuda(out, x, cos, sin)
    call("h3_rope", desc(out), desc(x), desc(cos), desc(sin), stream_of(x))
    return out


def h3_rope(x, cos, sin):
    return h3_rope_(torch.empty(x.shape, dtype=x.dtype, device=x.device), x, cos, sin)


def h3_qk_norm_rope_(out, x, weight, cos, sin, eps):
    """Per-head RMSNorm + RoPE of x [T,P,Hs,128] into out [T,P,Hs,128] (any strides)."""
    require_cuda(out, x, weight, cos, sin)
    call("h3_qk_norm_rope", desc(out), desc(x), desc(weight), desc(cos), desc(sin), float(eps), stream_of(x))
    return out


def rope_powers(sections=(16, 16, 16), theta: float = 10000.0, device="cuda") -> torch.Tensor:
    """Axis-major fp32 powers theta ** (2k / (2 f_a)), k < f_a, computed with fp32 pow
    like the pipeline (patches/InfiniLM.patch:7014-7025).  For the reference table
    pass only the first 16 to ``h3_rope_cache``."""
    parts = []
    for f in sections:
        exponent = torch.arange(0, 2 * f, 2, dtype=torch.float32) / (2 * f)
        parts.append(torch.full_like(exponent, theta) ** exponent)
    return torch.cat(parts).to(device)


def h3_rope_cache(position, power):
    """position [T,3] fp64, power [16] fp32 -> [T,96] bf16 (cat(cos, sin))."""
    require_cuda(position, power)
    out = torch.empty(position.shape[0], 96, dtype=torch.bfloat16, device=position.device)
    call("h3_rope_cache", desc(out), desc(position), desc(power), stream_of(position))
    return out


def h3_rope_cache_sectioned(position, power, sections):
    f0, f1, f2 = (int(s) for s in sections)
    require_cuda(position, power)
    out = torch.empty(position.shape[0], 2 * (f0 + f1 + f2), dtype=torch.bfloat16, device=position.device)
    call("h3_rope_cache_sectioned", desc(out), desc(position), desc(power), f0, f1, f2, stream_of(position))
    return out


def timestep_embedding(t, dim, max_period=10000.0):
    require_cuda(t)
    t = t.float()
    out = torch.empty(t.shape[0], dim, dtype=torch.float32, device=t.device)
    call("h3_timestep_embedding", desc(out), desc(t), float(max_period), stream_of(t))
    return out


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def mha_(out, q, k, v, scale=None):
    """Non-causal attention, q/out [B,Sq,H,D], k/v [B,Sk,H,D] (the reference mha layout)."""
    require_cuda(out, q, k, v)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    call("h3_mha", desc(out), desc(q), desc(k), desc(v), float(scale), stream_of(q))
    return out


def mha(q, k, v, scale=None):
    return mha_(torch.empty(q.shape, dtype=q.dtype, device=q.device), q, k, v, scale)


# ---------------------------------------------------------------------------
# projections
# ---------------------------------------------------------------------------
def _flat(x):
    return x.reshape(-1, x.shape[-1])


def linear_(out, x, weight):
    require_cuda(out, x, weight)
    call("h3_linear", desc(_flat(out)), desc(_flat(x)), desc(weight), stream_of(x))
    return out


def linear(x, weight):
    out = torch.empty(*x.shape[:-1], weight.shape[0], dtype=x.dtype, device=x.device)
    return linear_(out, x, weight)


def _desc_array(ts):
    return (_lib.H3Tensor * len(ts))(*[desc(t) for t in ts])


def linear_qkv_norm_rope_(q_outs, k_outs, v_outs, x, weight, norm_q, norm_k, cos, sin, eps):
    """q, k, v = x W^T with q/k RMSNorm + RoPE in the GEMM epilogue; head h goes to
    q_outs[h // hpd][:, h % hpd] (lists of [T, hpd, 128] tensors; bitwise
    h3_linear followed by h3_qk_norm_rope)."""
    require_cuda(x, weight, norm_q, norm_k, cos, sin, *q_outs, *k_outs, *v_outs)
    call("h3_linear_qkv_norm_rope", desc(_flat(x)), desc(weight), _desc_array(q_outs), _desc_array(k_outs),
         _desc_array(v_outs), len(q_outs), desc(norm_q), desc(norm_k), desc(cos), desc(sin), float(eps),
         stream_of(x))


def pack_gate_up(weight):
    """[up; gate] rows [2F, K] -> 128-row blocks [up_0|gate_0|up_1|gate_1|...] for linear_swiglu."""
    require_cuda(weight)
    out = torch.empty_like(weight)
    call("h3_pack_gate_up", desc(out), desc(weight), stream_of(weight))
    return out


def linear_swiglu(x, packed_weight, out=None):
    f = packed_weight.shape[0] // 2
    if out is None:
        out = torch.empty(*x.shape[:-1], f, dtype=x.dtype, device=x.device)
    require_cuda(out, x, packed_weight)
    call("h3_linear_swiglu", desc(_flat(out)), desc(_flat(x)), desc(packed_weight), stream_of(x))
    return out


def linear_gated_residual(x, weight, residual, gate, out=None):
    """out = bf16(residual + bf16(gate * (x W^T)))."""
    if out is None:
        out = torch.empty_like(residual)
    r2 = _flat(residual)
    g2 = _rowlike(gate, r2) if gate.dim() == 1 else _flat(gate)
    require_cuda(out, x, weight, residual, g2)
    call("h3_linear_gated_residual", desc(_flat(out)), desc(_flat(x)), desc(weight), desc(r2), desc(g2),
         stream_of(x))
    return out


SQ_TILE = 256   # columns per partial sum of squares (the projection's output tile width)


def sq_partials_shape(rows: int, width: int) -> tuple[int, int]:
    """Shape of the per-tile sums of squares of a [rows, width] output."""
    return rows, (width + SQ_TILE - 1) // SQ_TILE


def linear_gated_residual_sq(x, weight, residual, gate, out=None, sq=None):
    """(out, sq): out = bf16(residual + bf16(gate * (x W^T))) and its per-tile
    row sums of squares sq [M, ceil(N/256)] F32 for ``h3_rms_modulate_sq_``."""
    if out is None:
        out = torch.empty_like(residual)
    o2 = _flat(out)
    if sq is None:
        sq = torch.empty(sq_partials_shape(*o2.shape), dtype=torch.float32, device=out.device)
    r2 = _flat(residual)
    g2 = _rowlike(gate, r2) if gate.dim() == 1 else _flat(gate)
    require_cuda(out, sq, x, weight, residual, g2)
    call("h3_linear_gated_residual_sq", desc(o2), desc(sq), desc(_flat(x)), desc(weight), desc(r2), desc(g2),
         stream_of(x))
    return out, sq


def h3_rms_modulate_sq_(out, x, sq, weight, scale, shift, eps):
    """h3_rms_modulate_ with the row sums of squares taken from ``sq`` (written by
    ``linear_gated_residual_sq``)."""
    scale, shift = _rowlike(scale, x), _rowlike(shift, x)
    require_cuda(out, x, sq, weight, scale, shift)
    call("h3_rms_modulate_sq", desc(out), desc(x), desc(sq), desc(weight), desc(scale), desc(shift), float(eps),
         stream_of(x))
    return out


def _segments(rows, lengths):
    if len(rows) != len(lengths) or not rows:
        raise ValueError("one modulation row per segment")
    return _desc_array(rows), (ctypes.c_int64 * len(lengths))(*[int(n) for n in lengths]), len(rows)


def linear_gated_residual_segmented(x, weight, residual, gates, lengths, out=None, sq=None):
    """out = bf16(residual + bf16(gate_s * (x W^T))) with gate row ``gates[s]`` for the
    ``lengths[s]`` rows of segment s (consecutive, one launch); with ``sq``, also the
    per-tile sums of squares of out."""
    if out is None:
        out = torch.empty_like(residual)
    g, n, k = _segments(gates, lengths)
    require_cuda(out, sq, x, weight, residual, *gates)
    call("h3_linear_gated_residual_segmented", desc(_flat(out)), desc(sq), desc(_flat(x)), desc(weight),
         desc(_flat(residual)), g, n, k, stream_of(x))
    return out


def h3_rms_modulate_segmented_(out, x, sq, weight, scales, shifts, lengths, eps):
    """h3_rms_modulate_ with scale/shift rows per segment of consecutive rows (one
    launch); with ``sq`` the row sums of squares come from the partials."""
    sc, n, k = _segments(scales, lengths)
    sh, _, _ = _segments(shifts, lengths)
    require_cuda(out, x, sq, weight, *scales, *shifts)
    call("h3_rms_modulate_segmented", desc(out), desc(x), desc(sq), desc(weight), sc, sh, n, k, float(eps),
         stream_of(x))
    return out


def linear_gated_residual_rms_modulate(x, weight, residual, gate, norm_weight, scale, shift, eps,
                                       residual_out=None, out=None, workspace=None):
    """(residual_out, out) of the out-projection fused with
    h3_gated_residual_rms_modulate; ``workspace`` [M, ceil(N/256)] F32 is scratch."""
    residual_out = torch.empty_like(residual) if residual_out is None else residual_out
    out = torch.empty_like(residual) if out is None else out
    r2 = _flat(residual)
    if workspace is None:
        workspace = torch.empty(sq_partials_shape(*r2.shape), dtype=torch.float32, device=r2.device)
    g2 = _rowlike(gate, r2) if gate.dim() == 1 else _flat(gate)
    sc, sh = _rowlike(scale, r2), _rowlike(shift, r2)
    require_cuda(residual_out, out, x, weight, residual, g2, norm_weight, sc, sh, workspace)
    call("h3_linear_gated_residual_rms_modulate", desc(_flat(residual_out)), desc(_flat(out)), desc(_flat(x)),
         desc(weight), desc(r2), desc(g2), desc(norm_weight), desc(sc), desc(sh), float(eps), desc(workspace),
         stream_of(x))
    return residual_out, out


ADALN_MAX_ROWS = 4


def adaln_projection(x, weight, bias=None, out=None):
    """[M, N] = bf16(bf16(x W^T) + bias) for M <= 4 conditioning rows (the AdaLN
    projection's linear + bias, patches/InfiniLM.patch:1260-1279), a
    weight-streaming kernel; a column slice of W gives bitwise the same columns."""
    x2 = _flat(x)
    if out is None:
        out = torch.empty(x2.shape[0], weight.shape[0], dtype=torch.bfloat16, device=x.device)
    require_cuda(out, x2, weight, bias)
    call("h3_adaln_projection", desc(out), desc(x2), desc(weight), desc(bias), stream_of(x))
    return out


# ---------------------------------------------------------------------------
# model wrapper ops (outside the block loop)
# ---------------------------------------------------------------------------
def linear_f32_(out, x, weight, bias=None):
    """out [M,N] = x [M,K] (BF16 or F32) * weight[N,K]^T (+ bias) in fp32, stored as out's dtype
    (F32, or BF16 rounded once) -- linear_forward on the F32 modules of MiniMaxH3Transformer."""
    require_cuda(out, x, weight, bias)
    call("h3_linear_f32", desc(_flat(out)), desc(_flat(x)), desc(weight), desc(bias), stream_of(x))
    return out


def linear_f32(x, weight, bias=None, out_dtype=torch.float32):
    out = torch.empty(*x.shape[:-1], weight.shape[0], dtype=out_dtype, device=x.device)
    return linear_f32_(out, x, weight, bias)


def gather_rows_(out, table, indices):
    """out[r] = table[indices[r]] (gather_rows / op::embedding)."""
    require_cuda(out, table, indices)
    call("h3_gather_rows", desc(out), desc(table), desc(indices), stream_of(table))
    return out


def gather_rows(table, indices):
    out = torch.empty(indices.shape[0], table.shape[1], dtype=table.dtype, device=table.device)
    return gather_rows_(out, table, indices)


def index_copy_rows_(out, indices, src):
    """out[indices[r]] = src[r] in place (op::index_copy along the token dim)."""
    require_cuda(out, src, indices)
    call("h3_index_copy_rows", desc(out), desc(indices), desc(src), stream_of(src))
    return out


def silu_(out, x):
    """out = silu(x) in fp32, stored as out's dtype (F32 or BF16)."""
    require_cuda(out, x)
    call("h3_silu", desc(out), desc(x), stream_of(x))
    return out


def silu(x, dtype=torch.float32):
    return silu_(torch.empty(x.shape, dtype=dtype, device=x.device), x)


def library_loaded() -> bool:
    return _lib._lib is not None
