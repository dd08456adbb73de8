"""Host composition of one MiniMax-H3 DiT block and of the 40-block denoising
step over the sm_100a C-ABI kernels.

Follows ``MiniMaxH3TransformerBlock::forward_segmented`` (patches/InfiniLM.patch:
1353-1397) and ``MiniMaxH3Transformer::forward`` (:1626-1826):

    per segment  n1  = h3_rms_modulate(x, norm1.w, scale_msa, shift_msa)      (K6)
                 q,k,v = n1 W_qkv^T, q/k RMSNorm + RoPE in the epilogue        (K10+K2, tcgen05)
                 a   = mha(q, k, v)                                            (K1, tcgen05)
    per segment  res = bf16(x + bf16(gate_msa * bf16(a W_o^T)))  + sums of squares   (K10+K8a)
                 n2  = RMSNorm + AdaLN of res from those sums                  (K8b, element-wise)
                 h   = swiglu(n2 W_up^T, n2 W_gate^T)   (fused epilogue)       (K10+K9)
    per segment  out = bf16(res + bf16(gate_mlp * bf16(h W_down^T)))  + sums of squares (K10+K7)
    (the next block's K6 then reads out's sums instead of reducing its rows again;
    the "per segment" ops run as one launch over up to 4 segments, each row picking
    its segment's modulation row)

Modulation columns are ordered shift_msa, scale_msa, gate_msa, shift_mlp,
scale_mlp, gate_mlp (:1313-1318); a segment's row is broadcast over its tokens
with stride 0 (:1360-1364).  Under sequence parallelism (``ulysses``) the
attention part runs on the all-to-all-exchanged heads; everything else is
token-local.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import ops
from .phases import mark


@dataclass
class Segment:
    """Tokens [start, start+length) of this rank share modulation row ``row``
    (MiniMaxH3ModulationSegment, patches/InfiniLM.patch:2041-2045)."""
    start: int
    length: int
    row: int


@dataclass
class BlockWeights:
    w_qkv: torch.Tensor          # [3*Hd, Hd], rows [q | k | v], head-major
    norm_q: torch.Tensor         # [D]
    norm_k: torch.Tensor         # [D]
    w_o: torch.Tensor            # [Hd, Hd]
    w_gate_up: torch.Tensor      # [2F, Hd], rows [up; gate] (Diffusers ff.net.0.proj order)
    w_down: torch.Tensor         # [Hd, F]
    norm1: torch.Tensor          # [Hd]
    norm2: torch.Tensor          # [Hd]
    w_adaln: torch.Tensor | None = None   # [modalities*6*Hd, Hd]
    b_adaln: torch.Tensor | None = None   # [modalities*6*Hd]
    w_gate_up_packed: torch.Tensor | None = field(default=None, repr=False)

    def prepare(self) -> "BlockWeights":
        """One-time weight layout for the fused SwiGLU epilogue (like the
        reference's first-call QKV regroup, patches/InfiniLM.patch:1020-1045)."""
        if self.w_gate_up_packed is None:
            self.w_gate_up_packed = ops.pack_gate_up(self.w_gate_up)
        return self


@dataclass
class BlockConfig:
    hidden: int = 5120
    heads: int = 40
    head_dim: int = 128
    ffn: int = 13824
    eps: float = 1e-6
    qk_eps: float = 1e-6
    modalities: int = 3


def random_block_weights(cfg: BlockConfig, device, seed: int = 0, std: float = 0.02,
                         adaln: bool = True, temb_dim: int | None = None) -> BlockWeights:
    """Random-init weights ~N(0, std) (benchmark configs 3-5), norm weights ones,
    qk-norm weights ones.  Generated on the device (no checkpoint is used).  The
    AdaLN projection reads a time embedding of ``temb_dim`` (default: hidden)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    hd, f, d = cfg.hidden, cfg.ffn, cfg.head_dim

    def rnd(*shape):
        return (torch.randn(*shape, generator=g, device=device) * std).to(torch.bfloat16)

    w = BlockWeights(
        w_qkv=rnd(3 * hd, hd), norm_q=torch.ones(d, dtype=torch.bfloat16, device=device),
        norm_k=torch.ones(d, dtype=torch.bfloat16, device=device), w_o=rnd(hd, hd),
        w_gate_up=rnd(2 * f, hd), w_down=rnd(hd, f),
        norm1=torch.ones(hd, dtype=torch.bfloat16, device=device),
        norm2=torch.ones(hd, dtype=torch.bfloat16, device=device))
    if adaln:
        w.w_adaln = rnd(cfg.modalities * 6 * hd, temb_dim or hd)
        w.b_adaln = rnd(cfg.modalities * 6 * hd)
    return w.prepare()


class Workspace:
    """Per-shape activation buffers reused across blocks (the step allocates
    nothing per block, which also keeps CUDA-graph capture simple)."""

    def __init__(self, tokens: int, cfg: BlockConfig, device):
        hd, f = cfg.hidden, cfg.ffn
        e = dict(dtype=torch.bfloat16, device=device)
        self.tokens = tokens
        self.normalized = torch.empty(tokens, hd, **e)
        self.qkv = torch.empty(tokens, 3 * hd, **e)
        self.q = torch.empty(tokens, cfg.heads, cfg.head_dim, **e)
        self.k = torch.empty(tokens, cfg.heads, cfg.head_dim, **e)
        self.v = torch.empty(tokens, cfg.heads, cfg.head_dim, **e)
        self.attn = torch.empty(tokens, cfg.heads, cfg.head_dim, **e)
        self.attn_out = torch.empty(tokens, hd, **e)
        self.residual = torch.empty(tokens, hd, **e)
        self.normalized2 = torch.empty(tokens, hd, **e)
        self.hidden = torch.empty(tokens, f, **e)
        self.out = [torch.empty(tokens, hd, **e), torch.empty(tokens, hd, **e)]
        # per-256-column sums of squares written by the projections' epilogues for
        # the RMSNorm passes that follow: of the residual, and of each output buffer
        sq = ops.sq_partials_shape(tokens, hd)
        self.sq = torch.empty(sq, dtype=torch.float32, device=device)
        self.out_sq = [torch.empty(sq, dtype=torch.float32, device=device) for _ in range(2)]


def qkv_fused(heads: int, cos: torch.Tensor) -> bool:
    """Whether the QKV projection can carry the q/k norm + RoPE in its epilogue
    (two heads per 256-column tile; the reference's 48 rotated pairs, or the 64 of
    the full-D 44/42/42 layout)."""
    return heads % 2 == 0 and cos.shape[-1] in (48, 64)


def _col(modulation: torch.Tensor, index: int, hidden: int, seg: Segment) -> torch.Tensor:
    """Column block ``index`` of the segment's modulation row, broadcast over its tokens."""
    row = modulation[seg.row, index * hidden:(index + 1) * hidden]
    return row.unsqueeze(0).expand(seg.length, hidden)


MAX_SEGMENTS = 4   # modulation segments one segmented launch takes (H3_MAX_SEGMENTS)


def _one_launch_segments(segments: list[Segment], tokens: int) -> list[int] | None:
    """Segment lengths when the segments tile [0, tokens) in order and are few enough
    for the one-launch (segmented) kernels, else None."""
    if not segments or len(segments) > MAX_SEGMENTS:
        return None
    start = 0
    for sg in segments:
        if sg.start != start or sg.length < 0:
            return None
        start += sg.length
    return [sg.length for sg in segments] if start == tokens else None


def block_forward(x: torch.Tensor, modulation: torch.Tensor, segments: list[Segment], w: BlockWeights,
                  cos: torch.Tensor, sin: torch.Tensor, cfg: BlockConfig, ws: Workspace,
                  out: torch.Tensor | None = None, sp=None, x_sq: torch.Tensor | None = None,
                  out_sq: torch.Tensor | None = None, fused_norms: bool = True) -> torch.Tensor:
    """One block on this rank's tokens x [T, Hd] -> out [T, Hd].

    modulation [rows, 6*Hd]; cos/sin [T, half] for this rank's tokens.  ``sp``
    is a ``ulysses.SequenceParallel`` (None on one GPU).

    With ``fused_norms`` (the default) the out-projection's epilogue computes the
    gated residual and its per-tile sums of squares, and the post-attention
    RMSNorm + AdaLN reads those sums instead of reducing the row again
    (``h3_rms_modulate_sq``); the down-projection does the same for the block's
    output into ``out_sq`` when given, and the pre-attention RMSNorm uses
    ``x_sq`` (x's sums from the previous block) when given.  The residuals are
    bitwise those of the unfused ops; the normalised rows differ from them only by
    the order of the fp32 sum of squares."""
    t, hd = x.shape
    h, d = cfg.heads, cfg.head_dim
    out = ws.out[0] if out is None else out
    # the norms and gated-residual projections run once over all segments when they fit
    # the segmented launches (segment s uses modulation row s's column blocks)
    lengths = _one_launch_segments(segments, t) if fused_norms else None
    rows = (lambda i: [modulation[sg.row, i * hd:(i + 1) * hd] for sg in segments])  # noqa: E731
    mark("norm1")
    if lengths is not None:
        ops.h3_rms_modulate_segmented_(ws.normalized, x, x_sq, w.norm1, rows(1), rows(0), lengths, cfg.eps)
    else:
        for s in segments:
            r = slice(s.start, s.start + s.length)
            if fused_norms and x_sq is not None:
                ops.h3_rms_modulate_sq_(ws.normalized[r], x[r], x_sq[r], w.norm1, _col(modulation, 1, hd, s),
                                        _col(modulation, 0, hd, s), cfg.eps)
            else:
                ops.h3_rms_modulate_(ws.normalized[r], x[r], w.norm1, _col(modulation, 1, hd, s),
                                     _col(modulation, 0, hd, s), cfg.eps)
    if sp is None or sp.world == 1:
        mark("qkv_norm_rope")
        if qkv_fused(h, cos):
            # one GEMM whose epilogue normalises and rotates q/k and stores q, k, v per head
            ops.linear_qkv_norm_rope_([ws.q], [ws.k], [ws.v], ws.normalized, w.w_qkv, w.norm_q, w.norm_k,
                                      cos, sin, cfg.qk_eps)
            v = ws.v
        else:
            ops.linear_(ws.qkv, ws.normalized, w.w_qkv)
            qkv = ws.qkv.view(t, 3, h, d)
            ops.h3_qk_norm_rope_(ws.q.unsqueeze(1), qkv[:, 0].unsqueeze(1), w.norm_q, cos, sin, cfg.qk_eps)
            ops.h3_qk_norm_rope_(ws.k.unsqueeze(1), qkv[:, 1].unsqueeze(1), w.norm_k, cos, sin, cfg.qk_eps)
            v = qkv[:, 2]
        mark("attention")
        ops.mha_(ws.attn.unsqueeze(0), ws.q.unsqueeze(0), ws.k.unsqueeze(0), v.unsqueeze(0), 1.0 / math.sqrt(d))
        attn_flat = ws.attn.view(t, hd)
    else:
        attn_flat = sp.attention(ws.normalized, w.w_qkv, w.norm_q, w.norm_k, cos, sin, cfg.qk_eps)
    mark("out_proj_norm")
    if lengths is not None:
        ops.linear_gated_residual_segmented(attn_flat, w.w_o, x, rows(2), lengths, out=ws.residual, sq=ws.sq)
        ops.h3_rms_modulate_segmented_(ws.normalized2, ws.residual, ws.sq, w.norm2, rows(4), rows(3), lengths,
                                       cfg.eps)
    elif fused_norms:
        for s in segments:
            r = slice(s.start, s.start + s.length)
            ops.linear_gated_residual_sq(attn_flat[r], w.w_o, x[r], modulation[s.row, 2 * hd:3 * hd],
                                         out=ws.residual[r], sq=ws.sq[r])
            ops.h3_rms_modulate_sq_(ws.normalized2[r], ws.residual[r], ws.sq[r], w.norm2,
                                    _col(modulation, 4, hd, s), _col(modulation, 3, hd, s), cfg.eps)
    else:
        ops.linear_(ws.attn_out, attn_flat, w.w_o)
        for s in segments:
            r = slice(s.start, s.start + s.length)
            ops.h3_gated_residual_rms_modulate_(ws.residual[r], ws.normalized2[r], x[r],
                                                _col(modulation, 2, hd, s), ws.attn_out[r], w.norm2,
                                                _col(modulation, 4, hd, s), _col(modulation, 3, hd, s), cfg.eps)
    mark("gate_up_swiglu")
    ops.linear_swiglu(ws.normalized2, w.w_gate_up_packed, out=ws.hidden)
    mark("down_gated_residual")
    if lengths is not None:
        ops.linear_gated_residual_segmented(ws.hidden, w.w_down, ws.residual, rows(5), lengths, out=out, sq=out_sq)
        return out
    for s in segments:
        r = slice(s.start, s.start + s.length)
        gate_mlp = modulation[s.row, 5 * hd:6 * hd]
        if fused_norms and out_sq is not None:
            ops.linear_gated_residual_sq(ws.hidden[r], w.w_down, ws.residual[r], gate_mlp, out=out[r],
                                         sq=out_sq[r])
        else:
            ops.linear_gated_residual(ws.hidden[r], w.w_down, ws.residual[r], gate_mlp, out=out[r])
    return out


# ---------------------------------------------------------------------------
# step-level pieces (patches/InfiniLM.patch:1489-1517, 1718-1793)
# ---------------------------------------------------------------------------
@dataclass
class TimeEmbedderWeights:
    """fp32 time MLP: linear_1 [Hd, 256] + bias, silu, linear_2 [Hd, Hd] + bias."""
    w1: torch.Tensor
    b1: torch.Tensor
    w2: torch.Tensor
    b2: torch.Tensor


def random_time_embedder(hidden: int, device, in_dim: int = 256, seed: int = 1,
                         out_dim: int | None = None) -> TimeEmbedderWeights:
    """fp32 time MLP in_dim -> hidden -> out_dim (default hidden), ~N(0, 0.02)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, device=device) * 0.02  # noqa: E731
    out_dim = out_dim or hidden
    return TimeEmbedderWeights(r(hidden, in_dim), r(hidden), r(out_dim, hidden), r(out_dim))


def time_embedding(t: torch.Tensor, tw: TimeEmbedderWeights, in_dim: int = 256) -> torch.Tensor:
    """temb [N, out] fp32 = linear_2(silu(linear_1(sinusoid(t))))
    (MiniMaxH3TimeEmbedder::forward, patches/InfiniLM.patch:1494-1517): the fp32
    linears and the SiLU are the h3_linear_f32 / h3_silu kernels."""
    emb = ops.timestep_embedding(t, in_dim)
    hidden = ops.silu(ops.linear_f32(emb, tw.w1, tw.b1))
    return ops.linear_f32(hidden, tw.w2, tw.b2)


_UNIT: dict = {}


def unit_gate(width: int, device) -> torch.Tensor:
    """A BF16 row of ones [width] (cached), the gate that turns a gated residual
    into a plain add: bf16(x + bf16(1 * y)) = bf16(x + y)."""
    key = (width, str(device))
    if key not in _UNIT:
        _UNIT[key] = torch.ones(width, dtype=torch.bfloat16, device=device)
    return _UNIT[key]


def add_bias(y: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """y + bias in BF16 (one rounding), in place: the gated-residual kernel with a
    unit gate."""
    flat = y.reshape(-1, y.shape[-1])
    ops.h3_gated_residual_(flat, flat, unit_gate(flat.shape[-1], y.device), bias.expand(flat.shape))
    return y


def adaln_modulation(temb: torch.Tensor, w: BlockWeights, cfg: BlockConfig) -> torch.Tensor:
    """[N*modalities, 6*Hd] BF16 modulation rows of one block: silu(temb) -> bf16,
    projected by the block's AdaLN linear plus bias
    (MiniMaxH3AdaLNProjection::forward, patches/InfiniLM.patch:1260-1279)."""
    activated = ops.silu(temb, dtype=torch.bfloat16)
    return adaln_project(activated, w.w_adaln, w.b_adaln).view(temb.shape[0] * cfg.modalities, 6 * cfg.hidden)


def adaln_project(activated: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """bf16(bf16(activated W^T) + bias): the weight-streaming kernel for the usual
    few conditioning rows, else the tcgen05 GEMM and the bias pass.  (The two sum
    the K products in different orders; every rank takes the same branch.)"""
    if activated.shape[0] <= ops.ADALN_MAX_ROWS:
        return ops.adaln_projection(activated, weight, bias)
    return add_bias(ops.linear(activated, weight), bias)


def segments_from_indices(indices) -> list[Segment]:
    """Run-length segments of per-token modulation rows (:1770-1792)."""
    segs: list[Segment] = []
    for i, row in enumerate(indices):
        row = int(row)
        if segs and segs[-1].row == row:
            segs[-1].length += 1
        else:
            segs.append(Segment(i, 1, row))
    return segs
