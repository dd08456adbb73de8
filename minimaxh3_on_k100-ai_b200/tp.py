"""Tensor-parallel block: the reference's mode for fewer GPUs
(``MiniMaxH3TransformerBlock::forward_overlapped``, patches/InfiniLM.patch:1399-1476,
with column-parallel QKV / gate_up and row-parallel out / down linears,
:734-741, 1163-1169).

Every rank holds all tokens.  Rank r owns heads [r*H/W, (r+1)*H/W) (its rows of
the QKV weight and columns of the output projection) and FFN columns
[r*F/W, (r+1)*F/W) (its rows of gate_up and columns of down).  Per block:

    n1      = RMSNorm + AdaLN(x)                                   (replicated)
    q, k, v = n1 W_qkv_r^T, q/k RMSNorm + RoPE                     (local heads)
    a       = mha(q, k, v)                                         (local heads, all tokens)
    o       = all-reduce(a W_o_r^T)                                (row-parallel)
    res, n2 = gated residual + RMSNorm + AdaLN(x, o)               (replicated)
    h       = swiglu(n2 W_gate_up_r^T)                             (local FFN columns)
    out     = gated residual(res, all-reduce(h W_down_r^T))        (row-parallel)

The all-reduce runs over peer memory (``TensorParallel``): the projection GEMM
writes its BF16 partial into this rank's exchange region; after a flag exchange
each rank sums its 1/W of the rows over all ranks' partials in fp32, in rank
order (``h3_peer_reduce_rows``), and stores the BF16 sum into every rank's sum
region; a second flag exchange publishes it.  The reference all-reduces BF16
partials with a collective whose summation order is the library's; here the
order is fixed, so every rank and every run gets the same sum.  Results differ
from the 1-GPU block by that summation (fp32 sum of W BF16 partials instead of
one fp32 accumulation), within the block tolerance.
"""
from __future__ import annotations

import math

import torch

from . import _lib, ops
from .block import BlockConfig, BlockWeights, Segment, _col, qkv_fused
from .ulysses import PeerExchange


class TensorParallel:
    """All-reduce of a [tokens, hidden] BF16 partial over peer memory."""

    SLOT_PARTIAL, SLOT_SUM = 0, 1

    def __init__(self, world: int, rank: int, group, tokens: int, hidden: int, device):
        self.world, self.rank = world, rank
        nbytes = tokens * hidden * 2
        self.px = PeerExchange(world, rank, group, device, {"part": nbytes, "sum": nbytes})
        self.part = self.px.local("part", (tokens, hidden))
        self.sum = self.px.local("sum", (tokens, hidden))
        chunk = (tokens + world - 1) // world
        r0, r1 = min(tokens, rank * chunk), min(tokens, (rank + 1) * chunk)
        self.rows = r1 - r0
        shape = (self.rows, hidden)
        self.srcs = (_lib.H3Tensor * world)(*[self.px.peer_desc(p, "part", shape, r0 * hidden) for p in range(world)])
        self.dsts = (_lib.H3Tensor * world)(*[self.px.peer_desc(p, "sum", shape, r0 * hidden) for p in range(world)])
        self.device = torch.device(device)

    def allreduce(self) -> torch.Tensor:
        """Sum of every rank's ``self.part`` (written by the caller on the current
        stream), returned as ``self.sum``."""
        stream = torch.cuda.current_stream(self.device).cuda_stream
        self.px.signal(self.SLOT_PARTIAL, stream)
        self.px.wait(self.SLOT_PARTIAL, stream)
        if self.rows > 0:
            _lib.call("h3_peer_reduce_rows", self.dsts, self.srcs, self.world, stream)
        self.px.signal(self.SLOT_SUM, stream)
        self.px.wait(self.SLOT_SUM, stream)
        return self.sum

    def close(self) -> None:
        self.px.close()


def shard_block_weights(w: BlockWeights, cfg: BlockConfig, world: int, rank: int,
                        prepare: bool = True) -> BlockWeights:
    """Rank r's slices of a block's projections (AdaLN and norm weights unchanged);
    ``prepare`` packs the gate_up slice for the SwiGLU epilogue (a device op)."""
    h, d, hd, f = cfg.heads, cfg.head_dim, cfg.hidden, cfg.ffn
    if h % world or f % world:
        raise ValueError("heads and FFN width must be divisible by the tensor-parallel size")
    hl, fr = h // world, f // world
    if fr % 128:
        raise ValueError("each rank's FFN slice must be a multiple of 128 columns (SwiGLU epilogue blocks)")
    qkv = w.w_qkv.view(3, h, d, hd)[:, rank * hl:(rank + 1) * hl].reshape(3 * hl * d, hd).contiguous()
    w_o = w.w_o[:, rank * hl * d:(rank + 1) * hl * d].contiguous()
    up = w.w_gate_up[:f][rank * fr:(rank + 1) * fr]
    gate = w.w_gate_up[f:][rank * fr:(rank + 1) * fr]
    gate_up = torch.cat([up, gate]).contiguous()
    w_down = w.w_down[:, rank * fr:(rank + 1) * fr].contiguous()
    out = BlockWeights(w_qkv=qkv, norm_q=w.norm_q, norm_k=w.norm_k, w_o=w_o, w_gate_up=gate_up, w_down=w_down,
                       norm1=w.norm1, norm2=w.norm2, w_adaln=w.w_adaln, b_adaln=w.b_adaln)
    return out.prepare() if prepare else out


class TPWorkspace:
    def __init__(self, tokens: int, cfg: BlockConfig, world: int, device):
        e = dict(dtype=torch.bfloat16, device=device)
        hl, fr = cfg.heads // world, cfg.ffn // world
        self.normalized = torch.empty(tokens, cfg.hidden, **e)
        self.qkv = torch.empty(tokens, 3 * hl * cfg.head_dim, **e)
        self.q = torch.empty(tokens, hl, cfg.head_dim, **e)
        self.k = torch.empty(tokens, hl, cfg.head_dim, **e)
        self.v = torch.empty(tokens, hl, cfg.head_dim, **e)
        self.attn = torch.empty(tokens, hl, cfg.head_dim, **e)
        self.residual = torch.empty(tokens, cfg.hidden, **e)
        self.normalized2 = torch.empty(tokens, cfg.hidden, **e)
        self.hidden = torch.empty(tokens, fr, **e)
        self.out = [torch.empty(tokens, cfg.hidden, **e), torch.empty(tokens, cfg.hidden, **e)]


def tp_block_forward(x: torch.Tensor, modulation: torch.Tensor, segments: list[Segment], w: BlockWeights,
                     cos: torch.Tensor, sin: torch.Tensor, cfg: BlockConfig, ws: TPWorkspace, tp: TensorParallel,
                     out: torch.Tensor) -> torch.Tensor:
    """One block on all tokens x [N, Hd] with this rank's weight slices."""
    n, hd = x.shape
    d = cfg.head_dim
    hl = w.w_qkv.shape[0] // (3 * d)
    for s in segments:
        r = slice(s.start, s.start + s.length)
        ops.h3_rms_modulate_(ws.normalized[r], x[r], w.norm1, _col(modulation, 1, hd, s),
                             _col(modulation, 0, hd, s), cfg.eps)
    if qkv_fused(hl, cos):
        ops.linear_qkv_norm_rope_([ws.q], [ws.k], [ws.v], ws.normalized, w.w_qkv, w.norm_q, w.norm_k, cos, sin,
                                  cfg.qk_eps)
        v = ws.v
    else:
        ops.linear_(ws.qkv, ws.normalized, w.w_qkv)
        qkv = ws.qkv.view(n, 3, hl, d)
        ops.h3_qk_norm_rope_(ws.q.unsqueeze(1), qkv[:, 0].unsqueeze(1), w.norm_q, cos, sin, cfg.qk_eps)
        ops.h3_qk_norm_rope_(ws.k.unsqueeze(1), qkv[:, 1].unsqueeze(1), w.norm_k, cos, sin, cfg.qk_eps)
        v = qkv[:, 2]
    ops.mha_(ws.attn.unsqueeze(0), ws.q.unsqueeze(0), ws.k.unsqueeze(0), v.unsqueeze(0), 1.0 / math.sqrt(d))
    ops.linear_(tp.part, ws.attn.view(n, hl * d), w.w_o)
    o = tp.allreduce()
    for s in segments:
        r = slice(s.start, s.start + s.length)
        ops.h3_gated_residual_rms_modulate_(ws.residual[r], ws.normalized2[r], x[r], _col(modulation, 2, hd, s),
                                            o[r], w.norm2, _col(modulation, 4, hd, s),
                                            _col(modulation, 3, hd, s), cfg.eps)
    ops.linear_swiglu(ws.normalized2, w.w_gate_up_packed, out=ws.hidden)
    ops.linear_(tp.part, ws.hidden, w.w_down)
    mlp = tp.allreduce()
    for s in segments:
        r = slice(s.start, s.start + s.length)
        ops.h3_gated_residual_(out[r], ws.residual[r], modulation[s.row, 5 * hd:6 * hd], mlp[r])
    return out
