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
from .phases import mark
from .ulysses import PeerExchange


class TensorParallel:
    """All-reduce of a [tokens, hidden] BF16 partial over peer memory.

    ``allreduce_overlapped`` is the reference's chunked overlap
    (``forward_overlapped``, patches/InfiniLM.patch:1399-1476, ``H3_TP_OVERLAP``):
    the rows are cut into ``chunks`` row blocks; the producer (the row-parallel
    GEMM) writes block c on the compute stream while block c-1 is being summed on
    a side stream, so the exchange hides behind the next block's GEMM tiles.  Each
    block's rows are split among the ranks; every row is summed exactly as in the
    unchunked all-reduce (fp32, rank order, one rounding), so both give the same
    bits."""

    SLOT_PARTIAL, SLOT_SUM = 0, 1

    def __init__(self, world: int, rank: int, group, tokens: int, hidden: int, device, chunks: int = 4):
        self.world, self.rank = world, rank
        nbytes = tokens * hidden * 2
        self.px = PeerExchange(world, rank, group, device, {"part": nbytes, "sum": nbytes})
        self.part = self.px.local("part", (tokens, hidden))
        self.sum = self.px.local("sum", (tokens, hidden))
        self.srcs, self.dsts, self.rows = self._owned(0, tokens, hidden)
        self.device = torch.device(device)
        # row blocks of the overlapped form: multiples of the GEMM's 128-row tiles
        per_block = -(-tokens // max(1, chunks))
        step = max(128, -(-per_block // 128) * 128)
        self.blocks = [(c0, min(tokens, c0 + step)) for c0 in range(0, tokens, step)]
        self.block_descs = [self._owned(c0, c1, hidden) for c0, c1 in self.blocks]
        self.side = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None

    def _owned(self, r0: int, r1: int, hidden: int):
        """(srcs, dsts, rows): this rank's share of rows [r0, r1) in every rank's
        partial (srcs) and sum (dsts) buffers, as mapped here."""
        share = -(-(r1 - r0) // self.world)
        a = min(r1, r0 + self.rank * share)
        b = min(r1, a + share)
        shape = (b - a, hidden)
        srcs = (_lib.H3Tensor * self.world)(*[self.px.peer_desc(p, "part", shape, a * hidden)
                                              for p in range(self.world)])
        dsts = (_lib.H3Tensor * self.world)(*[self.px.peer_desc(p, "sum", shape, a * hidden)
                                              for p in range(self.world)])
        return srcs, dsts, b - a

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

    def allreduce_overlapped(self, produce) -> torch.Tensor:
        """``produce(r0, r1)`` writes rows [r0, r1) of ``self.part`` on the current
        stream; returns ``self.sum`` (complete on the current stream).

        Per row block: the compute stream produces it and raises this rank's
        PARTIAL flag; the side stream waits for every peer's PARTIAL flag of that
        block (the flags are epochs: a later value also covers this block), sums
        this rank's share into every rank's sum buffer and raises SUM.  The
        compute stream goes on with the next block meanwhile, and at the end waits
        for every peer's SUM flag of the last block, which covers all blocks.
        Buffer reuse is safe for the same reasons as ``allreduce``: nobody writes
        a partial again before every rank has summed all blocks."""
        main = torch.cuda.current_stream(self.device)
        m, s = main.cuda_stream, self.side.cuda_stream
        for (r0, r1), (srcs, dsts, rows) in zip(self.blocks, self.block_descs):
            produce(r0, r1)
            self.px.signal(self.SLOT_PARTIAL, m)
            self.side.wait_stream(main)
            self.px.wait(self.SLOT_PARTIAL, s)
            if rows > 0:
                _lib.call("h3_peer_reduce_rows", dsts, srcs, self.world, s)
            self.px.signal(self.SLOT_SUM, s)
        main.wait_stream(self.side)
        self.px.wait(self.SLOT_SUM, m)
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
                     out: torch.Tensor, overlap: bool = True) -> torch.Tensor:
    """One block on all tokens x [N, Hd] with this rank's weight slices.  With
    ``overlap`` the two all-reduces run chunked behind their GEMMs
    (``TensorParallel.allreduce_overlapped``); the result is the same bits."""
    n, hd = x.shape
    d = cfg.head_dim
    hl = w.w_qkv.shape[0] // (3 * d)
    mark("norm1")
    for s in segments:
        r = slice(s.start, s.start + s.length)
        ops.h3_rms_modulate_(ws.normalized[r], x[r], w.norm1, _col(modulation, 1, hd, s),
                             _col(modulation, 0, hd, s), cfg.eps)
    mark("qkv_norm_rope")
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
    mark("attention")
    ops.mha_(ws.attn.unsqueeze(0), ws.q.unsqueeze(0), ws.k.unsqueeze(0), v.unsqueeze(0), 1.0 / math.sqrt(d))
    mark("out_proj_allreduce")
    attn = ws.attn.view(n, hl * d)
    if overlap:
        o = tp.allreduce_overlapped(lambda r0, r1: ops.linear_(tp.part[r0:r1], attn[r0:r1], w.w_o))
    else:
        ops.linear_(tp.part, attn, w.w_o)
        o = tp.allreduce()
    mark("norm2")
    for s in segments:
        r = slice(s.start, s.start + s.length)
        ops.h3_gated_residual_rms_modulate_(ws.residual[r], ws.normalized2[r], x[r], _col(modulation, 2, hd, s),
                                            o[r], w.norm2, _col(modulation, 4, hd, s),
                                            _col(modulation, 3, hd, s), cfg.eps)
    mark("gate_up_swiglu")
    ops.linear_swiglu(ws.normalized2, w.w_gate_up_packed, out=ws.hidden)
    mark("down_allreduce")
    if overlap:
        mlp = tp.allreduce_overlapped(lambda r0, r1: ops.linear_(tp.part[r0:r1], ws.hidden[r0:r1], w.w_down))
    else:
        ops.linear_(tp.part, ws.hidden, w.w_down)
        mlp = tp.allreduce()
    mark("residual")
    for s in segments:
        r = slice(s.start, s.start + s.length)
        ops.h3_gated_residual_(out[r], ws.residual[r], modulation[s.row, 5 * hd:6 * hd], mlp[r])
    return out
