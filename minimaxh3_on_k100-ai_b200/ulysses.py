"""Ulysses sequence parallelism for the H3 DiT attention (head <-> sequence
all-to-all), after ``MiniMaxH3Attention`` in patches/InfiniLM.patch:895-1137.

Rank r owns tokens [r*T, (r+1)*T) of the sequence (zero-padded to W*T rows,
padding only after the real tokens, :1676-1716).  For attention each rank
needs H/W heads over the whole sequence:

  send block p   = heads [p*Hl, (p+1)*Hl) of my T tokens      (gather_sequence :895-910)
  recv block q   = rank q's tokens, so the token axis is global order
  attention      on [W*T, Hl, D] queries, keys/values narrowed to the real length
  return block q = my output rows for rank q's tokens;  back home, block q holds
                   heads q*Hl + h of the local tokens           (scatter_sequence :1127-1137)

The q/k RMSNorm + RoPE kernel writes straight into the permuted view of the
send buffer ([T, W, Hl, D] view of [W, T, Hl, D]), as the reference's
h3_qk_norm_rope_ does (:1092-1103), so no separate pack pass is needed for q/k.

The exchange logic is written against a small ``kernels`` interface so the same
host code runs with the CUDA ops on NCCL and, in the CPU tests, with the oracle
on gloo ranks.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


@dataclass
class Kernels:
    """The three device ops the exchange needs.
    qk_norm_rope(out, x, weight, cos, sin, eps); mha(out, q, k, v, scale); copy(dst, src)."""
    qk_norm_rope: Callable
    mha: Callable
    copy: Callable = lambda dst, src: dst.copy_(src)


def cuda_kernels() -> Kernels:
    from . import ops
    return Kernels(qk_norm_rope=ops.h3_qk_norm_rope_, mha=ops.mha_)


@dataclass
class ExchangeBuffers:
    send: list          # 3 x [W, T, Hl, D]  (q, k, v)
    recv: list          # 3 x [W, T, Hl, D]
    attn: torch.Tensor  # [W*T, Hl, D]
    back: torch.Tensor  # [W, T, Hl, D]

    @staticmethod
    def allocate(world, tokens, heads_local, head_dim, device, dtype=torch.bfloat16):
        e = dict(device=device, dtype=dtype)
        return ExchangeBuffers(
            send=[torch.empty(world, tokens, heads_local, head_dim, **e) for _ in range(3)],
            recv=[torch.empty(world, tokens, heads_local, head_dim, **e) for _ in range(3)],
            attn=torch.empty(world * tokens, heads_local, head_dim, **e),
            back=torch.empty(world, tokens, heads_local, head_dim, **e))


def local_rows(total_tokens: int, world: int, rank: int) -> tuple[int, int, int]:
    """(T, start, padded_total): T = ceil(S/W) tokens per rank, rank r owns [r*T, (r+1)*T)."""
    t = (total_tokens + world - 1) // world
    return t, rank * t, t * world


class SequenceParallel:
    def __init__(self, world: int, rank: int, group, valid_tokens: int, local_tokens: int, heads: int,
                 head_dim: int, device, kernels: Kernels | None = None):
        if heads % world != 0:
            # same constraint as the reference (patches/InfiniLM.patch:717-721)
            raise ValueError("heads must be divisible by the sequence-parallel size")
        if valid_tokens > world * local_tokens:
            raise ValueError("invalid sequence-parallel token layout")
        self.world, self.rank, self.group = world, rank, group
        self.valid = valid_tokens
        self.tokens = local_tokens
        self.heads, self.head_dim = heads, head_dim
        self.heads_local = heads // world
        self.kernels = kernels or cuda_kernels()
        self.bufs = ExchangeBuffers.allocate(world, local_tokens, self.heads_local, head_dim, device)

    def _all_to_all(self, outs, ins):
        for o, i in zip(outs, ins):
            dist.all_to_all_single(o, i, group=self.group)

    def attention_from_qkv(self, qkv: torch.Tensor, norm_q, norm_k, cos, sin, qk_eps: float) -> torch.Tensor:
        """qkv [T, 3*H*D] (rows [q|k|v] head-major) of this rank's tokens ->
        attention output [T, H*D] of the same tokens (all heads)."""
        t, w, hl, d = self.tokens, self.world, self.heads_local, self.head_dim
        k = self.kernels
        b = self.bufs
        parts = qkv.view(t, 3, w, hl, d)
        # tokens -> heads: q/k normalised + rotated straight into the send layout
        k.qk_norm_rope(b.send[0].permute(1, 0, 2, 3), parts[:, 0], norm_q, cos, sin, qk_eps)
        k.qk_norm_rope(b.send[1].permute(1, 0, 2, 3), parts[:, 1], norm_k, cos, sin, qk_eps)
        k.copy(b.send[2].permute(1, 0, 2, 3), parts[:, 2])
        self._all_to_all(b.recv, b.send)
        q = b.recv[0].view(1, w * t, hl, d)
        kk = b.recv[1].view(1, w * t, hl, d)[:, :self.valid]
        v = b.recv[2].view(1, w * t, hl, d)[:, :self.valid]
        k.mha(b.attn.unsqueeze(0), q, kk, v, 1.0 / math.sqrt(d))
        # heads -> tokens
        self._all_to_all([b.back], [b.attn.view(w, t, hl, d)])
        return b.back.permute(1, 0, 2, 3).reshape(t, w * hl * d)

    def attention(self, ws, weights, cos, sin, cfg) -> torch.Tensor:
        from . import ops
        ops.linear_(ws.qkv, ws.normalized, weights.w_qkv)
        return self.attention_from_qkv(ws.qkv, weights.norm_q, weights.norm_k, cos, sin, cfg.qk_eps)
