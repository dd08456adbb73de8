"""Ulysses sequence parallelism for the H3 DiT attention (head <-> sequence
all-to-all), after ``MiniMaxH3Attention`` in patches/InfiniLM.patch:895-1137.

Rank r owns tokens [r*T, (r+1)*T) of the sequence (zero-padded to W*T rows,
padding only after the real tokens, :1676-1716).  For attention each rank
needs its Hl = H/W heads over the whole sequence:

  send block p   = heads p*Hl + off_g + j of my T tokens    (gather_sequence :895-910)
  recv block q   = rank q's tokens, so the token axis is global order
  attention      on [W*T, Hs_g, D] queries, keys/values narrowed to the real length
  return block q = my output rows for rank q's tokens; back home block q holds
                   heads q*Hl + off_g + h of the local tokens  (:1006-1014)

Heads can be processed in groups (``pipelined_sequence_attention`` :1047-1125,
``attend_exchanged_groups`` :960-1018): the QKV projection of group g+1 runs on
the compute stream while group g's all-to-all runs on a side stream, and group
g's output travels home while group g+1 attends.  The default is one group: on
B200 the NCCL all-to-all kernels need SMs that the attention and GEMM kernels
(one ~200 KB shared-memory CTA per SM) do not leave free, so the exchange does
not overlap anyway, and whole-wave attention calls matter more (measured:
8 GPUs 0.1204 s/step with two groups vs 0.1202 with one).  The QKV weight rows are
regrouped once so each group's projection is one contiguous GEMM (like the
reference's ``group_qkv_weight`` :1020-1045; same dot products, so the result is
bitwise the ungrouped one).  The q/k RMSNorm + RoPE kernel writes straight into
the permuted view of the send buffer ([T, W, Hs, D] view of [W, T, Hs, D]), so
no separate pack pass is needed for q/k.

On GPUs the exchange is peer-to-peer (``PeerExchange``): the receive buffers of
every rank live in CUDA-IPC-shared allocations, the QKV projection's epilogue
(q/k RMSNorm + RoPE included) stores each head row straight into its
destination rank's receive buffer over NVLink (no send buffer, no separate
collective), the attention epilogue stores each output row straight into the
token-major return rows of the rank that owns the token (``h3_mha_scatter``), so
the out-projection reads them in place, and an epoch flag per rank (bounded
device wait) replaces the collective's synchronisation.  ``exchange="collective"`` keeps the
torch.distributed all_to_all_single path (NCCL, or gloo in the CPU tests).

The exchange logic is written against a small ``kernels`` interface so the same
host code runs with the CUDA ops and, in the CPU tests, with the oracle on gloo
ranks.
"""
from __future__ import annotations

import contextlib
import ctypes
import math
from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib
from .phases import mark


@dataclass
class Kernels:
    """Device ops the exchange needs: linear(out, x, w), qk_norm_rope(out, x,
    weight, cos, sin, eps), mha(out, q, k, v, scale), copy(dst, src)."""
    linear: Callable
    qk_norm_rope: Callable
    mha: Callable
    copy: Callable = lambda dst, src: dst.copy_(src)


def cuda_kernels() -> Kernels:
    from . import ops
    return Kernels(linear=ops.linear_, qk_norm_rope=ops.h3_qk_norm_rope_, mha=ops.mha_)


def local_rows(total_tokens: int, world: int, rank: int) -> tuple[int, int, int]:
    """(T, start, padded_total): T = ceil(S/W) tokens per rank, rank r owns [r*T, (r+1)*T)."""
    t = (total_tokens + world - 1) // world
    return t, rank * t, t * world


def head_groups(heads_local: int, groups: int) -> list[int]:
    """Split Hl heads into `groups` nearly equal groups (uneven allowed, larger
    first), as the reference's sp_head_groups (:452-479) does for H3_SP_GROUPS.
    Even group sizes are preferred: the attention kernel runs two 128-row query
    tiles per CTA, so an even head count keeps each call's CTAs a whole number of
    waves when the sequence is a multiple of 2*128*148/2 rows."""
    groups = max(1, min(groups, heads_local))
    if heads_local % 2 == 0 and heads_local // 2 >= groups:
        base, extra = divmod(heads_local // 2, groups)
        return [2 * (base + (1 if g < extra else 0)) for g in range(groups)]
    base, extra = divmod(heads_local, groups)
    return [base + (1 if g < extra else 0) for g in range(groups)]


class _CudaBytes:
    """A raw device allocation seen through __cuda_array_interface__ (int16 units,
    reinterpreted as BF16 by the caller)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes // 2,), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3}


class PeerExchange:
    """Receive buffers every peer can store into, plus epoch flags
    (h3_ipc_* / h3_exchange_* of the C-ABI).  Layout of each rank's allocation:
    flags [SLOTS][MAX_RANKS] uint64 (256 B), then the named regions, 256-byte
    aligned.  Created collectively (every rank, same regions)."""

    MAX_RANKS, SLOTS, HANDLE = 8, 4, 64
    FLAGS_BYTES = 256

    def __init__(self, world: int, rank: int, group, device, regions: dict, timeout_s: float = 5.0):
        if world > self.MAX_RANKS:
            raise ValueError(f"at most {self.MAX_RANKS} ranks")
        self.world, self.rank, self.device = world, rank, torch.device(device)
        self.timeout_ns = int(timeout_s * 1e9)
        lib = _lib.load()
        self.offsets, off = {}, self.FLAGS_BYTES
        for name, nbytes in regions.items():
            self.offsets[name] = off
            off += (nbytes + 255) // 256 * 256
        self.bytes = off
        ptr, handle = ctypes.c_void_p(), (ctypes.c_char * self.HANDLE)()
        with torch.cuda.device(self.device):
            _lib.check(lib.h3_ipc_alloc(self.bytes, ctypes.byref(ptr), handle), "h3_ipc_alloc")
        self.own = ptr.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.bases, self.opened = [], []
        with torch.cuda.device(self.device):
            for p in range(world):
                if p == rank:
                    self.bases.append(self.own)
                    continue
                peer = ctypes.c_void_p()
                buf = (ctypes.c_char * self.HANDLE).from_buffer_copy(handles[p])
                _lib.check(lib.h3_ipc_open(buf, ctypes.byref(peer)), "h3_ipc_open")
                self.bases.append(peer.value)
                self.opened.append(peer.value)
        self.peer_flags = (ctypes.c_void_p * world)(*self.bases)
        self.epoch = torch.zeros(self.SLOTS, dtype=torch.int64, device=self.device)
        dist.barrier(group=group)

    def local(self, name: str, shape) -> torch.Tensor:
        """This rank's region as a BF16 tensor of ``shape``."""
        n = math.prod(shape)
        t = torch.as_tensor(_CudaBytes(self.own + self.offsets[name], 2 * n), device=self.device)
        return t.view(torch.bfloat16).view(*shape)

    def peer_desc(self, p: int, name: str, shape, elem_offset: int = 0, strides=None) -> _lib.H3Tensor:
        """Descriptor of a BF16 block inside rank p's region (as mapped here):
        contiguous, or with the given element strides."""
        d = _lib.H3Tensor()
        d.data = self.bases[p] + self.offsets[name] + 2 * elem_offset
        stride = 1
        for i in reversed(range(len(shape))):
            d.shape[i] = shape[i]
            d.strides[i] = stride if strides is None else strides[i]
            stride *= shape[i]
        d.ndim, d.dtype = len(shape), 0
        return d

    def signal(self, slot: int, stream: int) -> None:
        _lib.CALLS["n"] += 1
        _lib.check(_lib.load().h3_exchange_signal(self.peer_flags, ctypes.c_void_p(self.epoch.data_ptr()), slot,
                                                  self.rank, self.world, stream), "h3_exchange_signal")

    def wait(self, slot: int, stream: int) -> None:
        _lib.CALLS["n"] += 1
        _lib.check(_lib.load().h3_exchange_wait(ctypes.c_void_p(self.own), ctypes.c_void_p(self.epoch.data_ptr()),
                                                slot, self.rank, self.world, self.timeout_ns, stream),
                   "h3_exchange_wait")

    def close(self) -> None:
        lib = _lib.load()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for p in self.opened:
                lib.h3_ipc_close(ctypes.c_void_p(p))
            self.opened = []
            if self.own:
                lib.h3_ipc_free(ctypes.c_void_p(self.own))
                self.own = 0


class SequenceParallel:
    SLOT_QKV, SLOT_OUT = 0, 1

    def __init__(self, world: int, rank: int, group, valid_tokens: int, local_tokens: int, heads: int,
                 head_dim: int, device, kernels: Kernels | None = None, groups: int = 1,
                 exchange: str | None = None):
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
        self.group_heads = head_groups(self.heads_local, groups)
        self.device = torch.device(device)
        e = dict(device=device, dtype=torch.bfloat16)
        w, t, d = world, local_tokens, head_dim
        cuda = self.device.type == "cuda"
        self.exchange = exchange or ("p2p" if cuda else "collective")
        if self.exchange not in ("p2p", "collective"):
            raise ValueError("exchange must be 'p2p' or 'collective'")
        self.attn = [torch.empty(w * t, hs, d, **e) for hs in self.group_heads]
        self.qkv = torch.empty(t * 3 * w * max(self.group_heads) * d, **e)
        self.out = torch.empty(t, w, self.heads_local, d, **e)
        self.side = torch.cuda.Stream(self.device) if cuda else None
        self._weights = {}
        self.peers = None
        if self.exchange == "p2p":
            if len(self.group_heads) != 1:
                raise ValueError("the peer-to-peer exchange runs the heads as one group")
            hs = self.group_heads[0]
            block = w * t * hs * d * 2
            self.peers = PeerExchange(world, rank, group, self.device,
                                      {"q": block, "k": block, "v": block, "back": block})
            self.recv_p2p = [self.peers.local(n, (w, t, hs, d)) for n in ("q", "k", "v")]
            # the returning attention rows land token-major, [T, W, Hl, D] = [T, H*D]
            # with head p*Hl + j at slot (p, j): the out-projection's input as is
            self.back_p2p = self.peers.local("back", (t, w, hs, d))
            # destination descriptors: slot `rank` of every rank's regions, as mapped here
            slot = rank * t * hs * d
            arr = lambda name, shape: (_lib.H3Tensor * w)(  # noqa: E731
                *[self.peers.peer_desc(p, name, shape, slot) for p in range(w)])
            self.dst_q, self.dst_k = arr("q", (t, hs, d)), arr("k", (t, hs, d))
            self.dst_v = arr("v", (t, hs * d))
            self.dst_v3 = arr("v", (t, hs, d))
            # this rank's head slice (slot `rank` of the W head slices) of every rank's
            # return rows: [T, Hl, D] with row stride W*Hl*D
            self.dst_back = (_lib.H3Tensor * w)(*[
                self.peers.peer_desc(p, "back", (t, hs, d), rank * hs * d, strides=(w * hs * d, d, 1))
                for p in range(w)])
        else:
            self.send = [[torch.empty(w, t, hs, d, **e) for _ in range(3)] for hs in self.group_heads]
            self.recv = [[torch.empty(w, t, hs, d, **e) for _ in range(3)] for hs in self.group_heads]
            self.back = [torch.empty(w, t, hs, d, **e) for hs in self.group_heads]

    # -- weight layout --------------------------------------------------------
    def group_weights(self, w_qkv: torch.Tensor) -> list[torch.Tensor]:
        """Rows [q|k|v][head p*Hl + j][D] -> per group g one block of rows
        [q|k|v][p][j in g][D] (computed once per weight tensor)."""
        if len(self.group_heads) == 1:
            return [w_qkv]          # one group: the regrouped order is the original order
        key = w_qkv.data_ptr()
        if key not in self._weights:
            w, hl, d = self.world, self.heads_local, self.head_dim
            by_head = w_qkv.view(3, w, hl, d, w_qkv.shape[1])
            out, off = [], 0
            for hs in self.group_heads:
                out.append(by_head[:, :, off:off + hs].reshape(3 * w * hs * d, w_qkv.shape[1]).contiguous())
                off += hs
            self._weights[key] = out
        return self._weights[key]

    # -- streams ----------------------------------------------------------------
    def _on_side(self):
        return torch.cuda.stream(self.side) if self.side is not None else contextlib.nullcontext()

    def _side_waits_compute(self):
        if self.side is not None:
            self.side.wait_stream(torch.cuda.current_stream(self.device))

    def _event_on_side(self):
        if self.side is None:
            return None
        ev = torch.cuda.Event()
        ev.record(self.side)
        return ev

    def _all_to_all(self, outs, ins):
        for o, i in zip(outs, ins):
            dist.all_to_all_single(o, i, group=self.group)

    def close(self) -> None:
        if self.peers is not None:
            self.peers.close()
            self.peers = None

    # -- peer-to-peer exchange (GPU) --------------------------------------------
    def _attention_p2p(self, normalized, w_qkv, norm_q, norm_k, cos, sin, qk_eps):
        w, t, d, hl = self.world, self.tokens, self.head_dim, self.heads_local
        px = self.peers
        stream = torch.cuda.current_stream(self.device).cuda_stream
        cos_d, sin_d = _lib.desc(cos), _lib.desc(sin)
        # tokens -> heads: block p (heads p*Hl..) of my tokens goes to slot r of rank p,
        # stored by the producing kernels themselves
        from .block import qkv_fused
        mark("qkv_norm_rope_send")
        if qkv_fused(self.heads, cos):
            # the QKV GEMM's epilogue normalises/rotates q and k and stores every head row
            # into its destination rank's receive buffer (one launch for the whole send)
            _lib.call("h3_linear_qkv_norm_rope", _lib.desc(normalized), _lib.desc(w_qkv), self.dst_q, self.dst_k,
                      self.dst_v3, w, _lib.desc(norm_q), _lib.desc(norm_k), cos_d, sin_d, float(qk_eps), stream)
        else:
            qkv = self.qkv[:t * 3 * w * hl * d].view(t, 3 * w * hl * d)
            self.kernels.linear(qkv, normalized, w_qkv)
            parts = qkv.view(t, 3, w, hl, d)
            _lib.call("h3_qk_norm_rope_multi", self.dst_q, w, _lib.desc(parts[:, 0]), _lib.desc(norm_q), cos_d,
                      sin_d, float(qk_eps), stream)
            _lib.call("h3_qk_norm_rope_multi", self.dst_k, w, _lib.desc(parts[:, 1]), _lib.desc(norm_k), cos_d,
                      sin_d, float(qk_eps), stream)
            _lib.call("h3_copy_blocks", self.dst_v, w, _lib.desc(parts[:, 2].permute(1, 0, 2, 3).flatten(2)),
                      stream)
        mark("wait_qkv")
        px.signal(self.SLOT_QKV, stream)
        px.wait(self.SLOT_QKV, stream)
        q = self.recv_p2p[0].view(1, w * t, hl, d)
        kk = self.recv_p2p[1].view(1, w * t, hl, d)[:, :self.valid]
        v = self.recv_p2p[2].view(1, w * t, hl, d)[:, :self.valid]
        # heads -> tokens: the attention epilogue stores each output row straight into
        # the return rows of the rank that owns its token (this rank's head slot)
        mark("attention_send")
        _lib.call("h3_mha_scatter", self.dst_back, w, _lib.desc(q), _lib.desc(kk), _lib.desc(v),
                  1.0 / math.sqrt(d), stream)
        mark("wait_out")
        px.signal(self.SLOT_OUT, stream)
        px.wait(self.SLOT_OUT, stream)
        return self.back_p2p.view(t, w * hl * d)

    # -- the exchange -----------------------------------------------------------
    def attention(self, normalized: torch.Tensor, w_qkv: torch.Tensor, norm_q, norm_k, cos, sin,
                  qk_eps: float) -> torch.Tensor:
        """normalized [T, Hd] tokens of this rank -> attention output [T, H*D] of
        the same tokens (all heads, head-major), before the output projection."""
        if self.exchange == "p2p":
            return self._attention_p2p(normalized, w_qkv, norm_q, norm_k, cos, sin, qk_eps)
        k = self.kernels
        w, t, d, hl = self.world, self.tokens, self.head_dim, self.heads_local
        compute = torch.cuda.current_stream(self.device) if self.side is not None else None
        weights = self.group_weights(w_qkv)
        arrived = []
        # tokens -> heads, group by group: project, normalise/rotate into the send
        # layout, exchange on the side stream while the next group projects
        for g, hs in enumerate(self.group_heads):
            qkv = self.qkv[:t * 3 * w * hs * d].view(t, 3 * w * hs * d)
            k.linear(qkv, normalized, weights[g])
            parts = qkv.view(t, 3, w, hs, d)
            send = self.send[g]
            k.qk_norm_rope(send[0].permute(1, 0, 2, 3), parts[:, 0], norm_q, cos, sin, qk_eps)
            k.qk_norm_rope(send[1].permute(1, 0, 2, 3), parts[:, 1], norm_k, cos, sin, qk_eps)
            k.copy(send[2].permute(1, 0, 2, 3), parts[:, 2])
            self._side_waits_compute()
            with self._on_side():
                self._all_to_all(self.recv[g], send)
            arrived.append(self._event_on_side())
        # attention per group; each group's output goes home while the next attends
        off = 0
        for g, hs in enumerate(self.group_heads):
            if arrived[g] is not None:
                compute.wait_event(arrived[g])
            recv = self.recv[g]
            q = recv[0].view(1, w * t, hs, d)
            kk = recv[1].view(1, w * t, hs, d)[:, :self.valid]
            v = recv[2].view(1, w * t, hs, d)[:, :self.valid]
            k.mha(self.attn[g].unsqueeze(0), q, kk, v, 1.0 / math.sqrt(d))
            self._side_waits_compute()
            with self._on_side():
                self._all_to_all([self.back[g]], [self.attn[g].view(w, t, hs, d)])
        if self.side is not None:
            compute.wait_stream(self.side)
        for g, hs in enumerate(self.group_heads):
            k.copy(self.out[:, :, off:off + hs], self.back[g].permute(1, 0, 2, 3))
            off += hs
        return self.out.view(t, w * hl * d)
