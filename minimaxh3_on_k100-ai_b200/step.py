"""The 40-block DiT denoising step (benchmark config 5) on 1..W GPUs.

Mirrors ``MiniMaxH3Transformer::forward`` (patches/InfiniLM.patch:1626-1826)
for the parts on the hot path: RoPE table for the joint sequence, time
embedding at the step's timestep, every block's AdaLN modulation computed up
front (the batched AdaLN of :1718-1761), run-length modulation segments of the
local tokens (:1765-1792), then the block loop.  Under sequence parallelism
rank r runs the loop on its T = ceil(S/W) tokens and the blocks exchange heads
through ``ulysses``.

Inputs are the joint sequence's hidden states (video latent tokens followed by
conditioning tokens) already at model width, as benchmark config 5 specifies;
weights are random-init (no checkpoint).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _lib, ops
from .block import (BlockConfig, Segment, Workspace, adaln_modulation, adaln_project, block_forward,
                    random_block_weights, random_time_embedder, segments_from_indices, time_embedding)
from .health import bounded_collective, bounded_sync
from . import phases
from .phases import mark

# the phases that launch the attention kernel (one GPU / tensor parallel, and the
# sequence-parallel block, whose attention also stores the return rows)
ATTENTION_PHASES = ("attention", "attention_send")
from .ulysses import SequenceParallel, local_rows

# token tags video 0, text 1, audio 2 (patches/InfiniLM.patch:137); adaln row = 3 * timestep_index + tag (:1695-1697)
VIDEO_TAG, TEXT_TAG, AUDIO_TAG = 0, 1, 2


@dataclass
class StepConfig:
    blocks: int = 40
    video_grid: tuple = (32, 24, 24)
    cond_tokens: int = 512
    timestep: float = 500.0
    block: BlockConfig = field(default_factory=BlockConfig)

    @property
    def video_tokens(self) -> int:
        t, h, w = self.video_grid
        return t * h * w

    @property
    def tokens(self) -> int:
        return self.video_tokens + self.cond_tokens


def joint_positions(cfg: StepConfig) -> torch.Tensor:
    """[S, 3] fp64: the video latent grid enumerated t-major, then conditioning
    token j at (j, j, j) (text tokens advance all three axes together)."""
    t, h, w = cfg.video_grid
    tt, hh, ww = torch.meshgrid(torch.arange(t), torch.arange(h), torch.arange(w), indexing="ij")
    video = torch.stack((tt, hh, ww), -1).reshape(-1, 3)
    j = torch.arange(cfg.cond_tokens)
    cond = torch.stack((j, j, j), -1)
    return torch.cat([video, cond]).double()


class BlockStack:
    """The block loop shared by ``DiTStep`` and ``model.H3Transformer``: the
    blocks' weights (AdaLN projections column-split across ranks), the batched
    AdaLN of every block, the Ulysses exchange state and the per-shape
    activation buffers."""

    def __init__(self, bc: BlockConfig, blocks: int, device, world: int = 1, rank: int = 0, group=None,
                 seed: int = 0, temb_dim: int | None = None, parallel: str = "sp"):
        if parallel not in ("sp", "tp"):
            raise ValueError("parallel must be 'sp' (Ulysses sequence parallelism) or 'tp' (tensor parallelism)")
        self.cfg = bc
        self.device = torch.device(device)
        self.world, self.rank, self.group = world, rank, group
        self.parallel = parallel if world > 1 else "sp"
        self.weights = [random_block_weights(bc, self.device, seed=seed + 1000 * i, temb_dim=temb_dim)
                        for i in range(blocks)]
        if world > 1:
            # AdaLN projections stay column-parallel (as the reference keeps them,
            # patches/InfiniLM.patch:1286-1292, 1740-1761): rank r holds output columns
            # [r*n, (r+1)*n) of every block's projection and the rows are all-gathered
            # once per step.  Each column's dot product is computed the same way on any
            # rank, so the gathered modulation is bitwise the 1-GPU one.
            rows = self.weights[0].w_adaln.shape[0]
            if rows % world != 0 or (rows // world) % 32 != 0:
                raise ValueError("AdaLN projection width must split into multiples of 32 columns per rank")
            n = rows // world
            for w in self.weights:
                w.w_adaln = w.w_adaln[rank * n:(rank + 1) * n].contiguous()
                w.b_adaln = w.b_adaln[rank * n:(rank + 1) * n].contiguous()
        if self.parallel == "tp":
            from .tp import shard_block_weights
            self.weights = [shard_block_weights(w, bc, world, rank) for w in self.weights]
        self._ws: dict = {}
        self._sp: dict[tuple[int, int], SequenceParallel] = {}
        self._tp: dict = {}
        # tensor parallelism: all-reduces chunked behind their GEMMs (same bits either way)
        self.tp_overlap = True
        # host-side bound on the step's collectives (a late or missing rank -> CollectiveTimeout)
        self.collective_timeout_s = 120.0

    def workspace(self, tokens: int):
        if tokens not in self._ws:
            if self.parallel == "tp":
                from .tp import TPWorkspace
                self._ws[tokens] = TPWorkspace(tokens, self.cfg, self.world, self.device)
            else:
                self._ws[tokens] = Workspace(tokens, self.cfg, self.device)
        return self._ws[tokens]

    def _evict(self, cache: dict, key) -> None:
        """Keep only the exchange of the shape about to run: a previous shape's
        peer buffers (CUDA-IPC allocations mapped by every peer) are released
        collectively first.  Every rank changes shape at the same call, so the
        barrier pairs up; after it no peer still writes into the old buffers (each
        rank's last wait on them completed before it got here)."""
        stale = [k for k in cache if k != key]
        if not stale:
            return
        import torch.distributed as dist
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for k in stale:
            cache.pop(k).close()

    def tensor_parallel(self, tokens: int):
        if tokens not in self._tp:
            from .tp import TensorParallel
            self._evict(self._tp, tokens)
            self._tp[tokens] = TensorParallel(self.world, self.rank, self.group, tokens, self.cfg.hidden, self.device)
        return self._tp[tokens]

    def sequence_parallel(self, valid_tokens: int, local_tokens: int) -> SequenceParallel | None:
        if self.world == 1 or self.parallel == "tp":
            return None
        key = (valid_tokens, local_tokens)
        if key not in self._sp:
            self._evict(self._sp, key)
            self._sp[key] = SequenceParallel(self.world, self.rank, self.group, valid_tokens, local_tokens,
                                             self.cfg.heads, self.cfg.head_dim, self.device)
        return self._sp[key]

    def _project_rows(self, activated: torch.Tensor, rows) -> torch.Tensor | None:
        """This rank's columns of every block's AdaLN projection [blocks, t, n], only
        the modalities that ``rows`` (rows of the [t*modalities, 6*Hd] table the
        segments read) name -- the others are left unwritten and never read.  None
        when every modality is needed or the weight-streaming kernel does not apply."""
        bc = self.cfg
        t, mods, width = activated.shape[0], bc.modalities, 6 * bc.hidden
        if rows is None or t > ops.ADALN_MAX_ROWS:
            return None
        needed = sorted({int(r) % mods for r in rows})
        if len(needed) == mods:
            return None
        n = self.weights[0].w_adaln.shape[0]          # this rank's columns: [c0, c0 + n)
        c0 = self.rank * n if self.world > 1 else 0
        spans = []
        for m in needed:
            a, b = max(m * width, c0), min((m + 1) * width, c0 + n)
            if a >= b:
                continue
            if spans and spans[-1][1] == a - c0:
                spans[-1] = (spans[-1][0], b - c0)        # adjacent modalities: one launch
            else:
                spans.append((a - c0, b - c0))
        local = torch.empty(len(self.weights), t, n, dtype=torch.bfloat16, device=activated.device)
        for i, w in enumerate(self.weights):
            for a, b in spans:
                ops.adaln_projection(activated, w.w_adaln[a:b], w.b_adaln[a:b], out=local[i, :, a:b])
        return local

    def modulations(self, temb: torch.Tensor, rows=None) -> list[torch.Tensor]:
        """Every block's modulation rows [timesteps*modalities, 6*Hd], computed up
        front (the reference's batched AdaLN, patches/InfiniLM.patch:1718-1761).
        ``rows``: the table rows the segments will read (the reference computes every
        modality's rows; a modality no token uses is skipped -- its rows stay unwritten)."""
        bc = self.cfg
        mark("adaln_modulations")
        activated = ops.silu(temb, dtype=torch.bfloat16)
        local = self._project_rows(activated, rows)
        if self.world == 1:
            if local is None:
                return [adaln_modulation(temb, w, bc) for w in self.weights]
            return [local[i].view(temb.shape[0] * bc.modalities, 6 * bc.hidden) for i in range(local.shape[0])]
        import torch.distributed as dist
        if local is None:
            local = torch.stack([adaln_project(activated, w.w_adaln, w.b_adaln) for w in self.weights])
        gathered = torch.empty((self.world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
        if local.is_cuda and torch.cuda.is_current_stream_capturing():
            dist.all_gather_into_tensor(gathered, local, group=self.group)   # recorded into the graph
        else:
            # a peer that is late or gone becomes an error here, not a hang
            bounded_collective(lambda: dist.all_gather_into_tensor(gathered, local, group=self.group, async_op=True),
                               "AdaLN modulation all-gather", self.collective_timeout_s)
        blocks, t, n = local.shape
        full = gathered.permute(1, 2, 0, 3).reshape(blocks, t * self.world * n)   # rank-major columns
        rows = t * bc.modalities
        return [full[i].view(rows, 6 * bc.hidden) for i in range(blocks)]

    def close(self) -> None:
        """Unmap and free the peer-exchange buffers (call on every rank, after a
        barrier that follows the last step)."""
        for sp in self._sp.values():
            sp.close()
        for tp in self._tp.values():
            tp.close()
        self._sp, self._tp = {}, {}

    def run(self, h: torch.Tensor, mods: list[torch.Tensor], segments: list[Segment], cos: torch.Tensor,
            sin: torch.Tensor, valid_tokens: int) -> torch.Tensor:
        """The block loop on this rank's tokens h [T, Hd]; returns one of the two
        workspace output buffers."""
        ws = self.workspace(h.shape[0])
        if self.parallel == "tp":
            from .tp import tp_block_forward
            tp = self.tensor_parallel(h.shape[0])
            for i, w in enumerate(self.weights):
                h = tp_block_forward(h, mods[i], segments, w, cos, sin, self.cfg, ws, tp, out=ws.out[i % 2],
                                     overlap=self.tp_overlap)
            return h
        sp = self.sequence_parallel(valid_tokens, h.shape[0])
        for i, w in enumerate(self.weights):
            # block i > 0 reads block i-1's output together with its per-tile sums of
            # squares (written by the down-projection's epilogue)
            x_sq = ws.out_sq[(i - 1) % 2] if i > 0 else None
            h = block_forward(h, mods[i], segments, w, cos, sin, self.cfg, ws, out=ws.out[i % 2], sp=sp,
                              x_sq=x_sq, out_sq=ws.out_sq[i % 2])
        return h


class DiTStep:
    """One denoising step of the block stack.  ``forward`` takes this rank's
    tokens [T, Hd] on the device; ``__call__`` is the end-to-end entry point
    (host tensor in, host tensor out)."""

    def __init__(self, cfg: StepConfig, device, world: int = 1, rank: int = 0, group=None, seed: int = 0,
                 parallel: str = "sp"):
        self.cfg = cfg
        self.device = torch.device(device)
        bc = cfg.block
        self.world, self.rank = world, rank
        self.parallel = parallel if world > 1 else "sp"
        if self.parallel == "tp":
            # tensor parallelism: every rank runs all tokens on its slice of the weights
            self.local, start = cfg.tokens, 0
        else:
            self.local, start, padded = local_rows(cfg.tokens, world, rank)
        self.start = start
        self.group = group
        self.stack = BlockStack(bc, cfg.blocks, self.device, world, rank, group, seed, parallel=self.parallel)
        self.weights = self.stack.weights
        self.time = random_time_embedder(bc.hidden, self.device, seed=seed + 7)
        # per-token tables of the local rows; padded rows reuse row 0 (:1706-1710)
        pos = joint_positions(cfg)
        tags = torch.cat([torch.full((cfg.video_tokens,), VIDEO_TAG), torch.full((cfg.cond_tokens,), TEXT_TAG)])
        idx = torch.arange(start, start + self.local)
        idx = torch.where(idx < cfg.tokens, idx, torch.zeros_like(idx))
        power = ops.rope_powers((16, 16, 16), device=self.device)[:16].contiguous()
        table = ops.h3_rope_cache(pos[idx].to(self.device), power)
        self.cos, self.sin = table[:, :48], table[:, 48:]
        self.segments: list[Segment] = segments_from_indices((3 * 0 + tags[idx]).tolist())
        # the modulation rows any rank's tokens read (the same set on every rank)
        self.mod_rows = sorted(set((3 * 0 + tags).tolist()))
        self.ws = self.stack.workspace(self.local)
        self.sp = self.stack.sequence_parallel(cfg.tokens, self.local)
        self.timestep = torch.full((1,), cfg.timestep, dtype=torch.float32, device=self.device)
        self.x_dev = torch.empty(self.local, bc.hidden, dtype=torch.bfloat16, device=self.device)
        self.graph, self.graph_out, self.graph_marks = None, None, []
        # __call__ copies the host tokens in on a side stream; the step waits for that
        # copy only where it first reads them (after the AdaLN modulations, which do not),
        # so the copy overlaps the modulations -- in the captured graph an event wait node
        self.copy_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self.tokens_in = torch.cuda.Event(external=True) if self.device.type == "cuda" else None

    def modulations(self, timestep: torch.Tensor) -> list[torch.Tensor]:
        """Every block's modulation rows [timesteps*modalities, 6*Hd], computed up
        front (the reference's batched AdaLN)."""
        return self.stack.modulations(time_embedding(timestep, self.time), rows=self.mod_rows)

    def forward(self, x: torch.Tensor, timestep: torch.Tensor | None = None) -> torch.Tensor:
        ts = self.timestep if timestep is None else timestep
        mods = self.modulations(ts)
        if self.tokens_in is not None:
            self.tokens_in.wait(torch.cuda.current_stream(self.device))   # the tokens' copy (if any)
        return self.stack.run(x, mods, self.segments, self.cos, self.sin, self.cfg.tokens)

    def capture(self) -> None:
        """Record ``forward(self.x_dev)`` -- every kernel of the step and, under
        sequence parallelism, its NCCL all-to-alls -- into one CUDA graph that
        ``run()`` and ``__call__`` replay.  All ranks must capture together."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.forward(self.x_dev)          # warm-up outside the graph
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            # event record nodes around each attention launch (2 per block): after a
            # replay, graph_attention_ms() reads that replay's attention time
            with phases.capturing(ATTENTION_PHASES) as marks:
                out = self.forward(self.x_dev)
        self.graph, self.graph_out, self.graph_marks = graph, out, marks

    def graph_attention_ms(self) -> tuple[float, int]:
        """(device ms of all attention launches, number of launches) in the last
        replay of the captured step."""
        t = phases.totals(self.graph_marks, ATTENTION_PHASES)
        n = sum(1 for name, _ in self.graph_marks if name in ATTENTION_PHASES)
        return sum(t.values()), n

    def release_graph(self) -> None:
        """Drop the graph (required before destroying a process group whose
        collectives it holds)."""
        self.graph, self.graph_out, self.graph_marks = None, None, []

    def close(self) -> None:
        """Release the peer-exchange buffers (every rank, after the last step)."""
        self.release_graph()
        self.stack.close()
        self.sp = None

    def run(self) -> torch.Tensor:
        """One step on ``self.x_dev`` (graph replay when captured)."""
        if getattr(self, "graph", None) is not None:
            self.graph.replay()
            return self.graph_out
        return self.forward(self.x_dev)

    def __call__(self, x_host: torch.Tensor, out_host: torch.Tensor | None = None) -> torch.Tensor:
        """End to end: host (pinned) tokens in, host tokens out."""
        if self.copy_stream is not None:
            # on a side stream, after everything before this call on the step's stream
            # (the previous step has finished with x_dev); the step waits at first use
            self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.copy_stream):
                self.x_dev.copy_(x_host, non_blocking=True)
                self.tokens_in.record(self.copy_stream)
        else:
            self.x_dev.copy_(x_host, non_blocking=True)
        y = self.run()
        if out_host is None:
            out_host = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        out_host.copy_(y, non_blocking=True)
        # bounded: a replayed graph whose exchange or collective waits on a missing
        # peer raises DeviceTimeout here instead of blocking the host for good
        bounded_sync(torch.cuda.current_stream(self.device), self.stack.collective_timeout_s, "DiTStep")
        self.check()
        return out_host

    def check(self) -> None:
        """Raise if a bounded device-side wait of the step gave up (a peer that
        never signalled its exchange flag, an mbarrier that never completed) or the
        device reported an error: such kernels return normally and leave their
        outputs incomplete.  Synchronises the device."""
        with torch.cuda.device(self.device):
            _lib.check_device("DiTStep")
