"""The full MiniMax-H3 transformer forward around the block stack: input
projections, the text token refiner, packing of the joint sequence, the time
embedding, the batched AdaLN, the 40 blocks, the output norm and projections,
and the gather of the video/audio rows.

Mirrors ``MiniMaxH3Transformer::forward`` (patches/InfiniLM.patch:1626-1826) and
its modules:

    video  = bf16(proj_in(f32 video patches))                    :1662, h3_linear_f32
    audio  = bf16(audio_proj_in(f32 audio latents))              :1663
    text   = token_refiner(context_embedder(bf16 text))          :1664-1665, :1198-1241
    hidden = zeros[P*T, Hd]; index_copy(text | video | audio)    :1680-1690, h3_index_copy_rows
    temb   = time_embedder(timestep)                             :1692, :1494-1517
    adaln  = 3 * timestep_indices + token_tags                   :1697-1700
    blocks (sequence-parallel over ranks, batched AdaLN)         :1702-1806
    out    = norm_out(hidden, temb, timestep_indices)            :1810, :1519-1538
    video_out = proj_out(f32 out), audio_out = audio_proj_out    :1812-1814, h3_linear_f32
    (sequence parallel: all-gather rows in token order)          :1815-1820
    gather_rows(video_out, video_indices), (audio ...)           :1822-1823, h3_gather_rows

The token refiner (2 blocks over the text tokens, replicated on every rank,
:233-235) is RMSNorm -> attention (q/k RMSNorm over the head dim, no RoPE) ->
residual add -> RMSNorm -> SwiGLU MLP -> residual add, then a final RMSNorm.
Residual adds and biases of BF16 linears use the gated-residual kernels with a
unit gate: bf16(x + bf16(1 * y)) = bf16(x + y).

``MiniMaxH3DiffusersAdapter`` (below) gives it the reference's Diffusers-style
surface: same forward signature, packed-input record and output record.

Weights are random-init (no checkpoint in this environment); sizes follow the
benchmark block config (hidden 5120, 40 heads, FFN 13824) with the reference's
patch (24 latent channels x (1,2,2) = 96), audio (32) and text (5120) widths.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import _lib, ops
from .block import (BlockConfig, add_bias, random_time_embedder, segments_from_indices, time_embedding,
                    unit_gate)
from .step import AUDIO_TAG, TEXT_TAG, VIDEO_TAG, BlockStack
from .ulysses import local_rows


@dataclass
class H3ModelConfig:
    block: BlockConfig = field(default_factory=BlockConfig)
    blocks: int = 40
    refiner_blocks: int = 2
    patch_dim: int = 96           # latents_dim 24 x patch (1, 2, 2)
    audio_dim: int = 32           # audio_latents_dim
    text_dim: int = 5120          # text_dim
    time_in: int = 256            # timestep_input_dim
    time_hidden: int | None = None    # time_embed_hidden_size (default: hidden)
    time_embed_dim: int | None = None  # time_embed_dim (default: hidden)
    final_eps: float = 1e-6
    rope_sections: tuple = (16, 16, 16)


@dataclass
class RefinerBlockWeights:
    norm1: torch.Tensor
    w_qkv: torch.Tensor
    norm_q: torch.Tensor
    norm_k: torch.Tensor
    w_o: torch.Tensor
    norm2: torch.Tensor
    w_gate_up: torch.Tensor
    w_down: torch.Tensor
    w_gate_up_packed: torch.Tensor | None = field(default=None, repr=False)


@dataclass
class H3ModelWeights:
    proj_in_w: torch.Tensor        # F32 [Hd, patch]
    proj_in_b: torch.Tensor        # F32 [Hd]
    audio_in_w: torch.Tensor       # F32 [Hd, audio]
    audio_in_b: torch.Tensor
    ctx_w: torch.Tensor            # BF16 [Hd, text]
    ctx_b: torch.Tensor            # BF16 [Hd]
    refiner: list
    refiner_norm: torch.Tensor     # BF16 [Hd]
    norm_out: torch.Tensor         # BF16 [Hd]
    norm_out_w: torch.Tensor       # BF16 [2*Hd, temb]  rows [shift | scale]
    norm_out_b: torch.Tensor       # BF16 [2*Hd]
    proj_out_w: torch.Tensor       # F32 [patch, Hd]
    proj_out_b: torch.Tensor
    audio_out_w: torch.Tensor      # F32 [audio, Hd]
    audio_out_b: torch.Tensor


def random_model_weights(cfg: H3ModelConfig, device, seed: int = 0, std: float = 0.02) -> H3ModelWeights:
    g = torch.Generator(device=device)
    g.manual_seed(seed + 99991)
    bc = cfg.block
    hd, f, d = bc.hidden, bc.ffn, bc.head_dim
    temb = cfg.time_embed_dim or hd

    def f32(*shape):
        return torch.randn(*shape, generator=g, device=device) * std

    def b16(*shape):
        return f32(*shape).to(torch.bfloat16)

    def ones(n):
        return torch.ones(n, dtype=torch.bfloat16, device=device)

    refiner = []
    for _ in range(cfg.refiner_blocks):
        r = RefinerBlockWeights(norm1=ones(hd), w_qkv=b16(3 * hd, hd), norm_q=ones(d), norm_k=ones(d),
                                w_o=b16(hd, hd), norm2=ones(hd), w_gate_up=b16(2 * f, hd), w_down=b16(hd, f))
        r.w_gate_up_packed = ops.pack_gate_up(r.w_gate_up)
        refiner.append(r)
    return H3ModelWeights(
        proj_in_w=f32(hd, cfg.patch_dim), proj_in_b=f32(hd), audio_in_w=f32(hd, cfg.audio_dim),
        audio_in_b=f32(hd), ctx_w=b16(hd, cfg.text_dim), ctx_b=b16(hd), refiner=refiner,
        refiner_norm=ones(hd), norm_out=ones(hd), norm_out_w=b16(2 * hd, temb), norm_out_b=b16(2 * hd),
        proj_out_w=f32(cfg.patch_dim, hd), proj_out_b=f32(cfg.patch_dim),
        audio_out_w=f32(cfg.audio_dim, hd), audio_out_b=f32(cfg.audio_dim))


def refiner_block_forward(x: torch.Tensor, w: RefinerBlockWeights, bc: BlockConfig) -> torch.Tensor:
    """MiniMaxH3TokenRefinerBlock::forward (patches/InfiniLM.patch:1210-1216) on
    x [Nt, Hd]; returns a new tensor."""
    nt, hd = x.shape
    h, d = bc.heads, bc.head_dim
    one = unit_gate(hd, x.device)
    n1 = ops.h3_rms_norm(x, w.norm1, bc.eps)
    qkv = ops.linear(n1, w.w_qkv).view(nt, 3, h, d)
    q = ops.h3_rms_norm_(torch.empty(nt, h, d, dtype=x.dtype, device=x.device), qkv[:, 0], w.norm_q, bc.qk_eps)
    k = ops.h3_rms_norm_(torch.empty(nt, h, d, dtype=x.dtype, device=x.device), qkv[:, 1], w.norm_k, bc.qk_eps)
    a = ops.mha(q.unsqueeze(0), k.unsqueeze(0), qkv[:, 2].unsqueeze(0), 1.0 / math.sqrt(d))
    out = ops.linear_gated_residual(a.view(nt, hd), w.w_o, x, one)
    n2 = ops.h3_rms_norm(out, w.norm2, bc.eps)
    hidden = ops.linear_swiglu(n2, w.w_gate_up_packed)
    return ops.linear_gated_residual(hidden, w.w_down, out, one)


class H3Transformer:
    """``forward`` takes the reference's packed-input tensors on this rank's
    device and returns (video [1, Nv, patch] F32, audio [1, Na, audio] F32),
    the full outputs on every rank.  Under sequence parallelism (world > 1, one
    process per GPU) every rank calls ``forward`` with the same inputs."""

    def __init__(self, cfg: H3ModelConfig, device, world: int = 1, rank: int = 0, group=None, seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        bc = cfg.block
        self.world, self.rank, self.group = world, rank, group
        temb_dim = cfg.time_embed_dim or bc.hidden
        self.stack = BlockStack(bc, cfg.blocks, self.device, world, rank, group, seed, temb_dim=temb_dim)
        self.time = random_time_embedder(cfg.time_hidden or bc.hidden, self.device, in_dim=cfg.time_in,
                                         seed=seed + 7, out_dim=temb_dim)
        self.w = random_model_weights(cfg, self.device, seed)
        self.power = ops.rope_powers(cfg.rope_sections, device=self.device)[:cfg.rope_sections[0]].contiguous()

    # -- pieces ---------------------------------------------------------------
    def refine(self, text: torch.Tensor) -> torch.Tensor:
        """context_embedder + token refiner (:1664-1665, :1232-1241): [Nt, text] -> [Nt, Hd]."""
        bc, w = self.cfg.block, self.w
        x = add_bias(ops.linear(text, w.ctx_w), w.ctx_b)
        for blk in w.refiner:
            x = refiner_block_forward(x, blk, bc)
        return ops.h3_rms_norm(x, w.refiner_norm, self.cfg.final_eps)

    def output_norm(self, h: torch.Tensor, temb: torch.Tensor, segments) -> torch.Tensor:
        """MiniMaxH3OutputNorm::forward (:1529-1538): silu(temb) -> bf16 -> linear + bias ->
        per-token [shift | scale] rows -> RMSNorm + modulate."""
        hd = self.cfg.block.hidden
        mod = add_bias(ops.linear(ops.silu(temb, dtype=torch.bfloat16), self.w.norm_out_w), self.w.norm_out_b)
        out = torch.empty_like(h)
        for s in segments:
            r = slice(s.start, s.start + s.length)
            shift = mod[s.row, :hd].unsqueeze(0).expand(s.length, hd)
            scale = mod[s.row, hd:].unsqueeze(0).expand(s.length, hd)
            ops.h3_rms_modulate_(out[r], h[r], self.w.norm_out, scale, shift, self.cfg.final_eps)
        return out

    # -- forward --------------------------------------------------------------
    def forward(self, video: torch.Tensor, audio: torch.Tensor, text: torch.Tensor, timestep: torch.Tensor,
                timestep_indices: torch.Tensor, token_tags: torch.Tensor, position_ids: torch.Tensor,
                video_indices: torch.Tensor, audio_indices: torch.Tensor, text_indices: torch.Tensor):
        cfg, bc, w = self.cfg, self.cfg.block, self.w
        for name, t in (("video", video), ("audio", audio), ("text", text)):
            if t.dim() != 3 or t.shape[0] != 1:
                raise ValueError(f"{name} hidden states must be [1, n, width] (batch 1, as the reference)")
        if position_ids.dim() != 2 or position_ids.shape[1] != 3:
            raise ValueError("position_ids must be [sequence_length, 3]")
        seq = position_ids.shape[0]
        hd = bc.hidden
        video_embeds = ops.linear_f32(video[0], w.proj_in_w, w.proj_in_b, out_dtype=torch.bfloat16)
        audio_embeds = ops.linear_f32(audio[0], w.audio_in_w, w.audio_in_b, out_dtype=torch.bfloat16)
        text_embeds = self.refine(text[0].to(torch.bfloat16))

        local, start, padded = local_rows(seq, self.world, self.rank)
        hidden = torch.zeros(padded, hd, dtype=torch.bfloat16, device=self.device)
        ops.index_copy_rows_(hidden, text_indices, text_embeds)
        ops.index_copy_rows_(hidden, video_indices, video_embeds)
        ops.index_copy_rows_(hidden, audio_indices, audio_embeds)

        temb = time_embedding(timestep, self.time, cfg.time_in)
        # per-token rows of this rank (padded rows reuse row 0, :1706-1710); the index
        # vectors are read on the host once per forward, as the reference does (:1765-1792)
        rows = torch.arange(start, start + local)
        rows = torch.where(rows < seq, rows, torch.zeros_like(rows))
        ts_idx = timestep_indices.cpu()[rows]
        adaln_idx = 3 * ts_idx + token_tags.cpu()[rows]
        table = ops.h3_rope_cache(position_ids.double()[rows.to(position_ids.device)], self.power)
        half = table.shape[1] // 2
        cos, sin = table[:, :half], table[:, half:]

        h = hidden[start:start + local]
        # the modulation rows any token of the sequence reads (the same set on every rank)
        used = sorted(set((3 * timestep_indices.cpu() + token_tags.cpu()).tolist()))
        mods = self.stack.modulations(temb, rows=used)
        h = self.stack.run(h, mods, segments_from_indices(adaln_idx.tolist()), cos, sin, seq)
        normalized = self.output_norm(h, temb, segments_from_indices(ts_idx.tolist()))
        video_all = ops.linear_f32(normalized, w.proj_out_w, w.proj_out_b)
        audio_all = ops.linear_f32(normalized, w.audio_out_w, w.audio_out_b)
        if self.world > 1:
            video_all = self._gather_rows_of_ranks(video_all)[:seq]
            audio_all = self._gather_rows_of_ranks(audio_all)[:seq]
        video_out = ops.gather_rows(video_all, video_indices)
        audio_out = ops.gather_rows(audio_all, audio_indices)
        # a bounded wait that gave up, or an index outside its table, leaves rows
        # incomplete without a launch error: report it before handing results back
        with torch.cuda.device(self.device):
            _lib.check_device("H3Transformer.forward")
        return video_out.unsqueeze(0), audio_out.unsqueeze(0)

    __call__ = forward

    def close(self) -> None:
        """Release the peer-exchange buffers (every rank, after the last forward)."""
        self.stack.close()

    def _gather_rows_of_ranks(self, local: torch.Tensor) -> torch.Tensor:
        """All ranks' [T, C] blocks concatenated in rank (= token) order (:1815-1820)."""
        import torch.distributed as dist
        out = torch.empty((self.world * local.shape[0], local.shape[1]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=self.group)
        return out


def packed_inputs(cfg: H3ModelConfig, video_grid=(4, 8, 8), audio_tokens: int = 16, text_tokens: int = 24,
                  timestep: float = 500.0, seed: int = 0, device="cpu"):
    """Synthetic packed inputs of the reference's layout: text tokens first, then
    video, then audio in the joint sequence; video on its (t, h, w) grid, text
    and audio tokens advancing all three axes together; tags video 0, text 1,
    audio 2 (patches/InfiniLM.patch:137); one timestep."""
    g = torch.Generator().manual_seed(seed)
    t, hh, ww = video_grid
    nv = t * hh * ww
    s = text_tokens + nv + audio_tokens
    video = torch.randn(1, nv, cfg.patch_dim, generator=g)
    audio = torch.randn(1, audio_tokens, cfg.audio_dim, generator=g)
    text = torch.randn(1, text_tokens, cfg.text_dim, generator=g).to(torch.bfloat16)
    text_idx = torch.arange(text_tokens)
    video_idx = torch.arange(text_tokens, text_tokens + nv)
    audio_idx = torch.arange(text_tokens + nv, s)
    tags = torch.empty(s, dtype=torch.long)
    tags[video_idx], tags[text_idx], tags[audio_idx] = VIDEO_TAG, TEXT_TAG, AUDIO_TAG
    tt, yy, xx = torch.meshgrid(torch.arange(t), torch.arange(hh), torch.arange(ww), indexing="ij")
    pos = torch.zeros(s, 3, dtype=torch.float64)
    pos[video_idx] = torch.stack((tt, yy, xx), -1).reshape(-1, 3).double()
    pos[text_idx] = torch.arange(text_tokens).double().unsqueeze(1).expand(-1, 3)
    pos[audio_idx] = torch.arange(audio_tokens).double().unsqueeze(1).expand(-1, 3)
    inputs = dict(video=video, audio=audio, text=text, timestep=torch.tensor([timestep]),
                  timestep_indices=torch.zeros(s, dtype=torch.long), token_tags=tags, position_ids=pos,
                  video_indices=video_idx, audio_indices=audio_idx, text_indices=text_idx)
    return {k: v.to(device) for k, v in inputs.items()}


# ---------------------------------------------------------------------------
# Diffusers-style surface (patches/InfiniLM.patch:6536-6603, 7081-7131): the
# packed-input record, the output record and the adapter module a Diffusers
# pipeline calls in place of its transformer.
# ---------------------------------------------------------------------------
_INDEX_DTYPES = (torch.int32, torch.int64)


@dataclass(frozen=True)
class MiniMaxH3TransformerInputs:
    """Packed FL2VA inputs (MiniMaxH3TransformerInputs, :6536-6586), same checks."""

    video_hidden_states: torch.Tensor
    audio_hidden_states: torch.Tensor
    encoder_hidden_states: torch.Tensor
    timestep: torch.Tensor
    timestep_indices: torch.Tensor
    token_tags: torch.Tensor
    position_ids: torch.Tensor
    video_indices: torch.Tensor
    audio_indices: torch.Tensor
    text_indices: torch.Tensor

    def validate(self) -> None:
        """Reject malformed packed inputs before any device work.  Rules (the
        interface's contract): the positions table is [S, 3] and fixes S; the
        per-token tables (timestep index, modality tag) hold S integers; the three
        row-index vectors are flat integer vectors; timestep is a flat vector;
        every hidden-state input is one [1, tokens, channels] batch.  Shape
        problems raise ValueError, element-type problems TypeError."""
        def shape_of(t):
            return tuple(t.shape)

        def is_index(t):
            return t.dtype in _INDEX_DTYPES

        pos = self.position_ids
        if pos.ndim != 2 or pos.shape[1] != 3:
            raise ValueError(f"position_ids: expected a [S, 3] table, got {shape_of(pos)}")
        if not (pos.is_floating_point() or is_index(pos)):
            raise TypeError(f"position_ids: expected floating-point or integer elements, got {pos.dtype}")
        s = pos.shape[0]
        if self.timestep.ndim != 1:
            raise ValueError(f"timestep: expected a flat vector, got {shape_of(self.timestep)}")
        per_token = {"timestep_indices": self.timestep_indices, "token_tags": self.token_tags}
        row_sets = {"video_indices": self.video_indices, "audio_indices": self.audio_indices,
                    "text_indices": self.text_indices}
        for label, t in per_token.items():
            if shape_of(t) != (s,):
                raise ValueError(f"{label}: expected one entry per token ({s}), got {shape_of(t)}")
        for label, t in row_sets.items():
            if t.ndim != 1:
                raise ValueError(f"{label}: expected a flat vector, got {shape_of(t)}")
        for label, t in {**per_token, **row_sets}.items():
            if not is_index(t):
                raise TypeError(f"{label}: expected int32 or int64 elements, got {t.dtype}")
        streams = {"video_hidden_states": self.video_hidden_states,
                   "audio_hidden_states": self.audio_hidden_states,
                   "encoder_hidden_states": self.encoder_hidden_states}
        for label, t in streams.items():
            if t.ndim != 3 or t.shape[0] != 1:
                raise ValueError(f"{label}: expected one batch [1, tokens, channels], got {shape_of(t)}")


@dataclass(frozen=True)
class MiniMaxH3TransformerOutput:
    """The forward's result: ``sample`` holds the video rows, ``audio_sample`` the
    audio rows (field names of the interface's output record, :6589-6603);
    ``video`` / ``audio`` name the same tensors by modality."""
    sample: torch.Tensor
    audio_sample: torch.Tensor

    video = property(lambda self: self.sample)
    audio = property(lambda self: self.audio_sample)


def run_packed(model: H3Transformer, inputs: MiniMaxH3TransformerInputs) -> MiniMaxH3TransformerOutput:
    """The runner call (MiniMaxH3TransformerRunner.__call__): validate, move the
    inputs to the model's device with int64 indices and fp64 positions (the
    kernels' index and angle types), run the forward."""
    inputs.validate()
    dev = model.device
    idx = lambda t: t.to(dev, torch.int64)  # noqa: E731
    video, audio = model.forward(
        inputs.video_hidden_states.to(dev), inputs.audio_hidden_states.to(dev),
        inputs.encoder_hidden_states.to(dev), inputs.timestep.to(dev, torch.float32),
        idx(inputs.timestep_indices), idx(inputs.token_tags), inputs.position_ids.to(dev, torch.float64),
        idx(inputs.video_indices), idx(inputs.audio_indices), idx(inputs.text_indices))
    return MiniMaxH3TransformerOutput(sample=video, audio_sample=audio)


class MiniMaxH3DiffusersAdapter(torch.nn.Module):
    """Diffusers-style facade (MiniMaxH3DiffusersAdapter, :7081-7131) around an
    ``H3Transformer``: same forward signature, ``return_dict`` behaviour and
    ``dtype`` / ``config`` attributes."""

    def __init__(self, model: H3Transformer, *, dtype: torch.dtype = torch.bfloat16) -> None:
        super().__init__()
        self.model = model
        self._dtype = dtype
        bc = model.cfg.block
        from types import SimpleNamespace
        self.config = SimpleNamespace(
            hidden_size=bc.hidden, num_attention_heads=bc.heads, attention_head_dim=bc.head_dim,
            ffn_hidden_size=bc.ffn, num_layers=model.cfg.blocks, num_refiner_layers=model.cfg.refiner_blocks,
            text_dim=model.cfg.text_dim, audio_latents_dim=model.cfg.audio_dim, patch_dim=model.cfg.patch_dim,
            freq_dim=model.cfg.time_in, norm_eps=bc.eps, qk_norm_eps=bc.qk_eps, final_norm_eps=model.cfg.final_eps)

    @property
    def dtype(self) -> torch.dtype:
        return self._dtype

    def forward(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep, timestep_indices,
                token_tags, position_ids, video_indices, audio_indices, text_indices, attention_kwargs=None,
                return_dict: bool = True):
        del attention_kwargs
        output = run_packed(self.model, MiniMaxH3TransformerInputs(
            video_hidden_states=hidden_states, audio_hidden_states=audio_hidden_states,
            encoder_hidden_states=encoder_hidden_states, timestep=timestep, timestep_indices=timestep_indices,
            token_tags=token_tags, position_ids=position_ids, video_indices=video_indices,
            audio_indices=audio_indices, text_indices=text_indices))
        if return_dict:
            return output
        return output.sample, output.audio_sample
