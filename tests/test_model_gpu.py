"""The model wrapper around the block stack: fp32 linears, row gather/scatter,
SiLU (each against torch / the oracle), and the whole transformer forward
(input projections, token refiner, packing, blocks, output norm and
projections) against the CPU oracle's restatement of
MiniMaxH3Transformer::forward (patches/InfiniLM.patch:1626-1826)."""
import pytest
import torch

from oracle import h3_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def h3():
    import h3b200
    h3b200.load()
    return h3b200


@pytest.mark.parametrize("M,K,N,xdt,bias", [(200, 96, 300, torch.float32, True), (1, 256, 512, torch.float32, True),
                                            (333, 5120, 96, torch.bfloat16, True), (64, 32, 130, torch.float32, False),
                                            (1, 5120, 5120, torch.float32, True), (8, 77, 33, torch.bfloat16, False),
                                            (9, 64, 70, torch.float32, True)])
def test_linear_f32(h3, M, K, N, xdt, bias):
    torch.manual_seed(M + K + N)
    x = torch.randn(M, K).to(xdt)
    w = torch.randn(N, K) * 0.05
    b = torch.randn(N) if bias else None
    ref = O.linear_f32(x, w, b)
    out = h3.ops.linear_f32(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV)).cpu()
    tol = 1e-5 * (K ** 0.5) * float(ref.abs().max())
    assert float((out - ref).abs().max()) <= tol
    # BF16 output: the same fp32 result rounded once (cast_to after the F32 linear)
    out16 = h3.ops.linear_f32(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV), out_dtype=torch.bfloat16)
    assert torch.equal(out16.cpu(), out.to(torch.bfloat16))


@pytest.mark.parametrize("dt,C", [(torch.bfloat16, 5120), (torch.bfloat16, 33), (torch.float32, 96), (torch.float32, 7)])
def test_gather_and_index_copy_bit_exact(h3, dt, C):
    torch.manual_seed(C)
    table = torch.randn(50, C).to(dt).to(DEV)
    idx = torch.randint(0, 50, (77,)).to(DEV)
    assert torch.equal(h3.ops.gather_rows(table, idx), table[idx])
    perm = torch.randperm(50)[:30].to(DEV)
    src = torch.randn(30, C).to(dt).to(DEV)
    out = torch.zeros(50, C, dtype=dt, device=DEV)
    ref = out.clone()
    ref[perm] = src
    h3.ops.index_copy_rows_(out, perm, src)
    assert torch.equal(out, ref)
    assert h3.load().h3_device_error() == 0


def test_row_index_out_of_range_is_reported(h3):
    table = torch.arange(40, dtype=torch.float32, device=DEV).view(10, 4)
    out = torch.full((3, 4), -1.0, device=DEV)
    idx = torch.tensor([1, 10, 2], device=DEV)
    h3.ops.gather_rows_(out, table, idx)
    assert h3.load().h3_device_error() == 9          # H3_ERR_INDEX
    assert torch.equal(out[0], table[1]) and torch.equal(out[2], table[2])
    assert bool((out[1] == -1.0).all())              # the bad row is left untouched
    assert h3.load().h3_device_error() == 0          # read-and-clear


def test_silu(h3):
    x = torch.linspace(-30, 30, 10001)
    ref = O.silu(x)
    out = h3.ops.silu(x.to(DEV)).cpu()
    assert torch.allclose(out, ref, rtol=4e-7, atol=1e-30)
    out16 = h3.ops.silu(x.to(DEV), dtype=torch.bfloat16).cpu()
    assert int(O.bf16_ulp_distance(out16, ref.to(torch.bfloat16)).max()) <= 1


def _small_config(h3):
    from h3b200.block import BlockConfig
    from h3b200.model import H3ModelConfig
    bc = BlockConfig(hidden=256, heads=2, head_dim=128, ffn=512)
    return H3ModelConfig(block=bc, blocks=2, refiner_blocks=2, text_dim=256, time_in=256)


def _oracle_weights(model):
    cpu = lambda t: t.detach().cpu()  # noqa: E731
    w = model.w
    weights = {k: cpu(getattr(w, k)) for k in ("proj_in_w", "proj_in_b", "audio_in_w", "audio_in_b", "ctx_w", "ctx_b",
                                               "refiner_norm", "norm_out", "norm_out_w", "norm_out_b", "proj_out_w",
                                               "proj_out_b", "audio_out_w", "audio_out_b")}
    weights["refiner"] = [{k: cpu(getattr(r, k)) for k in ("norm1", "w_qkv", "norm_q", "norm_k", "w_o", "norm2",
                                                           "w_gate_up", "w_down")} for r in w.refiner]
    t = model.time
    weights.update(time_w1=cpu(t.w1), time_b1=cpu(t.b1), time_w2=cpu(t.w2), time_b2=cpu(t.b2))
    blocks = [{k: cpu(getattr(b, k)) for k in ("w_qkv", "norm_q", "norm_k", "w_o", "w_gate_up", "w_down", "norm1",
                                                "norm2", "w_adaln", "b_adaln")} for b in model.stack.weights]
    return weights, blocks


def test_model_forward_matches_oracle(h3):
    from h3b200.model import H3Transformer, packed_inputs
    cfg = _small_config(h3)
    model = H3Transformer(cfg, DEV, seed=3)
    inputs = packed_inputs(cfg, video_grid=(2, 4, 8), audio_tokens=16, text_tokens=24, seed=5)
    video, audio = model(**{k: v.to(DEV) for k, v in inputs.items()})
    assert video.shape == (1, 64, cfg.patch_dim) and audio.shape == (1, 16, cfg.audio_dim)
    assert video.dtype == torch.float32
    weights, blocks = _oracle_weights(model)
    ref_v, ref_a = O.model_forward(inputs, weights, blocks, heads=cfg.block.heads, eps=cfg.block.eps,
                                   qk_eps=cfg.block.qk_eps, final_eps=cfg.final_eps)
    assert O.max_abs_rel(video.cpu(), ref_v) <= 2e-2
    assert O.max_abs_rel(audio.cpu(), ref_a) <= 2e-2
    assert h3.load().h3_device_error() == 0
    # deterministic end to end
    video2, _ = model(**{k: v.to(DEV) for k, v in inputs.items()})
    assert torch.equal(video, video2)


def test_model_refiner_matches_oracle(h3):
    """The token refiner alone, tighter than the whole forward."""
    from h3b200.model import H3Transformer
    cfg = _small_config(h3)
    model = H3Transformer(cfg, DEV, seed=4)
    torch.manual_seed(9)
    text = torch.randn(40, cfg.text_dim).to(torch.bfloat16)
    out = model.refine(text.to(DEV)).cpu()
    weights, _ = _oracle_weights(model)
    x = O.add_bias(O.linear(text, weights["ctx_w"]), weights["ctx_b"])
    for rb in weights["refiner"]:
        x = O.refiner_block_forward(x, rb, cfg.block.heads, cfg.block.eps, cfg.block.qk_eps)
    ref = O.rms_norm(x, weights["refiner_norm"], cfg.final_eps)
    assert O.max_abs_rel(out, ref) <= 1e-2


def test_diffusers_adapter_equals_model_forward(h3):
    """The Diffusers-style facade (int32 indices, integer positions, CPU inputs)
    returns exactly the model forward's outputs, as a record or a tuple."""
    from h3b200.model import H3Transformer, MiniMaxH3DiffusersAdapter, packed_inputs
    cfg = _small_config(h3)
    model = H3Transformer(cfg, DEV, seed=6)
    inputs = packed_inputs(cfg, video_grid=(2, 4, 4), audio_tokens=8, text_tokens=12, seed=1)
    video, audio = model(**{k: v.to(DEV) for k, v in inputs.items()})
    adapter = MiniMaxH3DiffusersAdapter(model)
    kwargs = dict(hidden_states=inputs["video"], audio_hidden_states=inputs["audio"],
                  encoder_hidden_states=inputs["text"], timestep=inputs["timestep"],
                  timestep_indices=inputs["timestep_indices"].int(), token_tags=inputs["token_tags"].int(),
                  position_ids=inputs["position_ids"].long(), video_indices=inputs["video_indices"].int(),
                  audio_indices=inputs["audio_indices"].int(), text_indices=inputs["text_indices"].int())
    out = adapter(**kwargs)
    assert torch.equal(out.sample, video) and torch.equal(out.audio, audio)
    v2, a2 = adapter(**kwargs, return_dict=False)
    assert torch.equal(v2, video) and torch.equal(a2, audio)
    assert adapter.dtype == torch.bfloat16 and adapter.config.hidden_size == cfg.block.hidden


def test_model_forward_other_time_embedding_widths(h3):
    """time_embed_hidden_size and time_embed_dim differ from hidden (the reference's
    defaults are 5376 and 2688 at hidden 5376): the AdaLN and output-norm
    projections read the narrower time embedding."""
    from h3b200.block import BlockConfig
    from h3b200.model import H3ModelConfig, H3Transformer, packed_inputs
    cfg = H3ModelConfig(block=BlockConfig(hidden=256, heads=2, ffn=512), blocks=1, refiner_blocks=1,
                        text_dim=192, time_hidden=384, time_embed_dim=128)
    model = H3Transformer(cfg, DEV, seed=8)
    assert model.stack.weights[0].w_adaln.shape == (18 * 256, 128)
    inputs = packed_inputs(cfg, video_grid=(1, 4, 6), audio_tokens=3, text_tokens=9, seed=4)
    video, audio = model(**{k: v.to(DEV) for k, v in inputs.items()})
    weights, blocks = _oracle_weights(model)
    ref_v, ref_a = O.model_forward(inputs, weights, blocks, heads=2)
    assert O.max_abs_rel(video.cpu(), ref_v) <= 2e-2
    assert O.max_abs_rel(audio.cpu(), ref_a) <= 2e-2
