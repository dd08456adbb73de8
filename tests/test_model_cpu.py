"""Host-side checks of the model wrapper's Diffusers-style surface (no GPU):
the packed-input validation mirrors MiniMaxH3TransformerInputs.validate
(patches/InfiniLM.patch:6550-6586) and the synthetic packing is consistent."""
import dataclasses

import pytest
import torch


def _cfg():
    from h3b200.block import BlockConfig
    from h3b200.model import H3ModelConfig
    return H3ModelConfig(block=BlockConfig(hidden=256, heads=2, ffn=512), blocks=1, text_dim=256)


def _inputs():
    from h3b200.model import MiniMaxH3TransformerInputs, packed_inputs
    d = packed_inputs(_cfg(), video_grid=(2, 3, 4), audio_tokens=5, text_tokens=7)
    return MiniMaxH3TransformerInputs(video_hidden_states=d["video"], audio_hidden_states=d["audio"],
                                      encoder_hidden_states=d["text"], timestep=d["timestep"],
                                      timestep_indices=d["timestep_indices"], token_tags=d["token_tags"],
                                      position_ids=d["position_ids"], video_indices=d["video_indices"],
                                      audio_indices=d["audio_indices"], text_indices=d["text_indices"])


def test_packed_inputs_are_a_permutation_with_reference_tags():
    inp = _inputs()
    inp.validate()
    s = inp.position_ids.shape[0]
    allidx = torch.cat([inp.text_indices, inp.video_indices, inp.audio_indices]).sort().values
    assert torch.equal(allidx, torch.arange(s))
    assert bool((inp.token_tags[inp.video_indices] == 0).all())
    assert bool((inp.token_tags[inp.text_indices] == 1).all())
    assert bool((inp.token_tags[inp.audio_indices] == 2).all())


@pytest.mark.parametrize("field,value,exc", [
    ("position_ids", torch.zeros(36, 2), ValueError),
    ("timestep", torch.zeros(1, 1), ValueError),
    ("token_tags", torch.zeros(35, dtype=torch.long), ValueError),
    ("timestep_indices", torch.zeros(36), TypeError),
    ("video_indices", torch.zeros(2, 3, dtype=torch.long), ValueError),
    ("audio_indices", torch.zeros(5), TypeError),
    ("encoder_hidden_states", torch.zeros(2, 7, 256), ValueError),
    ("position_ids", torch.zeros(36, 3, dtype=torch.bool), TypeError),
])
def test_validation_matches_reference_checks(field, value, exc):
    bad = dataclasses.replace(_inputs(), **{field: value})
    with pytest.raises(exc):
        bad.validate()
