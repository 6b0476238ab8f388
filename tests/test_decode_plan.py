"""Host-side checks of cached decoding that need no GPU: the parameter tree and state validation."""

import dataclasses

import pytest

from minifield_training_b200.models import decode
from minifield_training_b200.workloads import DECODER
from oracle import decode_model


def test_parameter_tree_matches_the_oracle():
    small = dataclasses.replace(DECODER, hidden=128, ffn=256, heads=4, kv_heads=2, vocab=512,
                                layer_types=("conv", "full_attention", "conv"))
    for cfg in (DECODER, small):
        assert decode.parameter_shapes(cfg) == decode_model.parameter_shapes(cfg)


def test_parameter_tree_names_every_block():
    shapes = decode.parameter_shapes(DECODER)
    n_attn = sum(1 for k in DECODER.layer_types if k == "full_attention")
    n_conv = len(DECODER.layer_types) - n_attn
    assert sum(1 for n in shapes if n.endswith("self_attn.q_proj.weight")) == n_attn
    assert sum(1 for n in shapes if n.endswith("conv.conv.weight")) == n_conv
    assert shapes["model.embed_tokens.weight"] == (DECODER.vocab, DECODER.hidden)


@pytest.mark.parametrize("capacity", [0, -4, 3, 12, 2.0, True])
def test_state_rejects_a_capacity_that_is_not_a_power_of_two(capacity):
    with pytest.raises(ValueError):
        decode.new_state(DECODER, 2, capacity)


@pytest.mark.parametrize("batch", [0, -1, 1.5, False])
def test_state_rejects_a_bad_batch_size(batch):
    with pytest.raises(ValueError):
        decode.new_state(DECODER, batch, 16)


def test_overflow_is_a_value_error():
    assert issubclass(decode.DecodeOverflow, ValueError)
