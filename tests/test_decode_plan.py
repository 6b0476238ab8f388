"""Host-side checks of cached decoding that need no GPU: the parameter tree and state validation."""

import dataclasses

import numpy as np
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


def _tiny():
    return dataclasses.replace(DECODER, hidden=128, ffn=256, heads=4, kv_heads=2, vocab=512,
                               layer_types=("conv", "full_attention", "conv"))


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_oracle_prefill_then_cached_steps_equal_the_uninterrupted_prompt():
    """The reference's prefix/cached-step property (tests/layers/test_blocks.py:223-340) at model level."""
    cfg = _tiny()
    params = decode.init_parameters(cfg, 3)
    ids = np.random.default_rng(4).integers(0, cfg.vocab, (2, 6)).astype(np.int32)
    logits, state = decode_model.prefill(cfg, params, ids[:, :3], 8)
    assert state["pos"] == 3
    for t in range(3, 6):
        full, full_state = decode_model.prefill(cfg, params, ids[:, :t], 8)
        assert _rel(logits, full) < 1e-2, t
        for i, kind in enumerate(cfg.layer_types):
            if kind == "conv":
                assert _rel(state["hist"][i], full_state["hist"][i]) < 1e-2
            else:
                assert _rel(state["k"][i], full_state["k"][i]) < 1e-2
                assert not full_state["k"][i][:, t:].any() and not full_state["v"][i][:, t:].any()
        logits, state = decode_model.decode_one(cfg, params, ids[:, t], state)


def test_oracle_one_token_prefill_history_starts_with_zeros():
    cfg = _tiny()
    params = decode.init_parameters(cfg, 5)
    _, state = decode_model.prefill(cfg, params, np.array([[7], [9]], np.int32), 4)
    for i, kind in enumerate(cfg.layer_types):
        if kind == "conv":
            assert not state["hist"][i][:, 0].any() and state["hist"][i][:, 1].any()


def test_oracle_prefill_rejects_a_prompt_longer_than_the_capacity():
    cfg = _tiny()
    with pytest.raises(ValueError):
        decode_model.prefill(cfg, decode.init_parameters(cfg, 0), np.zeros((1, 5), np.int32), 4)
