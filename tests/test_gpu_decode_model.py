"""Cached single-token decoding of the LFM2.5 decoder (models.decode) against oracle/decode_model.py.

A 4-layer decoder (conv, attention, conv, attention; hidden 256, 4/2 heads)
decodes several tokens from a fresh state; every step's FP32 logits must match
the FP64 restatement within the attention tolerance (max-abs 2e-2 of the
output scale, rel-L2 1e-2), and the caches must hold the same K/V rows and
conv history (rel-L2 1e-2; max-abs 5e-2, as they sit several bf16 layers
deep). Writing past the capacity raises DecodeOverflow before any
kernel runs (decode.py:447-451).

Prefill (decode.py:373-416) of ragged prompt lengths (one token, a length
inside the first 128-token tile, one that crosses it, the full capacity)
must give the oracle's last-token logits, K/V cache rows (zero past the
prompt) and conv history, and decode_one must continue from that state.
"""

import dataclasses

import numpy as np
import pytest

from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu


def _cfg():
    from minifield_training_b200 import workloads
    return dataclasses.replace(workloads.DECODER, hidden=256, ffn=512, heads=4, kv_heads=2, vocab=1000,
                               layer_types=("conv", "full_attention", "conv", "full_attention"))


def _close(got, ref, what, tol=2e-2):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    unit = np.maximum(max(1.0, float(np.sqrt(np.mean(ref * ref)))), np.abs(ref))
    err = float(np.max(np.abs(got - ref) / unit))
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    assert err <= tol and rel <= 1e-2, (what, err, rel)


def test_decode_one_matches_the_oracle_over_steps():
    require_gpu()
    from minifield_training_b200.models import decode as dm
    from oracle import decode_model as odm

    cfg = _cfg()
    params = dm.init_parameters(cfg, 0)
    assert set(params) == set(odm.parameter_shapes(cfg))
    dec = dm.Decoder(cfg, params)
    state = dm.new_state(cfg, 4, 64)
    ref_state = odm.new_state(cfg, 4, 64)
    rng = np.random.default_rng(1)
    for step in range(6):
        ids = rng.integers(0, cfg.vocab, 4).astype(np.int32)
        logits = dec.decode_one(ids, state).numpy()
        ref, ref_state = odm.decode_one(cfg, params, ids, ref_state)
        assert logits.shape == (4, cfg.vocab) and logits.dtype == np.float32
        _close(logits, ref, f"logits step {step}")
        assert state.valid_length == ref_state["pos"] == step + 1
    for i, kind in enumerate(cfg.layer_types):
        if kind == "full_attention":
            for got, ref in ((state.keys[i], ref_state["k"][i]), (state.values[i], ref_state["v"][i])):
                # Intermediate state a few bf16 layers deep: a propagated 1-3 ulp flip is allowed.
                _close(got.numpy()[:, :6].astype(np.float32), ref[:, :6], f"cache layer {i}", tol=5e-2)
                assert not got.numpy()[:, 6:].any()
        else:
            _close(state.history[i].numpy().astype(np.float32), ref_state["hist"][i], f"conv history layer {i}",
                   tol=5e-2)


def test_decode_past_capacity_is_rejected():
    require_gpu()
    from minifield_training_b200.models import decode as dm

    cfg = _cfg()
    dec = dm.Decoder(cfg, dm.init_parameters(cfg, 0))
    state = dm.new_state(cfg, 2, 2)
    for _ in range(2):
        dec.decode_one(np.array([1, 2], np.int32), state)
    with pytest.raises(dm.DecodeOverflow):
        dec.decode_one(np.array([1, 2], np.int32), state)
    with pytest.raises(ValueError):
        dm.new_state(cfg, 2, 3)
    with pytest.raises(ValueError):
        dec.decode_one(np.array([1, 2, 3], np.int32), dm.new_state(cfg, 2, 4))


@pytest.mark.parametrize("t", [1, 37, 130, 256])
def test_prefill_then_decode_matches_the_oracle(t):
    require_gpu()
    from minifield_training_b200.models import decode as dm
    from oracle import decode_model as odm

    cfg, b, cap = _cfg(), 3, 256
    params = dm.init_parameters(cfg, 2)
    dec = dm.Decoder(cfg, params)
    rng = np.random.default_rng(t)
    prompt = rng.integers(0, cfg.vocab, (b, t)).astype(np.int32)
    state = dm.new_state(cfg, b, cap)
    logits, same = dm.prefill(dec, prompt, state)
    ref, ref_state = odm.prefill(cfg, params, prompt, cap)
    assert same is state and state.valid_length == t
    assert logits.shape == (b, cfg.vocab) and logits.dtype == "float32"
    _close(logits.numpy(), ref, f"prefill logits T={t}")
    for i, kind in enumerate(cfg.layer_types):
        if kind == "full_attention":
            for got, want in ((state.keys[i], ref_state["k"][i]), (state.values[i], ref_state["v"][i])):
                g = got.numpy()
                _close(g[:, :t].astype(np.float32), want[:, :t], f"prefill cache layer {i}", tol=5e-2)
                assert not g[:, t:].any()
        else:
            h = state.history[i].numpy().astype(np.float32)
            _close(h, ref_state["hist"][i], f"prefill conv history layer {i}", tol=5e-2)
            if t == 1:
                assert not h[:, 0].any()
    for step in range(3 if t < cap else 0):
        ids = rng.integers(0, cfg.vocab, b).astype(np.int32)
        got = dec.decode_one(ids, state).numpy()
        ref, ref_state = odm.decode_one(cfg, params, ids, ref_state)
        _close(got, ref, f"decode after prefill T={t} step {step}")
    if t == cap:
        with pytest.raises(dm.DecodeOverflow):
            dec.decode_one(np.zeros(b, np.int32), state)


def test_prefill_rejects_what_the_reference_rejects():
    require_gpu()
    from minifield_training_b200.models import decode as dm

    cfg = _cfg()
    dec = dm.Decoder(cfg, dm.init_parameters(cfg, 0))
    with pytest.raises(ValueError):  # longer than the capacity
        dec.prefill(np.zeros((2, 9), np.int32), dm.new_state(cfg, 2, 8))
    with pytest.raises(ValueError):  # batch mismatch
        dec.prefill(np.zeros((3, 4), np.int32), dm.new_state(cfg, 2, 8))
    with pytest.raises(ValueError):  # not [batch, tokens]
        dec.prefill(np.zeros(4, np.int32), dm.new_state(cfg, 2, 8))
    state = dm.new_state(cfg, 2, 8)
    dec.prefill(np.ones((2, 3), np.int32), state)
    with pytest.raises(ValueError):  # not a fresh state
        dec.prefill(np.ones((2, 3), np.int32), state)


def test_graph_replayed_decode_equals_the_eager_step():
    """decode_one(graph=True) replays one captured step for every position; logits match the eager path."""
    require_gpu()
    from minifield_training_b200 import _lib
    from minifield_training_b200.device import DeviceArray
    from minifield_training_b200.models import decode as dm
    import ctypes

    cfg = _cfg()
    params = dm.init_parameters(cfg, 4)
    stream = ctypes.c_void_p()
    _lib.call("mfb_stream_create", ctypes.byref(stream))
    try:
        eager, graphed = dm.Decoder(cfg, params), dm.Decoder(cfg, params, stream=stream.value)
        se, sg = dm.new_state(cfg, 4, 16), dm.new_state(cfg, 4, 16)
        prompt = np.random.default_rng(5).integers(0, cfg.vocab, (4, 5)).astype(np.int32)
        eager.prefill(prompt, se)
        graphed.prefill(prompt, sg)
        out = DeviceArray((4, cfg.vocab), "float32")
        rng = np.random.default_rng(6)
        for _ in range(4):
            ids = rng.integers(0, cfg.vocab, 4).astype(np.int32)
            want = eager.decode_one(ids, se).numpy()
            got = graphed.decode_one(ids, sg, out=out, graph=True)
            assert got is out
            _lib.call("mfb_stream_sync", stream)
            np.testing.assert_array_equal(got.numpy(), want)
        assert len(graphed._graphs) == 1
        graphed.close()
    finally:
        _lib.call("mfb_stream_sync", stream)
        _lib.call("mfb_stream_destroy", stream)
