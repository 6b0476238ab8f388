"""Pins oracle/adamw.py to the reference's AdamW and data-parallel known answers.

Fixtures are transcribed from tests/optimizers/test_adamw.py:17-134 (inventory,
parameters, gradients, moments, and the float64 oracle update :75-111) and
tests/engine/data_parallel_cases.py:40-130 (scalar affine model over 8
replicas: loss 41, m 3.5, v 61.25, weight 1.9). CPU only.
"""

import math

import numpy as np
import pytest

from oracle import adamw as oa

F = np.float32


def _params():
    return {"w.matrix": np.array([[0.5, -0.25, 0.125], [1.0, -0.5, 0.75]], F),
            "w.vector": np.array([0.25, -0.5, 1.5], F),
            "w.frozen_matrix": np.array([[1.0, 2.0], [3.0, 4.0]], F),
            "w.frozen_vector": np.array([5.0, 6.0, 7.0, 8.0], F)}


def _grads():
    return {"w.matrix": np.array([[0.1, 0.2, -0.1], [0.05, -0.2, 0.3]], F),
            "w.vector": np.array([-0.4, 0.1, 0.2], F)}


def _state():
    p = _params()
    m = {"w.matrix": np.array([[0.01, 0.0, -0.01], [0.02, 0.0, 0.01]], F),
         "w.vector": np.array([0.05, -0.05, 0.0], F),
         "w.frozen_matrix": np.zeros((2, 2), F), "w.frozen_vector": np.zeros(4, F)}
    v = {"w.matrix": np.array([[0.001, 0.002, 0.001], [0.0, 0.004, 0.002]], F),
         "w.vector": np.array([0.01, 0.0, 0.03], F),
         "w.frozen_matrix": np.zeros((2, 2), F), "w.frozen_vector": np.zeros(4, F)}
    return {"params": p, "m": m, "v": v, "step": 0}


TRAINABLE = {"w.matrix", "w.vector"}
DECAYED = {"w.matrix"}


def _cfg(**kw):
    c = dict(learning_rate=0.1, beta1=0.9, beta2=0.95, epsilon=1e-8, weight_decay=0.01, clip_norm=1.0)
    c.update(kw)
    return c


def _run(state=None, grads=None, loss=1.0, valid=True, **kw):
    return oa.transition(state or _state(), grads or _grads(), loss, valid, _cfg(**kw), TRAINABLE, DECAYED)


def _fp64_oracle(p, g, m, v, clip_scale, cfg, it, decayed):
    """tests/optimizers/test_adamw.py:75-111."""
    g = np.asarray(g, np.float64) * clip_scale
    m = cfg["beta1"] * np.asarray(m, np.float64) + (1 - cfg["beta1"]) * g
    v = cfg["beta2"] * np.asarray(v, np.float64) + (1 - cfg["beta2"]) * g * g
    mh, vh = m / (1 - cfg["beta1"] ** it), v / (1 - cfg["beta2"] ** it)
    d = np.where(mh == 0, 0.0, mh / (np.sqrt(vh) + cfg["epsilon"]))
    decay = cfg["weight_decay"] * np.asarray(p, np.float64) if decayed else 0.0
    return np.asarray(p, np.float64) - cfg["learning_rate"] * (d + decay), m, v


def test_commit_matches_the_reference_fp64_oracle():
    cfg = _cfg(clip_norm=10.0)
    new, committed, code, _, gnorm, clipped, unorm = _run(clip_norm=10.0)
    assert committed and code == oa.COMMITTED and new["step"] == 1
    ref_norm = math.sqrt(sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in _grads().values()))
    scale = min(1.0, cfg["clip_norm"] / ref_norm)
    np.testing.assert_allclose(gnorm, ref_norm, rtol=1e-5)
    np.testing.assert_allclose(clipped, ref_norm * scale, rtol=1e-5)
    deltas = []
    for name in ("w.matrix", "w.vector"):
        up, m, v = _fp64_oracle(_params()[name], _grads()[name], _state()["m"][name], _state()["v"][name], scale, cfg,
                                1, name in DECAYED)
        np.testing.assert_allclose(new["params"][name], up, rtol=1e-5)
        np.testing.assert_allclose(new["m"][name], m, rtol=1e-5)
        np.testing.assert_allclose(new["v"][name], v, rtol=1e-5)
        deltas.append(up - np.asarray(_params()[name], np.float64))
    np.testing.assert_allclose(unorm, math.sqrt(sum(float(np.sum(d ** 2)) for d in deltas)), rtol=1e-5)


def test_frozen_leaves_are_bit_identical():
    new = _run()[0]
    for name in ("w.frozen_matrix", "w.frozen_vector"):
        for group in ("params", "m", "v"):
            np.testing.assert_array_equal(new[group][name], _state()[group][name])


def test_clipping_reaches_the_declared_norm():
    grads = {k: v * F(100) for k, v in _grads().items()}
    res = _run(grads=grads, clip_norm=0.05)
    assert res[1]
    np.testing.assert_allclose(res[5], 0.05, rtol=1e-5)


@pytest.mark.parametrize("case,code", [("grad", oa.NONFINITE_GRADIENT), ("loss", oa.NONFINITE_LOSS),
                                       ("acc", oa.ACCUMULATION_INVALID), ("m_inf", oa.INVALID_STATE),
                                       ("v_neg", oa.INVALID_STATE), ("step", oa.STEP_OVERFLOW)])
def test_rejections_keep_the_state(case, code):
    state, grads, loss, valid = _state(), _grads(), 1.0, True
    if case == "grad":
        grads["w.vector"] = np.array([np.nan, 0, 0], F)
    elif case == "loss":
        loss = np.nan
    elif case == "acc":
        valid = False
    elif case == "m_inf":
        state["m"]["w.vector"] = np.array([np.inf, 0, 0], F)
    elif case == "v_neg":
        state["v"]["w.vector"] = np.array([-1.0, 0, 0], F)
    elif case == "step":
        state["step"] = 2**31 - 1
    new, committed, got, *_ = oa.transition(state, grads, loss, valid, _cfg(), TRAINABLE, DECAYED)
    assert not committed and got == code and new is state


@pytest.mark.parametrize("variance,valid", [(0.25, True), (0.0, True), (-0.0, True), (-0.25, False),
                                            (np.nan, False), (np.inf, False), (-np.inf, False)])
def test_second_moment_validation_accepts_signed_zero(variance, valid):
    state = _state()
    state["v"]["w.vector"] = np.array([variance, 0.0, 0.03], F)
    assert oa.state_valid(state) is valid
    assert _run(state=state)[1] is valid


def test_overflowing_candidate_is_rejected():
    state = _state()
    state["params"]["w.matrix"] = np.full((2, 3), 1e38, F)
    grads = {"w.matrix": np.zeros((2, 3), F), "w.vector": np.zeros(3, F)}
    new, committed, code, *_ = _run(state=state, grads=grads, learning_rate=1.0, weight_decay=4.0, clip_norm=1e30)
    assert code == oa.CANDIDATE_INVALID and not committed
    np.testing.assert_array_equal(new["params"]["w.matrix"], state["params"]["w.matrix"])


def test_zero_gradient_applies_decay_only():
    state = {"params": _params(), "m": {k: np.zeros_like(v) for k, v in _params().items()},
             "v": {k: np.zeros_like(v) for k, v in _params().items()}, "step": 0}
    grads = {"w.matrix": np.zeros((2, 3), F), "w.vector": np.zeros(3, F)}
    new = _run(state=state, grads=grads, weight_decay=0.5)[0]
    np.testing.assert_allclose(new["params"]["w.matrix"], _params()["w.matrix"] * (1 - 0.1 * 0.5), rtol=1e-6)
    np.testing.assert_array_equal(new["params"]["w.vector"], _params()["w.vector"])


def test_eight_replica_data_parallel_step():
    """data_parallel_cases.py:40-130: residuals 3,5,7,9 -> loss 41, m 3.5, v 61.25, w 1.9."""
    values = np.zeros((3, 16), F)
    masks = np.zeros_like(values)
    values[0, 0], values[0, 2] = 1, 2
    values[1, 0], values[1, 1] = 3, 4
    masks[0, (0, 2)] = 1
    masks[1, :2] = 1
    w, b = F(2), F(1)
    loss_sum = count_sum = grad_sum = F(0)
    for slot in range(2):  # the third slot is inactive and never evaluated
        for replica in range(8):  # rows split over the 8-way data mesh
            x, mk = values[slot, 2 * replica:2 * replica + 2], masks[slot, 2 * replica:2 * replica + 2]
            r = w * x + b
            loss_sum += F(np.sum(mk * r * r))
            count_sum += F(np.sum(mk))
            grad_sum += F(np.sum(mk * 2 * r * x))
    loss, grads, valid = oa.normalize(loss_sum, count_sum, {"weight": np.array(grad_sum, F)})
    state = {"params": {"weight": np.array(w, F), "bias": np.array(b, F)},
             "m": {"weight": np.array(0, F), "bias": np.array(0, F)},
             "v": {"weight": np.array(0, F), "bias": np.array(0, F)}, "step": 0}
    new, committed, code, got_loss, *_ = oa.transition(state, grads, loss, valid, _cfg(clip_norm=100), {"weight"},
                                                       set())
    assert committed and new["step"] == 1
    np.testing.assert_allclose(got_loss, 41, rtol=1e-6)
    np.testing.assert_allclose(new["m"]["weight"], 3.5, rtol=1e-6)
    np.testing.assert_allclose(new["v"]["weight"], 61.25, rtol=1e-6)
    np.testing.assert_allclose(new["params"]["weight"], 1.9, rtol=1e-6)
    assert new["params"]["bias"] == 1 and new["m"]["bias"] == 0 and new["v"]["bias"] == 0


_CONFIG_REJECTIONS = [
    # The reference's own cases (tests/optimizers/test_adamw.py:481-496) ...
    ({"learning_rate": 0.0}, "learning_rate must be positive"),
    ({"learning_rate": 0.1, "beta1": 1.0}, "beta1 must be in [0, 1)"),
    ({"learning_rate": 0.1, "epsilon": 0.0}, "epsilon must be positive"),
    ({"learning_rate": 0.1, "weight_decay": -0.1}, "weight_decay must be nonnegative"),
    ({"learning_rate": 0.1, "clip_norm": 0.0}, "clip_norm must be positive"),
    ({"learning_rate": float("nan")}, "learning_rate must be a finite float32 scalar"),
    ({"learning_rate": True}, "learning_rate must be a non-boolean finite number"),
    # ... and the remaining branches of its validation (optimizers/adamw.py:53-93).
    ({"learning_rate": "0.1"}, "learning_rate must be a non-boolean finite number"),
    ({"learning_rate": 1e39}, "learning_rate must be a finite float32 scalar"),
    ({"learning_rate": float("inf")}, "learning_rate must be a finite float32 scalar"),
    ({"learning_rate": 1e-50}, "learning_rate must be representable in float32"),
    ({"learning_rate": 1e-40}, "learning_rate must be zero or a normal float32 scalar"),
    ({"learning_rate": 0.1, "beta2": -0.5}, "beta2 must be in [0, 1)"),
    ({"learning_rate": 0.1, "beta2": 1.0}, "beta2 must be in [0, 1)"),
    ({"learning_rate": -1.0, "clip_norm": False}, "clip_norm must be a non-boolean finite number"),
    ({"learning_rate": 0.1, "beta1": 1.5, "epsilon": float("nan")}, "epsilon must be a finite float32 scalar"),
    ({"learning_rate": -1.0, "beta1": 2.0}, "learning_rate must be positive"),
    ({"learning_rate": 0.1, "beta1": 0.99999999999}, "beta1 must be in [0, 1)"),
]


@pytest.mark.parametrize("kwargs,message", _CONFIG_REJECTIONS)
def test_adamw_config_rejects_with_the_reference_messages(kwargs, message):
    """Each bad setting raises the reference's exact ValueError text; scalar problems of any
    field come before range problems, and fields are checked in declaration order."""
    from minifield_training_b200.optimizers.adamw import AdamWConfig

    with pytest.raises(ValueError) as err:
        AdamWConfig(**kwargs)
    assert str(err.value) == message


def test_adamw_config_stores_float32_values():
    from minifield_training_b200.optimizers.adamw import AdamWConfig

    c = AdamWConfig(learning_rate=3e-4, beta2=0.95, weight_decay=0, epsilon=1e-8, clip_norm=1)
    for name in ("learning_rate", "beta1", "beta2", "epsilon", "weight_decay", "clip_norm"):
        value = getattr(c, name)
        assert isinstance(value, float) and value == float(np.float32(value)), name
    assert c.learning_rate == float(np.float32(3e-4)) and c.weight_decay == 0.0
