"""Transactional clipped AdamW, restated in NumPy FP32 (TEST INFRASTRUCTURE ONLY).

Follows src/minifield_training/optimizers/adamw.py:
  CommitCode                 :30-39
  _stable_norm               :355-367
  make_transaction           :384-571 (code precedence :437-461, attempt :476-541,
                                       candidate check :543-569)
and the logical-step normalization of src/minifield_training/engine/step.py:384-395
(valid count, denominator, loss and gradient division).

The state is a dict ``{"params", "m", "v"}`` of name -> float32 arrays plus an
int ``step``; ``trainable`` and ``decayed`` are name sets. Every elementwise
operation is a separate float32 NumPy operation in the reference's order, so a
device kernel that rounds each step (no fused multiply-add) reproduces the
candidate leaves bit for bit given the same clip scale and bias corrections.
"""

import numpy as np

COMMITTED, ACCUMULATION_INVALID, NONFINITE_LOSS, INVALID_STATE = 0, 1, 2, 3
NONFINITE_GRADIENT, STEP_OVERFLOW, CANDIDATE_INVALID = 4, 5, 6
INT32_MAX = 2**31 - 1

F = np.float32


def stable_norm(values):
    """FP32 norm that scales by the largest magnitude first (adamw.py:355-367)."""
    maximum = F(0)
    for value in values:
        a = np.asarray(value, F)
        if a.size:
            maximum = max(maximum, F(np.max(np.abs(a))))
    safe = F(1) if maximum == 0 else maximum
    squared = F(0)
    for value in values:
        scaled = np.asarray(value, F) / safe
        squared = F(squared + F(np.sum(scaled * scaled, dtype=np.float32)))
    return F(maximum * F(np.sqrt(squared)))


def bias_correction(beta, step):
    """1 - beta**t in float32 for t = step + 1 (adamw.py:474-475, :491-492)."""
    t = F(step + 1)
    return F(F(1) - F(np.power(np.float64(F(beta)), np.float64(t))))


def _finite(a):
    return bool(np.all(np.isfinite(np.asarray(a, F))))


def state_valid(state):
    """Masters and moments finite, second moment >= 0, step >= 0 (adamw.py:331-352)."""
    ok = all(_finite(x) for x in state["params"].values()) and all(_finite(x) for x in state["m"].values())
    ok = ok and all(_finite(x) and bool(np.all(np.asarray(x, F) >= 0)) for x in state["v"].values())
    return ok and state["step"] >= 0


def leaf_update(p, g, m, v, clip_scale, cfg, bc1, bc2, decayed):
    """One trainable leaf's candidate (adamw.py:500-534), float32, reference order."""
    p, g, m, v = (np.asarray(x, F) for x in (p, g, m, v))
    b1, b2 = F(cfg["beta1"]), F(cfg["beta2"])
    gradient = g * F(clip_scale)
    first = b1 * m + (F(1) - b1) * gradient
    second = b2 * v + (F(1) - b2) * gradient * gradient
    first_hat = first / F(bc1)
    second_hat = second / F(bc2)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        direction = np.where(first_hat == 0, F(0), first_hat / (np.sqrt(second_hat) + F(cfg["epsilon"])))
        decay = F(cfg["weight_decay"]) * p if decayed else F(0)
        updated = p - F(cfg["learning_rate"]) * (direction + decay)
    return updated.astype(F), first.astype(F), second.astype(F)


def transition(state, grads, loss, accumulation_valid, cfg, trainable, decayed):
    """Commit once or return the incoming state (adamw.py:417-571).

    Returns (new_state, committed, code, loss, gradient_norm, clipped_norm, update_norm).
    """
    loss = F(loss)
    step = int(state["step"])
    code = COMMITTED
    if not state_valid(state):
        code = INVALID_STATE
    elif not accumulation_valid:
        code = ACCUMULATION_INVALID
    elif not np.isfinite(loss):
        code = NONFINITE_LOSS
    elif not all(_finite(grads[n]) for n in trainable):
        code = NONFINITE_GRADIENT
    elif step >= INT32_MAX:
        code = STEP_OVERFLOW
    nan = F(np.nan)
    if code != COMMITTED:
        return state, False, code, loss, nan, nan, nan
    names = sorted(trainable)
    gnorm = stable_norm([grads[n] for n in names])
    clip_scale = F(1) if gnorm == 0 else min(F(1), F(F(cfg["clip_norm"]) / gnorm))
    clipped = F(gnorm * clip_scale)
    bc1, bc2 = bias_correction(cfg["beta1"], step), bias_correction(cfg["beta2"], step)
    new = {k: dict(state[k]) for k in ("params", "m", "v")}
    deltas = []
    for n in names:
        up, first, second = leaf_update(state["params"][n], grads[n], state["m"][n], state["v"][n], clip_scale, cfg,
                                        bc1, bc2, n in decayed)
        new["params"][n], new["m"][n], new["v"][n] = up, first, second
        with np.errstate(over="ignore", invalid="ignore"):
            deltas.append(up - np.asarray(state["params"][n], F))
    with np.errstate(over="ignore", invalid="ignore"):
        unorm = stable_norm(deltas)
    candidate = {**new, "step": step + 1}
    ok = np.isfinite(gnorm) and np.isfinite(unorm) and state_valid(candidate)
    if not ok:
        return state, False, CANDIDATE_INVALID, loss, gnorm, clipped, unorm
    return candidate, True, COMMITTED, loss, gnorm, clipped, unorm


def normalize(loss_sum, count_sum, grad_sums, counts_valid=True):
    """Logical-step normalization (engine/step.py:384-395).

    Returns (loss, gradients, accumulation_valid).
    """
    count_sum = F(count_sum)
    valid = bool(counts_valid) and bool(np.isfinite(count_sum)) and count_sum > 0
    denominator = count_sum if valid else F(1)
    grads = {n: (np.asarray(g, F) / denominator).astype(F) for n, g in grad_sums.items()}
    return F(F(loss_sum) / denominator), grads, valid
