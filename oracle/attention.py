"""Masked GQA attention forward/backward restated in NumPy (test infrastructure).

Follows the reference's dense attention and mask builders:

* ``_dense_attention``            src/minifield_training/kernels/attention.py:12-34
* ``dense_causal_attention``      kernels/attention.py:206-222
* ``_prefix_valid_mask`` / prefix kernels/attention.py:37-76, 225-242
* ``_packed_valid_mask`` / packed kernels/attention.py:79-108, 245-261
* ``dense_cached_attention``      kernels/attention.py:264-282
* ``bidirectional.attention``     src/minifield_training/kernels/bidirectional.py:7-35
  (which calls ``jax.nn.dot_product_attention(implementation="xla")``;
  the documented semantics restated here: logits in FP32, scale D^-0.5,
  query head h reads KV head h // (H/Hk), masked logits set to
  -0.7 * finfo(f32).max, FP32 softmax).

The backward is the analytic gradient of those graphs (the reference obtains
it by JAX autodiff): masked logits receive no gradient because the mask is a
``where`` select; a row whose every key is masked is a uniform average over
all keys under the dense ``finfo.min`` fill (so dV receives dO / S there),
and is zeroed under the bidirectional / packed policies.

Mask encoding shared with the CUDA kernels: every query row t has an id
``qid[b, t]`` and every key s an id ``kid[b, s]``; the pair is valid iff
``qid != 0 and qid == kid and (not causal or s <= t + offset)``.  The
``*_ids`` builders map each reference mask shape onto that encoding, and the
``reference_*_valid`` functions restate the reference's own mask formulas so
tests can prove the encodings identical element by element.
"""

import numpy as np

F32_MIN = float(np.finfo(np.float32).min)
# jax.nn.dot_product_attention's masked-logit fill: -0.7 * finfo(f32).max.
JAX_LARGE_NEGATIVE = float(np.float32(-0.7 * np.finfo(np.float32).max))

POLICY_UNIFORM = "uniform"  # empty row -> uniform average over all keys
POLICY_ZERO = "zero"  # empty row -> zero output


# ---------------------------------------------------------------------------
# Reference mask formulas (restated literally for cross-checking).
# ---------------------------------------------------------------------------


def reference_causal_valid(attention_mask: np.ndarray) -> np.ndarray:
    """kernels/attention.py:219-221 -> bool [B, T, S]."""
    t = attention_mask.shape[1]
    positions = np.arange(t)
    valid = (positions[:, None] >= positions[None, :])[None, :, :]
    return valid & (attention_mask[:, None, :] != 0)


def reference_prefix_valid(prefix_mask: np.ndarray, suffix_mask: np.ndarray) -> np.ndarray:
    """kernels/attention.py:61-76 -> bool [B, T, P + T]."""
    batch, t = suffix_mask.shape
    positions = np.arange(t)
    causal = (positions[:, None] >= positions[None, :])[None, :, :]
    suffix_valid = causal & (suffix_mask[:, None, :] != 0)
    prefix_valid = np.broadcast_to(
        (prefix_mask[:, None, :] != 0), (batch, t, prefix_mask.shape[1])
    )
    return np.concatenate((prefix_valid, suffix_valid), axis=-1)


def reference_packed_valid(attention_mask: np.ndarray, segment_ids: np.ndarray):
    """kernels/attention.py:79-108 -> (valid bool [B, T, T], active [B, T])."""
    t = segment_ids.shape[1]
    positions = np.arange(t)
    causal = (positions[:, None] >= positions[None, :])[None, :, :]
    active = (attention_mask > 0) & (segment_ids != 0)
    same = segment_ids[:, :, None] == segment_ids[:, None, :]
    valid = causal & same & (segment_ids[:, :, None] != 0) & active[:, None, :] & active[:, :, None]
    self_only = positions[:, None] == positions[None, :]
    valid = valid | ((~active)[:, :, None] & self_only[None, :, :])
    return valid, active


def reference_bidirectional_valid(mask: np.ndarray, segment_ids=None):
    """kernels/bidirectional.py:21-31 -> (valid [B, T, S], present [B, T])."""
    mask = mask.astype(bool)
    if segment_ids is None:
        t = mask.shape[1]
        valid = np.broadcast_to(mask[:, None, :], (mask.shape[0], t, t))
        present = np.broadcast_to(np.any(mask, axis=-1)[:, None], mask.shape)
        return valid, present
    active = mask & (segment_ids != 0)
    valid = (segment_ids[:, :, None] == segment_ids[:, None, :]) & active[:, :, None] & active[:, None, :]
    return valid, active


def reference_cached_valid(valid_length, batch: int, capacity: int) -> np.ndarray:
    """kernels/attention.py:280-281 -> bool [B, 1, S] (valid_length scalar or [B])."""
    lengths = np.broadcast_to(np.asarray(valid_length, np.int64).reshape(-1), (batch,))
    positions = np.arange(capacity)
    return (positions[None, None, :] < lengths[:, None, None])


# ---------------------------------------------------------------------------
# The (qid, kid, causal, offset, policy) encoding used by the CUDA kernels.
# ---------------------------------------------------------------------------


def causal_ids(attention_mask: np.ndarray):
    b, t = attention_mask.shape
    qid = np.ones((b, t), np.int32)
    kid = (attention_mask != 0).astype(np.int32)
    return qid, kid, True, 0, POLICY_UNIFORM


def prefix_ids(prefix_mask: np.ndarray, suffix_mask: np.ndarray):
    b, t = suffix_mask.shape
    qid = np.ones((b, t), np.int32)
    kid = np.concatenate((prefix_mask != 0, suffix_mask != 0), axis=1).astype(np.int32)
    return qid, kid, True, prefix_mask.shape[1], POLICY_UNIFORM


def packed_ids(attention_mask: np.ndarray, segment_ids: np.ndarray):
    active = (attention_mask > 0) & (segment_ids != 0)
    ids = np.where(active, segment_ids, 0).astype(np.int32)
    return ids, ids.copy(), True, 0, POLICY_ZERO


def bidirectional_ids(mask: np.ndarray, segment_ids=None):
    b, t = mask.shape
    if segment_ids is None:
        kid = (mask != 0).astype(np.int32)
        return np.ones((b, t), np.int32), kid, False, 0, POLICY_ZERO
    active = (mask != 0) & (segment_ids != 0)
    ids = np.where(active, segment_ids, 0).astype(np.int32)
    return ids, ids.copy(), False, 0, POLICY_ZERO


def cached_ids(valid_length, batch: int, capacity: int):
    lengths = np.broadcast_to(np.asarray(valid_length, np.int64).reshape(-1), (batch,))
    kid = (np.arange(capacity)[None, :] < lengths[:, None]).astype(np.int32)
    return np.ones((batch, 1), np.int32), kid, False, 0, POLICY_UNIFORM


def valid_from_ids(qid: np.ndarray, kid: np.ndarray, causal: bool, offset: int) -> np.ndarray:
    """bool [B, T, S] validity of the shared id encoding."""
    valid = (qid[:, :, None] != 0) & (qid[:, :, None] == kid[:, None, :])
    if causal:
        t, s = qid.shape[1], kid.shape[1]
        valid &= np.arange(s)[None, None, :] <= (np.arange(t)[None, :, None] + offset)
    return valid


# ---------------------------------------------------------------------------
# Forward / backward.
# ---------------------------------------------------------------------------


def _probabilities(q, k, valid, policy, dtype):
    """Per-batch-element probabilities [H, T, S] and the row-present flags [T]."""
    h, hk = q.shape[1], k.shape[1]
    group = h // hk
    d = q.shape[-1]
    qh = np.ascontiguousarray(q.transpose(1, 0, 2), dtype=dtype)  # [H, T, D]
    kh = np.ascontiguousarray(np.repeat(k, group, axis=1).transpose(1, 2, 0), dtype=dtype)  # [H, D, S]
    scores = np.matmul(qh, kh) * dtype(d ** -0.5)
    fill = F32_MIN if policy == POLICY_UNIFORM else JAX_LARGE_NEGATIVE
    scores = np.where(valid[None, :, :], scores, dtype(fill))
    scores -= scores.max(axis=-1, keepdims=True)
    np.exp(scores, out=scores)
    scores /= scores.sum(axis=-1, keepdims=True)
    present = valid.any(axis=-1)
    return scores, present


def attention_forward(q, k, v, valid, policy, dtype=np.float64):
    """O [B, T, H, D] for q [B,T,H,D], k/v [B,S,Hk,D], valid bool [B,T,S]."""
    b, t, h, d = q.shape
    hk = k.shape[2]
    group = h // hk
    out = np.empty((b, t, h, d), dtype)
    for i in range(b):
        p, present = _probabilities(q[i], k[i], valid[i], policy, dtype)
        vh = np.ascontiguousarray(np.repeat(v[i], group, axis=1).transpose(1, 0, 2), dtype=dtype)
        o = np.matmul(p, vh).transpose(1, 0, 2)  # [T, H, D]
        if policy == POLICY_ZERO:
            o = np.where(present[:, None, None], o, 0)
        out[i] = o
    return out


def attention_backward(q, k, v, valid, policy, d_out, dtype=np.float64):
    """(dq, dk, dv) of sum(O * d_out) for the forward above."""
    b, t, h, d = q.shape
    s, hk = k.shape[1], k.shape[2]
    group = h // hk
    scale = dtype(d ** -0.5)
    dq = np.empty(q.shape, dtype)
    dk = np.empty(k.shape, dtype)
    dv = np.empty(v.shape, dtype)
    for i in range(b):
        p, present = _probabilities(q[i], k[i], valid[i], policy, dtype)  # [H,T,S]
        do = np.ascontiguousarray(d_out[i].transpose(1, 0, 2), dtype=dtype)  # [H,T,D]
        if policy == POLICY_ZERO:
            do = np.where(present[None, :, None], do, 0)
        vh = np.ascontiguousarray(np.repeat(v[i], group, axis=1).transpose(1, 0, 2), dtype=dtype)
        kh = np.ascontiguousarray(np.repeat(k[i], group, axis=1).transpose(1, 0, 2), dtype=dtype)
        qh = np.ascontiguousarray(q[i].transpose(1, 0, 2), dtype=dtype)
        dv_h = np.matmul(p.transpose(0, 2, 1), do)  # [H,S,D]
        dp = np.matmul(do, vh.transpose(0, 2, 1))  # [H,T,S]
        ds = p * (dp - (p * dp).sum(axis=-1, keepdims=True))
        ds = np.where(valid[i][None, :, :], ds, 0)
        dq_h = np.matmul(ds, kh) * scale  # [H,T,D]
        dk_h = np.matmul(ds.transpose(0, 2, 1), qh) * scale  # [H,S,D]
        dq[i] = dq_h.transpose(1, 0, 2)
        dk[i] = dk_h.reshape(hk, group, s, d).sum(axis=1).transpose(1, 0, 2)
        dv[i] = dv_h.reshape(hk, group, s, d).sum(axis=1).transpose(1, 0, 2)
    return dq, dk, dv


# ---------------------------------------------------------------------------
# Reference-named entry points.
# ---------------------------------------------------------------------------


def _run(q, k, v, ids, dtype, d_out=None):
    qid, kid, causal, offset, policy = ids
    valid = valid_from_ids(qid, kid, causal, offset)
    out = attention_forward(q, k, v, valid, policy, dtype)
    if d_out is None:
        return out
    return out, attention_backward(q, k, v, valid, policy, d_out, dtype)


def dense_causal_attention(q, k, v, attention_mask, dtype=np.float64, d_out=None):
    return _run(q, k, v, causal_ids(attention_mask), dtype, d_out)


def dense_prefix_causal_attention(q, pk, pv, k, v, prefix_mask, suffix_mask, dtype=np.float64, d_out=None):
    b = q.shape[0]
    if pk.shape[0] != b:
        pk = np.broadcast_to(pk, (b,) + pk.shape[1:])
        pv = np.broadcast_to(pv, (b,) + pv.shape[1:])
    kk = np.concatenate((pk, k), axis=1)
    vv = np.concatenate((pv, v), axis=1)
    return _run(q, kk, vv, prefix_ids(prefix_mask, suffix_mask), dtype, d_out)


def dense_packed_causal_attention(q, k, v, attention_mask, segment_ids, dtype=np.float64, d_out=None):
    return _run(q, k, v, packed_ids(attention_mask, segment_ids), dtype, d_out)


def bidirectional_attention(q, k, v, mask, segment_ids=None, dtype=np.float64, d_out=None):
    return _run(q, k, v, bidirectional_ids(mask, segment_ids), dtype, d_out)


def dense_cached_attention(q, k, v, valid_length, dtype=np.float64):
    b, cap = k.shape[0], k.shape[1]
    return _run(q, k, v, cached_ids(valid_length, b, cap), dtype)


# ---------------------------------------------------------------------------
# Work accounting shared by tests and the benchmark.
# ---------------------------------------------------------------------------


def valid_pair_count(qid, kid, causal, offset) -> int:
    """Number of valid (t, s) pairs summed over the batch (per head)."""
    total = 0
    for i in range(qid.shape[0]):
        total += int(valid_from_ids(qid[i : i + 1], kid[i : i + 1], causal, offset).sum())
    return total
