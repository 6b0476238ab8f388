"""The causal attention block on B200: full sequence, prefill into a fixed cache, and the cached step.

Mirrors src/minifield_training/layers/attention.py:
  ``AttentionWeights``        :45-58
  ``attention_block``         :111-138  (full-sequence causal block)
  ``attention_block_prefill`` :246-278  (the block plus keys/values in a fixed-capacity cache)
  ``attention_block_step``    :281-322  (one token per row against the cache)
  ``decode_attention_step``   the cache write + cached attention of :309-317 alone

Each block is operator RMSNorm -> q/k/v ``full_linear`` -> per-head q/k
RMSNorm -> RoPE (``_rope_qkv`` :80-97, ``project_qkv`` :61-77) -> attention
-> out-projection -> residual -> SwiGLU block (``_attention_residual``
:100-108). The q/k/v masters are cast to bf16 into one [Hq+2Hk, C] matrix, so
the three projections are one GEMM; q/k norm and RoPE are one kernel; in the
step the cache write is fused into the cached-attention kernel. Weights are
FP32 masters (host arrays or device arrays) or bf16 device arrays; the
activations and outputs are bf16 device arrays.

Per-row ``position`` / ``valid_length`` ([B]) generalise the reference's
scalar position (every row equal is the reference's case).
"""

import ctypes
from typing import NamedTuple

import numpy as np

from .. import _lib
from ..device import DeviceArray, as_device, workspace
from ..kernels import attention as _attn
from ..kernels.linear import gemm_nt
from .feed_forward import FeedForwardWeights

P = ctypes.c_void_p
BACKEND = _attn.BACKEND


class AttentionWeights(NamedTuple):
    """Operator norm gain, q/k/v/out projection masters and per-head q/k norm gains (:45-58)."""

    operator_norm: object
    query: object
    key: object
    value: object
    out: object
    query_norm: object
    key_norm: object


def _bf16_rows(mats, stream=None) -> DeviceArray:
    """The row-concatenation of ``mats`` ([N_i, K] FP32 masters or bf16 device arrays) as one bf16 matrix."""
    k = int(np.shape(mats[0])[1]) if not isinstance(mats[0], DeviceArray) else mats[0].shape[1]
    rows = [m.shape[0] if isinstance(m, DeviceArray) else int(np.shape(m)[0]) for m in mats]
    out = DeviceArray((sum(rows), k), "bfloat16")
    offset = 0
    for m, n in zip(mats, rows):
        dst = out.view(offset * k, (n, k))
        if isinstance(m, DeviceArray) and m.dtype == "bfloat16":
            dst.copy_(m, stream)
        else:
            src = as_device(m, "float32", stream)
            if src.shape != (n, k):
                raise ValueError("projection matrices must share their input width")
            _lib.call("mfb_cast_f32_bf16", P(src.ptr), P(dst.ptr), n * k, stream)
        offset += n
    return out


def _gain(w, stream=None) -> DeviceArray:
    return as_device(np.asarray(w, np.float32) if not isinstance(w, DeviceArray) else w, "float32", stream)


def _rms(x, residual, gain, sum_out, y, rstd, m, c, eps, stream):
    _lib.call("mfb_rmsnorm_fwd", P(x.ptr), P(residual.ptr) if residual is not None else None, P(gain.ptr), None,
              P(sum_out.ptr) if sum_out is not None else None, P(y.ptr), P(rstd.ptr), m, c, ctypes.c_float(eps),
              stream)


def _check_head_dim(weights: AttentionWeights, head_dim: int, c: int):
    if head_dim != 64:
        raise ValueError("the b200 attention block supports head_dim 64")
    shapes = [tuple(np.shape(w)) if not isinstance(w, DeviceArray) else w.shape
              for w in (weights.query, weights.key, weights.value, weights.out)]
    hq, hk = shapes[0][0], shapes[1][0]
    if hq % head_dim or hk % head_dim or shapes[2][0] != hk or any(s[1] != c for s in shapes[:3]):
        raise ValueError("Attention projection shapes are incompatible with head_dim")
    if shapes[3] != (c, hq):
        raise ValueError("Attention output projection must be [hidden, query heads * head_dim]")
    if (hq // head_dim) % (hk // head_dim):
        raise ValueError("Query heads must be divisible by KV heads")
    return hq // head_dim, hk // head_dim


def _project(x2, weights, positions, *, heads, kv_heads, head_dim, rope_theta, eps, stream):
    """(q [M,H,D], k [M,Hk,D], v [M,Hk,D]) of ``_rope_qkv`` for token rows x2 [M, C] at int32 positions [M]."""
    from ..models.encoder import rope_freqs

    m, c = x2.shape
    hn, rstd = DeviceArray((m, c), "bfloat16"), DeviceArray((m,), "float32")
    _rms(x2, None, _gain(weights.operator_norm, stream), None, hn, rstd, m, c, eps, stream)
    nq = (heads + 2 * kv_heads) * head_dim
    proj = gemm_nt(hn, _bf16_rows((weights.query, weights.key, weights.value), stream), stream=stream)
    q = DeviceArray((m, heads, head_dim), "bfloat16")
    k = DeviceArray((m, kv_heads, head_dim), "bfloat16")
    v = DeviceArray((m, kv_heads, head_dim), "bfloat16")
    rq, rk = DeviceArray((m, heads), "float32"), DeviceArray((m, kv_heads), "float32")
    freqs = as_device(rope_freqs(rope_theta, head_dim), "float32", stream)
    # Device copies are bound to names: a temporary would be freed before the launch reads it.
    wq, wk = _gain(weights.query_norm, stream), _gain(weights.key_norm, stream)
    _lib.call("mfb_qknorm_rope_fwd", P(proj.ptr), nq, P(wq.ptr), P(wk.ptr), P(positions.ptr), P(freqs.ptr), P(q.ptr),
              P(k.ptr), P(v.ptr), P(rq.ptr), P(rk.ptr), m, heads, kv_heads, ctypes.c_float(eps), stream)
    return q, k, v


def _attention_residual(x2, attended2, weights, ffn: FeedForwardWeights, eps, stream):
    """``swiglu_ffn(x + out(attended), ffn, eps)`` (:100-108, layers/feed_forward.py:24-35) for rows [M, C]."""
    m, c = x2.shape
    r = gemm_nt(attended2, _bf16_rows((weights.out,), stream), stream=stream)
    mid, h2, rstd = DeviceArray((m, c), "bfloat16"), DeviceArray((m, c), "bfloat16"), DeviceArray((m,), "float32")
    _rms(x2, r, _gain(ffn.norm, stream), mid, h2, rstd, m, c, eps, stream)
    gu = gemm_nt(h2, _bf16_rows((ffn.gate, ffn.up), stream), stream=stream)
    f = gu.shape[1] // 2
    a = DeviceArray((m, f), "bfloat16")
    _lib.call("mfb_swiglu_fwd", P(gu.ptr), P(a.ptr), m, f, stream)
    y = gemm_nt(a, _bf16_rows((ffn.down,), stream), stream=stream)
    out = DeviceArray((m, c), "bfloat16")
    _lib.call("mfb_add_bf16", P(mid.ptr), P(y.ptr), P(out.ptr), m * c, stream)
    return out


def _per_row(x, b, what, stream=None) -> DeviceArray:
    if isinstance(x, DeviceArray):
        if x.size != b:
            raise ValueError(f"{what} must be a scalar or one value per row")
        return as_device(x, "int32")
    a = np.asarray(x, np.int64).reshape(-1)
    if a.size not in (1, b):
        raise ValueError(f"{what} must be a scalar or one value per row")
    return as_device(np.broadcast_to(a, (b,)).astype(np.int32), "int32", stream)


def _check_backend(backend):
    if backend != BACKEND:
        raise ValueError(f"Unsupported causal attention backend: {backend}")


def attention_block(x, weights: AttentionWeights, ffn: FeedForwardWeights, attention_mask, *, head_dim: int,
                    rope_theta: float, eps: float, backend: str, positions=None, stream=None) -> DeviceArray:
    """Full-sequence causal block (:111-138): x [B, T, C] bf16 -> [B, T, C] bf16.

    ``positions`` ([T] or [B, T] int) overrides the default 0..T-1 RoPE positions.
    """
    _check_backend(backend)
    xd = as_device(x, "bfloat16", stream)
    if xd.ndim != 3:
        raise ValueError("attention_block input must be [batch, tokens, hidden]")
    b, t, c = xd.shape
    heads, kv_heads = _check_head_dim(weights, head_dim, c)
    pos = np.broadcast_to(np.arange(t, dtype=np.int32) if positions is None else np.asarray(positions, np.int32),
                          (b, t))
    q, k, v = _project(xd.reshape(b * t, c), weights, as_device(np.ascontiguousarray(pos), "int32", stream),
                       heads=heads, kv_heads=kv_heads, head_dim=head_dim, rope_theta=rope_theta, eps=eps,
                       stream=stream)
    o = _attn.b200_causal_attention(q.reshape(b, t, heads, head_dim), k.reshape(b, t, kv_heads, head_dim),
                                    v.reshape(b, t, kv_heads, head_dim), attention_mask, stream)
    return _attention_residual(xd.reshape(b * t, c), o.reshape(b * t, heads * head_dim), weights, ffn, eps,
                               stream).reshape(b, t, c)


def attention_block_prefill(x, weights: AttentionWeights, ffn: FeedForwardWeights, attention_mask, *, capacity: int,
                            head_dim: int, rope_theta: float, eps: float, backend: str, stream=None):
    """(y [B, T, C], cache_key, cache_value [B, capacity, Hk, D]) (:246-278).

    The caches hold the block's RoPE'd keys and values times the attention
    mask in their first T slots and zeros after them: the layout
    ``attention_block_step`` updates.
    """
    _check_backend(backend)
    xd = as_device(x, "bfloat16", stream)
    if xd.ndim != 3:
        raise ValueError("attention_block_prefill input must be [batch, tokens, hidden]")
    b, t, c = xd.shape
    if t > capacity:
        raise ValueError("Prompt length exceeds attention cache capacity")
    heads, kv_heads = _check_head_dim(weights, head_dim, c)
    mask = np.asarray(attention_mask.numpy() if isinstance(attention_mask, DeviceArray) else attention_mask)
    if mask.shape != (b, t):
        raise ValueError("attention_mask must be [batch, tokens]")
    pos = np.ascontiguousarray(np.broadcast_to(np.arange(t, dtype=np.int32), (b, t)))
    q, k, v = _project(xd.reshape(b * t, c), weights, as_device(pos, "int32", stream), heads=heads,
                       kv_heads=kv_heads, head_dim=head_dim, rope_theta=rope_theta, eps=eps, stream=stream)
    o = _attn.b200_causal_attention(q.reshape(b, t, heads, head_dim), k.reshape(b, t, kv_heads, head_dim),
                                    v.reshape(b, t, kv_heads, head_dim), mask, stream)
    row = kv_heads * head_dim * 2  # bytes of one token's K (or V) row
    caches = []
    for src in (k, v):
        cache = DeviceArray.zeros((b, capacity, kv_heads, head_dim), "bfloat16", stream)
        _lib.call("mfb_memcpy2d_d2d", P(cache.ptr), capacity * row, P(src.ptr), t * row, t * row, b, stream)
        for r in range(b):  # keys and values of masked tokens are zero in the cache (key * keep)
            dropped = np.flatnonzero(mask[r] == 0)
            for run in np.split(dropped, np.flatnonzero(np.diff(dropped) != 1) + 1) if dropped.size else ():
                _lib.call("mfb_memset", P(cache.ptr + (r * capacity + int(run[0])) * row), 0, run.size * row, stream)
        caches.append(cache)
    y = _attention_residual(xd.reshape(b * t, c), o.reshape(b * t, heads * head_dim), weights, ffn, eps, stream)
    return y.reshape(b, t, c), caches[0], caches[1]


def attention_block_step(x, weights: AttentionWeights, ffn: FeedForwardWeights, cache_key, cache_value, position,
                         valid_length, *, head_dim: int, rope_theta: float, eps: float, backend: str, stream=None):
    """One decode step (:281-322): (y [B, 1, C], cache_key, cache_value).

    ``x`` holds one token per row; ``position`` is the cache slot written
    this step and its RoPE position, ``valid_length`` the number of readable
    slots after the write (each a scalar or one value per row). The caches
    (bf16 device arrays [B, capacity, Hk, D]) are updated in place and
    returned.
    """
    if backend != BACKEND:
        raise ValueError(f"Unsupported cached attention backend: {backend}")
    xd = as_device(x, "bfloat16", stream)
    if xd.ndim != 3 or xd.shape[1] != 1:
        raise ValueError("attention_block_step input must be [batch, 1, hidden]")
    b, _, c = xd.shape
    heads, kv_heads = _check_head_dim(weights, head_dim, c)
    kc = as_device(cache_key, "bfloat16", stream)
    vc = as_device(cache_value, "bfloat16", stream)
    if kc.ndim != 4 or kc.shape[0] != b or kc.shape[2:] != (kv_heads, head_dim) or vc.shape != kc.shape:
        raise ValueError("KV cache must be [batch, capacity, kv_heads, head_dim]")
    pos = _per_row(position, b, "position", stream)
    q, k, v = _project(xd.reshape(b, c), weights, pos, heads=heads, kv_heads=kv_heads, head_dim=head_dim,
                       rope_theta=rope_theta, eps=eps, stream=stream)
    o, kc, vc = decode_attention_step(q.reshape(b, 1, heads, head_dim), k, v, kc, vc, pos,
                                      _per_row(valid_length, b, "valid_length", stream), stream=stream)
    y = _attention_residual(xd.reshape(b, c), o.reshape(b, heads * head_dim), weights, ffn, eps, stream)
    return y.reshape(b, 1, c), kc, vc


def _rows(x, b, stream=None):
    if isinstance(x, DeviceArray):
        return as_device(x, "int32")
    return as_device(np.broadcast_to(np.asarray(x, np.int32).reshape(-1), (b,)).copy(), "int32", stream)


def decode_attention_step(query, new_key, new_value, cache_key, cache_value, position, valid_length, stream=None,
                          out=None):
    """The cache write + cached attention half of the step (:309-317).

    query [B,1,H,D], new k/v [B,1,Hk,D], caches [B,cap,Hk,D] -> (out [B,1,H,D], cache_key, cache_value). The
    kernel fuses the write into the attention pass; the caches are updated in place.
    """
    q = as_device(query, "bfloat16", stream)
    nk = as_device(new_key, "bfloat16", stream)
    nv = as_device(new_value, "bfloat16", stream)
    kc = as_device(cache_key, "bfloat16", stream)
    vc = as_device(cache_value, "bfloat16", stream)
    b, cap, hk, d = kc.shape
    h = q.shape[-2]
    if vc.shape != kc.shape or q.shape[-1] != d or q.size != b * h * d or nk.size != b * hk * d:
        raise ValueError("Cached attention query/KV shapes are incompatible")
    if h % hk:
        raise ValueError("Query heads must be divisible by KV heads")
    pos = _rows(position, b, stream)
    vl = _rows(valid_length, b, stream)
    if out is None:
        out = DeviceArray((b, 1, h, d), "bfloat16")
    ws = workspace("decode", _lib.lib().mfb_decode_workspace_size(b, cap, h, d))
    _lib.call(
        "mfb_decode_attn", P(q.ptr), P(kc.ptr), P(vc.ptr), P(nk.ptr), P(nv.ptr), P(pos.ptr), P(vl.ptr), P(out.ptr),
        b, cap, h, hk, d, ctypes.c_float(d ** -0.5), P(ws.ptr), ws.nbytes, stream,
    )
    return out, kc, vc
