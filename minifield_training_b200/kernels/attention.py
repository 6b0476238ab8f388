"""GQA attention on the B200 kernels, behind the reference's function names.

Mirrors src/minifield_training/kernels/attention.py: the dense/cudnn/splash
backends of ``causal_attention`` (:526-540), ``prefix_causal_attention``
(:543-568), ``packed_causal_attention`` (:571-588) and ``cached_attention``
(:591-610) gain one backend name, ``"b200"``, served by hand-written sm_100a
kernels (libmfb200). Unknown backend names raise the reference's
``ValueError("Unsupported ... backend: <name>")``. There is no CPU fallback:
without the library or an sm_100 device the calls raise.

Arrays are ``bthd`` (q [B,T,H,D], k/v [B,S,Hk,D]) in bf16; masks and segment
ids int32 (bool accepted); outputs keep the query's layout. Every forward also
has a ``*_fwd`` variant returning ``(out, residuals)`` and a ``*_bwd(residuals,
d_out) -> (dq, dk, dv)``: the pair a ``jax.custom_vjp`` registration wires to
the FFI targets.
"""

import ctypes
from dataclasses import dataclass

import numpy as np

from .. import _lib
from ..device import DeviceArray, as_device, workspace

BACKEND = "b200"


@dataclass
class AttentionResiduals:
    q: DeviceArray
    k: DeviceArray
    v: DeviceArray
    out: DeviceArray
    lse: DeviceArray
    qid: DeviceArray
    kid: DeviceArray
    causal: int
    offset: int
    policy: int
    scale: float


def _mask_i32(x, stream=None):
    if x is None:
        return None
    if isinstance(x, DeviceArray):
        return as_device(x, "int32")
    return as_device(np.asarray(x).astype(np.int32), "int32", stream)


def _operands(query, key, value, stream=None):
    q = as_device(query, "bfloat16", stream)
    k = as_device(key, "bfloat16", stream)
    v = as_device(value, "bfloat16", stream)
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("attention operands must be [B, T, H, D]")
    if k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[-1] != k.shape[-1]:
        raise ValueError("Attention query/KV shapes are incompatible")
    if q.shape[2] % k.shape[2]:
        raise ValueError("Query heads must be divisible by KV heads")
    return q, k, v


def build_ids(mode, mask, segment_ids, aux, batch, t, s, p, stream=None):
    """Device (qid, kid) encoding plus (causal, offset, policy) for a mask shape."""
    qid = DeviceArray((batch, t), "int32")
    kid = DeviceArray((batch, s), "int32")
    c, o, pol = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()

    def ptr(a):
        return ctypes.c_void_p(a.ptr) if a is not None else None

    _lib.call(
        "mfb_attn_ids", mode, ptr(mask), ptr(segment_ids), ptr(aux), ptr(qid), ptr(kid),
        batch, t, s, p, ctypes.byref(c), ctypes.byref(o), ctypes.byref(pol), stream,
    )
    return qid, kid, c.value, o.value, pol.value


def attention_fwd_ids(q, k, v, qid, kid, causal, offset, policy, stream=None, scale=None):
    """Forward over an explicit id encoding -> (out, residuals).

    ``scale`` defaults to head_dim ** -0.5 (the reference's logit scale).
    """
    b, t, h, d = q.shape
    s, hk = k.shape[1], k.shape[2]
    scale = d ** -0.5 if scale is None else float(scale)
    out = DeviceArray((b, t, h, d), "bfloat16")
    lse = DeviceArray((b, h, t), "float32")
    need = _lib.lib().mfb_attn_workspace_size(b, t, s, h, hk, d)
    ws = workspace("attention", need)
    _lib.call(
        "mfb_attn_fwd", ctypes.c_void_p(q.ptr), ctypes.c_void_p(k.ptr), ctypes.c_void_p(v.ptr),
        ctypes.c_void_p(out.ptr), ctypes.c_void_p(lse.ptr), ctypes.c_void_p(qid.ptr), ctypes.c_void_p(kid.ptr),
        b, t, s, h, hk, d, causal, offset, policy, ctypes.c_float(scale), ctypes.c_void_p(ws.ptr), ws.nbytes, stream,
    )
    return out, AttentionResiduals(q, k, v, out, lse, qid, kid, causal, offset, policy, scale)


def attention_bwd(res: AttentionResiduals, d_out, stream=None):
    """(dq, dk, dv) for upstream gradient ``d_out`` [B,T,H,D]."""
    do = as_device(d_out, "bfloat16", stream)
    if do.shape != res.out.shape:
        raise ValueError("d_out must match the attention output shape")
    b, t, h, d = res.q.shape
    s, hk = res.k.shape[1], res.k.shape[2]
    dq = DeviceArray(res.q.shape, "bfloat16")
    dk = DeviceArray(res.k.shape, "bfloat16")
    dv = DeviceArray(res.v.shape, "bfloat16")
    need = _lib.lib().mfb_attn_workspace_size(b, t, s, h, hk, d)
    ws = workspace("attention", need)
    p = ctypes.c_void_p
    _lib.call(
        "mfb_attn_bwd", p(res.q.ptr), p(res.k.ptr), p(res.v.ptr), p(res.out.ptr), p(res.lse.ptr), p(do.ptr),
        p(dq.ptr), p(dk.ptr), p(dv.ptr), p(res.qid.ptr), p(res.kid.ptr), b, t, s, h, hk, d, res.causal, res.offset,
        res.policy, ctypes.c_float(res.scale), p(ws.ptr), ws.nbytes, stream,
    )
    return dq, dk, dv


# ---------------------------------------------------------------------------
# Reference-named b200 backends.
# ---------------------------------------------------------------------------


def b200_causal_attention_fwd(query, key, value, attention_mask, stream=None):
    q, k, v = _operands(query, key, value, stream)
    b, t = q.shape[0], q.shape[1]
    if k.shape[1] != t:
        raise ValueError("Causal attention needs equal query and key lengths")
    mask = _mask_i32(attention_mask, stream)
    ids = build_ids(_lib.MASK_CAUSAL, mask, None, None, b, t, t, 0, stream)
    return attention_fwd_ids(q, k, v, *ids, stream=stream)


def b200_causal_attention(query, key, value, attention_mask, stream=None):
    """dense_causal_attention (kernels/attention.py:206-222) on B200."""
    return b200_causal_attention_fwd(query, key, value, attention_mask, stream)[0]


def b200_packed_causal_attention_fwd(query, key, value, attention_mask, segment_ids, stream=None):
    q, k, v = _operands(query, key, value, stream)
    if q.shape[1] != k.shape[1]:
        raise ValueError("Packed attention query/KV shapes are incompatible")
    b, t = q.shape[0], q.shape[1]
    mask = _mask_i32(attention_mask, stream)
    seg = _mask_i32(segment_ids, stream)
    ids = build_ids(_lib.MASK_PACKED, mask, seg, None, b, t, t, 0, stream)
    return attention_fwd_ids(q, k, v, *ids, stream=stream)


def b200_packed_causal_attention(query, key, value, attention_mask, segment_ids, stream=None):
    """dense_packed_causal_attention (kernels/attention.py:245-261) on B200."""
    return b200_packed_causal_attention_fwd(query, key, value, attention_mask, segment_ids, stream)[0]


def _concat_rows(prefix: DeviceArray, rest: DeviceArray, batch: int) -> DeviceArray:
    """[B, P + T, ...] from prefix [B|1, P, ...] and rest [B, T, ...] by row copies."""
    pb = prefix.nbytes // prefix.shape[0]
    rb = rest.nbytes // rest.shape[0]
    out = DeviceArray((batch, prefix.shape[1] + rest.shape[1]) + rest.shape[2:], rest.dtype)
    for i in range(batch):
        src = prefix.ptr + (0 if prefix.shape[0] == 1 else i * pb)
        _lib.call("mfb_memcpy_d2d", ctypes.c_void_p(out.ptr + i * (pb + rb)), ctypes.c_void_p(src), pb, None)
        _lib.call("mfb_memcpy_d2d", ctypes.c_void_p(out.ptr + i * (pb + rb) + pb), ctypes.c_void_p(rest.ptr + i * rb), rb, None)
    return out


def b200_prefix_causal_attention_fwd(query, prefix_key, prefix_value, key, value, prefix_mask, suffix_mask,
                                     stream=None):
    q, k, v = _operands(query, key, value, stream)
    pk = as_device(prefix_key, "bfloat16", stream)
    pv = as_device(prefix_value, "bfloat16", stream)
    b, t = q.shape[0], q.shape[1]
    if pk.shape[0] not in (1, b):
        raise ValueError("Shared prefix batch is incompatible")
    pmask = _mask_i32(prefix_mask, stream)
    smask = _mask_i32(suffix_mask, stream)
    kk = _concat_rows(pk, k, b)
    vv = _concat_rows(pv, v, b)
    p = pk.shape[1]
    ids = build_ids(_lib.MASK_PREFIX, smask, None, pmask, b, t, p + t, p, stream)
    return attention_fwd_ids(q, kk, vv, *ids, stream=stream)


def b200_prefix_causal_attention(query, prefix_key, prefix_value, key, value, prefix_mask, suffix_mask, stream=None):
    """dense_prefix_causal_attention (kernels/attention.py:225-242) on B200."""
    return b200_prefix_causal_attention_fwd(query, prefix_key, prefix_value, key, value, prefix_mask, suffix_mask,
                                            stream)[0]


def b200_cached_attention(query, key, value, valid_length, stream=None):
    """dense_cached_attention (kernels/attention.py:264-282) on B200 (decode kernel)."""
    q, k, v = _operands(query, key, value, stream)
    if q.shape[1] != 1:
        raise ValueError("Cached attention expects one query per row")
    b, cap, hk, d = k.shape
    h = q.shape[2]
    lengths = np.broadcast_to(np.asarray(valid_length, np.int32).reshape(-1), (b,)) if not isinstance(
        valid_length, DeviceArray) else None
    vl = as_device(lengths, "int32", stream) if lengths is not None else as_device(valid_length, "int32")
    out = DeviceArray((b, 1, h, d), "bfloat16")
    ws = workspace("decode", _lib.lib().mfb_decode_workspace_size(b, cap, h, d))
    p = ctypes.c_void_p
    _lib.call(
        "mfb_decode_attn", p(q.ptr), p(k.ptr), p(v.ptr), None, None, None, p(vl.ptr), p(out.ptr),
        b, cap, h, hk, d, ctypes.c_float(d ** -0.5), p(ws.ptr), ws.nbytes, stream,
    )
    return out


# ---------------------------------------------------------------------------
# Dispatchers with the reference's signatures.
# ---------------------------------------------------------------------------


def causal_attention(query, key, value, attention_mask, *, backend):
    if backend != BACKEND:
        raise ValueError(f"Unsupported causal attention backend: {backend}")
    return b200_causal_attention(query, key, value, attention_mask)


def prefix_causal_attention(query, prefix_key, prefix_value, key, value, prefix_mask, suffix_mask, *,
                            backend=BACKEND):
    if backend != BACKEND:
        raise ValueError(f"Unsupported prefix attention backend: {backend}")
    return b200_prefix_causal_attention(query, prefix_key, prefix_value, key, value, prefix_mask, suffix_mask)


def packed_causal_attention(query, key, value, attention_mask, segment_ids, *, backend):
    if backend != BACKEND:
        raise ValueError(f"Unsupported packed attention backend: {backend}")
    return b200_packed_causal_attention(query, key, value, attention_mask, segment_ids)


def cached_attention(query, key, value, valid_length, *, backend=BACKEND):
    if backend != BACKEND:
        raise ValueError(f"Unsupported cached attention backend: {backend}")
    return b200_cached_attention(query, key, value, valid_length)


def attention_flops(b, t, s, h, d, valid_pairs=None, causal=False) -> float:
    """Forward FLOPs: 4 * H * D per valid (t, s) pair (two matmuls)."""
    if valid_pairs is None:
        valid_pairs = b * t * s / (2.0 if causal else 1.0)
    return 4.0 * h * d * valid_pairs


__all__ = [
    "AttentionResiduals", "attention_bwd", "attention_fwd_ids", "build_ids", "b200_causal_attention",
    "b200_causal_attention_fwd", "b200_packed_causal_attention", "b200_packed_causal_attention_fwd",
    "b200_prefix_causal_attention", "b200_prefix_causal_attention_fwd", "b200_cached_attention",
    "causal_attention", "prefix_causal_attention", "packed_causal_attention", "cached_attention",
    "attention_flops",
]
