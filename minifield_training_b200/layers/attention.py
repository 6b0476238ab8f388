"""The KV-cache half of the decode step on B200.

Mirrors the attention part of ``attention_block_step``
(src/minifield_training/layers/attention.py:281-322): the step's new key and
value are written into the caches at ``position`` (the ``dynamic_update_slice``
of :309-314) and the single query attends to slots ``< valid_length``
(:315-317). The B200 kernel fuses the write into the attention pass and takes
per-row positions and lengths (scalars broadcast, as in the reference). The
caches are updated in place and returned.
"""

import ctypes

import numpy as np

from .. import _lib
from ..device import DeviceArray, as_device, workspace


def _rows(x, b, stream=None):
    if isinstance(x, DeviceArray):
        return as_device(x, "int32")
    return as_device(np.broadcast_to(np.asarray(x, np.int32).reshape(-1), (b,)).copy(), "int32", stream)


def decode_attention_step(query, new_key, new_value, cache_key, cache_value, position, valid_length, stream=None,
                          out=None):
    """query [B,1,H,D], new k/v [B,1,Hk,D], caches [B,cap,Hk,D] -> (out [B,1,H,D], cache_key, cache_value)."""
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
    p = ctypes.c_void_p
    _lib.call(
        "mfb_decode_attn", p(q.ptr), p(kc.ptr), p(vc.ptr), p(nk.ptr), p(nv.ptr), p(pos.ptr), p(vl.ptr), p(out.ptr),
        b, cap, h, hk, d, ctypes.c_float(d ** -0.5), p(ws.ptr), ws.nbytes, stream,
    )
    return out, kc, vc
