"""Encoder (non-causal) GQA attention on B200.

Mirrors ``attention(query, key, value, mask, segment_ids=None)`` of
src/minifield_training/kernels/bidirectional.py:7-35: with ``segment_ids``
(int32 [B, T], 0 = padding) a query sees only active keys of its own nonzero
segment and inactive queries return zeros; without them every query sees the
mask-active keys and rows of an all-zero mask return zeros. Logits FP32,
softmax FP32, probabilities bf16 for the value product.

``attention_fwd`` / ``attention_bwd`` are the custom-VJP halves.
"""

from .. import _lib
from ..device import DeviceArray
from .attention import _mask_i32, _operands, attention_bwd as _bwd, attention_fwd_ids, build_ids


def attention_fwd(query, key, value, mask, segment_ids=None, stream=None):
    q, k, v = _operands(query, key, value, stream)
    b, t = q.shape[0], q.shape[1]
    if k.shape[1] != t:
        raise ValueError("Bidirectional attention needs equal query and key lengths")
    m = _mask_i32(mask, stream)
    seg = _mask_i32(segment_ids, stream)
    ids = build_ids(_lib.MASK_BIDIR, m, seg, None, b, t, t, 0, stream)
    return attention_fwd_ids(q, k, v, *ids, stream=stream)


def attention(query, key, value, mask, segment_ids=None, stream=None) -> DeviceArray:
    return attention_fwd(query, key, value, mask, segment_ids, stream)[0]


def attention_bwd(residuals, d_out, stream=None):
    return _bwd(residuals, d_out, stream)
