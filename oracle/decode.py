"""KV-cache append + single-query cached attention (test infrastructure only).

Restates the attention half of ``attention_block_step``
(src/minifield_training/layers/attention.py:281-322): the step's new key and
value are written into the cache at ``position`` with
``dynamic_update_slice`` (:309-314), then ``cached_attention`` attends the
single query to cache slots ``< valid_length`` (kernels/attention.py:264-282,
non-causal by design, ``valid_length`` scalar or ``[B]``). A row whose
``valid_length`` is 0 is a uniform average over every cache slot, the dense
``finfo.min`` fill's behaviour.

The benchmark's per-sequence positions generalise the reference's scalar
position (one write slot per row); the scalar case is the special case of
all rows equal.
"""

import numpy as np

from . import attention


def append_kv(k_cache, v_cache, new_k, new_v, positions):
    """Return caches with row b's slot positions[b] replaced.

    ``jax.lax.dynamic_update_slice`` clamps the start index so the update fits,
    so the slot is clamped into [0, capacity - 1].
    """
    k_cache = k_cache.copy()
    v_cache = v_cache.copy()
    cap = k_cache.shape[1]
    for b, p in enumerate(np.asarray(positions).reshape(-1)):
        p = min(max(int(p), 0), cap - 1)
        k_cache[b, p] = new_k[b]
        v_cache[b, p] = new_v[b]
    return k_cache, v_cache


def decode_attention(q, k_cache, v_cache, valid_length, new_k=None, new_v=None, positions=None, dtype=np.float64):
    """q [B, H, D], caches [B, cap, Hk, D] -> (o [B, H, D], k_cache, v_cache)."""
    if new_k is not None:
        k_cache, v_cache = append_kv(k_cache, v_cache, new_k, new_v, positions)
    b, cap = k_cache.shape[0], k_cache.shape[1]
    ids = attention.cached_ids(valid_length, b, cap)
    valid = attention.valid_from_ids(*ids[:4])
    out = attention.attention_forward(q[:, None], k_cache, v_cache, valid, ids[4], dtype)
    return out[:, 0], k_cache, v_cache


def decode_bytes(lengths, kv_heads: int, head_dim: int, heads: int, elem: int = 2) -> int:
    """Algorithmic HBM bytes of one layer's decode attention.

    K and V reads of the valid prefix, plus q read, o write and the new k/v
    read + cache write.
    """
    lengths = np.asarray(lengths, np.int64)
    kv = int(lengths.sum()) * kv_heads * head_dim * 2 * elem
    b = lengths.shape[0]
    qo = b * heads * head_dim * 2 * elem
    new = b * kv_heads * head_dim * 2 * elem * 2
    return kv + qo + new
