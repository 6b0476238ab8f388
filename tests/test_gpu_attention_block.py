"""The attention block at layer level: prefill plus cached steps equal the uninterrupted block.

Mirrors the reference's property test (tests/layers/test_blocks.py:223-291):
``attention_block_prefill`` over the first P tokens, then
``attention_block_step`` for each later token, must give the outputs of one
``attention_block`` over all T tokens, with the cache holding the block's
RoPE'd keys and values in its first T slots and zeros after them
(src/minifield_training/layers/attention.py:111-138, 246-322). Every output is
also checked against the FP64 oracle block (oracle/decode_model.py) under the
per-op gate (max-abs 2e-2, rel-L2 1e-2, per-element units).
"""

import types

import numpy as np
import pytest

from oracle.bf16 import round_bf16
from tests._util import assert_close
from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


CFG = types.SimpleNamespace(hidden=256, ffn=256, heads=4, kv_heads=2, head_dim=64, norm_eps=1e-5, rope_theta=1e6)


def _weights(seed):
    rng = np.random.default_rng(seed)
    c, f, hd = CFG.hidden, CFG.ffn, CFG.head_dim

    def mat(n, k, s=0.05):
        return (rng.standard_normal((n, k)) * s).astype(np.float32)

    def gain(n):
        return rng.uniform(0.5, 1.5, n).astype(np.float32)

    w = {"operator_norm.weight": gain(c), "self_attn.q_proj.weight": mat(CFG.heads * hd, c),
         "self_attn.k_proj.weight": mat(CFG.kv_heads * hd, c), "self_attn.v_proj.weight": mat(CFG.kv_heads * hd, c),
         "self_attn.out_proj.weight": mat(c, CFG.heads * hd), "self_attn.q_layernorm.weight": gain(hd),
         "self_attn.k_layernorm.weight": gain(hd), "ffn_norm.weight": gain(c), "feed_forward.w1.weight": mat(f, c),
         "feed_forward.w3.weight": mat(f, c), "feed_forward.w2.weight": mat(c, f)}
    return w


def _tuples(w):
    from minifield_training_b200.layers.attention import AttentionWeights
    from minifield_training_b200.layers.feed_forward import FeedForwardWeights

    att = AttentionWeights(w["operator_norm.weight"], w["self_attn.q_proj.weight"], w["self_attn.k_proj.weight"],
                           w["self_attn.v_proj.weight"], w["self_attn.out_proj.weight"],
                           w["self_attn.q_layernorm.weight"], w["self_attn.k_layernorm.weight"])
    ffn = FeedForwardWeights(w["ffn_norm.weight"], w["feed_forward.w1.weight"], w["feed_forward.w3.weight"],
                             w["feed_forward.w2.weight"])
    return att, ffn


def _kw():
    return dict(head_dim=CFG.head_dim, rope_theta=CFG.rope_theta, eps=CFG.norm_eps, backend="b200")


@pytest.mark.parametrize("b,t,prompt,cap", [(3, 37, 20, 64), (2, 130, 1, 256)])
def test_prefill_then_cached_steps_equal_the_uninterrupted_block(b, t, prompt, cap):
    from minifield_training_b200.layers import attention as la
    from oracle import decode_model as odm

    w = _weights(b + t)
    att, ffn = _tuples(w)
    x = round_bf16(np.random.default_rng(t).standard_normal((b, t, CFG.hidden)).astype(np.float32))
    full = la.attention_block(x, att, ffn, np.ones((b, t), np.int32), **_kw()).float32()
    pre, kc, vc = la.attention_block_prefill(x[:, :prompt], att, ffn, np.ones((b, prompt), np.int32), capacity=cap,
                                             **_kw())
    outs = [pre.float32()]
    for pos in range(prompt, t):
        y, kc, vc = la.attention_block_step(x[:, pos:pos + 1], att, ffn, kc, vc, pos, pos + 1, **_kw())
        outs.append(y.float32())
    stepped = np.concatenate(outs, axis=1)
    y_ref, k_ref, v_ref = odm.attention_block(CFG, w, x)
    assert_close(full, y_ref, scaled=True, what="uninterrupted block vs oracle")
    assert_close(stepped, y_ref, scaled=True, what="prefill + steps vs oracle")
    assert_close(stepped, full, scaled=True, what="prefill + steps vs uninterrupted block")
    k_got, v_got = kc.float32(), vc.float32()
    assert_close(k_got[:, :t], k_ref, scaled=True, what="cached keys")
    assert_close(v_got[:, :t], v_ref, scaled=True, what="cached values")
    assert not np.any(k_got[:, t:]) and not np.any(v_got[:, t:])


def test_prefill_zeroes_masked_cache_rows():
    """Keys and values of masked prompt tokens are zero in the cache (key * keep, :268-278)."""
    from minifield_training_b200.layers import attention as la

    b, t, cap = 2, 40, 64
    att, ffn = _tuples(_weights(5))
    x = round_bf16(np.random.default_rng(5).standard_normal((b, t, CFG.hidden)).astype(np.float32))
    mask = np.ones((b, t), np.int32)
    mask[0, 30:] = 0
    mask[1, 3:7] = 0
    _, kc, vc = la.attention_block_prefill(x, att, ffn, mask, capacity=cap, **_kw())
    _, kf, vf = la.attention_block_prefill(x, att, ffn, np.ones((b, t), np.int32), capacity=cap, **_kw())
    for got, ref in ((kc.float32(), kf.float32()), (vc.float32(), vf.float32())):
        keep = mask[:, :, None, None].astype(bool)
        np.testing.assert_array_equal(got[:, :t], np.where(keep, ref[:, :t], 0))
        assert not np.any(got[:, t:])


def test_step_takes_a_position_per_row():
    """Rows at different positions in one step (the per-row generalisation of the scalar position)."""
    from minifield_training_b200.layers import attention as la
    from oracle import decode_model as odm

    b, t, cap = 3, 24, 32
    w = _weights(9)
    att, ffn = _tuples(w)
    x = round_bf16(np.random.default_rng(9).standard_normal((b, t, CFG.hidden)).astype(np.float32))
    y_ref, _, _ = odm.attention_block(CFG, w, x)
    lengths = np.array([5, 11, 17])
    kc = vc = None
    caches = []
    for r in range(b):  # each row's prompt prefilled alone, then assembled into one batch cache
        _, k1, v1 = la.attention_block_prefill(x[r:r + 1, :lengths[r]], att, ffn,
                                               np.ones((1, lengths[r]), np.int32), capacity=cap, **_kw())
        caches.append((k1.float32(), v1.float32()))
    from minifield_training_b200.device import DeviceArray
    kc = DeviceArray.from_numpy(np.concatenate([c[0] for c in caches]), "bfloat16")
    vc = DeviceArray.from_numpy(np.concatenate([c[1] for c in caches]), "bfloat16")
    xs = np.stack([x[r, lengths[r]] for r in range(b)])[:, None]
    y, kc, vc = la.attention_block_step(xs, att, ffn, kc, vc, lengths, lengths + 1, **_kw())
    ref = np.stack([y_ref[r, lengths[r]] for r in range(b)])[:, None]
    assert_close(y.float32(), ref, scaled=True, what="per-row positions")
