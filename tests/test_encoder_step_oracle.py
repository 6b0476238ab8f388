"""Model-level properties of oracle/encoder_step.py, the FP64 step the GPU encoder is compared with.

The reference pins its encoder with two properties
(tests/models/lfm2_5/test_encoder.py): segments packed into one row encode
exactly as the same segments in rows of their own (:65-103), and padding
tokens never reach valid ones (:37-63). The same properties hold here for the
loss sum, the valid count and every trainable gradient of a tiny two-layer
(conv + attention) encoder. CPU only.
"""

import dataclasses

import numpy as np
import pytest

from minifield_training_b200 import workloads
from minifield_training_b200.models import encoder as me
from oracle import encoder_step as oes

T = 32


def _cfg():
    return dataclasses.replace(workloads.CONFIG5, global_batch=1, length=T, hidden=128, ffn=256, heads=2,
                               kv_heads=1, vocab=200, layer_types=("conv", "full_attention"))


def _row(segments, rng, pad_id=0):
    """One row holding the given segment lengths (ids 1..n, positions restarting at 0) then padding."""
    seg = np.zeros(T, np.int32)
    pos = np.zeros(T, np.int32)
    at = 0
    for i, n in enumerate(segments):
        seg[at:at + n] = i + 1
        pos[at:at + n] = np.arange(n)
        at += n
    ids = rng.integers(0, 200, T).astype(np.int32)
    ids[at:] = pad_id
    labels = rng.integers(0, 2, T).astype(np.int32)
    return ids, (seg != 0).astype(np.int32), seg, pos, labels


def _run(cfg, params, rows, bf16):
    stack = [np.stack([r[i] for r in rows]) for i in range(5)]
    return oes.loss_and_grads(cfg, params, *stack, rows=len(rows), bf16=bf16)


def test_packed_segments_equal_separate_rows():
    cfg = _cfg()
    params = me.init_parameters(cfg, 0)
    rng = np.random.default_rng(7)
    packed = _row((12, 15), rng)
    ids, mask, seg, pos, labels = packed
    first = [a.copy() for a in packed]
    second = [a.copy() for a in packed]
    for a in first:
        a[12:] = 0
    for a, b in zip(second, packed):
        a[:] = 0
        a[:15] = b[12:27]
    second[2][:15] = 1  # its own segment id
    first[3][:12] = np.arange(12)
    second[3][:15] = np.arange(15)
    loss_p, count_p, grads_p = _run(cfg, params, [packed], bf16=False)
    loss_s, count_s, grads_s = _run(cfg, params, [tuple(first), tuple(second)], bf16=False)
    assert count_p == count_s == 27
    np.testing.assert_allclose(loss_p, loss_s, rtol=1e-10)
    for name, g in grads_p.items():
        np.testing.assert_allclose(g, grads_s[name], rtol=1e-8, atol=1e-12 * max(1.0, np.abs(g).max()),
                                   err_msg=name)


@pytest.mark.parametrize("bf16", [False, True])
def test_padding_never_reaches_valid_tokens(bf16):
    cfg = _cfg()
    params = me.init_parameters(cfg, 1)
    a = _row((20,), np.random.default_rng(3), pad_id=0)
    b = [x.copy() for x in a]
    rng = np.random.default_rng(4)
    b[0][20:] = rng.integers(0, 200, T - 20)  # other padding ids
    b[4][20:] = rng.integers(0, 2, T - 20)  # other padding labels
    loss_a, count_a, grads_a = _run(cfg, params, [a], bf16)
    loss_b, count_b, grads_b = _run(cfg, params, [tuple(b)], bf16)
    assert count_a == count_b == 20
    assert loss_a == loss_b
    for name, g in grads_a.items():
        np.testing.assert_array_equal(g, grads_b[name], err_msg=name)
