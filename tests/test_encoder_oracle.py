"""oracle/encoder.py's analytic backward passes against FP64 central differences.

The forward functions are evaluated with the bf16 rounding replaced by the
identity and float64 arithmetic (monkeypatched), so the finite differences
measure the exact derivative the backward functions state. CPU only.
"""

import numpy as np
import pytest

from oracle import encoder as oe


@pytest.fixture
def exact(monkeypatch):
    monkeypatch.setattr(oe, "rb", lambda x: np.asarray(x, np.float64))
    monkeypatch.setattr(oe, "F", np.float64)
    return oe


def _fd(f, x, dy, eps=1e-6):
    """sum(dy * df/dx) directional check: returns the numeric gradient of <dy, f(x)>."""
    g = np.zeros_like(x)
    it = np.nditer(x, flags=["multi_index"])
    for _ in it:
        i = it.multi_index
        xp, xm = x.copy(), x.copy()
        xp[i] += eps
        xm[i] -= eps
        g[i] = (np.sum(dy * f(xp)) - np.sum(dy * f(xm))) / (2 * eps)
    return g


def test_rms_norm_bwd(exact):
    rng = np.random.default_rng(0)
    x, w, dy, mask = rng.standard_normal((3, 8)), rng.standard_normal(8), rng.standard_normal((3, 8)), np.array([1, 0, 1])
    dx, dw = exact.rms_norm_bwd(x, w, dy, mask=mask, eps=1e-5)
    np.testing.assert_allclose(dx, _fd(lambda v: exact.rms_norm(v, w, 1e-5, mask=mask)[1], x, dy), rtol=1e-5, atol=1e-8)
    np.testing.assert_allclose(dw, _fd(lambda v: exact.rms_norm(x, v, 1e-5, mask=mask)[1], w, dy), rtol=1e-5, atol=1e-8)


def test_qknorm_rope_bwd(exact):
    rng = np.random.default_rng(1)
    m, h, hk = 2, 2, 1
    qkv = rng.standard_normal((m, (h + 2 * hk) * 64))
    wq, wk = rng.standard_normal(64), rng.standard_normal(64)
    pos = np.array([3, 17])
    freqs = oe.rope_freqs(1e4).astype(np.float64)
    dq, dk, dv = rng.standard_normal((m, h, 64)), rng.standard_normal((m, hk, 64)), rng.standard_normal((m, hk, 64))
    d, dwq, dwk = exact.qknorm_rope_bwd(qkv, wq, wk, pos, freqs, h, hk, dq, dk, dv, 1e-5)

    def f(v):
        q, k, vv = exact.qknorm_rope(v, wq, wk, pos, freqs, h, hk, 1e-5)
        return np.concatenate((q.reshape(m, -1), k.reshape(m, -1), vv.reshape(m, -1)), axis=1)

    dy = np.concatenate((dq.reshape(m, -1), dk.reshape(m, -1), dv.reshape(m, -1)), axis=1)
    np.testing.assert_allclose(d, _fd(f, qkv, dy), rtol=1e-5, atol=1e-7)
    fq = lambda v: exact.qknorm_rope(qkv, v, wk, pos, freqs, h, hk, 1e-5)[0]
    np.testing.assert_allclose(dwq, _fd(fq, wq, dq), rtol=1e-5, atol=1e-7)


def test_gated_conv_bwd(exact):
    rng = np.random.default_rng(2)
    c, t = 8, 7
    seg = np.array([1, 1, 1, 0, 2, 2, 3, 1, 1, 2, 2, 2, 0, 0])
    bcx = rng.standard_normal((2 * t, 3 * c))
    taps = rng.standard_normal((c, 3))
    dm = rng.standard_normal((2 * t, c))
    d, dt = exact.gated_conv_bwd(bcx, taps, seg, t, dm)
    np.testing.assert_allclose(d, _fd(lambda v: exact.gated_conv(v, taps, seg, t), bcx, dm), rtol=1e-5, atol=1e-8)
    np.testing.assert_allclose(dt, _fd(lambda v: exact.gated_conv(bcx, v, seg, t), taps, dm), rtol=1e-5, atol=1e-8)


def test_head_loss_bwd(exact, monkeypatch):
    rng = np.random.default_rng(3)
    e, w = rng.standard_normal((5, 6)), rng.standard_normal((3, 6))
    labels, valid = np.array([0, 2, 1, 1, 0]), np.array([1, 1, 0, 1, 1])
    _, count, de, dw = exact.head_loss(e, w, labels, valid)
    assert count == 4
    loss = lambda ee, ww: exact.head_loss(ee, ww, labels, valid)[0]
    np.testing.assert_allclose(de, _fd(lambda v: np.array(loss(v, w)), e, np.array(1.0)), rtol=1e-5, atol=1e-8)
    np.testing.assert_allclose(dw, _fd(lambda v: np.array(loss(e, v)), w, np.array(1.0)), rtol=1e-5, atol=1e-8)
