"""Encoder-step kernels (RMSNorm, q/k norm + RoPE, gated conv, embedding, head) against oracle/encoder.py.

Forward outputs whose rounding chain the kernels reproduce step for step
(residual sums, the conv, the embedding) are compared bit for bit; the norms
(FP32 sums of squares in another order) and every backward use the stated
tolerance (max-abs 2e-2, rel-L2 1e-2; gradients in per-element units).
"""

import ctypes

import numpy as np
import pytest

from oracle import encoder as oe
from oracle.bf16 import round_bf16 as rb
from tests._util import assert_close
from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu
F = np.float32
P = ctypes.c_void_p


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


def _dev(x, dt):
    from minifield_training_b200.device import DeviceArray
    return DeviceArray.from_numpy(np.asarray(x), dt)


def _empty(shape, dt):
    from minifield_training_b200.device import DeviceArray
    return DeviceArray(shape, dt)


def _lib():
    from minifield_training_b200 import _lib
    return _lib


def _ws(nbytes):
    return _empty((max(int(nbytes), 16),), "uint8")


def _segments(rng, b, t):
    seg = np.zeros((b, t), np.int32)
    for r in range(b):
        pos, sid = 0, 1
        while pos < t:
            n = int(rng.integers(1, 40))
            seg[r, pos:pos + n] = sid if rng.random() > 0.15 else 0
            pos += n
            sid += 1
    return seg.reshape(-1)


@pytest.mark.parametrize("c,with_res,with_mask", [(1024, True, False), (1024, False, True), (256, True, True)])
def test_rmsnorm_forward_and_backward(c, with_res, with_mask):
    rng = np.random.default_rng(1)
    m = 333
    x = rb(rng.standard_normal((m, c), dtype=F))
    res = rb(rng.standard_normal((m, c), dtype=F)) if with_res else None
    w = (1 + 0.1 * rng.standard_normal(c)).astype(F)
    mask = (rng.random(m) > 0.2).astype(np.int32) if with_mask else None
    L = _lib()
    xd, wd = _dev(x, "bfloat16"), _dev(w, "float32")
    rd = _dev(res, "bfloat16") if with_res else None
    md = _dev(mask, "int32") if with_mask else None
    s_out, y, rstd = _empty((m, c), "bfloat16"), _empty((m, c), "bfloat16"), _empty((m,), "float32")
    L.call("mfb_rmsnorm_fwd", P(xd.ptr), P(rd.ptr) if rd else None, P(wd.ptr), P(md.ptr) if md else None,
           P(s_out.ptr) if with_res else None, P(y.ptr), P(rstd.ptr), m, c, F(1e-5), None)
    s_ref, y_ref, r_ref = oe.rms_norm(x, w, 1e-5, residual=res, mask=mask)
    if with_res:
        np.testing.assert_array_equal(s_out.float32(), s_ref)
    assert_close(y.float32(), y_ref, what="rms y")
    np.testing.assert_allclose(rstd.numpy(), r_ref, rtol=1e-5)
    # Backward with a residual-path gradient.
    dy = rb(rng.standard_normal((m, c), dtype=F))
    dres = rb(rng.standard_normal((m, c), dtype=F))
    s_in = s_out if with_res else xd
    dyd, dresd, dx, dw = _dev(dy, "bfloat16"), _dev(dres, "bfloat16"), _empty((m, c), "bfloat16"), _empty((c,), "float32")
    ws = _ws(L.lib().mfb_norm_workspace_size(m, c))
    L.call("mfb_rmsnorm_bwd", P(s_in.ptr), P(wd.ptr), P(rstd.ptr), P(md.ptr) if md else None, P(dyd.ptr),
           P(dresd.ptr), P(dx.ptr), P(dw.ptr), 0, m, c, P(ws.ptr), ws.nbytes, None)
    dx_ref, dw_ref = oe.rms_norm_bwd(s_ref, w, dy, dres=dres, mask=mask)
    assert_close(dx.float32(), dx_ref, scaled=True, what="rms dx")
    assert_close(dw.numpy(), dw_ref, scaled=True, what="rms dw")


def test_qknorm_rope_forward_and_backward():
    rng = np.random.default_rng(2)
    m, h, hk = 300, 16, 8
    ld = (h + 2 * hk) * 64
    qkv = rb(rng.standard_normal((m, ld), dtype=F) * F(2))
    wq, wk = (1 + 0.1 * rng.standard_normal(64)).astype(F), (1 + 0.1 * rng.standard_normal(64)).astype(F)
    pos = rng.integers(0, 2048, m).astype(np.int32)
    freqs = oe.rope_freqs(1e6)
    L = _lib()
    qd, wqd, wkd, pd, fd = _dev(qkv, "bfloat16"), _dev(wq, "float32"), _dev(wk, "float32"), _dev(pos, "int32"), \
        _dev(freqs, "float32")
    q, k, v = _empty((m, h, 64), "bfloat16"), _empty((m, hk, 64), "bfloat16"), _empty((m, hk, 64), "bfloat16")
    rq, rk = _empty((m, h), "float32"), _empty((m, hk), "float32")
    L.call("mfb_qknorm_rope_fwd", P(qd.ptr), ld, P(wqd.ptr), P(wkd.ptr), P(pd.ptr), P(fd.ptr), P(q.ptr), P(k.ptr),
           P(v.ptr), P(rq.ptr), P(rk.ptr), m, h, hk, F(1e-5), None)
    q_ref, k_ref, v_ref = oe.qknorm_rope(qkv, wq, wk, pos, freqs, h, hk, 1e-5)
    assert_close(q.float32(), q_ref, what="rope q")
    assert_close(k.float32(), k_ref, what="rope k")
    np.testing.assert_array_equal(v.float32(), v_ref)
    dq, dk, dv = (rb(rng.standard_normal(s, dtype=F)) for s in ((m, h, 64), (m, hk, 64), (m, hk, 64)))
    dqd, dkd, dvd = _dev(dq, "bfloat16"), _dev(dk, "bfloat16"), _dev(dv, "bfloat16")
    dqkv, dwq, dwk = _empty((m, ld), "bfloat16"), _empty((64,), "float32"), _empty((64,), "float32")
    ws = _ws(L.lib().mfb_norm_workspace_size(m, 128))
    L.call("mfb_qknorm_rope_bwd", P(qd.ptr), ld, P(wqd.ptr), P(wkd.ptr), P(pd.ptr), P(fd.ptr), P(rq.ptr), P(rk.ptr),
           P(dqd.ptr), P(dkd.ptr), P(dvd.ptr), P(dqkv.ptr), P(dwq.ptr), P(dwk.ptr), 0, m, h, hk, P(ws.ptr), ws.nbytes,
           None)
    d_ref, dwq_ref, dwk_ref = oe.qknorm_rope_bwd(qkv, wq, wk, pos, freqs, h, hk, dq, dk, dv, 1e-5)
    assert_close(dqkv.float32(), d_ref, scaled=True, what="rope dqkv")
    assert_close(dwq.numpy(), dwq_ref, scaled=True, what="dwq")
    assert_close(dwk.numpy(), dwk_ref, scaled=True, what="dwk")


@pytest.mark.parametrize("c,b,t", [(1024, 2, 192), (256, 3, 100)])
def test_gated_conv_forward_and_backward(c, b, t):
    rng = np.random.default_rng(3)
    m = b * t
    bcx = rb(rng.standard_normal((m, 3 * c), dtype=F))
    taps = (0.5 * rng.standard_normal((c, 3))).astype(F)
    seg = _segments(rng, b, t)
    L = _lib()
    bd, td, sd = _dev(bcx, "bfloat16"), _dev(taps, "float32"), _dev(seg, "int32")
    mixed = _empty((m, c), "bfloat16")
    L.call("mfb_conv_fwd", P(bd.ptr), P(td.ptr), P(sd.ptr), P(mixed.ptr), m, t, c, None)
    np.testing.assert_array_equal(mixed.float32(), oe.gated_conv(bcx, taps, seg, t))
    dm = rb(rng.standard_normal((m, c), dtype=F))
    dmd, dbcx, dtaps = _dev(dm, "bfloat16"), _empty((m, 3 * c), "bfloat16"), _empty((c, 3), "float32")
    ws = _ws(L.lib().mfb_encoder_workspace_size(c, 2))
    L.call("mfb_conv_bwd", P(bd.ptr), P(td.ptr), P(sd.ptr), P(dmd.ptr), P(dbcx.ptr), P(dtaps.ptr), 0, m, t, c,
           P(ws.ptr), ws.nbytes, None)
    d_ref, dt_ref = oe.gated_conv_bwd(bcx, taps, seg, t, dm)
    assert_close(dbcx.float32(), d_ref, scaled=True, what="conv dbcx")
    assert_close(dtaps.numpy(), dt_ref, scaled=True, what="conv dtaps")


def test_embedding_gather_clamps_ids():
    rng = np.random.default_rng(4)
    table = rng.standard_normal((1000, 1024), dtype=F)
    ids = rng.integers(-5, 1010, 257).astype(np.int32)
    L = _lib()
    td, idd, out = _dev(table, "float32"), _dev(ids, "int32"), _empty((257, 1024), "bfloat16")
    L.call("mfb_embed_gather", P(td.ptr), P(idd.ptr), P(out.ptr), 257, 1024, 1000, None)
    np.testing.assert_array_equal(out.float32(), oe.embed(table, ids))


def test_head_loss_forward_and_backward():
    rng = np.random.default_rng(5)
    m, c, k = 777, 1024, 2
    e = rb(rng.standard_normal((m, c), dtype=F))
    w = (0.05 * rng.standard_normal((k, c))).astype(F)
    labels = rng.integers(0, k, m).astype(np.int32)
    valid = (rng.random(m) > 0.3).astype(np.int32)
    L = _lib()
    ed, wd, ld, vd = _dev(e, "bfloat16"), _dev(w, "float32"), _dev(labels, "int32"), _dev(valid, "int32")
    de, dw, lc = _empty((m, c), "bfloat16"), _empty((k, c), "float32"), _empty((2,), "float32")
    ws = _ws(L.lib().mfb_encoder_workspace_size(c, k))
    L.call("mfb_head_loss", P(ed.ptr), P(wd.ptr), P(ld.ptr), P(vd.ptr), P(de.ptr), P(dw.ptr), P(lc.ptr), m, c, k,
           P(ws.ptr), ws.nbytes, None)
    loss, count, de_ref, dw_ref = oe.head_loss(e, w, labels, valid)
    got = lc.numpy()
    np.testing.assert_allclose(got[0], loss, rtol=1e-4)
    assert got[1] == count
    assert_close(de.float32(), de_ref, scaled=True, what="head d_encoded")
    assert_close(dw.numpy(), dw_ref, scaled=True, what="head dW")
