"""tcgen05 GEMM and the QAT SwiGLU FFN chain vs the oracle."""

import numpy as np
import pytest

from oracle import linear as olin
from oracle import quant as oq
from oracle.bf16 import round_bf16
from tests._util import assert_close, report_errors
from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


def _dev(x, dtype="bfloat16"):
    from minifield_training_b200.device import DeviceArray

    return DeviceArray.from_numpy(x, dtype)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (296, 520, 200), (1000, 768, 1024), (64, 40, 136)])
@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_gemm_all_majors(m, n, k, a_mn, b_mn):
    from minifield_training_b200 import _lib
    from minifield_training_b200.device import DeviceArray
    from minifield_training_b200.kernels.linear import _gemm

    rng = np.random.default_rng(m * 7 + n + k + 3 * a_mn + b_mn)
    a = round_bf16(rng.standard_normal((m, k), dtype=np.float32))
    b = round_bf16(rng.standard_normal((n, k), dtype=np.float32))
    ka = np.ascontiguousarray(a.T) if a_mn else a
    kb = np.ascontiguousarray(b.T) if b_mn else b
    ad, bd = _dev(ka), _dev(kb)
    for out_dtype, code in (("float32", _lib.DTYPE_F32), ("bfloat16", _lib.DTYPE_BF16)):
        ldc = n + 3  # unaligned output rows exercise the scalar-store epilogue
        c = DeviceArray((m, ldc), out_dtype)
        _gemm(ad, a_mn, ka.shape[1], bd, b_mn, kb.shape[1], c, ldc, code, m, n, k)
        got = c.float32()[:, :n]
        ref = a.astype(np.float64) @ b.astype(np.float64).T
        if out_dtype == "float32":
            np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-4 * np.sqrt(k))
        else:
            assert_close(got, ref, scaled=True, what="bf16 gemm")
    code = np.zeros(1, np.int32)
    from minifield_training_b200 import _lib as L
    import ctypes

    st = ctypes.c_int()
    L.call("mfb_gemm_status", ctypes.byref(st))
    assert st.value == 0


def test_full_linear_reference_kats(golden):
    """KATs of tests/kernels/test_linear.py, zero-padded to the TMA's 8-element
    stride granularity (padding rows/columns are zero, so the sums are unchanged)."""
    from minifield_training_b200.kernels.linear import full_linear, full_linear_bwd

    x = np.zeros((8, 64), np.float32)
    x[0, :2] = golden["linear_cast_x"][0]
    w = np.zeros((8, 64), np.float32)
    w[0, :2] = golden["linear_cast_w"][0]
    y = full_linear(x, w)
    np.testing.assert_array_equal(y.float32()[:1, :1], golden["linear_cast_out"])
    dy = np.zeros((8, 8), np.float32)
    dy[0, 0] = 1.0
    dx, dw = full_linear_bwd(x, w, dy)
    np.testing.assert_array_equal(dx.float32()[:1, :2], golden["linear_cast_dx"])
    np.testing.assert_array_equal(dw.float32()[:1, :2], golden["linear_cast_dw"])
    gx, gw, probe = golden["linear_x"], golden["linear_w"], golden["linear_probe"]
    xp = np.zeros((8, 64), np.float32)
    xp[:2, :2] = gx.reshape(2, 2)
    wp = np.zeros((8, 64), np.float32)
    wp[:2, :2] = gw
    np.testing.assert_array_equal(full_linear(xp, wp).float32()[:2, :2], golden["linear_out"].reshape(2, 2))
    dyp = np.zeros((8, 8), np.float32)
    dyp[:2, :2] = probe.reshape(2, 2)
    dx, dw = full_linear_bwd(xp, wp, dyp)
    np.testing.assert_array_equal(dx.float32()[:2, :2], golden["linear_dx"].reshape(2, 2))
    np.testing.assert_array_equal(dw.float32()[:2, :2], golden["linear_dw"])


def test_gemm_rejects_unaligned_tma_strides():
    from minifield_training_b200.kernels.linear import gemm_tn

    a = _dev(np.zeros((16, 300), np.float32))
    b = _dev(np.zeros((16, 64), np.float32))
    with pytest.raises(ValueError, match="multiples of 8"):
        gemm_tn(a, b)


@pytest.mark.parametrize("kind", [oq.KIND_INT8_CHANNEL, oq.KIND_INT4_G128, oq.KIND_NF4_G128])
def test_swiglu_qat_small(kind):
    from minifield_training_b200.layers.feed_forward import swiglu_qat_bwd, swiglu_qat_fwd

    rng = np.random.default_rng(17)
    m, c, f = 384, 256, 640
    x = rng.standard_normal((m, c), dtype=np.float32)
    w_gu = (rng.standard_normal((2 * f, c)) * 0.05).astype(np.float32)
    w_d = (rng.standard_normal((c, f)) * 0.05).astype(np.float32)
    dy = rng.standard_normal((m, c), dtype=np.float32)
    y, res = swiglu_qat_fwd(x, w_gu, w_d, kind)
    dx, dwgu, dwd = swiglu_qat_bwd(res, dy)
    ry, _, _ = olin.swiglu_qat_forward(x, w_gu, w_d, kind)
    rdx, rdwgu, rdwd = olin.swiglu_qat_backward(x, w_gu, w_d, kind, dy)
    assert_close(y.float32(), ry, scaled=True, what="y")
    assert_close(dx.float32(), rdx, scaled=True, what="dx")
    assert_close(dwgu.float32(), rdwgu, scaled=True, what="dW_gate_up")
    assert_close(dwd.float32(), rdwd, scaled=True, what="dW_down")


@pytest.mark.parametrize("kind", ["int8-channel-absmax-v1", "int4-g128-absmax-v1"])
def test_swiglu_qat_config4_full_size(kind):
    """Full config-4 shapes, both quantizer kinds, every checked value from the oracle: forward and
    dX rows, and dW_down / dW_gate_up columns from the oracle's own gate/up and SwiGLU intermediates
    over all 16384 tokens."""
    from minifield_training_b200 import workloads
    from minifield_training_b200.layers.feed_forward import swiglu_qat_bwd, swiglu_qat_fwd

    cfg = workloads.CONFIG4
    x, w_gu, w_d, dy = workloads.qat_inputs(cfg, seed=0)
    y, res = swiglu_qat_fwd(x, w_gu, w_d, kind)
    dx, dwgu, dwd = swiglu_qat_bwd(res, dy)
    rows = np.arange(0, cfg.tokens, 997)
    ry, _, _ = olin.swiglu_qat_forward(x[rows], w_gu, w_d, kind, dtype=np.float32)
    assert_close(y.float32()[rows], ry, scaled=True, what=f"cfg4 {kind} y rows")
    rdx, _, _ = olin.swiglu_qat_backward(x[rows], w_gu, w_d, kind, dy[rows], dtype=np.float32)
    assert_close(dx.float32()[rows], rdx, scaled=True, what=f"cfg4 {kind} dx rows")
    cols = np.arange(0, cfg.ffn, 331)
    rdwd, rdg, rdu = olin.swiglu_qat_weight_grad_columns(x, w_gu, w_d, kind, dy, cols, dtype=np.float32)
    dwd_h, dwgu_h = dwd.float32(), dwgu.float32()
    assert_close(dwd_h[:, cols], rdwd, scaled=True, what=f"cfg4 {kind} dW_down cols")
    assert_close(dwgu_h[cols], rdg, scaled=True, what=f"cfg4 {kind} dW_gate rows")
    assert_close(dwgu_h[cfg.ffn + cols], rdu, scaled=True, what=f"cfg4 {kind} dW_up rows")
    for what, a, e in (("dW_down", dwd_h[:, cols], rdwd), ("dW_gate", dwgu_h[cols], rdg),
                       ("dW_up", dwgu_h[cfg.ffn + cols], rdu), ("y", y.float32()[rows], ry),
                       ("dx", dx.float32()[rows], rdx)):
        report_errors(f"cfg4 {kind} {what}", a, e)


@pytest.mark.parametrize("m,n,k", [(64, 1024, 6656), (64, 3072, 1024), (1, 1024, 1024), (100, 520, 200),
                                   (64, 13312, 1024)])
@pytest.mark.parametrize("ws_fraction", [1.0, 0.3])
def test_split_k_gemm_for_small_m(m, n, k, ws_fraction):
    """mfb_gemm_bf16_ws: K-sliced partials summed in slice order (deterministic), any workspace size,
    launched plainly and as a programmatic dependent (MFB_GEMM_PDL) with the same result."""
    import ctypes

    from minifield_training_b200 import _lib as L
    from minifield_training_b200.device import DeviceArray

    rng = np.random.default_rng(m + n + k)
    a = round_bf16(rng.standard_normal((m, k), dtype=np.float32))
    b = round_bf16(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.05))
    ad, bd = _dev(a), _dev(b)
    need = int(L.lib().mfb_gemm_workspace_size(m, n, k))
    ws = DeviceArray((max(16, int(need * ws_fraction) // 16 * 16),), "uint8")
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    stream = ctypes.c_void_p()
    L.call("mfb_stream_create", ctypes.byref(stream))
    for out_dtype, code in (("float32", L.DTYPE_F32), ("bfloat16", L.DTYPE_BF16)):
        outs = []
        for flags, s in ((0, None), (L.GEMM_PDL, stream)):  # plain, then as a programmatic dependent
            c = DeviceArray((m, n), out_dtype)
            L.call("mfb_gemm_bf16_ws", ctypes.c_void_p(ad.ptr), L.MAJOR_K, k, ctypes.c_void_p(bd.ptr), L.MAJOR_K, k,
                   ctypes.c_void_p(c.ptr), n, code, m, n, k, ctypes.c_float(0.5), None, flags,
                   ctypes.c_void_p(ws.ptr), ws.nbytes, s)
            L.call("mfb_stream_sync", s)
            outs.append(c.float32())
        np.testing.assert_array_equal(outs[0], outs[1])  # deterministic slice order
        if out_dtype == "float32":
            np.testing.assert_allclose(outs[0], 0.5 * ref, rtol=1e-5, atol=1e-4 * np.sqrt(k))
        else:
            assert_close(outs[0], 0.5 * ref, scaled=True, what="split-K bf16 gemm")
    L.call("mfb_stream_destroy", stream)
    st = ctypes.c_int()
    L.call("mfb_gemm_status", ctypes.byref(st))
    assert st.value == 0


def test_split_k_workspace_is_needed_only_for_few_tiles():
    from minifield_training_b200 import _lib as L

    assert L.lib().mfb_gemm_workspace_size(64, 1024, 6656) > 0
    assert L.lib().mfb_gemm_workspace_size(16384, 13312, 1024) == 0  # enough tiles: no split
    assert L.lib().mfb_gemm_workspace_size(64, 1024, 64) == 0  # one k-block: nothing to split
    # A 64-row product runs swapped: the 13312 weight rows give 104 tiles, no split.
    assert L.lib().mfb_gemm_workspace_size(64, 13312, 1024) == 0
    # Weight gradients over 65536 tokens: 16 and 104 pair tiles get K slices.
    assert L.lib().mfb_gemm_workspace_size(1024, 1024, 65536) > 0
    assert L.lib().mfb_gemm_workspace_size(1024, 6656, 65536) > 0


@pytest.mark.parametrize("m,n,k", [(1024, 1024, 8192), (520, 776, 4100)])
def test_split_k_weight_gradient_on_pairs(m, n, k):
    """The weight-gradient layout (dW = dY^T X: both operands MN-major, FP32 out, STE mask) on CTA
    pairs with K slices: equal to the FP64 product within FP32 summation noise, to the unsplit
    product within the same, and deterministic across calls."""
    import ctypes

    from minifield_training_b200 import _lib as L
    from minifield_training_b200.device import DeviceArray

    rng = np.random.default_rng(m + n + k)
    dy = round_bf16(rng.standard_normal((k, m), dtype=np.float32))  # [tokens, out]
    x = round_bf16(rng.standard_normal((k, n), dtype=np.float32))   # [tokens, in]
    mask = (rng.random((m, n)) > 0.1).astype(np.uint8)
    dyd, xd = _dev(dy), _dev(x)
    md = DeviceArray.from_numpy(mask, "uint8")
    need = int(L.lib().mfb_gemm_workspace_size(m, n, k))
    assert need > 0
    ws = DeviceArray((need,), "uint8")
    ref = (dy.astype(np.float64).T @ x.astype(np.float64)) * mask

    def run(workspace):
        c = DeviceArray((m, n), "float32")
        L.call("mfb_gemm_bf16_ws", ctypes.c_void_p(dyd.ptr), L.MAJOR_MN, m, ctypes.c_void_p(xd.ptr), L.MAJOR_MN, n,
               ctypes.c_void_p(c.ptr), n, L.DTYPE_F32, m, n, k, ctypes.c_float(1.0), ctypes.c_void_p(md.ptr), 0,
               ctypes.c_void_p(workspace.ptr) if workspace is not None else None,
               workspace.nbytes if workspace is not None else 0, None)
        return c.float32()

    split_a, split_b, whole = run(ws), run(ws), run(None)
    np.testing.assert_array_equal(split_a, split_b)
    tol = 1e-4 * np.sqrt(k)
    np.testing.assert_allclose(split_a, ref, rtol=1e-5, atol=tol)
    np.testing.assert_allclose(split_a, whole, rtol=1e-5, atol=tol)
    assert np.all(split_a[mask == 0] == 0)
    st = ctypes.c_int()
    L.call("mfb_gemm_status", ctypes.byref(st))
    assert st.value == 0
