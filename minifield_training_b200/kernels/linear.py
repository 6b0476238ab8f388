"""``full_linear`` on the tcgen05 GEMM.

Mirrors src/minifield_training/kernels/linear.py:7-13:
``full_linear(x, weight) = x @ weight.astype(x.dtype).T`` -- the FP32 master
is rounded to bf16 *before* the product (KAT tests/kernels/test_linear.py:46-62)
and the output is bf16. ``full_linear_bwd`` gives the two transposed
products: dx = dy @ W (bf16) and dW = dy^T @ x (FP32, optionally times the
QAT STE mask), both read in place (MN-major operands) without a transpose.
"""

import ctypes

from .. import _lib
from ..device import DeviceArray, as_device


def _gemm(a, a_major, lda, b, b_major, ldb, c, ldc, out_dtype, m, n, k, alpha=1.0, mask=None, stream=None,
          ws=None):
    p = ctypes.c_void_p
    _lib.call(
        "mfb_gemm_bf16_ws", p(a.ptr), a_major, lda, p(b.ptr), b_major, ldb, p(c.ptr), ldc, out_dtype, m, n, k,
        ctypes.c_float(alpha), p(mask.ptr) if mask is not None else None, 0, p(ws.ptr) if ws is not None else None,
        ws.nbytes if ws is not None else 0, stream,
    )


def gemm_nt(a: DeviceArray, b: DeviceArray, out_dtype="bfloat16", stream=None) -> DeviceArray:
    """C[M,N] = A[M,K] . B[N,K]^T (both K-major)."""
    m, k = a.shape
    n = b.shape[0]
    c = DeviceArray((m, n), out_dtype)
    _gemm(a, _lib.MAJOR_K, k, b, _lib.MAJOR_K, k, c, n, _lib.DTYPE_BF16 if out_dtype == "bfloat16" else _lib.DTYPE_F32,
          m, n, k, stream=stream)
    return c


def gemm_nn(a: DeviceArray, b: DeviceArray, out_dtype="bfloat16", stream=None) -> DeviceArray:
    """C[M,N] = A[M,K] . B[K,N] (B read MN-major in place)."""
    m, k = a.shape
    n = b.shape[1]
    c = DeviceArray((m, n), out_dtype)
    _gemm(a, _lib.MAJOR_K, k, b, _lib.MAJOR_MN, n, c, n, _lib.DTYPE_BF16 if out_dtype == "bfloat16" else _lib.DTYPE_F32,
          m, n, k, stream=stream)
    return c


def gemm_tn(a: DeviceArray, b: DeviceArray, out_dtype="float32", mask=None, stream=None) -> DeviceArray:
    """C[M,N] = A[K,M]^T . B[K,N] (both read MN-major in place), optional mask. The weight
    gradient: few output tiles over a deep K (the tokens), so K is split through a workspace
    when that fills the GPU better (its release waits for the product)."""
    k, m = a.shape
    n = b.shape[1]
    c = DeviceArray((m, n), out_dtype)
    need = int(_lib.lib().mfb_gemm_workspace_size(m, n, k))
    ws = DeviceArray((need,), "uint8") if need else None
    _gemm(a, _lib.MAJOR_MN, m, b, _lib.MAJOR_MN, n, c, n, _lib.DTYPE_BF16 if out_dtype == "bfloat16" else _lib.DTYPE_F32,
          m, n, k, mask=mask, stream=stream, ws=ws)
    return c


def cast_bf16(x: DeviceArray, stream=None) -> DeviceArray:
    y = DeviceArray(x.shape, "bfloat16")
    _lib.call("mfb_cast_f32_bf16", ctypes.c_void_p(x.ptr), ctypes.c_void_p(y.ptr), x.size, stream)
    return y


def _weight_bf16(weight, stream=None) -> DeviceArray:
    if isinstance(weight, DeviceArray) and weight.dtype == "bfloat16":
        return weight
    return cast_bf16(as_device(weight, "float32", stream), stream)


def full_linear(x, weight, stream=None) -> DeviceArray:
    """x [..., K] bf16, weight [N, K] (FP32 master or bf16) -> [..., N] bf16."""
    xd = as_device(x, "bfloat16", stream)
    w = _weight_bf16(weight, stream)
    if w.ndim != 2 or xd.shape[-1] != w.shape[1]:
        raise ValueError("full_linear: x [..., K] and weight [N, K] are incompatible")
    lead = xd.shape[:-1]
    y = gemm_nt(xd.reshape(-1, w.shape[1]), w, stream=stream)
    return y.reshape(*lead, w.shape[0])


def full_linear_bwd(x, weight, d_y, ste_mask=None, stream=None):
    """(dx bf16 [..., K], dW FP32 [N, K]) for y = full_linear(x, weight)."""
    xd = as_device(x, "bfloat16", stream)
    w = _weight_bf16(weight, stream)
    dy = as_device(d_y, "bfloat16", stream)
    n, k = w.shape
    lead = xd.shape[:-1]
    x2 = xd.reshape(-1, k)
    dy2 = dy.reshape(-1, n)
    dx = gemm_nn(dy2, w, stream=stream).reshape(*lead, k)
    dw = gemm_tn(dy2, x2, "float32", mask=ste_mask, stream=stream)
    return dx, dw
