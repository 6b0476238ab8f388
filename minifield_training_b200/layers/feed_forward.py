"""QAT SwiGLU feed-forward GEMM chain on B200.

Mirrors the GEMMs of ``swiglu_ffn`` (src/minifield_training/layers/
feed_forward.py:24-35) under QAT (strategies/quantization.py:114-126): each
projection master is fake-quantized, cast to bf16 and multiplied on the
tensor cores; the weight gradients pass through the STE mask in the GEMM
epilogue. ``w_gate_up`` is [2F, C] (gate rows, then up rows), ``w_down`` is
[C, F]. The SwiGLU product runs in the gate|up GEMM's epilogue and its
backward in the epilogue of the down projection's input gradient. The RMSNorm
and residual around the chain are not part of it.
"""

import ctypes
from dataclasses import dataclass
from typing import NamedTuple

from .. import _lib
from ..device import DeviceArray, as_device
from ..kernels.linear import gemm_nn, gemm_nt, gemm_tn
from ..kernels.quantization import effective_bf16


class FeedForwardWeights(NamedTuple):
    """Pre-norm gain and the three SwiGLU projection masters (feed_forward.py:11-21).

    FP32 masters (host or device) or bf16 device arrays: gate and up [F, C], down [C, F].
    """

    norm: object
    gate: object
    up: object
    down: object


@dataclass
class FfnResiduals:
    x: DeviceArray
    gu: DeviceArray
    h: DeviceArray
    w_gu: DeviceArray
    ste_gu: DeviceArray
    w_d: DeviceArray
    ste_d: DeviceArray


def quantize_weights(w_gate_up, w_down, kind, stream=None):
    w_gu, ste_gu = effective_bf16(w_gate_up, kind, stream)
    w_d, ste_d = effective_bf16(w_down, kind, stream)
    return w_gu, ste_gu, w_d, ste_d


def swiglu_qat_fwd(x, w_gate_up, w_down, kind, stream=None, weights=None):
    """(y [M, C] bf16, residuals). ``weights`` reuses quantize_weights() output."""
    xd = as_device(x, "bfloat16", stream)
    w_gu, ste_gu, w_d, ste_d = weights if weights is not None else quantize_weights(w_gate_up, w_down, kind, stream)
    m, c = xd.shape
    f = w_d.shape[1]
    gu = DeviceArray((m, 2 * f), "bfloat16")
    h = DeviceArray((m, f), "bfloat16")
    P = ctypes.c_void_p
    # gate|up GEMM with silu(gate) * up in its epilogue (gu kept for the backward)
    _lib.call("mfb_gemm_swiglu_fwd", P(xd.ptr), _lib.MAJOR_K, c, P(w_gu.ptr), c, P(gu.ptr), P(h.ptr), m, f, c,
              stream)
    y = gemm_nt(h, w_d, stream=stream)
    return y, FfnResiduals(xd, gu, h, w_gu, ste_gu, w_d, ste_d)


def swiglu_qat_bwd(res: FfnResiduals, d_y, stream=None):
    """(dx bf16 [M, C], dW_gate_up FP32 [2F, C], dW_down FP32 [C, F])."""
    dy = as_device(d_y, "bfloat16", stream)
    m, c = dy.shape
    f = res.w_d.shape[1]
    dw_d = gemm_tn(dy, res.h, "float32", mask=res.ste_d, stream=stream)
    dgu = DeviceArray((m, 2 * f), "bfloat16")
    P = ctypes.c_void_p
    # dH = dY . W_down with the SwiGLU backward in its epilogue (dH itself is never stored)
    _lib.call("mfb_gemm_swiglu_bwd", P(dy.ptr), _lib.MAJOR_K, c, P(res.w_d.ptr), _lib.MAJOR_MN, f, P(res.gu.ptr),
              P(dgu.ptr), m, f, c, stream)
    dx = gemm_nn(dgu, res.w_gu, stream=stream)
    dw_gu = gemm_tn(dgu, res.x, "float32", mask=res.ste_gu, stream=stream)
    return dx, dw_gu, dw_d
