"""Projection GEMM and the QAT SwiGLU FFN restated in NumPy (test infrastructure).

* ``full_linear``  src/minifield_training/kernels/linear.py:7-13 -- the FP32
  master is cast to the activation dtype *before* the dot
  (KAT: tests/kernels/test_linear.py:46-62); the weight gradient is the
  dot's transpose widened back to FP32.
* ``swiglu_ffn``   src/minifield_training/layers/feed_forward.py:24-35 -- the
  gate/up/down GEMM chain with SiLU(gate) * up between them. The benchmark
  configuration times the three QAT GEMMs and the SiLU product; the RMSNorm
  and residual of the full block are not part of that timed chain.
* QAT: ``strategies/quantization.py:114-126`` replaces each selected master by
  ``Quantizer.effective(master)``; the STE passes the effective weight's
  gradient to the master, multiplied by the quantizer's STE mask.

The oracle computes in FP64 (or FP32) from bf16-rounded operands. With
``bf16_casts=True`` (the default; the benchmark configurations run bf16
activations) it also rounds to bf16 where the reference's bf16 graph does:
``full_linear`` returns ``x.dtype`` (kernels/linear.py:9-13), so the gate/up
output, the SiLU product and, in the backward, dH and dGate/dUp (gradients of
bf16 tensors) are bf16 values; every product is still exact FP64 arithmetic.
"""

import numpy as np

from . import quant
from .bf16 import round_bf16


def full_linear(x: np.ndarray, weight: np.ndarray, dtype=np.float64) -> np.ndarray:
    """x @ bf16(weight).T accumulated in ``dtype``."""
    return np.matmul(np.asarray(x, dtype), round_bf16(weight).astype(dtype).T)


def silu(g):
    return g / (1.0 + np.exp(-g))


def silu_grad(g):
    s = 1.0 / (1.0 + np.exp(-g))
    return s * (1.0 + g * (1.0 - s))


def qat_weights(w_gate_up: np.ndarray, w_down: np.ndarray, kind: str):
    """Effective bf16-rounded weights and STE masks for the two QAT GEMMs."""
    _, _, ste_gu, eff_gu = quant.fake_quant(w_gate_up, kind)
    _, _, ste_d, eff_d = quant.fake_quant(w_down, kind)
    return round_bf16(eff_gu), ste_gu, round_bf16(eff_d), ste_d


def _cast(a, on, dtype):
    return round_bf16(a).astype(dtype) if on else a


def swiglu_qat_forward(x, w_gate_up, w_down, kind, dtype=np.float64, bf16_casts=True):
    """Return (y, gu, h): gu = x W_gu^T, h = silu(gate) * up, y = h W_d^T.

    ``w_gate_up`` is [2F, C] with the gate rows first; ``w_down`` is [C, F].
    ``h`` is rounded to bf16 before the down GEMM, the cast point of the
    reference's bf16 activations.
    """
    eff_gu, _, eff_d, _ = qat_weights(w_gate_up, w_down, kind)
    f = w_down.shape[1]
    xb = round_bf16(x).astype(dtype)
    gu = _cast(xb @ eff_gu.astype(dtype).T, bf16_casts, dtype)
    g, u = gu[:, :f], gu[:, f:]
    h = round_bf16(silu(g) * u).astype(dtype)
    y = h @ eff_d.astype(dtype).T
    return y, gu, h


def swiglu_qat_backward(x, w_gate_up, w_down, kind, d_y, dtype=np.float64, bf16_casts=True):
    """Return (dx, dw_gate_up, dw_down) of sum(y * d_y) with the STE masks."""
    eff_gu, ste_gu, eff_d, ste_d = qat_weights(w_gate_up, w_down, kind)
    f = w_down.shape[1]
    xb = round_bf16(x).astype(dtype)
    gu = _cast(xb @ eff_gu.astype(dtype).T, bf16_casts, dtype)
    g, u = gu[:, :f], gu[:, f:]
    h = round_bf16(silu(g) * u).astype(dtype)
    dy = round_bf16(d_y).astype(dtype)
    dh = _cast(dy @ eff_d.astype(dtype), bf16_casts, dtype)
    dw_down = (dy.T @ h) * ste_d
    dg = dh * u * silu_grad(g)
    du = dh * silu(g)
    dgu = _cast(np.concatenate((dg, du), axis=1), bf16_casts, dtype)
    dx = dgu @ eff_gu.astype(dtype)
    dw_gate_up = (dgu.T @ xb) * ste_gu
    return dx, dw_gate_up, dw_down


def swiglu_qat_step(x, w_gate_up, w_down, kind, d_y, dtype=np.float64, bf16_casts=True):
    """One forward + backward of the chain with each product computed once.

    Returns (y, gu, h, dx, dw_gate_up, dw_down): the values of
    ``swiglu_qat_forward`` and ``swiglu_qat_backward`` without the backward's
    recomputation of the forward products (what a training step runs).
    """
    eff_gu, ste_gu, eff_d, ste_d = qat_weights(w_gate_up, w_down, kind)
    f = w_down.shape[1]
    xb = round_bf16(x).astype(dtype)
    gu = _cast(xb @ eff_gu.astype(dtype).T, bf16_casts, dtype)
    g, u = gu[:, :f], gu[:, f:]
    h = round_bf16(silu(g) * u).astype(dtype)
    y = h @ eff_d.astype(dtype).T
    dy = round_bf16(d_y).astype(dtype)
    dh = _cast(dy @ eff_d.astype(dtype), bf16_casts, dtype)
    dw_down = (dy.T @ h) * ste_d
    dgu = _cast(np.concatenate((dh * u * silu_grad(g), dh * silu(g)), axis=1), bf16_casts, dtype)
    dx = dgu @ eff_gu.astype(dtype)
    dw_gate_up = (dgu.T @ xb) * ste_gu
    return y, gu, h, dx, dw_gate_up, dw_down


def swiglu_qat_weight_grad_columns(x, w_gate_up, w_down, kind, d_y, ffn_cols, dtype=np.float64):
    """Selected columns of the two weight gradients, from the oracle's own forward.

    For the FFN columns ``ffn_cols`` (indices into F) returns
    (dw_down[:, ffn_cols], dw_gate_up[ffn_cols], dw_gate_up[F + ffn_cols]) --
    exactly those entries of ``swiglu_qat_backward`` -- computing only the
    gate/up/h/dh columns they need, so a full-size batch stays cheap.
    """
    eff_gu, ste_gu, eff_d, ste_d = qat_weights(w_gate_up, w_down, kind)
    f = w_down.shape[1]
    cols = np.asarray(ffn_cols)
    xb = round_bf16(x).astype(dtype)
    dy = round_bf16(d_y).astype(dtype)
    g = round_bf16(xb @ eff_gu[cols].astype(dtype).T).astype(dtype)
    u = round_bf16(xb @ eff_gu[f + cols].astype(dtype).T).astype(dtype)
    h = round_bf16(silu(g) * u).astype(dtype)
    dh = round_bf16(dy @ eff_d[:, cols].astype(dtype)).astype(dtype)
    dw_down = (dy.T @ h) * ste_d[:, cols]
    dg = round_bf16(dh * u * silu_grad(g)).astype(dtype)
    du = round_bf16(dh * silu(g)).astype(dtype)
    return dw_down, (dg.T @ xb) * ste_gu[cols], (du.T @ xb) * ste_gu[f + cols]


def qat_linear_forward(x, weight, kind, dtype=np.float64):
    """``full_linear(x, effective(weight))`` for one QAT projection."""
    _, _, _, eff = quant.fake_quant(weight, kind)
    return full_linear(round_bf16(x), eff, dtype)


def qat_linear_backward(x, weight, kind, d_y, dtype=np.float64):
    """(dx, dw_master) for ``full_linear(x, effective(weight))``."""
    _, _, ste, eff = quant.fake_quant(weight, kind)
    dy = round_bf16(d_y).astype(dtype)
    dx = dy @ round_bf16(eff).astype(dtype)
    dw = (dy.T @ round_bf16(x).astype(dtype)) * ste
    return dx, dw


def ffn_flops(tokens: int, hidden: int, ffn: int) -> float:
    """Forward GEMM FLOPs of the gate/up + down chain (x3 for fwd+bwd)."""
    return 2.0 * tokens * hidden * (2 * ffn) + 2.0 * tokens * ffn * hidden
