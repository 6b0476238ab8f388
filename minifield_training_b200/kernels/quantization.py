"""Fake quantizers on B200 behind the reference's ``Quantizer`` protocol.

Mirrors src/minifield_training/kernels/quantization.py: ``Quantizer``
(:11-22: ``identity``, ``effective(weight)``, ``validate_shape(shape)``) and
``Group128Quantizer`` (:107-134) for the reference kinds
``ternary-g128-absmax-f16-v1`` / ``nf4-g128-absmax-f16-v1``, plus
``SymmetricQuantizer`` for the benchmark's ``int8-channel-absmax-v1`` and
``int4-g128-absmax-v1`` kinds (no reference implementation). ``effective``
returns the decoded FP32 weight; ``quantize`` returns every kernel output
(codes, scales, STE mask, FP32 and bf16 decoded weights); the backward of
``effective`` is ``grad * ste`` (identity for the reference kinds).
"""

import ctypes
from dataclasses import dataclass
from typing import Protocol

import numpy as np

from .. import _lib
from ..device import DeviceArray, as_device

REFERENCE_KINDS = ("ternary-g128-absmax-f16-v1", "nf4-g128-absmax-f16-v1")
SYMMETRIC_KINDS = ("int8-channel-absmax-v1", "int4-g128-absmax-v1")


class Quantizer(Protocol):
    @property
    def identity(self) -> str: ...

    def effective(self, weight) -> DeviceArray: ...

    def validate_shape(self, shape) -> None: ...


@dataclass
class Quantized:
    codes: DeviceArray
    scales: DeviceArray
    ste: DeviceArray
    effective: DeviceArray
    effective_bf16: DeviceArray


def _master(weight, stream=None) -> DeviceArray:
    if isinstance(weight, DeviceArray):
        if weight.dtype != "float32":
            raise ValueError("Quantized master must be FP32")
        return weight
    w = np.asarray(weight)
    if w.dtype != np.float32:
        raise ValueError("Quantized master must be FP32")
    return as_device(w, "float32", stream)


def fake_quant(weight, kind: str, stream=None) -> Quantized:
    """Run the fake-quant kernel for ``kind`` on an FP32 master [rows, cols]."""
    if kind not in _lib.QUANT_KINDS:
        raise ValueError("Unknown quantizer")
    w = _master(weight, stream)
    if w.ndim != 2 or 0 in w.shape or (kind != "int8-channel-absmax-v1" and w.shape[1] % 128):
        raise ValueError("Quantized matrix requires rank 2 and K divisible by 128")
    rows, cols = w.shape
    groups = 1 if kind == "int8-channel-absmax-v1" else cols // 128
    out = Quantized(
        DeviceArray((rows, cols), "int8"),
        DeviceArray((rows, groups), "float32"),
        DeviceArray((rows, cols), "uint8"),
        DeviceArray((rows, cols), "float32"),
        DeviceArray((rows, cols), "bfloat16"),
    )
    p = ctypes.c_void_p
    _lib.call(
        "mfb_fakequant", p(w.ptr), _lib.QUANT_KINDS[kind], rows, cols, p(out.codes.ptr), p(out.scales.ptr),
        p(out.ste.ptr), p(out.effective.ptr), p(out.effective_bf16.ptr), stream,
    )
    return out


def effective_bf16(weight, kind: str, stream=None):
    """(decoded weight cast to bf16, STE mask) -- what the QAT GEMMs consume."""
    if kind not in _lib.QUANT_KINDS:
        raise ValueError("Unknown quantizer")
    w = _master(weight, stream)
    rows, cols = w.shape
    eff = DeviceArray((rows, cols), "bfloat16")
    ste = DeviceArray((rows, cols), "uint8")
    p = ctypes.c_void_p
    _lib.call("mfb_fakequant", p(w.ptr), _lib.QUANT_KINDS[kind], rows, cols, None, None, p(ste.ptr), None,
              p(eff.ptr), stream)
    return eff, ste


class _Base:
    def __init__(self, kind: str, allowed):
        if kind not in allowed:
            raise ValueError("Unknown group-128 quantizer" if allowed is REFERENCE_KINDS else "Unknown quantizer")
        self._kind = kind

    @property
    def identity(self) -> str:
        return self._kind

    def quantize(self, weight, stream=None) -> Quantized:
        return fake_quant(weight, self._kind, stream)

    def effective(self, weight, stream=None) -> DeviceArray:
        return fake_quant(weight, self._kind, stream).effective


class Group128Quantizer(_Base):
    """Reference ternary / NF4 g128 with FP16-stored scales and identity STE."""

    def __init__(self, kind: str):
        super().__init__(kind, REFERENCE_KINDS)

    def validate_shape(self, shape) -> None:
        if len(shape) != 2 or 0 in shape or shape[1] % 128:
            raise ValueError("Group-128 quantizer needs a complete matrix")


class SymmetricQuantizer(_Base):
    """Symmetric int8 per-output-channel or int4 group-128 absmax fake quant."""

    def __init__(self, kind: str):
        super().__init__(kind, SYMMETRIC_KINDS)

    def validate_shape(self, shape) -> None:
        if len(shape) != 2 or 0 in shape:
            raise ValueError("Quantized matrix requires rank 2")
        if self._kind == "int4-g128-absmax-v1" and shape[1] % 128:
            raise ValueError("Group-128 quantizer needs a complete matrix")


def make_quantizer(kind: str):
    return Group128Quantizer(kind) if kind in REFERENCE_KINDS else SymmetricQuantizer(kind)
