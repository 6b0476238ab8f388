"""Fake quantizers restated in NumPy (test infrastructure only).

Reference kinds (``src/minifield_training/kernels/quantization.py``):

* ``_groups``   :68-79  -- rank-2 FP32 master, K % 128 == 0, absmax per
                            128-column group, scale stored as FP16 then widened.
* ``_decoded``  :82-104 -- ternary: +-1 where |w| >= 0.5 * scale (ties away),
                            NF4: code = number of transitions <= w / scale.
* ``_nf4_transitions`` :46-61 -- first FP32 value above each exact midpoint.
* ``Group128Quantizer.effective`` :124-129 -- identity STE.

New kinds stated by the benchmark definition (no reference implementation,
parity unpinned): symmetric int8 per output channel (scale = max|w_row| / 127)
and symmetric int4 per 128-column group (scale = max|w_group| / 7). Codes are
``clamp(rint_half_even(w / scale), -qmax, qmax)``; the STE mask is 1 where the
clamp is inactive (``rint(w / scale)`` already inside the range); a zero scale
gives code 0, mask 1 and a zero decoded value, mirroring ``quantization.py:86``.
All arithmetic is FP32 with IEEE correctly rounded division, so the CUDA
kernel must agree bit for bit.
"""

import numpy as np

KIND_INT8_CHANNEL = "int8-channel-absmax-v1"
KIND_INT4_G128 = "int4-g128-absmax-v1"
KIND_TERNARY_G128 = "ternary-g128-absmax-f16-v1"
KIND_NF4_G128 = "nf4-g128-absmax-f16-v1"
KINDS = (KIND_INT8_CHANNEL, KIND_INT4_G128, KIND_TERNARY_G128, KIND_NF4_G128)

NF4_LEVELS = np.asarray(
    (
        -1.0,
        -0.6961928009986877,
        -0.5250730514526367,
        -0.39491748809814453,
        -0.28444138169288635,
        -0.18477343022823334,
        -0.09105003625154495,
        0.0,
        0.07958029955625534,
        0.16093020141124725,
        0.24611230194568634,
        0.33791524171829224,
        0.44070982933044434,
        0.5626170039176941,
        0.7229568362236023,
        1.0,
    ),
    dtype=np.float32,
)


def nf4_transitions() -> np.ndarray:
    """First FP32 value at or above each exact level midpoint (quantization.py:46-61)."""
    out = []
    levels = [float(x) for x in NF4_LEVELS]
    for left, right in zip(levels[:-1], levels[1:]):
        midpoint = (left + right) * 0.5
        rounded = np.float32(midpoint)
        if float(rounded) <= midpoint:
            rounded = np.nextafter(rounded, np.float32(np.inf))
        out.append(rounded)
    return np.asarray(out, np.float32)


NF4_TRANSITIONS = nf4_transitions()


def group_size(kind: str, cols: int) -> int:
    return cols if kind == KIND_INT8_CHANNEL else 128


def validate_shape(kind: str, shape) -> None:
    if kind not in KINDS:
        raise ValueError("Unknown quantizer")
    if len(shape) != 2 or 0 in shape:
        raise ValueError("Quantized matrix requires rank 2")
    if kind != KIND_INT8_CHANNEL and shape[1] % 128:
        raise ValueError("Quantized matrix requires rank 2 and K divisible by 128")


def fake_quant(weight: np.ndarray, kind: str):
    """Return (codes int8, scales f32 [rows, groups], ste uint8, effective f32)."""
    w = np.asarray(weight)
    if w.dtype != np.float32:
        raise ValueError("Quantized master must be FP32")
    validate_shape(kind, w.shape)
    rows, cols = w.shape
    g = group_size(kind, cols)
    grouped = w.reshape(rows, cols // g, g)
    absmax = np.max(np.abs(grouped), axis=-1, keepdims=True)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        if kind in (KIND_INT8_CHANNEL, KIND_INT4_G128):
            qmax = np.float32(127 if kind == KIND_INT8_CHANNEL else 7)
            scale = (absmax / qmax).astype(np.float32)
            ratio = np.where(scale == 0, np.float32(0), grouped / scale).astype(np.float32)
            rounded = np.rint(ratio)
            codes = np.clip(rounded, -qmax, qmax)
            ste = (rounded == codes)
            values = codes.astype(np.float32)
        else:
            scale = absmax.astype(np.float16).astype(np.float32)
            if kind == KIND_TERNARY_G128:
                threshold = np.float32(0.5) * scale
                codes = np.where(
                    scale == 0,
                    0,
                    np.where(grouped >= threshold, 1, np.where(grouped <= -threshold, -1, 0)),
                ).astype(np.float32)
                values = codes
            else:
                normalized = np.where(scale == 0, np.float32(0), grouped / scale).astype(np.float32)
                codes = np.zeros(normalized.shape, np.int32)
                for threshold in NF4_TRANSITIONS:
                    codes += (normalized >= threshold).astype(np.int32)
                values = NF4_LEVELS[codes]
                codes = codes.astype(np.float32)
            ste = np.ones(grouped.shape, bool)
        effective = (values * scale).astype(np.float32)
    return (
        codes.astype(np.int8).reshape(rows, cols),
        scale.reshape(rows, cols // g).astype(np.float32),
        ste.astype(np.uint8).reshape(rows, cols),
        effective.reshape(rows, cols),
    )


def effective(weight: np.ndarray, kind: str) -> np.ndarray:
    """Decoded FP32 weight (``Quantizer.effective`` forward value)."""
    return fake_quant(weight, kind)[3]
