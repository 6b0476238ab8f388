"""bfloat16 rounding helpers for the oracle (test infrastructure only).

JAX's ``astype(jnp.bfloat16)`` rounds FP32 to nearest, ties to even; so does
``ml_dtypes.bfloat16``. These helpers give the oracle the same cast points as
the reference (``kernels/linear.py:11`` casts the master before the dot;
``kernels/attention.py:31`` casts probabilities to the query dtype).
"""

import ml_dtypes
import numpy as np

BF16 = ml_dtypes.bfloat16


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round to bfloat16 (RNE) and return FP32 values."""
    return np.asarray(x, np.float32).astype(BF16).astype(np.float32)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round to bfloat16 (RNE) and return the raw uint16 payload."""
    return np.asarray(x, np.float32).astype(BF16).view(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    """Interpret uint16 payloads as bfloat16 and widen to FP32."""
    return np.asarray(bits, np.uint16).view(BF16).astype(np.float32)
