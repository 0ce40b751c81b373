"""Rounding helpers so numpy float32 arrays can stand in for bf16 / fp16 tensors.

The reference casts fp32 results to the input dtype with torch's
round-to-nearest-even conversion (``.to(x.dtype)`` in
``flashdec/paged_reference.py:123`` and ``flashdec/rope.py:81``).  These
helpers perform the same rounding on float32 arrays and return float32 arrays
whose values are exactly representable in the target type.
"""

from __future__ import annotations

import numpy as np


def bf16_round(x) -> np.ndarray:
    """Round float32 values to bfloat16 (round to nearest, ties to even).

    NaN stays NaN (quiet); infinities and overflow behave like torch's cast.
    """
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) >> 16) << 16
    out = (rounded & 0xFFFFFFFF).astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.float32("nan")
    return out


def fp16_round(x) -> np.ndarray:
    """Round float32 values to float16 (numpy's cast is round-to-nearest-even)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to_dtype(x, dtype: str) -> np.ndarray:
    """Round to ``dtype`` in {"float32", "float16", "bfloat16"}; returns float32."""
    if dtype == "float32":
        return np.asarray(x, dtype=np.float32).copy()
    if dtype == "float16":
        return fp16_round(x)
    if dtype == "bfloat16":
        return bf16_round(x)
    raise ValueError(f"unsupported dtype {dtype!r}")


def bf16_bits(x) -> np.ndarray:
    """Return the uint16 bit pattern of bf16-representable float32 values."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    return (a.view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits) -> np.ndarray:
    """Inverse of :func:`bf16_bits`."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)
