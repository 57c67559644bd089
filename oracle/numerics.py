"""Bit-level helpers shared by the oracle modules (test infrastructure only)."""
from __future__ import annotations

import numpy as np


def bf16_round(values) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32.

    This is the value torch stores for ``tensor.to(torch.bfloat16)``."""
    x = np.ascontiguousarray(values, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32).reshape(x.shape)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def f16_round(values) -> np.ndarray:
    return np.asarray(values, dtype=np.float32).astype(np.float16).astype(np.float32)


def bf16_to_bits(values) -> np.ndarray:
    """fp32 values already on the bf16 grid -> uint16 bit patterns."""
    x = bf16_round(values)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def bits_to_bf16(bits) -> np.ndarray:
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


def max_rel_err(actual, expected) -> float:
    """Norm-wise relative error: max|a - e| / max(max|e|, tiny)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    denom = max(float(np.max(np.abs(e))) if e.size else 0.0, 1e-30)
    return float(np.max(np.abs(a - e))) / denom if e.size else 0.0
