"""W8A8 oracle (test infrastructure only).

Follows engine/kernels/w8a8.py:67-125 (`w8a8_matmul`) and :33-64 (`_int8_gemm`):
per-token dynamic activation scale amax/127 (0 -> 1), codes = round_half_even(x / scale)
clamped to ±127, exact int32 accumulation, then ``acc * act_scale * weight_scale`` in fp32
(left to right). Optional exact fp32 side path for protected (outlier) columns.
"""
from __future__ import annotations

import numpy as np


def quantize_activations(x: np.ndarray, keep: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    src = np.asarray(x, np.float32)
    if keep is not None:
        src = (src * np.asarray(keep, np.float32)).astype(np.float32)
    act_scale = (np.abs(src).max(axis=1, keepdims=True) / np.float32(127.0)).astype(np.float32)
    act_scale = np.where(act_scale == 0, np.float32(1.0), act_scale).astype(np.float32)
    codes = np.round(src / act_scale).clip(-127, 127).astype(np.int8)
    return codes, act_scale


def int8_gemm(qx: np.ndarray, qw: np.ndarray) -> np.ndarray:
    """[T, in] int8 @ [out, in] int8 -> [T, out] int32, exact."""
    acc = qx.astype(np.int64) @ qw.astype(np.int64).T
    return acc.astype(np.int32)


def protect_columns(x: np.ndarray, k: int) -> np.ndarray:
    """Top-k columns by column max-abs (descending; ties -> lower column first)."""
    col_max = np.abs(np.asarray(x, np.float32)).max(axis=0)
    k = min(int(k), col_max.shape[0])
    order = np.argsort(-col_max, kind="stable")
    return order[:k]


def w8a8_matmul(qw, sw, x, *, protect_idx=None, protect_k: int = 0) -> np.ndarray:
    x2 = np.asarray(x, np.float32).reshape(-1, np.asarray(x).shape[-1])
    qw = np.asarray(qw, np.int8)
    sw = np.asarray(sw, np.float32)
    if protect_idx is None and protect_k > 0:
        protect_idx = protect_columns(x2, protect_k)
    y = np.zeros((x2.shape[0], qw.shape[0]), np.float32)
    keep = None
    if protect_idx is not None and len(protect_idx):
        idx = np.asarray(protect_idx, np.int64)
        wp = qw[:, idx].astype(np.float32) * sw[:, None]
        y = y + x2[:, idx] @ wp.T
        keep = np.ones(x2.shape[1], np.float32)
        keep[idx] = 0.0
    qx, act_scale = quantize_activations(x2, keep)
    acc = int8_gemm(qx, qw)
    y = y + (acc.astype(np.float32) * act_scale * sw[None, :]).astype(np.float32)
    return y.astype(np.float32).reshape(*np.asarray(x).shape[:-1], qw.shape[0])
