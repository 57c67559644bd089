"""QStore int8 linear oracle (test infrastructure only).

References (mrun project paths):
  * quantiser        engine/kernels/qstore_build.py:496-501   `_quant_row_int8`
  * fp32 dequant     engine/kernels/qstore.py:385-399          `_dequant_qrow`
  * fp32 matmul      engine/kernels/qstore.py:1082-1092        `QStore.matmul`
  * W8A16 contract   engine/kernels/dense_qstore_cuda.py:1003-1013 `dequantized_reference_matmul`
  * paired SwiGLU    engine/kernels/dense_qstore_cuda.py:1037-1049 `fused_qrow_swiglu_reference`
  * residual RMSNorm engine/kernels/dense_qstore_cuda.py:1390-1408
  * RMSNorm          engine/kernels/dense_qstore_cuda.py:1462-1470
  * embed rows       engine/kernels/qstore.py:1099-1128         `QStore.embed_rows`
  * exact head       engine/dense_qstore_cuda.py:838-896        streamed fp32 head + argmax
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_round


def quant_row_int8(weight: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-row symmetric int8: scale = max|w|/127 (0 -> 1), code = rint(w/scale) clip ±127."""
    w = np.asarray(weight, dtype=np.float32)
    scale = np.abs(w).max(axis=1, keepdims=True) / np.float32(127.0)
    scale = np.where(scale == 0.0, np.float32(1.0), scale).astype(np.float32)
    codes = np.round(w / scale).clip(-127, 127).astype(np.int8)
    return codes, scale[:, 0].astype(np.float32)


def dequant_qrow(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """int8 [out, in] * fp32 [out] -> fp32 [out, in] (exact widen, one fp32 multiply)."""
    return codes.astype(np.float32) * np.asarray(scales, np.float32)[:, None]


def qrow_matmul_fp32(x: np.ndarray, codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """``QStore.matmul`` on CPU: x fp32 @ dequant(codes, scales).T in fp32."""
    return np.asarray(x, np.float32) @ dequant_qrow(codes, scales).T


def qrow_matmul_w8a16(x: np.ndarray, codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """The W8A16 contract: weight rounded to bf16 before an fp32-accumulated dot; the output
    is returned as the bf16 value stored by the kernel (fp32 array on the bf16 grid)."""
    w = bf16_round(dequant_qrow(codes, scales))
    xb = bf16_round(x)
    return bf16_round(xb.astype(np.float64) @ w.T.astype(np.float64))


def qrow_matmul_exact(x: np.ndarray, codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Float64 value of x @ (codes * scale).T — the infinitely precise target both the
    reference and the B200 kernel approximate (used for error budgets)."""
    return (np.asarray(x, np.float64) @ codes.astype(np.float64).T) * np.asarray(scales, np.float64)[None, :]


def sigmoid_f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32)
    with np.errstate(over="ignore"):
        return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def swiglu_w8a16(x, gate_codes, gate_scales, up_codes, up_scales) -> np.ndarray:
    """bf16(silu(bf16 g)) * bf16(u) -> bf16, with g/u the W8A16 projections."""
    g = qrow_matmul_w8a16(x, gate_codes, gate_scales)
    u = qrow_matmul_w8a16(x, up_codes, up_scales)
    s = bf16_round(g * sigmoid_f32(g))
    return bf16_round(s * u)


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float, out_bf16: bool) -> np.ndarray:
    xf = np.asarray(x, np.float32)
    inv = (np.float32(1.0) / np.sqrt(np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps))).astype(np.float32)
    y = (xf * inv).astype(np.float32) * np.asarray(weight, np.float32)
    return bf16_round(y) if out_bf16 else y.astype(np.float32)


def residual_rms_norm(residual, update, weight, eps) -> tuple[np.ndarray, np.ndarray]:
    r = bf16_round(np.asarray(residual, np.float32) + np.asarray(update, np.float32))
    return r, rms_norm(r, weight, eps, out_bf16=True)


def embed_rows(codes: np.ndarray, scales: np.ndarray, ids) -> np.ndarray:
    ids = np.asarray(ids, dtype=np.int64)
    return dequant_qrow(codes[ids], scales[ids])


def exact_head_argmax(hidden: np.ndarray, codes: np.ndarray, scales: np.ndarray, semantic_rows: int | None = None):
    """fp32 logits = hidden @ dequant(W).T; first maximal index over the semantic prefix."""
    logits = np.asarray(hidden, np.float32) @ dequant_qrow(codes, scales).T
    n = logits.shape[-1] if semantic_rows is None else int(semantic_rows)
    return np.argmax(logits[..., :n], axis=-1), logits
