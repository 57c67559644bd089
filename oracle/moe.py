"""Routed-MoE oracle (test infrastructure only).

References (mrun project paths):
  * router: engine/qwen3_moe_cuda.py:3700-3707 — softmax(fp32 logits) -> topk -> renorm -> bf16
  * route compiler, CPU branch: engine/olmoe_cuda.py:1064-1089 — stable argsort by expert,
    bincount, exclusive prefix, inverse bijection
  * grouped expert projection: engine/qwen3_moe_cuda.py:2740-2761 (per expert
    ``rows[start:start+count] @ W_e.T``, then silu(g) * u); expert pages per
    ``ExpertPageLayout`` engine/qwen3_moe_cuda.py:187-231
  * stable combine, CPU branch: engine/qwen3_moe_cuda.py:2654-2664 — fp32 products, summed
    in original route-rank order
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_round
from .qrow import dequant_qrow, sigmoid_f32


def softmax_f32(logits: np.ndarray) -> np.ndarray:
    x = np.asarray(logits, np.float32)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp((x - m).astype(np.float32)).astype(np.float32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def router_topk(logits: np.ndarray, k: int, renorm: bool = True) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Returns (indices int64 [T,k], fp32 weights before bf16, bf16-valued weights)."""
    p = softmax_f32(logits)
    order = np.argsort(-p, axis=-1, kind="stable")[:, :k]
    w = np.take_along_axis(p, order, axis=-1)
    if renorm:
        w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return order.astype(np.int64), w, bf16_round(w)


def route_tensors(top_indices: np.ndarray, top_weights: np.ndarray, num_experts: int):
    """(token_ids, coefficients, starts, counts, inverse) exactly as the CPU branch."""
    rows, k = top_indices.shape
    flat_e = top_indices.reshape(-1)
    flat_w = np.asarray(top_weights).reshape(-1)
    flat_t = np.repeat(np.arange(rows, dtype=np.int64), k)
    order = np.argsort(flat_e, kind="stable")
    token_ids = flat_t[order]
    coefficients = flat_w[order]
    counts = np.bincount(flat_e, minlength=num_experts).astype(np.int32)
    starts = np.concatenate(([0], np.cumsum(counts)[:-1])).astype(np.int32)
    inverse = np.empty(flat_e.size, np.int64)
    inverse[order] = np.arange(flat_e.size, dtype=np.int64)
    return token_ids, coefficients, starts, counts, inverse


def stable_route_reduce(expert_output, coefficients, inverse, rows: int, k: int) -> np.ndarray:
    eo = np.asarray(expert_output, np.float32)[inverse].reshape(rows, k, -1)
    co = np.asarray(coefficients, np.float32)[inverse].reshape(rows, k)
    contrib = (eo * co[..., None]).astype(np.float32)
    out = contrib[:, 0]
    for r in range(1, k):
        out = (out + contrib[:, r]).astype(np.float32)
    return out


def expert_swiglu_exact(x_rows: np.ndarray, gate_up_codes, gate_up_scales, down_codes, down_scales) -> np.ndarray:
    """One expert in float64 with the bf16 boundaries of the B200 path:
    gu = bf16(x @ W_gu.T); a = bf16(bf16(silu(g)) * u); y = bf16(a @ W_d.T)."""
    f = gate_up_codes.shape[0] // 2
    x = np.asarray(x_rows, np.float64)
    gu = bf16_round(x @ dequant_qrow(gate_up_codes, gate_up_scales).T.astype(np.float64))
    g, u = gu[:, :f], gu[:, f:]
    a = bf16_round(bf16_round(g * sigmoid_f32(g)) * u)
    return bf16_round(a.astype(np.float64) @ dequant_qrow(down_codes, down_scales).T.astype(np.float64))
