"""Ragged MoE decode-step oracle on the CPU (test infrastructure only; never on a product path).

Restates one step of ``Qwen3MoeDecodeRuntime.forward_decode_rows``
(engine/qwen3_moe_cuda.py:3790-3960) for int8 qrow weights with the reference's boundaries:
  * ``rms_norm`` (:3282-3285): fp32 mean of squares, normalised value rounded to bf16, times
    the weight, rounded to bf16 — for the input/post/final norms and per head for q/k;
  * projections (qkv, o, router): bf16 activations times the dequantised int8 weight,
    fp32 accumulation, bf16 output (the W8A16 contract);
  * RoPE at each row's own position (rotate-half, fp32 tables), bf16 output;
  * attention over the row's committed K/V plus the new token, fp32 softmax, bf16 output;
  * router: softmax(fp32(logits)), top-k with ties to the lower expert, renorm, bf16 weights;
  * experts: ``expert_swiglu_exact`` (bf16 gate/up, bf16 SwiGLU, bf16 down), fp32 combine of
    the k outputs in route-rank order, bf16;
  * head: fp32 logits of the bf16 final-normed hidden state.
The committed context (K/V of earlier positions) is an input, so one step can be checked
against the device step that saw the same cache.
"""
from __future__ import annotations

import numpy as np

from .attention import gqa_decode_rows, rope, rope_tables
from .moe import expert_swiglu_exact, router_topk
from .numerics import bf16_round
from .qrow import dequant_qrow


def _rms(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.asarray(x, np.float32)
    inv = 1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True) + eps)
    return bf16_round(bf16_round(x * inv) * w)


def _linear(x: np.ndarray, codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    return bf16_round(np.asarray(x, np.float64) @ dequant_qrow(codes, scales).T.astype(np.float64))


def _expert_tensors(layout: dict, page: np.ndarray):
    f, h = layout["intermediate_size"], layout["hidden_size"]

    def view(off, nbytes, dtype, shape):
        return page[off:off + nbytes].view(dtype).reshape(shape)

    gu = view(layout["gate_up_codes_offset"], layout["gate_up_codes_bytes"], np.int8, (2 * f, h))
    gus = view(layout["gate_up_scales_offset"], layout["gate_up_scales_bytes"], np.float32, (2 * f,))
    dn = view(layout["down_codes_offset"], layout["down_codes_bytes"], np.int8, (h, f))
    dns = view(layout["down_scales_offset"], layout["down_scales_bytes"], np.float32, (h,))
    return gu, gus, dn, dns


def moe_decode_step(w: dict, cfg, ids, positions, context_k, context_v, *, new_kv: list | None = None):
    """One decode token per row.

    w: ``MoeWeights.to_host()``; ids [R]; positions [R] (= committed lengths);
    context_k[layer][row] / context_v: [positions[row], Hkv, D] float arrays.
    Returns (fp32 logits [R, vocab], per-layer router indices [R, k]). With ``new_kv`` (a
    list), the step's own K/V rows are appended to it per layer as (k [R, Hkv, D], v), so a
    caller can grow the context and run several steps."""
    ids = np.asarray(ids, np.int64)
    pos = np.asarray(positions, np.int64)
    rows = ids.size
    hq, hkv, d = cfg.heads, cfg.kv_heads, cfg.head_dim
    ec, es = w["embed"]
    hidden = bf16_round(dequant_qrow(ec[ids], es[ids]))
    cos, sin = rope_tables(d, cfg.rope_theta, pos)
    routes = []
    for li, L in enumerate(w["layers"]):
        normed = _rms(hidden, L["ln1"], cfg.eps)
        qkv = _linear(normed, *L["qkv"])
        q = qkv[:, : hq * d].reshape(rows, hq, d)
        k = qkv[:, hq * d: (hq + hkv) * d].reshape(rows, hkv, d)
        v = qkv[:, (hq + hkv) * d:].reshape(rows, hkv, d)
        if L["q_norm"] is not None:  # Qwen3 layers; Mixtral-family layers have no q/k norm
            q, k = _rms(q, L["q_norm"], cfg.eps), _rms(k, L["k_norm"], cfg.eps)
        q = rope(q, cos, sin)
        k = rope(k, cos, sin)
        if new_kv is not None:
            new_kv.append((k, v))
        keys = [np.concatenate([context_k[li][r], k[r:r + 1]], 0) for r in range(rows)]
        vals = [np.concatenate([context_v[li][r], v[r:r + 1]], 0) for r in range(rows)]
        ctx = bf16_round(gqa_decode_rows(q, keys, vals)).reshape(rows, hq * d)
        resid = bf16_round(hidden + _linear(ctx, *L["o"]))
        moe_in = _rms(resid, L["ln2"], cfg.eps)
        logits = _linear(moe_in, *L["router"])
        top_idx, _, top_w = router_topk(logits, cfg.top_k, renorm=cfg.norm_topk)
        routes.append(top_idx)
        out = np.zeros((rows, cfg.hidden), np.float32)
        for r in range(rows):
            acc = None
            for j in range(cfg.top_k):
                e = int(top_idx[r, j])
                y = expert_swiglu_exact(moe_in[r:r + 1], *_expert_tensors(w["layout"], L["pages"][e]))[0]
                c = (y.astype(np.float32) * np.float32(top_w[r, j])).astype(np.float32)
                acc = c if acc is None else (acc + c).astype(np.float32)
            out[r] = acc
        hidden = bf16_round(resid + bf16_round(out))
    normed = _rms(hidden, w["final_norm"], cfg.eps)
    hc, hs = w["head"]
    logits = np.asarray(normed, np.float32) @ dequant_qrow(hc, hs).T.astype(np.float32)
    return logits, routes
