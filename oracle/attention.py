"""Decode attention oracle (test infrastructure only).

References (mrun project paths):
  * one-token GQA, committed + provisional segment:
      engine/kernels/dense_qstore_cuda.py:1690-1760 `segmented_decode_attention_reference`
  * ragged compact GQA over [slots, Hkv, cap, D]:
      engine/kernels/segmented_gqa_decode.py:85-126 `segmented_gqa_decode_reference`
  * one-position K/V scatter: engine/kernels/segmented_gqa_decode.py:458-524
  * 16-token block-paged layout: runtime/mlx_paged_attention.py:56-67 — element
    ((page_slots[token // PAGE] * Hkv + kvh) * PAGE + token % PAGE) * D + d
  * RoPE (rotate-half): engine/dense_qstore_cuda.py:689-704 `_rope`
The gathers are integer indexing (exact). Softmax is evaluated in float64 here; kernels are
compared within the bf16 tolerance.
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_round

PAGE = 16


def gqa_decode_rows(q: np.ndarray, keys: list[np.ndarray], values: list[np.ndarray], scale: float | None = None) -> np.ndarray:
    """q [rows, Hq, D]; keys[r]/values[r] [len_r, Hkv, D] -> fp32 [rows, Hq, D] (not rounded)."""
    rows, hq, d = q.shape
    out = np.zeros((rows, hq, d), np.float64)
    sc = (1.0 / np.sqrt(d)) if scale is None else float(scale)
    for r in range(rows):
        k = np.asarray(keys[r], np.float64)
        v = np.asarray(values[r], np.float64)
        hkv = k.shape[1]
        group = hq // hkv
        for h in range(hq):
            kvh = h // group
            s = (k[:, kvh, :] @ np.asarray(q[r, h], np.float64)) * sc
            s = s - s.max()
            p = np.exp(s)
            p /= p.sum()
            out[r, h] = p @ v[:, kvh, :]
    return out.astype(np.float32)


def segmented_gqa_decode(q, key_cache, value_cache, physical_slots, sequence_lengths, scale=None) -> np.ndarray:
    keys = [key_cache[s, :, :n].transpose(1, 0, 2) for s, n in zip(physical_slots, sequence_lengths)]
    values = [value_cache[s, :, :n].transpose(1, 0, 2) for s, n in zip(physical_slots, sequence_lengths)]
    return bf16_round(gqa_decode_rows(q, keys, values, scale))


def segmented_decode_attention(q, cache_key, cache_value, key_new, value_new, lengths, row_indices=None) -> np.ndarray:
    """q [B,1,Hq,D]; cache [slots,S,Hkv,D]; new [B,1,Hkv,D] -> bf16-valued [B,1,Hq,D]."""
    b = q.shape[0]
    rows = range(b) if row_indices is None else row_indices
    keys, values = [], []
    for i, (slot, n) in enumerate(zip(rows, lengths)):
        keys.append(np.concatenate([cache_key[slot, :n], key_new[i, :1]], axis=0))
        values.append(np.concatenate([cache_value[slot, :n], value_new[i, :1]], axis=0))
    return bf16_round(gqa_decode_rows(q[:, 0], keys, values))[:, None]


def paged_gather(pages: np.ndarray, block_table_row, length: int) -> np.ndarray:
    """pages [P, Hkv, PAGE, D], logical tokens [0, length) -> [length, Hkv, D] (exact)."""
    p, hkv, page, d = pages.shape
    out = np.empty((length, hkv, d), pages.dtype)
    for t in range(length):
        phys = int(block_table_row[t // page])
        out[t] = pages[phys, :, t % page, :]
    return out


def paged_gqa_decode(q, k_pages, v_pages, block_table, seq_lens, scale=None) -> np.ndarray:
    keys = [paged_gather(k_pages, block_table[r], int(n)) for r, n in enumerate(seq_lens)]
    values = [paged_gather(v_pages, block_table[r], int(n)) for r, n in enumerate(seq_lens)]
    return bf16_round(gqa_decode_rows(q, keys, values, scale))


def rope_tables(head_dim: int, theta: float, positions) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin [len(positions), head_dim] as the reference builds them in fp32."""
    import torch  # the reference computes the table with torch fp32 ops

    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    freqs = torch.as_tensor(np.asarray(positions), dtype=torch.float32)[:, None] * inv
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().numpy(), emb.sin().numpy()


def rope(values: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """values [T, H, D] (bf16-valued), cos/sin [T, D] -> bf16-valued rotated values."""
    v = np.asarray(values, np.float32)
    half = v.shape[-1] // 2
    rotated = np.concatenate((-v[..., half:], v[..., :half]), axis=-1)
    c = cos[:, None, :].astype(np.float32)
    s = sin[:, None, :].astype(np.float32)
    return bf16_round((v * c).astype(np.float32) + (rotated * s).astype(np.float32))
