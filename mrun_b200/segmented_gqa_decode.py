"""B200 decode attention: drop-ins for mrun's segmented GQA decode and the paged-KV kernel.

Reference interfaces (same names, arguments and validation errors):
  * ``segmented_gqa_decode`` / ``scatter_segmented_decode_kv``
    (engine/kernels/segmented_gqa_decode.py:458-607)
  * ``segmented_decode_attention`` (engine/kernels/dense_qstore_cuda.py:1763-1854)
All of them run one native split-K kernel (``mrb_paged_attention``) that reads K/V through a
page table; the contiguous reference caches are single-page views of it.
"""
from __future__ import annotations

import math
import threading
from collections.abc import Sequence

import torch

from . import _lib

IMPL_SEGMENTED = "b200-paged-splitk-gqa-decode-v1"


class SegmentedGQADecodeError(RuntimeError):
    """The compact segmented-GQA execution contract was violated."""


# ------------------------------------------------------------------ workspace


class AttentionWorkspace:
    """Grow-only, zero-initialised split-K scratch per device (counters self-reset)."""

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._buffers: dict[int, torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor | None:
        if nbytes <= 0:
            return None
        index = device.index if device.index is not None else torch.cuda.current_device()
        with self._lock:
            buf = self._buffers.get(index)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                self._buffers[index] = buf
            return buf


_WORKSPACE = AttentionWorkspace()


def paged_attention_workspace_bytes(rows: int, hq: int, hkv: int, head_dim: int, max_total_tokens: int) -> int:
    return int(_lib.load().mrb_paged_attention_workspace(rows, hq, hkv, head_dim, max_total_tokens))


def paged_attention(
    query: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    *,
    strides: tuple[int, int, int],
    page_size: int,
    block_table: torch.Tensor,
    row_len: torch.Tensor,
    max_total_tokens: int,
    row_seq: torch.Tensor | None = None,
    k_new: torch.Tensor | None = None,
    v_new: torch.Tensor | None = None,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    kv_heads: int | None = None,
) -> torch.Tensor:
    """Low-level call: query [rows, hq, d] bf16 -> [rows, hq, d] bf16.

    ``kv_heads`` defaults to ``k_cache.shape[1]`` (the [pages, Hkv, page, D] layouts)."""
    rows, hq, d = (int(v) for v in query.shape)
    hkv = int(k_cache.shape[1]) if kv_heads is None else int(kv_heads)
    device = _lib.require_cuda(query, k_cache, v_cache, block_table, row_len, what="paged attention")
    if query.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise TypeError("paged attention runs on bf16 queries and caches")
    if block_table.dtype != torch.int32 or row_len.dtype != torch.int32:
        raise TypeError("block tables and lengths must be int32")
    q = query.contiguous()
    if out is None:
        out = torch.empty_like(q)
    need = paged_attention_workspace_bytes(rows, hq, hkv, d, max_total_tokens)
    if workspace is None:
        workspace = _WORKSPACE.get(device, need)
    elif need and workspace.numel() < need:
        raise ValueError(f"workspace too small: {workspace.numel()} < {need} bytes")
    sc = (1.0 / math.sqrt(d)) if scale is None else float(scale)
    _lib.call(
        "mrb_paged_attention",
        q.data_ptr(), rows, hq, hkv, d,
        k_cache.data_ptr(), v_cache.data_ptr(), strides[0], strides[1], strides[2], page_size,
        block_table.data_ptr(), int(block_table.stride(0)) if block_table.ndim > 1 else 1,
        _lib.ptr(row_seq), row_len.data_ptr(), _lib.ptr(k_new), _lib.ptr(v_new), sc,
        int(max_total_tokens), out.data_ptr(), _lib.ptr(workspace),
        0 if workspace is None else workspace.numel(), _lib.stream_handle(device),
    )
    return out


def rope_kv_append(
    k_in: torch.Tensor,
    v_in: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    *,
    strides: tuple[int, int, int],
    page_size: int,
    block_table: torch.Tensor,
    positions: torch.Tensor,
    token_rows: torch.Tensor | None,
    q_in: torch.Tensor | None = None,
    q_out: torch.Tensor | None = None,
    rope: tuple[torch.Tensor, torch.Tensor] | None = None,
    in_row_stride: int | None = None,
    num_heads: int = 0,
    error_flag: torch.Tensor | None = None,
    qk_norm: tuple[torch.Tensor, torch.Tensor] | None = None,
    norm_eps: float = 1e-6,
) -> None:
    """Rotate (optional) and append one K/V position per token into a paged cache.

    ``qk_norm`` = (q weight, k weight), bf16 [head_dim]: per-head RMSNorm of queries and keys
    before the rotation (the Qwen3 q/k norm)."""
    tokens = int(positions.numel())
    hkv, d = int(k_cache.shape[1]), int(k_cache.shape[-1])
    device = _lib.require_cuda(k_in, v_in, k_cache, v_cache, block_table, positions, what="KV append")
    stride = int(in_row_stride if in_row_stride is not None else k_in.stride(0))
    cos, sin = rope if rope is not None else (None, None)
    _lib.call(
        "mrb_rope_kv_append",
        _lib.ptr(q_in), k_in.data_ptr(), v_in.data_ptr(), stride, tokens, int(num_heads), hkv, d,
        positions.data_ptr(), _lib.ptr(token_rows), _lib.ptr(cos), _lib.ptr(sin),
        0 if cos is None else int(cos.shape[0]), _lib.ptr(q_out), k_cache.data_ptr(), v_cache.data_ptr(),
        strides[0], strides[1], strides[2], page_size, block_table.data_ptr(),
        int(block_table.stride(0)) if block_table.ndim > 1 else 1, int(k_cache.shape[0]),
        _lib.ptr(error_flag), _lib.ptr(qk_norm[0] if qk_norm else None), _lib.ptr(qk_norm[1] if qk_norm else None),
        float(norm_eps), _lib.stream_handle(device),
    )


def rope_append_attention(
    q_in: torch.Tensor,
    k_in: torch.Tensor,
    v_in: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    *,
    strides: tuple[int, int, int],
    page_size: int,
    block_table: torch.Tensor,
    positions: torch.Tensor,
    row_seq: torch.Tensor | None,
    num_heads: int,
    max_total_tokens: int,
    in_row_stride: int | None = None,
    rope: tuple[torch.Tensor, torch.Tensor] | None = None,
    qk_norm: tuple[torch.Tensor, torch.Tensor] | None = None,
    norm_eps: float = 1e-6,
    error_flag: torch.Tensor | None = None,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    state_ready: bool = False,
) -> torch.Tensor:
    """One decode token per row in one launch: ``rope_kv_append`` of the row's new position
    followed by ``paged_attention`` over positions ``[0, positions[r]]``.

    Every row must continue a different sequence (``row_seq`` distinct): a row reads only
    cache entries written before this call plus its own new token. ``state_ready``: the
    positions, block table and cached K/V are not written by a kernel still in flight, so the
    kernel may read them before waiting on the previous launch. Returns bf16
    ``[rows, num_heads, head_dim]``."""
    rows = int(positions.numel())
    hkv, d = int(k_cache.shape[1]), int(k_cache.shape[-1])
    device = _lib.require_cuda(q_in, k_in, v_in, k_cache, v_cache, block_table, positions,
                               what="fused decode attention")
    if k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16 or q_in.dtype != torch.bfloat16:
        raise TypeError("fused decode attention runs on bf16 rows and caches")
    if block_table.dtype != torch.int32 or positions.dtype != torch.int32:
        raise TypeError("block tables and positions must be int32")
    if out is None:
        out = torch.empty(rows, int(num_heads), d, dtype=torch.bfloat16, device=device)
    elif out.shape != (rows, int(num_heads), d) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 [rows, num_heads, head_dim] tensor")
    stride = int(in_row_stride if in_row_stride is not None else q_in.stride(0))
    cos, sin = rope if rope is not None else (None, None)
    sc = (1.0 / math.sqrt(d)) if scale is None else float(scale)
    _lib.call(
        "mrb_rope_append_attention",
        q_in.data_ptr(), k_in.data_ptr(), v_in.data_ptr(), stride, rows, int(num_heads), hkv, d,
        positions.data_ptr(), _lib.ptr(row_seq), _lib.ptr(cos), _lib.ptr(sin),
        0 if cos is None else int(cos.shape[0]), _lib.ptr(qk_norm[0] if qk_norm else None),
        _lib.ptr(qk_norm[1] if qk_norm else None), float(norm_eps), k_cache.data_ptr(), v_cache.data_ptr(),
        strides[0], strides[1], strides[2], page_size, block_table.data_ptr(),
        int(block_table.stride(0)) if block_table.ndim > 1 else 1, int(k_cache.shape[0]), _lib.ptr(error_flag), sc,
        int(max_total_tokens), 1 if state_ready else 0, out.data_ptr(), _lib.stream_handle(device),
    )
    return out


def paged_prefill_attention(
    query: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    *,
    strides: tuple[int, int, int],
    page_size: int,
    block_row: torch.Tensor,
    start: int,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    error_flag: torch.Tensor | None = None,
) -> torch.Tensor:
    """Causal attention of ``query`` [n, hq, 128] (bf16): token i of one sequence sits at
    position ``start + i`` and attends to positions ``[0, start + i]`` of the pages listed in
    ``block_row`` (its int32 page-table row); the block's K/V must already be appended."""
    n, hq, d = (int(v) for v in query.shape)
    hkv = int(k_cache.shape[1])
    device = _lib.require_cuda(query, k_cache, v_cache, block_row, what="prefill attention")
    if query.dtype != torch.bfloat16 or not query.is_contiguous():
        raise TypeError("prefill attention runs on contiguous bf16 queries")
    if block_row.dtype != torch.int32 or not block_row.is_contiguous():
        raise TypeError("the page-table row must be contiguous int32")
    if out is None:
        out = torch.empty_like(query)
    sc = (1.0 / math.sqrt(d)) if scale is None else float(scale)
    _lib.call("mrb_paged_prefill_attention", query.data_ptr(), n, hq, hkv, d, int(start), k_cache.data_ptr(),
              v_cache.data_ptr(), strides[0], strides[1], strides[2], page_size, block_row.data_ptr(),
              int(k_cache.shape[0]), _lib.ptr(error_flag), sc, out.data_ptr(), _lib.stream_handle(device))
    return out


def rope_append_attention_cluster(rows: int, hq: int, hkv: int, head_dim: int, max_total_tokens: int) -> int:
    """CTAs per (row, KV head) the fused decode step uses for these sizes."""
    return int(_lib.load().mrb_rope_append_attention_cluster(rows, hq, hkv, head_dim, max_total_tokens))


# ------------------------------------------------------------------ reference-shaped API


def _validate_shapes(query, key_cache, value_cache, physical_slots, sequence_lengths):
    if query.ndim != 3:
        raise ValueError(f"query must have shape [rows,query_heads,head_dim], got {query.shape}")
    if key_cache.ndim != 4 or value_cache.ndim != 4:
        raise ValueError("segmented K/V caches must have shape [slots,kv_heads,capacity,head_dim]")
    if key_cache.shape != value_cache.shape:
        raise ValueError("segmented key and value cache shapes must match")
    rows, query_heads, head_dim = map(int, query.shape)
    slots, kv_heads, capacity, cache_head_dim = map(int, key_cache.shape)
    if rows <= 0 or query_heads <= 0 or kv_heads <= 0 or head_dim <= 0 or capacity <= 0:
        raise ValueError("segmented GQA dimensions must be positive")
    if head_dim != cache_head_dim:
        raise ValueError("segmented query and K/V head dimensions must match")
    if query_heads % kv_heads:
        raise ValueError("query heads must be an exact multiple of K/V heads")
    if physical_slots.ndim != 1 or tuple(physical_slots.shape) != (rows,):
        raise ValueError("physical_slots must contain one slot per query row")
    if sequence_lengths.ndim != 1 or tuple(sequence_lengths.shape) != (rows,):
        raise ValueError("sequence_lengths must contain one length per query row")
    if physical_slots.dtype not in (torch.int32, torch.int64):
        raise TypeError("physical_slots must use an integer tensor dtype")
    if sequence_lengths.dtype not in (torch.int32, torch.int64):
        raise TypeError("sequence_lengths must use an integer tensor dtype")
    tensors = (query, key_cache, value_cache, physical_slots, sequence_lengths)
    if len({tensor.device for tensor in tensors}) != 1:
        raise ValueError("segmented GQA tensors must share one device")
    if query.dtype != key_cache.dtype or query.dtype != value_cache.dtype:
        raise TypeError("segmented query and K/V cache dtypes must match")
    return rows, query_heads, kv_heads, capacity, head_dim


def _slot_view(cache: torch.Tensor) -> tuple[tuple[int, int, int], int]:
    """[slots, Hkv, cap, D] as pages of `cap` tokens."""
    if not cache.is_contiguous():
        raise ValueError("segmented K/V caches must be contiguous")
    slots, hkv, cap, d = map(int, cache.shape)
    return (hkv * cap * d, cap * d, d), cap


def segmented_gqa_decode(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    physical_slots: torch.Tensor,
    sequence_lengths: torch.Tensor,
    *,
    max_sequence_length: int | None = None,
    scale: float | None = None,
) -> torch.Tensor:
    """Ragged one-token GQA over [slots, Hkv, cap, D] (reference: segmented_gqa_decode.py:526)."""
    rows, query_heads, kv_heads, capacity, head_dim = _validate_shapes(
        query, key_cache, value_cache, physical_slots, sequence_lengths
    )
    attention_scale = 1.0 / math.sqrt(head_dim) if scale is None else float(scale)
    if not math.isfinite(attention_scale) or attention_scale <= 0:
        raise ValueError("segmented GQA scale must be finite and positive")
    if query.device.type != "cuda":
        raise SegmentedGQADecodeError("B200 segmented GQA runs on CUDA only")
    if query.dtype != torch.bfloat16:
        raise TypeError("B200 segmented GQA supports bf16")
    if max_sequence_length is None:
        raise ValueError("CUDA segmented GQA requires an explicit host max_sequence_length")
    if (
        isinstance(max_sequence_length, bool)
        or not isinstance(max_sequence_length, int)
        or max_sequence_length <= 0
        or max_sequence_length > capacity
    ):
        raise ValueError("max_sequence_length must be in 1..cache capacity")
    strides, page = _slot_view(key_cache)
    return paged_attention(
        query, key_cache, value_cache, strides=strides, page_size=page,
        block_table=physical_slots.to(torch.int32).reshape(rows, 1).contiguous(),
        row_len=sequence_lengths.to(torch.int32).contiguous(), max_total_tokens=max_sequence_length,
        scale=attention_scale,
    )


def scatter_segmented_decode_kv(
    key: torch.Tensor,
    value: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    physical_slots: torch.Tensor,
    parent_lengths: torch.Tensor,
) -> None:
    """Write one provisional K/V position per row (reference: segmented_gqa_decode.py:458)."""
    rows, _, kv_heads, capacity, head_dim = _validate_shapes(
        key, key_cache, value_cache, physical_slots, parent_lengths + 1
    )
    if key.shape != value.shape:
        raise ValueError("provisional key and value shapes must match")
    if key.device != value.device or key.dtype != value.dtype:
        raise ValueError("provisional key and value must share one device and dtype")
    if int(key.shape[1]) != kv_heads:
        raise ValueError("provisional key/value head count must match the cache")
    if key.device.type != "cuda":
        raise SegmentedGQADecodeError("B200 segmented K/V scatter runs on CUDA only")
    if key.dtype != torch.bfloat16:
        raise TypeError("B200 segmented K/V scatter supports bf16")
    strides, page = _slot_view(key_cache)
    k = key.contiguous()
    v = value.contiguous()
    rope_kv_append(
        k, v, key_cache, value_cache, strides=strides, page_size=page,
        block_table=physical_slots.to(torch.int32).reshape(rows, 1).contiguous(),
        positions=parent_lengths.to(torch.int32).contiguous(),
        token_rows=torch.arange(rows, device=key.device, dtype=torch.int32),
        in_row_stride=kv_heads * head_dim,
    )


def segmented_decode_attention(
    query: torch.Tensor,
    cache_key: torch.Tensor,
    cache_value: torch.Tensor,
    key_new: torch.Tensor,
    value_new: torch.Tensor,
    lengths: torch.Tensor | Sequence[int],
    *,
    cache_row_indices: torch.Tensor | None = None,
    require_triton: bool = False,
    sequence_tile: int = 64,
    max_committed: int | None = None,
    validate_lengths: bool = True,
) -> tuple[torch.Tensor, str]:
    """One-token GQA over committed [B,S,Hkv,D] K/V plus one provisional token
    (reference: engine/kernels/dense_qstore_cuda.py:1763-1854)."""
    del require_triton
    if query.ndim != 4 or cache_key.ndim != 4 or cache_value.shape != cache_key.shape:
        raise ValueError("query and key/value need [B,T,H,D] and [B,S,Hkv,D]")
    batch, token_count, num_heads, head_dim = map(int, query.shape)
    slots, max_total, num_kv_heads, key_dim = map(int, cache_key.shape)
    if token_count != 1:
        raise ValueError("segmented decode attention takes exactly one query token")
    if key_dim != head_dim or num_heads % num_kv_heads:
        raise ValueError("attention batch/head dimensions are incompatible")
    if tuple(key_new.shape) != (batch, 1, num_kv_heads, head_dim) or key_new.shape != value_new.shape:
        raise ValueError("provisional key/value need [B,1,Hkv,D]")
    if isinstance(sequence_tile, bool) or not isinstance(sequence_tile, int):
        raise TypeError("sequence_tile must be an integer")
    if sequence_tile < 16 or sequence_tile > 256 or sequence_tile & (sequence_tile - 1):
        raise ValueError("sequence_tile must be a power of two in [16, 256]")
    device = _lib.require_cuda(query, cache_key, cache_value, key_new, value_new, what="segmented decode")
    length_tensor = torch.as_tensor(lengths, device=device).to(torch.int32).reshape(batch)
    if max_committed is None:
        max_committed = int(length_tensor.max().item())
    if max_committed < 0 or max_committed > max_total:
        raise ValueError("max_committed must fit inside committed KV storage")
    if validate_lengths and bool(((length_tensor < 0) | (length_tensor > max_committed)).any().item()):
        raise ValueError("max_committed does not cover every committed request length")
    if cache_row_indices is not None:
        if tuple(cache_row_indices.shape) != (batch,):
            raise ValueError("cache_row_indices must have shape [B]")
        if validate_lengths and bool(((cache_row_indices < 0) | (cache_row_indices >= slots)).any().item()):
            raise ValueError("cache_row_indices select a slot outside committed KV storage")
        table = cache_row_indices.to(torch.int32).reshape(batch, 1).contiguous()
    else:
        table = torch.arange(batch, device=device, dtype=torch.int32).reshape(batch, 1)
    if not cache_key.is_contiguous() or not cache_value.is_contiguous():
        raise ValueError("committed K/V caches must be contiguous")
    strides = (max_total * num_kv_heads * head_dim, head_dim, num_kv_heads * head_dim)
    out = paged_attention(
        query.reshape(batch, num_heads, head_dim), cache_key, cache_value, strides=strides,
        page_size=max_total, block_table=table, row_len=length_tensor.contiguous(),
        max_total_tokens=max_committed + 1,
        k_new=key_new.reshape(batch, num_kv_heads, head_dim).contiguous(),
        v_new=value_new.reshape(batch, num_kv_heads, head_dim).contiguous(),
        kv_heads=num_kv_heads,
    )
    return out.reshape(batch, 1, num_heads, head_dim), IMPL_SEGMENTED


__all__ = [
    "IMPL_SEGMENTED",
    "SegmentedGQADecodeError",
    "paged_attention",
    "paged_attention_workspace_bytes",
    "rope_kv_append",
    "scatter_segmented_decode_kv",
    "segmented_decode_attention",
    "segmented_gqa_decode",
]
