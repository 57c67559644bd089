"""Block-paged KV cache in HBM: 16-token pages, one page table row per sequence.

Layout per layer: K and V pools ``[num_pages, Hkv, 16, D]`` bf16 (a page of one KV head is
4 KiB contiguous at D=128), the block-paged layout of mrun's paged attention
(runtime/mlx_paged_attention.py:56-67, runtime/mlx_paged_kv.py:37-50). Pages are handed out
from a host free list; the device block table ``[max_seqs, max_pages_per_seq]`` int32 maps a
sequence's logical page to its physical page (-1 = unmapped).
"""
from __future__ import annotations

import torch

from .segmented_gqa_decode import (paged_attention, paged_attention_workspace_bytes, paged_prefill_attention,
                                   rope_append_attention, rope_kv_append)

PAGE = 16


class PagedKVCache:
    def __init__(
        self,
        *,
        num_layers: int,
        num_pages: int,
        kv_heads: int,
        head_dim: int,
        max_seqs: int,
        max_pages_per_seq: int,
        device: torch.device,
        page_size: int = PAGE,
    ) -> None:
        if page_size % 16:
            raise ValueError("page_size must be a multiple of 16 tokens")
        self.num_layers = int(num_layers)
        self.num_pages = int(num_pages)
        self.kv_heads = int(kv_heads)
        self.head_dim = int(head_dim)
        self.page_size = int(page_size)
        self.max_seqs = int(max_seqs)
        self.max_pages_per_seq = int(max_pages_per_seq)
        self.device = device
        shape = (self.num_layers, self.num_pages, self.kv_heads, self.page_size, self.head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.block_table = torch.full((self.max_seqs, self.max_pages_per_seq), -1, dtype=torch.int32, device=device)
        self._host_table = [[] for _ in range(self.max_seqs)]
        self._free = list(range(self.num_pages - 1, -1, -1))
        self.lengths = [0] * self.max_seqs

    # strides of one layer's pool, in elements
    @property
    def strides(self) -> tuple[int, int, int]:
        return (self.kv_heads * self.page_size * self.head_dim, self.page_size * self.head_dim, self.head_dim)

    @property
    def bytes_per_token(self) -> int:
        return 2 * self.num_layers * self.kv_heads * self.head_dim * 2

    def free_pages(self) -> int:
        return len(self._free)

    def reserve(self, seq: int, total_tokens: int) -> None:
        """Map enough pages for ``total_tokens`` positions of ``seq`` (grow only)."""
        need = (int(total_tokens) + self.page_size - 1) // self.page_size
        if need > self.max_pages_per_seq:
            raise OverflowError(f"sequence needs {need} pages > {self.max_pages_per_seq}")
        pages = self._host_table[seq]
        if need - len(pages) > len(self._free):
            raise MemoryError("paged KV pool exhausted")
        new = []
        while len(pages) < need:
            page = self._free.pop()
            pages.append(page)
            new.append(page)
        if new:
            row = torch.tensor(pages, dtype=torch.int32)
            self.block_table[seq, : len(pages)].copy_(row, non_blocking=False)

    def release(self, seq: int) -> None:
        pages = self._host_table[seq]
        self._free.extend(reversed(pages))
        self._host_table[seq] = []
        self.lengths[seq] = 0
        self.block_table[seq].fill_(-1)

    def pages_of(self, seq: int) -> list[int]:
        return list(self._host_table[seq])

    def append(
        self,
        layer: int,
        k_rows: torch.Tensor,
        v_rows: torch.Tensor,
        positions: torch.Tensor,
        token_rows: torch.Tensor,
        *,
        q_rows: torch.Tensor | None = None,
        q_out: torch.Tensor | None = None,
        rope: tuple[torch.Tensor, torch.Tensor] | None = None,
        in_row_stride: int | None = None,
        num_heads: int = 0,
        error_flag: torch.Tensor | None = None,
        qk_norm: tuple[torch.Tensor, torch.Tensor] | None = None,
        norm_eps: float = 1e-6,
    ) -> None:
        rope_kv_append(
            k_rows, v_rows, self.k[layer], self.v[layer], strides=self.strides, page_size=self.page_size,
            block_table=self.block_table, positions=positions, token_rows=token_rows, q_in=q_rows, q_out=q_out,
            rope=rope, in_row_stride=in_row_stride, num_heads=num_heads, error_flag=error_flag, qk_norm=qk_norm,
            norm_eps=norm_eps,
        )

    def append_attend(
        self,
        layer: int,
        q_rows: torch.Tensor,
        k_rows: torch.Tensor,
        v_rows: torch.Tensor,
        positions: torch.Tensor,
        row_seq: torch.Tensor | None,
        *,
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
        """``append`` then ``attend`` for one decode token per sequence, in one launch."""
        return rope_append_attention(
            q_rows, k_rows, v_rows, self.k[layer], self.v[layer], strides=self.strides, page_size=self.page_size,
            block_table=self.block_table, positions=positions, row_seq=row_seq, num_heads=num_heads,
            max_total_tokens=max_total_tokens, in_row_stride=in_row_stride, rope=rope, qk_norm=qk_norm,
            norm_eps=norm_eps, error_flag=error_flag, scale=scale, out=out, state_ready=state_ready,
        )

    def attend_prefill(self, layer: int, query: torch.Tensor, seq: int, start: int, *, scale: float | None = None,
                       out: torch.Tensor | None = None, error_flag: torch.Tensor | None = None) -> torch.Tensor:
        """Causal attention of a prefill block of sequence `seq` starting at position `start`
        (its K/V already appended)."""
        return paged_prefill_attention(query, self.k[layer], self.v[layer], strides=self.strides,
                                       page_size=self.page_size, block_row=self.block_table[seq], start=start,
                                       scale=scale, out=out, error_flag=error_flag)

    def workspace_bytes(self, rows: int, num_heads: int, max_total_tokens: int) -> int:
        return paged_attention_workspace_bytes(rows, num_heads, self.kv_heads, self.head_dim, max_total_tokens)

    def attend(
        self,
        layer: int,
        query: torch.Tensor,
        row_len: torch.Tensor,
        *,
        max_total_tokens: int,
        row_seq: torch.Tensor | None = None,
        out: torch.Tensor | None = None,
        workspace: torch.Tensor | None = None,
        scale: float | None = None,
    ) -> torch.Tensor:
        return paged_attention(
            query, self.k[layer], self.v[layer], strides=self.strides, page_size=self.page_size,
            block_table=self.block_table, row_len=row_len, max_total_tokens=max_total_tokens, row_seq=row_seq,
            out=out, workspace=workspace, scale=scale, kv_heads=self.kv_heads,
        )
