"""The dense engine's store protocol over the B200 QStore: ``DenseQStore``.

mrun's dense CUDA engine talks to its weights through the duck-typed ``DenseQStore``
(engine/kernels/dense_qstore_cuda.py:1857-2611): ``compact_page`` hands out device-resident
int8 pages, ``matmul`` / ``fused_swiglu`` project through them, ``selected_rows_fp32`` reads a
few head rows, ``prebind`` pins pages that CUDA graphs point at, and ``stats_snapshot`` reports
what moved. This module gives the same methods, arguments, return values, counters and
errors on top of ``mrun_b200.qstore.QStore``: pages come off disk by the parallel ``pread``
reader into pinned staging and one host-to-device copy, and every projection is the B200
W8A16 kernel (``mrb_qrow_matmul`` / ``mrb_qrow_swiglu``), never a widened fp32 weight.

Bookkeeping differences from the reference, all internal: one ``OrderedDict`` LRU holds the
evictable pages and a plain dict the prebound ones, both keyed by the physical (alias-free)
block name; the implementation tags the projections return start with ``"b200-"``, and the
reference's ``triton_*`` counters count these native calls (its ``reference_*`` counters, the
eager fallback, stay at zero: there is no fallback).
"""
from __future__ import annotations

from collections import OrderedDict
from collections.abc import Mapping, Sequence
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any

import numpy as np
import torch

from .dense_qstore_cuda import CompactQRowPage, _tensor_bytes, fused_qrow_matmul, fused_qrow_swiglu
from .qstore import QStore


@dataclass
class DenseQStoreStats:
    """Counters of ``DenseQStore`` (the reference's ``DenseQStoreStats`` fields,
    engine/kernels/dense_qstore_cuda.py:142-170)."""

    projection_calls: int = 0
    triton_projection_calls: int = 0
    reference_projection_calls: int = 0
    paired_swiglu_calls: int = 0
    triton_paired_swiglu_calls: int = 0
    reference_paired_swiglu_calls: int = 0
    selected_head_calls: int = 0
    selected_head_rows: int = 0
    selected_head_compact_bytes: int = 0
    page_loads: int = 0
    cache_hits: int = 0
    compact_h2d_bytes: int = 0
    compact_logical_bytes: int = 0
    expanded_fp32_bytes_avoided: int = 0
    expanded_compute_bytes_avoided: int = 0
    peak_compact_resident_bytes: int = 0
    fp32_aux_cache_loads: int = 0
    resident_exact_head_loads: int = 0

    def snapshot(self, *, resident_bytes: int, cache_entries: int) -> dict[str, Any]:
        out = asdict(self)
        out["compact_resident_bytes"] = int(resident_bytes)
        out["cache_entries"] = int(cache_entries)
        return out


def load_compact_qrow_page(store: Any, name: str, *, start_row: int = 0,
                           end_row: int | None = None) -> CompactQRowPage:
    """Rows [start_row, end_row) of a qrow block as a device page
    (engine/kernels/dense_qstore_cuda.py:963-1000).

    A B200 ``QStore`` reads exactly those rows from disk into its pinned staging and copies
    them to HBM; a store exposing the reference's memory-mapped ``w`` / ``s`` arrays is read
    through them. Raises ValueError for a non-qrow block or an empty / out-of-range span."""
    block = store._resolve(name)
    if block.get("kind") != "qrow":
        raise ValueError(f"{name} is not a qrow block")
    rows, cols = (int(v) for v in block["shape"])
    start = int(start_row)
    stop = rows if end_row is None else int(end_row)
    if not 0 <= start < stop <= rows:
        raise ValueError(f"invalid row range [{start}, {stop}) for {name}")
    if isinstance(store, QStore):
        codes, scales = store._direct(block, start, stop)
    else:
        w0 = int(block["w_off"]) + start * cols
        codes = torch.from_numpy(np.array(store.w[w0:w0 + (stop - start) * cols], dtype=np.int8))
        codes = codes.reshape(stop - start, cols)
        s0 = int(block["s_off"]) // 4 + start
        scales = torch.from_numpy(np.array(store.s[s0:s0 + stop - start], dtype=np.float32))
        device = torch.device(store.device)
        if device.type != "cpu":
            codes, scales = codes.to(device), scales.to(device)
    return CompactQRowPage(name=name, start_row=start, end_row=stop, in_features=cols, codes=codes, scales=scales)


class DenseQStore(QStore):
    """Int8 QStore with a byte-bounded device page cache, non-evictable prebound pages and the
    fused W8A16 projections (the reference's ``DenseQStore``, dense_qstore_cuda.py:1857)."""

    def __init__(self, model_name: str, *, root: str | Path, device: str = "cuda", compute_dtype: str = "bf16",
                 compact_cache_mb: float = 0.0, require_triton: bool = True, stable_block_m: int = 16,
                 pin_fp32_aux: bool = False) -> None:
        # the dense engine reads pages, never weight(): the successor ring would only hold
        # pinned slots for nothing, so it stays off as in the reference
        super().__init__(model_name, root=root, device=device, enable_prefetch_ring=False)
        self.disable_ring()
        if stable_block_m not in (16, 32, 64):
            raise ValueError("stable_block_m must be one of 16, 32, or 64")
        dtypes = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}
        if compute_dtype not in dtypes:
            raise ValueError(f"compute_dtype must be one of {sorted(dtypes)}")
        self.compute_dtype = dtypes[compute_dtype]
        self.require_triton = bool(require_triton)  # accepted; the native kernels are always required
        self.stable_block_m = int(stable_block_m)
        self.compact_cache_budget = int(float(compact_cache_mb) * 1e6)
        self.compact_cache: OrderedDict[str, CompactQRowPage] = OrderedDict()
        self.compact_cache_bytes = 0
        self._prebound_pages: dict[str, CompactQRowPage] = {}
        self._prebound_compact_bytes = 0
        self._prebound_fp32: dict[str, torch.Tensor] = {}
        self._prebound_fp32_bytes = 0
        self.pin_fp32_aux = bool(pin_fp32_aux)
        self.fp32_aux_cache: dict[str, torch.Tensor] = {}
        self.fp32_aux_cache_bytes = 0
        self.resident_exact_heads: dict[str, torch.Tensor] = {}
        self.resident_exact_head_budget_bytes = 0
        self.resident_exact_head_bytes = 0
        self.stats = DenseQStoreStats()
        if self.pin_fp32_aux:
            try:
                self._pin_fp32_blocks()
            except BaseException:
                super().close()
                raise

    # ---- names and accounting

    def _physical_key(self, name: str) -> str:
        """The alias-free name of the block ``name`` resolves to (KeyError if absent)."""
        key, hops = str(name), 0
        while True:
            block = self.blocks.get(key)
            if not isinstance(block, Mapping):
                raise KeyError(f"QStore has no block {key!r}")
            if "alias" not in block:
                return key
            key, hops = str(block["alias"]), hops + 1
            if hops > len(self.blocks):
                raise ValueError(f"cyclic QStore alias at {name!r}")

    _compact_cache_key = _physical_key

    def _resident_total(self) -> int:
        return (self.compact_cache_bytes + self._prebound_compact_bytes + self.fp32_aux_cache_bytes
                + self._prebound_fp32_bytes)

    def _note_peak(self, extra: int = 0) -> None:
        self.stats.peak_compact_resident_bytes = max(self.stats.peak_compact_resident_bytes,
                                                     self._resident_total() + extra)

    def reset_stats(self) -> None:
        self.stats = DenseQStoreStats(peak_compact_resident_bytes=self._resident_total())

    def stats_snapshot(self) -> dict[str, Any]:
        snap = self.stats.snapshot(resident_bytes=self.compact_cache_bytes + self._prebound_compact_bytes,
                                   cache_entries=len(self.compact_cache) + len(self._prebound_pages))
        snap.update({
            "stable_block_m": self.stable_block_m,
            "compact_cache_budget_bytes": self.compact_cache_budget,
            "cache_kind": "compact-device-lru",
            "fp32_aux_pinning_enabled": self.pin_fp32_aux,
            "fp32_aux_cache_entries": len(self.fp32_aux_cache),
            "fp32_aux_resident_bytes": self.fp32_aux_cache_bytes,
            "resident_physical_bytes": self._resident_total() + self.resident_exact_head_bytes,
            "resident_exact_head_entries": len(self.resident_exact_heads),
            "resident_exact_head_budget_bytes": self.resident_exact_head_budget_bytes,
            "resident_exact_head_bytes": self.resident_exact_head_bytes,
            "prebound_page_entries": len(self._prebound_pages),
            "prebound_compact_bytes": self._prebound_compact_bytes,
            "prebound_fp32_entries": len(self._prebound_fp32),
            "prebound_fp32_bytes": self._prebound_fp32_bytes,
        })
        return snap

    # ---- fp32 auxiliaries

    def _fp32_names(self) -> list[str]:
        names = {self._physical_key(n) for n, b in self.blocks.items() if isinstance(b, Mapping)}
        return sorted(n for n in names if self.blocks[n].get("kind") == "fp32")

    def _pin_fp32_blocks(self) -> None:
        names = self._fp32_names()
        need = sum(int(self.blocks[n]["e_len"]) for n in names)
        if need > self.compact_cache_budget:
            raise MemoryError("pinned FP32 auxiliary residency exceeds the provider cache budget "
                              f"({need} > {self.compact_cache_budget} bytes)")
        pinned = {n: super(DenseQStore, self).fp32(n).contiguous() for n in names}
        held = sum(_tensor_bytes(t) for t in pinned.values())
        if held != need:
            raise RuntimeError(f"pinned FP32 auxiliary bytes disagree with the verified manifest ({held} != {need})")
        self.fp32_aux_cache, self.fp32_aux_cache_bytes = pinned, held
        self.stats.fp32_aux_cache_loads += len(pinned)
        self._note_peak()

    def fp32(self, name: str) -> torch.Tensor:
        key = self._physical_key(name)
        held = self._prebound_fp32.get(key)
        if held is None:
            held = self.fp32_aux_cache.get(key)
        if held is not None:
            return held
        if self.pin_fp32_aux and self.blocks[key].get("kind") == "fp32":
            raise RuntimeError(f"pinned FP32 auxiliary {name!r} is unexpectedly absent")
        return super().fp32(name)

    # ---- pages

    def _evict_to(self, ceiling: int) -> None:
        while self.compact_cache and self.compact_cache_bytes > ceiling:
            _, old = self.compact_cache.popitem(last=False)
            self.compact_cache_bytes -= old.compact_bytes

    def compact_page(self, name: str) -> CompactQRowPage:
        """The device page of a qrow block: a prebound page, else the LRU's copy, else a fresh
        read that joins the LRU when it fits the budget left after pinned fp32 blocks."""
        key = self._physical_key(name)
        page = self._prebound_pages.get(key)
        if page is None and key in self.compact_cache:
            page = self.compact_cache[key]
            self.compact_cache.move_to_end(key)
        if page is not None:
            self.stats.cache_hits += 1
            return page
        page = load_compact_qrow_page(self, key)
        self.stats.page_loads += 1
        self.stats.compact_h2d_bytes += page.compact_bytes
        self._note_peak(page.compact_bytes)
        room = self.compact_cache_budget - self.fp32_aux_cache_bytes
        if 0 < page.compact_bytes <= room:
            self.compact_cache[key] = page
            self.compact_cache_bytes += page.compact_bytes
            self._evict_to(room)
        return page

    def page(self, name: str) -> CompactQRowPage:
        """``QStore.page`` goes through the compact cache here, so ``weight`` and the base
        class's helpers see the same pages."""
        return self.compact_page(name)

    def set_compact_cache_budget(self, cache_mb: float) -> None:
        """Resize the page LRU and evict down to the new ceiling now."""
        budget = max(0, int(float(cache_mb) * 1e6))
        if budget < self.fp32_aux_cache_bytes:
            raise MemoryError("provider cache budget cannot evict pinned FP32 auxiliaries "
                              f"({budget} < {self.fp32_aux_cache_bytes} bytes)")
        self.compact_cache_budget = budget
        self._evict_to(budget - self.fp32_aux_cache_bytes)

    def clear_compact_cache(self) -> None:
        self.compact_cache.clear()
        self.compact_cache_bytes = 0

    def prebind(self, names: Sequence[str], *, max_resident_bytes: int | None = None) -> dict[str, int]:
        """Pin qrow pages and fp32 blocks that captured graphs point at: they never leave the
        device and aliases share one copy. With ``max_resident_bytes`` the whole pinned set is
        checked against that budget and against free device memory before anything loads."""
        if not names:
            return {"qrow_pages": 0, "fp32_tensors": 0, "resident_bytes": 0}
        wanted = list(dict.fromkeys(self._physical_key(n) for n in names))
        qrows, fp32s, need = [], [], 0
        for key in wanted:
            block = self.blocks[key]
            if block.get("kind") == "qrow":
                if key not in self._prebound_pages:
                    qrows.append(key)
                    need += int(block["w_len"]) + int(block["s_len"])
            elif block.get("kind") == "fp32":
                if key not in self._prebound_fp32:
                    fp32s.append(key)
                    need += int(block["e_len"])
            else:
                raise ValueError(f"cannot prebind unsupported block {key!r}")
        if max_resident_bytes is not None:
            budget = int(max_resident_bytes)
            if budget <= 0:
                raise ValueError("prebound residency budget must be positive")
            held = self._prebound_compact_bytes + self._prebound_fp32_bytes
            if held + need > budget:
                raise MemoryError(f"prebound linked pages exceed their explicit residency budget "
                                  f"({held + need} > {budget} bytes)")
            free, _ = torch.cuda.mem_get_info(self.device)
            if need and held + need > int(free):
                raise MemoryError(f"prebound linked pages exceed currently free device memory "
                                  f"({held + need} > {int(free)} bytes)")
        for key in qrows:
            page = self.compact_cache.pop(key, None)
            if page is not None:
                self.compact_cache_bytes -= page.compact_bytes
            else:
                page = load_compact_qrow_page(self, key)
                self.stats.page_loads += 1
                self.stats.compact_h2d_bytes += page.compact_bytes
            self._prebound_pages[key] = page
            self._prebound_compact_bytes += page.compact_bytes
            self._note_peak()
        for key in fp32s:
            tensor = super().fp32(key).contiguous()
            self._prebound_fp32[key] = tensor
            self._prebound_fp32_bytes += _tensor_bytes(tensor)
            self._note_peak()
        return {"qrow_pages": len(qrows), "fp32_tensors": len(fp32s),
                "resident_bytes": self._prebound_compact_bytes + self._prebound_fp32_bytes}

    def prepare_resident_exact_head(self, name: str = "lm_head", *, max_resident_bytes: int) -> torch.Tensor:
        """Keep one qrow head dequantised to fp32 on the device (admitted against the budget
        and free memory from the manifest before allocating; no silent fallback)."""
        if max_resident_bytes <= 0:
            raise ValueError("resident exact-head budget must be positive")
        key = self._physical_key(name)
        held = self.resident_exact_heads.get(key)
        if held is not None:
            if _tensor_bytes(held) > max_resident_bytes:
                raise MemoryError("existing resident exact head exceeds the requested budget")
            return held
        block = self.blocks[key]
        if block.get("kind") != "qrow":
            raise ValueError(f"resident exact head {name!r} is not a qrow block")
        rows, cols = (int(v) for v in block["shape"])
        need = rows * cols * 4
        if need > max_resident_bytes:
            raise MemoryError(f"resident exact FP32 head exceeds its admission budget "
                              f"({need} > {max_resident_bytes} bytes)")
        free, _ = torch.cuda.mem_get_info(self.device)
        if need > int(free):
            raise MemoryError(f"resident exact FP32 head exceeds currently free device memory ({need} > {int(free)} bytes)")
        page = self.compact_page(name)
        head = (page.codes.float() * page.scales[:, None]).contiguous()
        self.resident_exact_heads[key] = head
        self.resident_exact_head_budget_bytes = int(max_resident_bytes)
        self.resident_exact_head_bytes += _tensor_bytes(head)
        self.stats.resident_exact_head_loads += 1
        return head

    def resident_exact_head_fp32(self, name: str = "lm_head") -> torch.Tensor | None:
        return self.resident_exact_heads.get(self._physical_key(name))

    # ---- projections

    def _count_projection(self, pages: Sequence[CompactQRowPage], impl: str, *, paired: bool) -> None:
        st = self.stats
        n = len(pages)
        st.projection_calls += n
        st.compact_logical_bytes += sum(p.compact_bytes for p in pages)
        if paired:
            st.paired_swiglu_calls += 1
        native = impl.startswith("b200")
        if native:
            st.triton_projection_calls += n
            st.triton_paired_swiglu_calls += int(paired)
            st.expanded_fp32_bytes_avoided += sum(p.expanded_fp32_bytes for p in pages)
            st.expanded_compute_bytes_avoided += sum(p.expanded_compute_bytes(self.compute_dtype) for p in pages)
        else:  # pragma: no cover - every projection here is native
            st.reference_projection_calls += n
            st.reference_paired_swiglu_calls += int(paired)

    def _matmul_page(self, page: CompactQRowPage, activations: torch.Tensor) -> torch.Tensor:
        out, impl = fused_qrow_matmul(page, activations, require_triton=self.require_triton,
                                      block_m=self.stable_block_m)
        self._count_projection((page,), impl, paired=False)
        return out

    def _fused_swiglu_pages(self, gate_page: CompactQRowPage, up_page: CompactQRowPage,
                            activations: torch.Tensor) -> tuple[torch.Tensor, str]:
        out, impl = fused_qrow_swiglu(gate_page, up_page, activations, require_triton=self.require_triton,
                                      block_m=self.stable_block_m)
        self._count_projection((gate_page, up_page), impl, paired=True)
        return out, impl

    def fused_swiglu(self, gate_name: str, up_name: str, activations: torch.Tensor) -> tuple[torch.Tensor, str]:
        return self._fused_swiglu_pages(self.compact_page(gate_name), self.compact_page(up_name), activations)

    def matmul(self, name: str, x: torch.Tensor) -> torch.Tensor:
        return self._matmul_page(self.compact_page(name), x)

    def embed_rows(self, name: str, ids) -> torch.Tensor:
        """Rows of a qrow block dequantised in the compute dtype, from its device page."""
        from .qstore_build import embed_rows as gather_rows

        page = self.compact_page(name)
        index = torch.as_tensor(ids, dtype=torch.long, device=page.codes.device)
        if index.numel() and (int(index.min()) < 0 or int(index.max()) >= page.out_features):
            raise IndexError("embedding id out of range")
        rows = gather_rows(page.codes, page.scales, index.reshape(-1), dtype=self.compute_dtype)
        return rows.reshape(*index.shape, page.in_features)

    @torch.inference_mode()
    def selected_rows_fp32(self, name: str, ids) -> torch.Tensor:
        """fp32 [len(ids), in] for only the named rows, read straight from disk (a head
        scored on a few candidate rows never loads the whole vocabulary page)."""
        key = self._physical_key(name)
        block = self.blocks[key]
        if block.get("kind") != "qrow":
            raise ValueError(f"{name} is not a qrow block")
        index = torch.as_tensor(ids, dtype=torch.long).detach().cpu().numpy()
        if index.ndim != 1 or not index.size:
            raise ValueError("selected qrow IDs must be a non-empty one-dimensional array")
        rows, cols = (int(v) for v in block["shape"])
        if int(index.min()) < 0 or int(index.max()) >= rows:
            raise IndexError(f"selected qrow ID outside [0, {rows})")
        codes = np.empty((index.size, cols), dtype=np.int8)
        scales = np.empty(index.size, dtype=np.float32)
        w_off, s_off = int(block["w_off"]), int(block["s_off"])
        for i, r in enumerate(index.tolist()):
            self.w.read_into(w_off + r * cols, cols, codes[i])
            self.s.read_into(s_off + r * 4, 4, scales[i:i + 1])
        moved = codes.nbytes + scales.nbytes
        st = self.stats
        st.compact_h2d_bytes += moved
        st.selected_head_calls += 1
        st.selected_head_rows += int(index.size)
        st.selected_head_compact_bytes += moved
        st.compact_logical_bytes += moved
        self._note_peak(moved)
        dev_codes = torch.from_numpy(codes).to(self.device)
        dev_scales = torch.from_numpy(scales).to(self.device)
        return dev_codes.float() * dev_scales[:, None]

    def close(self) -> None:
        self.clear_compact_cache()
        self._prebound_pages.clear()
        self._prebound_fp32.clear()
        self.fp32_aux_cache.clear()
        self.resident_exact_heads.clear()
        self._prebound_compact_bytes = self._prebound_fp32_bytes = 0
        self.fp32_aux_cache_bytes = self.resident_exact_head_bytes = 0
        super().close()


__all__ = ["DenseQStore", "DenseQStoreStats", "load_compact_qrow_page"]
