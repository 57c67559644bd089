"""Weight-page streaming: expert pages live in pinned host memory and are copied into a
fixed pool of HBM slots on a side stream, overlapped with compute.

Mirrors mrun's ``HostPageTier`` / ``ExpertPageCache`` (engine/qwen3_moe_cuda.py:878-1817):
a pinned host tier holds every expert page; an HBM slot cache (capacity from a byte budget,
LRU) serves the experts a layer routes to; misses and predicted next-layer pages are
copied by ``mrb_copy_pages`` (one cudaMemcpyAsync per page) on a copy stream, and the
compute stream waits on per-slot ready events. A slot is only overwritten after the compute
stream has passed its last use (per-slot release events), so streaming never changes a
result: pages in HBM are byte-identical to the host tier.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass

import torch

from . import _lib
from .moe import ExpertPageLayout


@dataclass
class PageCacheStats:
    hits: int = 0
    misses: int = 0
    prefetched: int = 0
    prefetch_hits: int = 0
    evictions: int = 0
    bytes_h2d: int = 0

    def as_dict(self) -> dict[str, int]:
        return dict(self.__dict__)


class HostPageTier:
    """Pinned host copy of every expert page: [layers, experts, page_stride] uint8."""

    def __init__(self, layout: ExpertPageLayout, layers: int, experts: int) -> None:
        self.layout = layout
        self.layers = layers
        self.experts = experts
        self.pages = torch.empty((layers, experts, layout.page_stride), dtype=torch.uint8, pin_memory=True)

    @property
    def nbytes(self) -> int:
        return self.pages.numel()

    def page_index(self, layer: int, expert: int) -> int:
        return layer * self.experts + expert


class ExpertPageCache:
    """HBM slot cache over a HostPageTier (LRU; prefetch on a side stream)."""

    def __init__(self, host: HostPageTier, *, budget_bytes: int, device: torch.device) -> None:
        self.host = host
        self.layout = host.layout
        self.device = device
        stride = self.layout.page_stride
        self.capacity = max(1, int(budget_bytes // stride))
        self.slots = torch.empty((self.capacity, stride), dtype=torch.uint8, device=device)
        self.where: OrderedDict[tuple[int, int], int] = OrderedDict()  # LRU order: oldest first
        self.owner: list[tuple[int, int] | None] = [None] * self.capacity
        self.ready = [torch.cuda.Event() for _ in range(self.capacity)]
        self.released = [torch.cuda.Event() for _ in range(self.capacity)]
        self.prefetched: set[tuple[int, int]] = set()
        self.copy_stream = torch.cuda.Stream(device)
        self.stats = PageCacheStats()
        self.slot_of = torch.full((host.experts,), -1, dtype=torch.int32, device=device)
        # pinned staging for the slot map, rotated so an in-flight copy is never overwritten
        self._maps = [torch.full((host.experts,), -1, dtype=torch.int32, pin_memory=True) for _ in range(4)]
        self._map_events: list[torch.cuda.Event | None] = [None] * 4
        self._map_next = 0

    @property
    def device_bytes(self) -> int:
        return self.slots.numel()

    def reset(self, *, clear_pages: bool) -> None:
        self.stats = PageCacheStats()
        if clear_pages:
            self.where.clear()
            self.owner = [None] * self.capacity
            self.prefetched.clear()

    # ------------------------------------------------------------------ slot management

    def _victim(self, protect: set[tuple[int, int]]) -> int:
        for slot, owner in enumerate(self.owner):
            if owner is None:
                return slot
        for key in self.where:  # oldest first
            if key not in protect:
                slot = self.where.pop(key)
                self.owner[slot] = None
                self.prefetched.discard(key)
                self.stats.evictions += 1
                return slot
        raise MemoryError("expert page cache has no evictable slot (capacity below one layer's working set)")

    def _copy(self, keys: list[tuple[int, int]], protect: set[tuple[int, int]]) -> None:
        """Assign slots to `keys` and copy their pages on the copy stream."""
        if not keys:
            return
        slots, pages = [], []
        for key in keys:
            slot = self._victim(protect | set(keys))
            self.owner[slot] = key
            self.where[key] = slot
            # the compute stream must be done with the slot's previous page
            self.copy_stream.wait_event(self.released[slot])
            slots.append(slot)
            pages.append(self.host.page_index(*key))
        stride = self.layout.page_stride
        s_arr = (torch.tensor(slots, dtype=torch.int32)).contiguous()
        p_arr = (torch.tensor(pages, dtype=torch.int32)).contiguous()
        done = torch.cuda.Event()
        with torch.cuda.stream(self.copy_stream):
            _lib.call("mrb_copy_pages", self.slots.data_ptr(), stride, self.host.pages.data_ptr(), stride,
                      s_arr.data_ptr(), p_arr.data_ptr(), len(slots), stride, self.copy_stream.cuda_stream, None)
            done.record(self.copy_stream)
        for slot in slots:
            self.ready[slot] = done
        self.stats.bytes_h2d += len(slots) * stride

    def prefetch(self, layer: int, experts: list[int], *, protect_layer: int | None = None) -> None:
        """Start copying `layer`'s predicted experts (no wait)."""
        protect = {k for k in self.where if k[0] == protect_layer} if protect_layer is not None else set()
        missing = [(layer, e) for e in experts if (layer, e) not in self.where]
        self._copy(missing, protect)
        self.prefetched.update(missing)
        self.stats.prefetched += len(missing)

    def layer_pages(self, layer: int, top_indices: torch.Tensor, *, prefill: bool = False):
        """(slot buffer, slot_of [E] int32) for the experts `top_indices` route to; the
        current stream is ordered after their copies."""
        del prefill
        needed = sorted(int(e) for e in torch.unique(top_indices).tolist())  # host sync, as the reference
        keys = [(layer, e) for e in needed]
        missing = [k for k in keys if k not in self.where]
        for k in keys:
            if k in self.where:
                self.where.move_to_end(k)
                self.stats.hits += 1
                if k in self.prefetched:
                    self.stats.prefetch_hits += 1
                    self.prefetched.discard(k)
        self.stats.misses += len(missing)
        self._copy(missing, set(keys))
        compute = torch.cuda.current_stream(self.device)
        i = self._map_next
        self._map_next = (i + 1) % len(self._maps)
        if self._map_events[i] is not None:
            self._map_events[i].synchronize()
        mapping = self._maps[i]
        mapping.fill_(-1)
        waited = set()
        for k in keys:
            slot = self.where[k]
            mapping[k[1]] = slot
            ev = self.ready[slot]
            if id(ev) not in waited:
                compute.wait_event(ev)
                waited.add(id(ev))
        self.slot_of.copy_(mapping, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(compute)
        self._map_events[i] = ev
        self._pending_release = [self.where[k] for k in keys]
        return self.slots, self.slot_of

    def release_layer(self) -> None:
        """Mark the slots used by the last layer_pages() as free once the compute stream
        reaches this point (call after enqueuing the layer's kernels)."""
        compute = torch.cuda.current_stream(self.device)
        for slot in getattr(self, "_pending_release", []):
            ev = torch.cuda.Event()
            ev.record(compute)
            self.released[slot] = ev
        self._pending_release = []

    def report(self) -> dict:
        return {"kind": "streamed", "capacity_pages": self.capacity, "device_bytes": self.device_bytes,
                "host_bytes": self.host.nbytes, **self.stats.as_dict()}


__all__ = ["ExpertPageCache", "HostPageTier", "PageCacheStats"]
