"""Weight-page streaming: expert pages live in pinned host memory and are copied into a
fixed pool of HBM slots on a side stream, overlapped with compute.

Mirrors mrun's ``HostPageTier`` / ``ExpertPageCache`` (engine/qwen3_moe_cuda.py:878-1817):
a pinned host tier holds every expert page; an HBM slot cache (capacity from a byte budget)
serves the experts a layer routes to. Which pages stay and which slot each occupies is
planned by ``page_policy.ExpertResidency`` (the reference's global-LRU and layer-frequency
policies, transient-frequency prefill, route-history prefetch); this module executes the
plans: host pages are copied by ``mrb_copy_pages`` (one cudaMemcpyAsync per page) on a copy
stream and the compute stream waits on per-slot ready events. A slot is only overwritten
after the compute stream has passed its last use (per-slot release events), so streaming
never changes a result: pages in HBM are byte-identical to the host tier.
"""
from __future__ import annotations

import weakref
from dataclasses import dataclass

import torch

from . import _lib
from .moe import ExpertPageLayout
from .page_policy import TRANSIENT_FREQUENCY_PREFILL, ExpertResidency, PageTrace, options_from_env


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


EXPERT_STORE_SCHEMA = "mrun-b200-int8-expert-store-v1"
EXPERT_STORE_FILE = "expert_pages.u8"


def write_expert_store(directory, layout: ExpertPageLayout, pages) -> dict:
    """Write expert pages [layers, experts, page_stride] uint8 as an on-disk expert store: one
    data file of pages in (layer, expert) order plus ``manifest.json`` (the reference's packed
    expert-store manifest keys, engine/qwen3_moe_cuda.py:780-842, for this build's int8 page
    layout). Returns the manifest."""
    import json
    from pathlib import Path

    import numpy as np

    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    data = pages.cpu().numpy() if isinstance(pages, torch.Tensor) else np.asarray(pages)
    if data.dtype != np.uint8 or data.ndim != 3 or data.shape[2] != layout.page_stride:
        raise ValueError("pages must be uint8 [layers, experts, page_stride]")
    np.ascontiguousarray(data).tofile(directory / EXPERT_STORE_FILE)
    manifest = {"schema_version": EXPERT_STORE_SCHEMA, "layout": layout.as_dict(), "layers": int(data.shape[0]),
                "num_experts": int(data.shape[1]), "data_file": EXPERT_STORE_FILE}
    (directory / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    return manifest


class ExpertPageStore:
    """On-disk expert pages read with the library's parallel positional reader (the
    reference's ``PackedFP8ExpertStore`` role, engine/qwen3_moe_cuda.py:780-842, with the int8
    page layout): the manifest names the layout, the layer and expert counts and the data file
    of [layers * experts, page_stride] bytes."""

    def __init__(self, store_dir) -> None:
        import json
        from pathlib import Path

        from .qstore import StoreFile

        self.store_dir = Path(store_dir)
        manifest = json.loads((self.store_dir / "manifest.json").read_text(encoding="utf-8"))
        if manifest.get("schema_version") != EXPERT_STORE_SCHEMA:
            raise ValueError("unsupported expert store schema")
        self.layout = ExpertPageLayout(**{k: int(v) for k, v in manifest["layout"].items()})
        if self.layout != ExpertPageLayout.create(self.layout.hidden_size, self.layout.intermediate_size):
            raise ValueError("expert store layout does not match the int8 page layout")
        self.layers, self.experts = int(manifest["layers"]), int(manifest["num_experts"])
        if self.layers < 1 or self.experts < 1:
            raise ValueError("expert store must contain layers and experts")
        self.file = StoreFile(self.store_dir / manifest["data_file"])
        if self.file.size != self.layers * self.experts * self.layout.page_stride:
            self.file.close()
            raise ValueError("expert store byte length does not match its page geometry")

    def global_page(self, layer: int, expert: int) -> int:
        return layer * self.experts + expert

    def gather(self, layer: int, expert_ids, target: torch.Tensor, *, threads: int = 4) -> None:
        """Pages of `layer`'s `expert_ids` into host uint8 rows target[:len(expert_ids)]."""
        stride = self.layout.page_stride
        if target.is_cuda or target.dtype != torch.uint8 or target.shape[-1] != stride:
            raise ValueError("expert page staging target must be a host uint8 [n, page_stride] tensor")
        for i, expert in enumerate(expert_ids):
            if not 0 <= int(expert) < self.experts or not 0 <= int(layer) < self.layers:
                raise IndexError(f"expert page ({layer}, {expert}) outside the store")
            self.file.read_into(self.global_page(int(layer), int(expert)) * stride, stride, target[i], threads=threads)

    def close(self) -> None:
        self.file.close()


_REGISTER_BYTES = 1 << 30


def _host_unregister(pages: torch.Tensor) -> None:
    torch.cuda.cudart().cudaHostUnregister(pages.data_ptr())


class HostPageTier:
    """Pinned host copy of every expert page: [layers, experts, page_stride] uint8."""

    def __init__(self, layout: ExpertPageLayout, layers: int, experts: int, *, pin: bool = True) -> None:
        self.layout = layout
        self.layers = layers
        self.experts = experts
        shape = (layers, experts, layout.page_stride)
        nbytes = layers * experts * layout.page_stride
        if pin and nbytes >= _REGISTER_BYTES:
            # torch's pinned allocator rounds every block up to a power of two (a 45 GB tier
            # would take 64 GB); page-locking an ordinary allocation costs exactly its size
            self.pages = torch.empty(shape, dtype=torch.uint8)
            rc = torch.cuda.cudart().cudaHostRegister(self.pages.data_ptr(), nbytes, 0)
            if int(rc) != 0:
                raise RuntimeError(f"cudaHostRegister of the {nbytes} B host tier failed ({int(rc)})")
            weakref.finalize(self, _host_unregister, self.pages)
        else:
            self.pages = torch.empty(shape, dtype=torch.uint8, pin_memory=pin)
        self.stats = {"warmed_pages": 0, "warm_seconds": 0.0, "pinned": bool(pin)}

    @classmethod
    def from_store(cls, store: ExpertPageStore, *, pin: bool = True, threads: int | None = None) -> "HostPageTier":
        """Fill the tier from an on-disk store in one sequential pass of parallel reads
        straight into the (pinned) tier -- the reference's pread warm-up of
        ``HostPageTier.warm`` (engine/qwen3_moe_cuda.py:925-951), without a memory map."""
        import time

        from .qstore import DEFAULT_READ_THREADS

        tier = cls(store.layout, store.layers, store.experts, pin=pin)
        started = time.perf_counter()
        store.file.read_into(0, tier.pages.numel(), tier.pages, threads=threads or DEFAULT_READ_THREADS)
        tier.stats.update(warmed_pages=store.layers * store.experts, warm_seconds=time.perf_counter() - started)
        return tier

    @property
    def nbytes(self) -> int:
        return self.pages.numel()

    def page_index(self, layer: int, expert: int) -> int:
        return layer * self.experts + expert


class BudgetedHostPageTier:
    """Host-RAM tier of at most ``host_cache_mb`` of an on-disk expert store, for callers that
    stage pages themselves (the reference's ``HostPageTier`` contract,
    engine/qwen3_moe_cuda.py:878-980): ``warm()`` fills the tier with the first pages in one
    sequential pass of parallel reads; ``gather`` serves pages from the tier, else from disk,
    admitting disk pages while room remains (fill once, no eviction). Pinned when possible."""

    def __init__(self, store: ExpertPageStore, *, host_cache_mb: float, try_pin: bool = True) -> None:
        import numpy as np

        self.store = store
        stride = store.layout.page_stride
        total = store.layers * store.experts
        self.capacity = min(total, int(float(host_cache_mb) * 1e6) // stride)
        if self.capacity < 1:
            raise ValueError("host_cache_mb smaller than one expert page")
        self.pinned = False
        buf = None
        if try_pin:
            try:
                buf = torch.empty((self.capacity, stride), dtype=torch.uint8, pin_memory=True)
                self.pinned = True
            except RuntimeError:
                buf = None
        self.buf = buf if buf is not None else torch.empty((self.capacity, stride), dtype=torch.uint8)
        self._rows = np.full(total, -1, dtype=np.int64)
        self._next = 0
        self.stats = {"capacity_pages": self.capacity, "pinned": self.pinned, "warmed_pages": 0, "warm_seconds": 0.0,
                      "served_pages": 0, "admitted_pages": 0, "disk_pages": 0}

    def warm(self, *, threads: int | None = None) -> dict:
        import time

        import numpy as np

        from .qstore import DEFAULT_READ_THREADS

        started = time.perf_counter()
        stride = self.store.layout.page_stride
        if self._next < self.capacity:
            first = self._next
            self.store.file.read_into(first * stride, (self.capacity - first) * stride, self.buf[first:],
                                      threads=threads or DEFAULT_READ_THREADS)
            self._rows[first:self.capacity] = np.arange(first, self.capacity)
            self._next = self.capacity
        self.stats["warm_seconds"] = time.perf_counter() - started
        self.stats["warmed_pages"] = self._next
        return dict(self.stats)

    def gather(self, layer: int, expert_ids, target: torch.Tensor) -> None:
        """Pages of `layer`'s `expert_ids` into host uint8 rows target[:len(expert_ids)]."""
        for i, expert in enumerate(expert_ids):
            gid = self.store.global_page(int(layer), int(expert))
            row = int(self._rows[gid]) if 0 <= gid < self._rows.size else -1
            if row >= 0:
                target[i].copy_(self.buf[row])
                self.stats["served_pages"] += 1
                continue
            self.store.gather(layer, [expert], target[i:i + 1])
            self.stats["disk_pages"] += 1
            if self._next < self.capacity:
                self.buf[self._next].copy_(target[i])
                self._rows[gid] = self._next
                self._next += 1
                self.stats["admitted_pages"] += 1


class ExpertPageCache:
    """HBM slot cache over a HostPageTier, copies on a side stream.

    cache_policy / prefill_page_policy / route_prefetch select the residency rules (see
    ``page_policy``); page_trace records every acquisition's routed pages for offline replay
    (``page_policy.replay``). Options left as None come from the reference's environment
    switches (``page_policy.options_from_env``)."""

    plans_on_host = True  # every acquisition reads its routes on the host (no graph capture)

    def __init__(self, host: HostPageTier, *, budget_bytes: int, device: torch.device,
                 cache_policy: str | None = None, prefill_page_policy: str | None = None,
                 route_prefetch: bool | None = None, page_trace: bool | None = None,
                 max_active_pages: int | None = None) -> None:
        opts = options_from_env(cache_policy=cache_policy, prefill_page_policy=prefill_page_policy,
                                route_prefetch=route_prefetch, page_trace=page_trace)
        cache_policy, prefill_page_policy = opts["cache_policy"], opts["prefill_page_policy"]
        route_prefetch, page_trace = opts["route_prefetch"], opts["page_trace"]
        self.host = host
        self.layout = host.layout
        self.device = device
        stride = self.layout.page_stride
        self.capacity = max(1, int(budget_bytes // stride))
        self.max_active_pages = int(max_active_pages or min(host.experts, self.capacity))
        self.residency = ExpertResidency(layers=host.layers, experts=host.experts, capacity=self.capacity,
                                         page_bytes=stride, max_active_pages=self.max_active_pages,
                                         cache_policy=cache_policy, prefill_page_policy=prefill_page_policy,
                                         route_prefetch=route_prefetch)
        self.slots = torch.empty((self.capacity, stride), dtype=torch.uint8, device=device)
        self.ready = [torch.cuda.Event() for _ in range(self.capacity)]
        self.released = [torch.cuda.Event() for _ in range(self.capacity)]
        # transient prefill slab (pages a prefill layer runs from without keeping them)
        self.slab = (torch.empty((self.max_active_pages, stride), dtype=torch.uint8, device=device)
                     if prefill_page_policy == TRANSIENT_FREQUENCY_PREFILL else None)
        self.slab_released = torch.cuda.Event()
        self._slab_in_use = False
        self.prefetched: set[tuple[int, int]] = set()
        self.copy_stream = torch.cuda.Stream(device)
        self.stats = PageCacheStats()
        self.trace = PageTrace(host.layers, stride) if page_trace else None
        self.step = 0
        self.slot_of = torch.full((host.experts,), -1, dtype=torch.int32, device=device)
        # pinned staging for the slot map, rotated so an in-flight copy is never overwritten
        self._maps = [torch.full((host.experts,), -1, dtype=torch.int32, pin_memory=True) for _ in range(4)]
        self._map_events: list[torch.cuda.Event | None] = [None] * 4
        self._map_next = 0
        self._pending_release: list[int] = []

    @property
    def device_bytes(self) -> int:
        return self.slots.numel() + (self.slab.numel() if self.slab is not None else 0)

    @property
    def where(self):
        """Resident pages: (layer, expert) -> slot, least recently used first."""
        return self.residency.entries

    def reset(self, *, clear_pages: bool) -> None:
        self.stats = PageCacheStats()
        self.residency.reset(clear_pages=clear_pages)
        if clear_pages:
            self.prefetched.clear()

    # ------------------------------------------------------------------ copies

    def _copy_host(self, layer: int, copies: list[tuple[int, int]], dst: torch.Tensor, *, slot_events: bool) -> None:
        """Copy host pages (expert, index) of `layer` into dst[index] on the copy stream."""
        if not copies:
            return
        stride = self.layout.page_stride
        if slot_events:  # the compute stream must be done with each slot's previous page
            for _, slot in copies:
                self.copy_stream.wait_event(self.released[slot])
        idx = torch.tensor([i for _, i in copies], dtype=torch.int32)
        pages = torch.tensor([self.host.page_index(layer, e) for e, _ in copies], dtype=torch.int32)
        done = torch.cuda.Event()
        with torch.cuda.stream(self.copy_stream):
            _lib.call("mrb_copy_pages", dst.data_ptr(), stride, self.host.pages.data_ptr(), stride, idx.data_ptr(),
                      pages.data_ptr(), len(copies), stride, self.copy_stream.cuda_stream, None)
            done.record(self.copy_stream)
        if slot_events:
            for _, slot in copies:
                self.ready[slot] = done
        self.stats.bytes_h2d += len(copies) * stride

    def _evictions_since(self, before: int) -> None:
        self.stats.evictions += self.residency.stats["evictions"] - before

    def prefetch(self, layer: int, experts: list[int], *, protect_layer: int | None = None) -> None:
        """Start copying `layer`'s predicted experts (no wait); the resident pages of
        `protect_layer` are not evicted for them."""
        protect = {k for k in self.where if k[0] == protect_layer} if protect_layer is not None else set()
        before = self.residency.stats["evictions"]
        copies = self.residency.reserve(layer, experts, protect)
        self._evictions_since(before)
        self._copy_host(layer, copies, self.slots, slot_events=True)
        self.prefetched.update((layer, e) for e, _ in copies)
        self.stats.prefetched += len(copies)

    # ------------------------------------------------------------------ acquisitions

    def _publish_map(self, entries: dict[int, int], waits: list[torch.cuda.Event]) -> torch.Tensor:
        compute = torch.cuda.current_stream(self.device)
        i = self._map_next
        self._map_next = (i + 1) % len(self._maps)
        if self._map_events[i] is not None:
            self._map_events[i].synchronize()
        mapping = self._maps[i]
        mapping.fill_(-1)
        for expert, where in entries.items():
            mapping[expert] = where
        seen = set()
        for ev in waits:
            if id(ev) not in seen:
                compute.wait_event(ev)
                seen.add(id(ev))
        self.slot_of.copy_(mapping, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(compute)
        self._map_events[i] = ev
        return self.slot_of

    def layer_pages(self, layer: int, top_indices: torch.Tensor, *, prefill: bool = False):
        """(page buffer, slot_of [E] int32) for the experts `top_indices` route to; the
        current stream is ordered after their copies. Decode acquisitions (prefill False) mark
        their pages decode-protected, as the reference's decode path does."""
        routed = [int(e) for e in top_indices.reshape(-1).tolist()]  # host sync, as the reference
        if self.trace is not None:
            self.trace.record(phase="prefill" if prefill else "decode", step=self.step, layer=layer, routed=routed)
        res = self.residency
        before = res.stats["evictions"]
        if prefill and res.prefill_page_policy == TRANSIENT_FREQUENCY_PREFILL:
            return self._transient(layer, routed, before)
        plan = res.acquire(layer, routed, protect=not prefill)
        self._evictions_since(before)
        missed = {e for e, _ in plan.copies}
        for e in plan.experts:
            if e not in missed:
                self.stats.hits += 1
                if (layer, e) in self.prefetched:
                    self.stats.prefetch_hits += 1
                    self.prefetched.discard((layer, e))
        self.stats.misses += len(plan.copies)
        self._copy_host(layer, plan.copies, self.slots, slot_events=True)
        if res.route_prefetch:
            before = res.stats["evictions"]
            ahead = res.prefetch_next_layer(layer, {(layer, e) for e in plan.experts})
            self._evictions_since(before)
            self._copy_host(layer + 1, ahead, self.slots, slot_events=True)
            self.prefetched.update((layer + 1, e) for e, _ in ahead)
            self.stats.prefetched += len(ahead)
        self._pending_release = list(plan.slots)
        slot_of = self._publish_map(dict(zip(plan.experts, plan.slots)), [self.ready[s] for s in plan.slots])
        if layer == res.layers - 1 and not prefill:
            self.step += 1
        return self.slots, slot_of

    def _transient(self, layer: int, routed: list[int], evictions_before: int):
        res = self.residency
        if self._slab_in_use:
            raise RuntimeError("release_layer() must follow each transient prefill layer")
        plan = res.acquire_transient_prefill(layer, routed)
        self._evictions_since(evictions_before)
        stride = self.layout.page_stride
        self.stats.hits += len(plan.resident_slots)
        self.stats.misses += plan.host_count
        # the slab is reused only after the previous transient layer's kernels
        self.copy_stream.wait_event(self.slab_released)
        self._copy_host(layer, [(e, i) for i, e in enumerate(plan.slab_experts[:plan.host_count])], self.slab,
                        slot_events=False)
        with torch.cuda.stream(self.copy_stream):
            if plan.resident_slots:  # resident pages as they are now, before any slot is reused
                for s in plan.resident_slots:
                    self.copy_stream.wait_event(self.ready[s])
                src = torch.tensor(plan.resident_slots, dtype=torch.long, device=self.device)
                torch.index_select(self.slots, 0, src, out=self.slab[plan.host_count:len(plan.slab_experts)])
            if plan.admissions:  # the hottest new pages stay: slab -> their cache slots
                for _, s in plan.admissions:
                    self.copy_stream.wait_event(self.released[s])
                dst = torch.tensor([s for _, s in plan.admissions], dtype=torch.long, device=self.device)
                pos = torch.tensor([p for p, _ in plan.admissions], dtype=torch.long, device=self.device)
                self.slots.index_copy_(0, dst, self.slab.index_select(0, pos))
            done = torch.cuda.Event()
            done.record(self.copy_stream)
        for _, s in plan.admissions:
            self.ready[s] = done
        self._slab_in_use = True
        self._pending_release = []
        return self.slab, self._publish_map(dict(zip(plan.experts, plan.group_slots)), [done])

    def release_layer(self) -> None:
        """Mark the pages used by the last layer_pages() as free once the compute stream
        reaches this point (call after enqueuing the layer's kernels)."""
        compute = torch.cuda.current_stream(self.device)
        for slot in self._pending_release:
            ev = torch.cuda.Event()
            ev.record(compute)
            self.released[slot] = ev
        self._pending_release = []
        if self._slab_in_use:
            self.slab_released = torch.cuda.Event()
            self.slab_released.record(compute)
            self._slab_in_use = False

    def report(self) -> dict:
        return {"kind": "streamed", "capacity_pages": self.capacity, "device_bytes": self.device_bytes,
                "host_bytes": self.host.nbytes, "cache_policy": self.residency.cache_policy,
                "prefill_page_policy": self.residency.prefill_page_policy, **self.stats.as_dict(),
                "residency": self.residency.stats.as_dict(), "prefetch": dict(self.residency.prefetch_stats)}


__all__ = ["ExpertPageCache", "HostPageTier", "PageCacheStats"]
