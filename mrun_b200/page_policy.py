"""Residency planning for the HBM expert-page cache: which (layer, expert) pages stay, which
slot each page occupies, what to copy for an acquisition, plus route-history prefetch, a
compact page trace and its offline replay.

Host-side integer bookkeeping, separate from the copies it plans (``streaming.ExpertPageCache``
executes the plans on a copy stream). The rules are the reference's
(engine/qwen3_moe_cuda.py:1221-1817, replayed offline by science/qwen3_moe_page_trace.py):

* ``global-lru-v1``: evict the least recently used page outside the acquisition.
* ``layer-frequency-lru-v1``: every layer owns a quota (capacity split evenly, the first
  ``capacity % layers`` layers one more); an incoming page first replaces its own layer's
  least recently used page once the layer is at quota, else the oldest page of a layer over
  its quota, else the least recently used page; an acquisition admits its least-routed pages
  first so its most-routed pages end up most recently used.
* decode acquisitions mark their pages decode-protected (counted when evicted anyway);
  ``transient-frequency-v1`` prefill runs a layer from a transient slab, keeps the layer's
  decode-protected pages and admits only the layer's most-routed pages up to its quota,
  releasing the layer's other unprotected pages.
* route prefetch: after layer L the pages the previous step routed at layer L+1 are reserved
  and copied ahead.

One rule is this build's own, for decode steps that touch every page of every layer in
layer order (every expert hit at large batch): under that cyclic scan any LRU rule with a
budget below the working set evicts each page just before its next use (hit rate 0).
``resident-prefix-v1`` keeps the first ``capacity - ring`` pages ever admitted resident for
good and runs LRU over the remaining ``ring = 2 x max_active_pages`` slots (one layer's active
set plus the next layer's prefetch), so a 25 % budget saves the prefix's share of the copies.

Slots come from a free stack (slot 0 first; released slots are reused last-in first-out),
so physical slot numbers match the reference's for the same sequence of acquisitions.
"""
from __future__ import annotations

import hashlib
import json
from collections import Counter, OrderedDict
from collections.abc import Iterable, Sequence
from dataclasses import dataclass, field

GLOBAL_LRU = "global-lru-v1"
LAYER_FREQUENCY_LRU = "layer-frequency-lru-v1"
RESIDENT_PREFIX = "resident-prefix-v1"
CACHE_POLICIES = (GLOBAL_LRU, LAYER_FREQUENCY_LRU, RESIDENT_PREFIX)
CACHE_FILL_PREFILL = "cache-fill-v1"
TRANSIENT_FREQUENCY_PREFILL = "transient-frequency-v1"
PREFILL_POLICIES = (CACHE_FILL_PREFILL, TRANSIENT_FREQUENCY_PREFILL)

PageKey = tuple[int, int]  # (layer, expert)

_COUNTERS = (
    "page_requests", "page_hits", "page_misses", "host_to_device_bytes", "layer_acquires", "active_experts_sum",
    "evictions", "same_layer_evictions", "over_quota_evictions", "fallback_evictions",
    "transient_prefill_acquires", "transient_prefill_pages", "transient_prefill_admitted_pages",
    "transient_prefill_preserved_pages", "transient_prefill_h2d_bytes",
    "transient_prefill_resident_materialization_d2d_bytes", "transient_prefill_admission_d2d_bytes",
    "transient_prefill_replaced_pages", "transient_prefill_skipped_protected_pages",
    "decode_protected_promotions", "decode_protected_demotions",
)


class ResidencyStats(dict):
    """The reference cache's counters (``PageCacheStats``) with its derived rates."""

    def __init__(self) -> None:
        super().__init__({name: 0 for name in _COUNTERS})

    def as_dict(self) -> dict:
        out = dict(self)
        out["hit_rate"] = self["page_hits"] / max(1, self["page_requests"])
        out["host_to_device_gb"] = self["host_to_device_bytes"] / 1e9
        out["mean_active_experts"] = self["active_experts_sum"] / max(1, self["layer_acquires"])
        return out


@dataclass
class AcquirePlan:
    """A resident acquisition: ``experts`` sorted, ``slots[i]`` holds ``experts[i]``'s page;
    ``copies`` are the (expert, slot) pages to bring from the host, in admission order."""

    layer: int
    experts: list[int]
    slots: list[int]
    copies: list[tuple[int, int]]


@dataclass
class TransientPlan:
    """A transient prefill acquisition. The slab holds ``slab_experts`` in order: the newly
    admitted misses, the other misses (both copied from the host), then the resident pages
    (copied from ``resident_slots`` before any slot is reused). ``admissions`` are the
    (slab position, slot) pages to copy from the slab into the cache afterwards;
    ``group_slots[i]`` is the slab position of ``experts[i]``."""

    layer: int
    experts: list[int]
    slab_experts: list[int]
    host_count: int
    resident_slots: list[int]
    admissions: list[tuple[int, int]]
    group_slots: list[int]


class ExpertResidency:
    def __init__(self, *, layers: int, experts: int, capacity: int, page_bytes: int, max_active_pages: int,
                 cache_policy: str = GLOBAL_LRU, prefill_page_policy: str = CACHE_FILL_PREFILL,
                 route_prefetch: bool = False) -> None:
        if cache_policy not in CACHE_POLICIES:
            raise ValueError(f"unsupported cache policy {cache_policy!r}; expected one of {sorted(CACHE_POLICIES)}")
        if prefill_page_policy not in PREFILL_POLICIES:
            raise ValueError(f"unsupported prefill page policy {prefill_page_policy!r}; "
                             f"expected one of {sorted(PREFILL_POLICIES)}")
        if prefill_page_policy == TRANSIENT_FREQUENCY_PREFILL and cache_policy != LAYER_FREQUENCY_LRU:
            raise ValueError("transient-frequency-v1 prefill needs layer-frequency-lru-v1 (per-layer quotas)")
        if prefill_page_policy == TRANSIENT_FREQUENCY_PREFILL and route_prefetch:
            raise ValueError("transient-frequency-v1 prefill excludes route prefetch (speculative pages would "
                             "evict decode-protected ones)")
        if capacity < 1 or layers < 1 or experts < 1:
            raise ValueError("capacity, layers and experts must be positive")
        self.layers, self.experts = int(layers), int(experts)
        self.capacity = int(capacity)
        self.page_bytes = int(page_bytes)
        self.max_active_pages = int(max_active_pages)
        self.cache_policy = cache_policy
        self.prefill_page_policy = prefill_page_policy
        self.route_prefetch = bool(route_prefetch)
        base, extra = divmod(self.capacity, self.layers)
        self.layer_quotas = tuple(base + (1 if layer < extra else 0) for layer in range(self.layers))
        ring = 2 * self.max_active_pages
        self.prefix_pages = max(0, self.capacity - ring) if cache_policy == RESIDENT_PREFIX else 0
        self.reset(clear_pages=True)

    # ---- state

    def reset(self, *, clear_pages: bool) -> None:
        self.stats = ResidencyStats()
        self.prefetch_stats = {"prefetched_pages": 0, "prefetch_rounds": 0}
        self.prev_routes: dict[int, list[int]] = {}
        if clear_pages:
            self.entries: OrderedDict[PageKey, int] = OrderedDict()  # LRU order, oldest first
            self.decode_protected: set[PageKey] = set()
            self.free_slots = list(range(self.capacity - 1, -1, -1))
            self.layer_counts = [0] * self.layers
            self.pinned: set[PageKey] = set()

    def slot_of(self, key: PageKey) -> int | None:
        return self.entries.get(key)

    def _victim(self, key: PageKey, protected: set[PageKey]) -> tuple[PageKey | None, str]:
        def first(pred) -> PageKey | None:
            return next((k for k in self.entries if k not in protected and pred(k)), None)

        if self.cache_policy == RESIDENT_PREFIX:
            return first(lambda k: k not in self.pinned), "fallback"

        if self.cache_policy == LAYER_FREQUENCY_LRU:
            layer = key[0]
            own = first(lambda k: k[0] == layer)
            if own is not None and self.layer_counts[layer] >= self.layer_quotas[layer]:
                return own, "same_layer"
            over = first(lambda k: self.layer_counts[k[0]] > self.layer_quotas[k[0]])
            if over is not None:
                return over, "over_quota"
        return first(lambda k: True), "fallback"

    def _reserve(self, key: PageKey, protected: set[PageKey]) -> int | None:
        """A slot for `key` (free, else the policy's victim's); None when all are protected."""
        if self.free_slots:
            slot = self.free_slots.pop()
        else:
            victim, reason = self._victim(key, protected)
            if victim is None:
                return None
            slot = self.entries.pop(victim)
            if victim in self.decode_protected:
                self.decode_protected.discard(victim)
                self.stats["decode_protected_demotions"] += 1
            self.layer_counts[victim[0]] -= 1
            self.stats["evictions"] += 1
            self.stats[f"{reason}_evictions"] += 1
        self.entries[key] = slot
        self.layer_counts[key[0]] += 1
        if len(self.pinned) < self.prefix_pages:
            self.pinned.add(key)
        return slot

    def _count_request(self, n: int, misses: int) -> None:
        self.stats["page_requests"] += n
        self.stats["page_hits"] += n - misses
        self.stats["page_misses"] += misses
        self.stats["host_to_device_bytes"] += misses * self.page_bytes
        self.stats["layer_acquires"] += 1
        self.stats["active_experts_sum"] += n

    # ---- acquisitions

    def acquire(self, layer: int, routed: Iterable[int], *, protect: bool) -> AcquirePlan:
        """Make every expert routed at `layer` resident (protect: a decode acquisition)."""
        freq = Counter(int(e) for e in routed)
        experts = sorted(freq)
        if len(experts) > self.max_active_pages:
            raise RuntimeError(f"active expert set {len(experts)} exceeds staging limit {self.max_active_pages}")
        keys = [(int(layer), e) for e in experts]
        protected = set(keys)
        order = keys
        if self.cache_policy == LAYER_FREQUENCY_LRU:
            order = sorted(keys, key=lambda k: (freq[k[1]], k[1]))  # most-routed admitted last
        copies = []
        for key in order:
            if key in self.entries:
                self.entries.move_to_end(key)
                continue
            slot = self._reserve(key, protected)
            if slot is None:
                raise RuntimeError("expert cache cannot evict a page from the active set")
            copies.append((key[1], slot))
        self._count_request(len(keys), len(copies))
        if protect:
            fresh = protected - self.decode_protected
            self.decode_protected |= protected
            self.stats["decode_protected_promotions"] += len(fresh)
        plan = AcquirePlan(int(layer), experts, [self.entries[k] for k in keys], copies)
        if self.route_prefetch:
            self.prev_routes[int(layer)] = experts
        return plan

    def reserve(self, layer: int, experts: Sequence[int], protected: set[PageKey]) -> list[tuple[int, int]]:
        """Caller-predicted pages of `layer` (a prefetch): (expert, slot) for each expert not
        yet resident, never evicting `protected`; stops when only protected pages remain."""
        copies = []
        for expert in experts:
            key = (int(layer), int(expert))
            if key in self.entries:
                continue
            slot = self._reserve(key, protected | {key})
            if slot is None:
                break
            copies.append((key[1], slot))
        if copies:
            self.stats["host_to_device_bytes"] += len(copies) * self.page_bytes
            self.prefetch_stats["prefetched_pages"] += len(copies)
            self.prefetch_stats["prefetch_rounds"] += 1
        return copies

    def prefetch_next_layer(self, layer: int, protected: set[PageKey]) -> list[tuple[int, int]]:
        """(expert, slot) pages to copy ahead for layer + 1: what the previous step routed
        there and is not resident. Call after `acquire(layer)` of the current step, before
        that acquisition's routes replace the history."""
        nxt = int(layer) + 1
        predicted = self.prev_routes.get(nxt)
        if not predicted:
            return []
        copies = []
        for expert in [e for e in predicted if (nxt, e) not in self.entries][: self.max_active_pages]:
            slot = self._reserve((nxt, expert), protected)
            if slot is None:
                break  # the protected set fills the cache
            copies.append((expert, slot))
        if copies:
            self.stats["host_to_device_bytes"] += len(copies) * self.page_bytes
            self.prefetch_stats["prefetched_pages"] += len(copies)
            self.prefetch_stats["prefetch_rounds"] += 1
        return copies

    def acquire_transient_prefill(self, layer: int, routed: Iterable[int]) -> TransientPlan:
        """Run a prefill layer from a transient slab and keep only its hottest pages."""
        if self.prefill_page_policy != TRANSIENT_FREQUENCY_PREFILL:
            raise RuntimeError("transient prefill acquisition requires transient-frequency-v1")
        layer = int(layer)
        freq = Counter(int(e) for e in routed)
        experts = sorted(freq)
        if len(experts) > self.max_active_pages:
            raise RuntimeError(f"active expert set {len(experts)} exceeds staging limit {self.max_active_pages}")
        keys = [(layer, e) for e in experts]
        resident = [k for k in keys if k in self.entries]
        resident_set = set(resident)
        held = sum(1 for k in self.decode_protected if k[0] == layer and k in self.entries)
        seed = sorted((k for k in keys if k not in self.decode_protected),
                      key=lambda k: (-freq[k[1]], k[1]))[: max(0, self.layer_quotas[layer] - held)]
        seed_set = set(seed)
        stale = [k for k in self.entries if k[0] == layer and k not in self.decode_protected and k not in seed_set]
        admit = [k for k in seed if k not in self.entries]
        admit_set = set(admit)
        host_keys = admit + [k for k in keys if k not in resident_set and k not in admit_set]
        slab_keys = host_keys + resident
        resident_slots = [self.entries[k] for k in resident]  # read before stale slots are reused
        for key in stale:
            self.free_slots.append(self.entries.pop(key))
            self.layer_counts[layer] -= 1
        admissions = []
        protected = self.decode_protected | set(keys)
        for position, key in enumerate(admit):
            slot = self._reserve(key, protected)
            if slot is None:
                break
            admissions.append((position, slot))
        where = {k[1]: i for i, k in enumerate(slab_keys)}
        page = self.page_bytes
        st = self.stats
        self._count_request(len(keys), len(host_keys))
        st["transient_prefill_acquires"] += 1
        st["transient_prefill_pages"] += len(keys)
        st["transient_prefill_admitted_pages"] += len(admissions)
        st["transient_prefill_preserved_pages"] += len(resident_set.difference(stale))
        st["transient_prefill_h2d_bytes"] += len(host_keys) * page
        st["transient_prefill_resident_materialization_d2d_bytes"] += len(resident) * page
        st["transient_prefill_admission_d2d_bytes"] += len(admissions) * page
        st["transient_prefill_replaced_pages"] += len(stale)
        st["transient_prefill_skipped_protected_pages"] += len(admit) - len(admissions)
        return TransientPlan(layer, experts, [k[1] for k in slab_keys], len(host_keys), resident_slots, admissions,
                             [where[e] for e in experts])


def options_from_env(*, cache_policy: str | None = None, prefill_page_policy: str | None = None,
                     route_prefetch: bool | None = None, page_trace: bool | None = None,
                     environ=None) -> dict:
    """Fill the options a caller left as None from the reference's environment switches
    (engine/qwen3_moe_cuda.py:1239-1330): MRUN_QWEN3_MOE_CACHE_POLICY (default global-lru-v1),
    MRUN_QWEN3_MOE_PREFILL_PAGE_POLICY (default cache-fill-v1), MRUN_QWEN3_MOE_ROUTE_PREFETCH
    (on unless empty or "0") and MRUN_QWEN3_MOE_PAGE_TRACE (off for empty, 0, false, no, off).
    Explicit arguments win."""
    import os

    env = os.environ if environ is None else environ
    if cache_policy is None:
        cache_policy = env.get("MRUN_QWEN3_MOE_CACHE_POLICY", GLOBAL_LRU)
    if prefill_page_policy is None:
        prefill_page_policy = env.get("MRUN_QWEN3_MOE_PREFILL_PAGE_POLICY", CACHE_FILL_PREFILL)
    if route_prefetch is None:
        route_prefetch = env.get("MRUN_QWEN3_MOE_ROUTE_PREFETCH", "").strip() not in ("", "0")
    if page_trace is None:
        page_trace = env.get("MRUN_QWEN3_MOE_PAGE_TRACE", "").strip().lower() not in ("", "0", "false", "no", "off")
    return {"cache_policy": str(cache_policy).strip().lower(),
            "prefill_page_policy": str(prefill_page_policy).strip().lower(),
            "route_prefetch": bool(route_prefetch), "page_trace": bool(page_trace)}


# ------------------------------------------------------------------ page trace and replay


@dataclass
class PageTrace:
    """Compact acquisition trace: per event the phase, decode step, layer and the
    (expert, route count) pairs -- page ids and counts only, never page bytes (the reference's
    trace format, science/qwen3_moe_page_trace.py:97-234)."""

    layer_count: int
    page_bytes: int
    events: list[dict] = field(default_factory=list)
    max_events: int = 250_000

    def record(self, *, phase: str, step: int, layer: int, routed: Iterable[int]) -> None:
        if phase not in ("prefill", "decode"):
            raise ValueError("phase must be 'prefill' or 'decode'")
        if len(self.events) >= self.max_events:
            raise RuntimeError(f"page trace exceeds {self.max_events} events")
        pages = sorted(Counter(int(e) for e in routed).items())
        if not pages:
            raise ValueError("an event routes at least one page")
        self.events.append({"phase": phase, "step": int(step), "layer": int(layer),
                            "pages": [[e, c] for e, c in pages]})

    def as_dict(self) -> dict:
        return {"schema": "mrun-qwen3-moe-page-trace-v1", "layer_count": self.layer_count,
                "page_bytes": self.page_bytes, "events": self.events}

    def sha256(self) -> str:
        text = json.dumps(self.as_dict(), sort_keys=True, separators=(",", ":")).encode()
        return hashlib.sha256(text).hexdigest()

    @classmethod
    def from_dict(cls, payload: dict) -> "PageTrace":
        trace = cls(int(payload["layer_count"]), int(payload["page_bytes"]))
        for ev in payload["events"]:
            routed = [e for e, c in ev["pages"] for _ in range(int(c))]
            trace.record(phase=ev["phase"], step=ev.get("step", 0), layer=ev["layer"], routed=routed)
        return trace


def replay(trace: PageTrace, *, capacity_pages: int, cache_policy: str, prefill_page_policy: str,
           max_active_pages: int | None = None) -> dict:
    """Replay a trace through the residency rules (no copies): the counters a live cache of
    `capacity_pages` pages would report, and the resident set at the end."""
    res = ExpertResidency(layers=trace.layer_count, experts=1 + max(e for ev in trace.events for e, _ in ev["pages"]),
                          capacity=capacity_pages, page_bytes=trace.page_bytes,
                          max_active_pages=max_active_pages or capacity_pages, cache_policy=cache_policy,
                          prefill_page_policy=prefill_page_policy)
    peak = 0
    for ev in trace.events:
        if len(ev["pages"]) > capacity_pages:
            raise ValueError(f"event requests {len(ev['pages'])} pages; the budget holds {capacity_pages}")
        routed = [e for e, c in ev["pages"] for _ in range(int(c))]
        if ev["phase"] == "prefill" and prefill_page_policy == TRANSIENT_FREQUENCY_PREFILL:
            res.acquire_transient_prefill(ev["layer"], routed)
        else:
            res.acquire(ev["layer"], routed, protect=ev["phase"] == "decode")
        peak = max(peak, len(res.entries))
    out = res.stats.as_dict()
    out.update({"peak_resident_pages": peak, "final_resident_pages": len(res.entries),
                "resident": [[k[0], k[1]] for k in res.entries], "layer_quotas": list(res.layer_quotas)})
    return out


def replay_ab(trace: PageTrace, *, capacity_pages: int) -> dict:
    """Both policy arms over one trace and budget (science/qwen3_moe_page_trace.py:548-614):
    baseline global-LRU with cache-fill prefill, candidate layer-frequency LRU with transient
    prefill, and the transfer bytes the candidate saves. A policy simulation, not a runtime
    measurement."""
    base = replay(trace, capacity_pages=capacity_pages, cache_policy=GLOBAL_LRU, prefill_page_policy=CACHE_FILL_PREFILL)
    cand = replay(trace, capacity_pages=capacity_pages, cache_policy=LAYER_FREQUENCY_LRU,
                  prefill_page_policy=TRANSIENT_FREQUENCY_PREFILL)
    saved = base["host_to_device_bytes"] - cand["host_to_device_bytes"]
    return {
        "trace_sha256": trace.sha256(),
        "capacity_pages": capacity_pages,
        "arms": {"baseline": base, "candidate": cand},
        "comparison": {
            "candidate_minus_baseline_hits": cand["page_hits"] - base["page_hits"],
            "candidate_minus_baseline_misses": cand["page_misses"] - base["page_misses"],
            "candidate_minus_baseline_evictions": cand["evictions"] - base["evictions"],
            "signed_h2d_bytes_saved": saved,
            "transfer_reduction_fraction": max(0, saved) / base["host_to_device_bytes"]
            if base["host_to_device_bytes"] else 0.0,
        },
    }


def main(argv: Sequence[str] | None = None) -> int:
    """``python -m mrun_b200.page_policy TRACE.json --capacity-pages N``: print the A/B replay."""
    import argparse

    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("trace")
    ap.add_argument("--capacity-pages", type=int, required=True)
    args = ap.parse_args(argv)
    with open(args.trace, encoding="utf-8") as f:
        trace = PageTrace.from_dict(json.load(f))
    print(json.dumps(replay_ab(trace, capacity_pages=args.capacity_pages), indent=1, sort_keys=True))
    return 0


__all__ = ["AcquirePlan", "CACHE_FILL_PREFILL", "CACHE_POLICIES", "ExpertResidency", "GLOBAL_LRU", "RESIDENT_PREFIX",
           "LAYER_FREQUENCY_LRU", "PREFILL_POLICIES", "PageTrace", "ResidencyStats", "TRANSIENT_FREQUENCY_PREFILL",
           "TransientPlan", "options_from_env", "replay", "replay_ab"]


if __name__ == "__main__":
    raise SystemExit(main())
