"""Generate the expert-page residency fixtures from the reference implementation.

Run where the reference sources are available (path as the first argument or in
MRUN_REFERENCE_SRC); the output ``page_policy.json`` is committed so the tests need no
reference at run time. A seeded synthetic route trace (one prefill pass over every layer,
then decode steps with skewed top-k routes) is fed to the reference's live
``ExpertPageCache`` on the CPU (a fake page store; slot numbers and counters do not depend
on page bytes) under three policy arms, recording every acquisition's selected experts and
physical slots and the final counters, and to the reference's offline replay simulator.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LAYERS, EXPERTS, TOP_K, ROWS = 4, 24, 2, 2
CAPACITY, MAX_ACTIVE = 30, 12
PAGE = 64
ARMS = [
    ("global-lru-v1", "cache-fill-v1"),
    ("layer-frequency-lru-v1", "cache-fill-v1"),
    ("layer-frequency-lru-v1", "transient-frequency-v1"),
]


def synthetic_trace() -> list[dict]:
    """Events: phase, step, layer, routed expert ids (with repeats, as top-k rows give)."""
    rng = np.random.default_rng(424242)
    weights = 1.0 / (1.0 + np.arange(EXPERTS)) ** 1.3
    events = []
    # prefill: 16 prompt tokens per layer, top-k each (many distinct experts, capped)
    for layer in range(LAYERS):
        perm = rng.permutation(EXPERTS)
        routed = []
        for _ in range(16):
            routed += [int(perm[e]) for e in rng.choice(EXPERTS, TOP_K, replace=False, p=weights / weights.sum())]
        distinct = sorted(set(routed))[:MAX_ACTIVE]
        routed = [e for e in routed if e in distinct]
        events.append({"phase": "prefill", "step": 0, "layer": layer, "routed": routed})
    for step in range(1, 15):
        for layer in range(LAYERS):
            routed = []
            for _ in range(ROWS):
                routed += [int(e) for e in rng.choice(EXPERTS, TOP_K, replace=False, p=weights / weights.sum())]
            events.append({"phase": "decode", "step": step, "layer": layer, "routed": routed})
    return events


class _Layout:
    page_stride = PAGE


class FakeStore:
    layout = _Layout()
    layers = LAYERS
    experts = EXPERTS

    def gather(self, layer, expert_ids, target):
        for i, e in enumerate(expert_ids):
            target[i].fill_((layer * EXPERTS + int(e)) % 251)

    def view_pages(self, raw):
        return raw


def run_live(ref, events, cache_policy, prefill_policy):
    import torch

    cache = ref.ExpertPageCache(FakeStore(), device="cpu", cache_mb=CAPACITY * PAGE / 1e6, max_active_pages=MAX_ACTIVE,
                                route_prefetch=False, cache_policy=cache_policy, page_binding_policy="slot-indirect-v1",
                                prefill_page_policy=prefill_policy, page_trace=False)
    log = []
    for ev in events:
        top = torch.tensor(ev["routed"], dtype=torch.long)
        if ev["phase"] == "prefill" and prefill_policy == "transient-frequency-v1":
            selected, _, group_slots = cache.acquire_transient_prefill(ev["layer"], top)
            log.append({"selected": selected.tolist(), "group_slots": group_slots.tolist()})
        else:
            selected, _, slots = cache.acquire_slot_binding(ev["layer"], top, protect=ev["phase"] == "decode")
            log.append({"selected": selected.tolist(), "slots": slots.tolist()})
    resident = [[k[0], k[1], s] for k, s in cache.entries.items()]
    return {"acquires": log, "stats": cache.stats.as_dict(), "resident": resident,
            "capacity": cache.capacity, "quotas": list(cache.layer_quotas)}


def run_replay(trace_mod, events, cache_policy, prefill_policy):
    from collections import Counter

    trace_events = tuple(
        trace_mod.PageTraceEvent(phase=ev["phase"], step=ev["step"], layer=ev["layer"],
                                 pages=tuple(sorted(Counter(ev["routed"]).items())))
        for ev in events)
    trace = trace_mod.PageAccessTrace(layer_count=LAYERS, page_bytes=PAGE, events=trace_events)
    budget = trace_mod.PageCacheBudget(page_bytes=PAGE, capacity_pages=CAPACITY)
    result = trace_mod._simulate_arm(trace, budget, name="arm", cache_policy=cache_policy,
                                     prefill_policy=prefill_policy)
    result.pop("final_resident_sha256")
    return result


def main() -> None:
    ref_src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MRUN_REFERENCE_SRC")
    if not ref_src:
        raise SystemExit("usage: make_page_policy_fixtures.py <reference src directory>")
    sys.path.insert(0, ref_src)
    from mrun.engine import qwen3_moe_cuda as ref
    from mrun.science import qwen3_moe_page_trace as trace_mod

    events = synthetic_trace()
    out = {"layers": LAYERS, "experts": EXPERTS, "capacity": CAPACITY, "max_active_pages": MAX_ACTIVE,
           "page_bytes": PAGE, "events": events, "arms": []}
    for cache_policy, prefill_policy in ARMS:
        out["arms"].append({"cache_policy": cache_policy, "prefill_page_policy": prefill_policy,
                            "live": run_live(ref, events, cache_policy, prefill_policy),
                            "replay": run_replay(trace_mod, events, cache_policy, prefill_policy)})
    (HERE / "page_policy.json").write_text(json.dumps(out, indent=0, sort_keys=True) + "\n")
    for arm in out["arms"]:
        st = arm["live"]["stats"]
        print(arm["cache_policy"], arm["prefill_page_policy"], "hits", st["page_hits"], "misses", st["page_misses"],
              "evictions", st["evictions"])


if __name__ == "__main__":
    main()
