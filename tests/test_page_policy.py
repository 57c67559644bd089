"""Expert-page residency planning against the reference: every acquisition's experts and
physical slots, the final counters and the resident set are identical to the reference's live
``ExpertPageCache`` on the same route trace, and the offline replay matches the reference's
replay simulator (integer bookkeeping: exact). No GPU."""
from __future__ import annotations

import json
from pathlib import Path

import pytest

from mrun_b200.page_policy import (CACHE_FILL_PREFILL, GLOBAL_LRU, LAYER_FREQUENCY_LRU, TRANSIENT_FREQUENCY_PREFILL,
                                   ExpertResidency, PageTrace, replay)

FIXTURE = json.loads((Path(__file__).resolve().parent / "golden" / "page_policy.json").read_text())


def _residency(arm, **kw):
    return ExpertResidency(layers=FIXTURE["layers"], experts=FIXTURE["experts"], capacity=arm["live"]["capacity"],
                           page_bytes=FIXTURE["page_bytes"], max_active_pages=FIXTURE["max_active_pages"],
                           cache_policy=arm["cache_policy"], prefill_page_policy=arm["prefill_page_policy"], **kw)


@pytest.mark.parametrize("index", range(len(FIXTURE["arms"])))
def test_live_cache_slots_and_counters_match_reference(index):
    arm = FIXTURE["arms"][index]
    res = _residency(arm)
    assert list(res.layer_quotas) == arm["live"]["quotas"]
    transient = arm["prefill_page_policy"] == TRANSIENT_FREQUENCY_PREFILL
    for i, (ev, want) in enumerate(zip(FIXTURE["events"], arm["live"]["acquires"])):
        if ev["phase"] == "prefill" and transient:
            plan = res.acquire_transient_prefill(ev["layer"], ev["routed"])
            assert plan.experts == want["selected"] and plan.group_slots == want["group_slots"], i
        else:
            plan = res.acquire(ev["layer"], ev["routed"], protect=ev["phase"] == "decode")
            assert plan.experts == want["selected"] and plan.slots == want["slots"], i
    got = res.stats.as_dict()
    for name, value in arm["live"]["stats"].items():
        assert got[name] == pytest.approx(value, rel=0, abs=1e-12), name
    assert [[k[0], k[1], s] for k, s in res.entries.items()] == arm["live"]["resident"]


@pytest.mark.parametrize("index", range(len(FIXTURE["arms"])))
def test_replay_matches_reference_simulator(index):
    arm = FIXTURE["arms"][index]
    trace = PageTrace(FIXTURE["layers"], FIXTURE["page_bytes"])
    for ev in FIXTURE["events"]:
        trace.record(phase=ev["phase"], step=ev["step"], layer=ev["layer"], routed=ev["routed"])
    got = replay(PageTrace.from_dict(trace.as_dict()), capacity_pages=FIXTURE["capacity"],
                 cache_policy=arm["cache_policy"], prefill_page_policy=arm["prefill_page_policy"])
    want = arm["replay"]
    assert got["host_to_device_bytes"] == want["h2d_bytes"]
    assert got["layer_acquires"] == want["acquisitions"]
    for name in ("page_requests", "page_hits", "page_misses", "evictions", "same_layer_evictions",
                 "over_quota_evictions", "fallback_evictions", "peak_resident_pages", "final_resident_pages",
                 "layer_quotas", "transient_prefill_admitted_pages", "transient_prefill_replaced_pages",
                 "transient_prefill_skipped_protected_pages", "decode_protected_promotions",
                 "decode_protected_demotions"):
        assert got[name] == want[name], name
    assert got["transient_prefill_acquires"] == want["transient_prefill_acquisitions"]


def test_route_prefetch_turns_repeated_routes_into_hits():
    """With route prefetch, a step that repeats the previous step's routes finds every layer
    after the first already resident; prefetches never evict the acquisition's own pages."""
    res = ExpertResidency(layers=4, experts=16, capacity=24, page_bytes=64, max_active_pages=8,
                          cache_policy=LAYER_FREQUENCY_LRU, route_prefetch=True)
    routes = {0: [1, 2, 2, 5], 1: [3, 4], 2: [7, 7, 9], 3: [0, 15]}
    for step in range(3):
        hits_before = res.stats["page_hits"]
        for layer in range(4):
            plan = res.acquire(layer, routes[layer], protect=True)
            protected = {(layer, e) for e in plan.experts}
            copies = res.prefetch_next_layer(layer, protected)
            assert all(res.slot_of((layer, e)) is not None for e in plan.experts)
            assert all(slot not in plan.slots for _, slot in copies)
        if step >= 1:
            assert res.stats["page_hits"] - hits_before == sum(len(set(r)) for r in routes.values())
    assert res.prefetch_stats["prefetched_pages"] >= 0


def test_policy_arguments_and_trace_limits():
    with pytest.raises(ValueError, match="unsupported cache policy"):
        ExpertResidency(layers=2, experts=4, capacity=4, page_bytes=8, max_active_pages=4, cache_policy="mru")
    with pytest.raises(ValueError, match="needs layer-frequency"):
        ExpertResidency(layers=2, experts=4, capacity=4, page_bytes=8, max_active_pages=4, cache_policy=GLOBAL_LRU,
                        prefill_page_policy=TRANSIENT_FREQUENCY_PREFILL)
    with pytest.raises(ValueError, match="excludes route prefetch"):
        ExpertResidency(layers=2, experts=4, capacity=4, page_bytes=8, max_active_pages=4,
                        cache_policy=LAYER_FREQUENCY_LRU, prefill_page_policy=TRANSIENT_FREQUENCY_PREFILL,
                        route_prefetch=True)
    res = ExpertResidency(layers=2, experts=8, capacity=3, page_bytes=8, max_active_pages=2,
                          prefill_page_policy=CACHE_FILL_PREFILL)
    with pytest.raises(RuntimeError, match="staging limit"):
        res.acquire(0, [1, 2, 3], protect=False)
    trace = PageTrace(2, 8, max_events=1)
    trace.record(phase="decode", step=1, layer=0, routed=[1, 1, 2])
    assert trace.events[0]["pages"] == [[1, 2], [2, 1]] and len(trace.sha256()) == 64
    with pytest.raises(RuntimeError, match="exceeds"):
        trace.record(phase="decode", step=1, layer=1, routed=[0])


def test_replay_ab_matches_reference_arms(tmp_path):
    """The A/B replay (baseline global-LRU/cache-fill vs candidate layer-frequency/transient)
    reproduces the reference simulator's two arms, also through the command line."""
    import subprocess
    import sys

    from mrun_b200.page_policy import replay_ab

    trace = PageTrace(FIXTURE["layers"], FIXTURE["page_bytes"])
    for ev in FIXTURE["events"]:
        trace.record(phase=ev["phase"], step=ev["step"], layer=ev["layer"], routed=ev["routed"])
    report = replay_ab(trace, capacity_pages=FIXTURE["capacity"])
    arms = {(a["cache_policy"], a["prefill_page_policy"]): a["replay"] for a in FIXTURE["arms"]}
    base = arms[(GLOBAL_LRU, CACHE_FILL_PREFILL)]
    cand = arms[(LAYER_FREQUENCY_LRU, TRANSIENT_FREQUENCY_PREFILL)]
    assert report["arms"]["baseline"]["page_hits"] == base["page_hits"]
    assert report["arms"]["candidate"]["page_hits"] == cand["page_hits"]
    assert report["comparison"]["signed_h2d_bytes_saved"] == base["h2d_bytes"] - cand["h2d_bytes"]
    path = tmp_path / "trace.json"
    path.write_text(json.dumps(trace.as_dict()))
    out = subprocess.run([sys.executable, "-m", "mrun_b200.page_policy", str(path), "--capacity-pages",
                          str(FIXTURE["capacity"])], capture_output=True, text=True, check=True,
                         cwd=Path(__file__).resolve().parents[1])
    assert json.loads(out.stdout)["comparison"] == report["comparison"]


def test_reference_environment_switches():
    """Options left unset follow the reference's environment variables; explicit ones win."""
    from mrun_b200.page_policy import options_from_env
    from mrun_b200.qstore import store_options_from_env

    assert options_from_env(environ={}) == {"cache_policy": GLOBAL_LRU, "prefill_page_policy": CACHE_FILL_PREFILL,
                                            "route_prefetch": False, "page_trace": False}
    env = {"MRUN_QWEN3_MOE_CACHE_POLICY": "Layer-Frequency-LRU-v1 ", "MRUN_QWEN3_MOE_ROUTE_PREFETCH": "1",
           "MRUN_QWEN3_MOE_PAGE_TRACE": "yes", "MRUN_QWEN3_MOE_PREFILL_PAGE_POLICY": "cache-fill-v1"}
    got = options_from_env(environ=env)
    assert got == {"cache_policy": LAYER_FREQUENCY_LRU, "prefill_page_policy": CACHE_FILL_PREFILL,
                   "route_prefetch": True, "page_trace": True}
    assert options_from_env(route_prefetch=False, environ=env)["route_prefetch"] is False
    assert options_from_env(environ={"MRUN_QWEN3_MOE_PAGE_TRACE": "off"})["page_trace"] is False
    assert store_options_from_env(environ={}) == {"ring": True, "ring_slots": 3, "cache_policy": "pin-fill"}
    assert store_options_from_env(environ={"MRUN_PAGED_RING": "0"})["ring"] is False
    assert store_options_from_env(environ={"MRUN_PAGED_RING": "5"})["ring_slots"] == 5
    assert store_options_from_env(environ={"MRUN_QSTORE_CACHE_POLICY": "LRU"})["cache_policy"] == "lru"
    with pytest.warns(UserWarning, match="unknown"):
        assert store_options_from_env(environ={"MRUN_QSTORE_CACHE_POLICY": "mru"})["cache_policy"] == "pin-fill"
    assert store_options_from_env(cache_policy="lru", environ={"MRUN_QSTORE_CACHE_POLICY": "mru"})["cache_policy"] == "lru"


def test_resident_prefix_keeps_its_pages_under_a_cyclic_scan():
    """Decode steps that touch every page of every layer in layer order: the reference's LRU
    rules evict each page just before its next use (no hits at a 25 % budget);
    resident-prefix-v1 keeps the first capacity - 2 x active pages admitted for good, so every
    step after the first hits exactly those."""
    from mrun_b200.page_policy import RESIDENT_PREFIX

    layers, experts, cap = 32, 8, 64
    trace = PageTrace(layers, 8)
    steps = 5
    for step in range(steps):
        for layer in range(layers):
            trace.record(phase="decode", step=step, layer=layer, routed=list(range(experts)) * 4)
    lru = replay(trace, capacity_pages=cap, cache_policy=GLOBAL_LRU, prefill_page_policy=CACHE_FILL_PREFILL,
                 max_active_pages=experts)
    assert lru["page_hits"] == 0
    got = replay(trace, capacity_pages=cap, cache_policy=RESIDENT_PREFIX, prefill_page_policy=CACHE_FILL_PREFILL,
                 max_active_pages=experts)
    prefix = cap - 2 * experts
    assert got["page_hits"] == (steps - 1) * prefix
    assert sorted(map(tuple, got["resident"]))[:prefix] == [(l, e) for l in range(prefix // experts)
                                                            for e in range(experts)]
    # the ring alone: with no room for a prefix the rule is plain LRU
    small = replay(trace, capacity_pages=16, cache_policy=RESIDENT_PREFIX, prefill_page_policy=CACHE_FILL_PREFILL,
                   max_active_pages=experts)
    assert small["page_hits"] == 0 and small["evictions"] == lru["evictions"] + (cap - 16)
