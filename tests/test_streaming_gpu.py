"""Weight-page streaming: expert pages copied from pinned host memory into an HBM slot cache
on a side stream must be byte-identical to the host tier, and a streamed MoE layer loop
(with next-layer prefetch and LRU eviction) must give bit-identical outputs to resident
pages."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

L, E, K, H, F, T = 4, 8, 2, 256, 128, 16


def _build(cuda):
    from mrun_b200.moe import ExpertPageLayout, pack_expert_page
    from mrun_b200.streaming import HostPageTier
    from oracle import qrow as oq

    rng = np.random.default_rng(3)
    ly = ExpertPageLayout.create(H, F)
    host = HostPageTier(ly, L, E)
    host.pages.zero_()
    for layer in range(L):
        for e in range(E):
            gu = oq.quant_row_int8((rng.standard_normal((2 * F, H)) * 0.02).astype(np.float32))
            dn = oq.quant_row_int8((rng.standard_normal((H, F)) * 0.02).astype(np.float32))
            pack_expert_page(ly, torch.from_numpy(gu[0]), torch.from_numpy(gu[1]), torch.from_numpy(dn[0]),
                             torch.from_numpy(dn[1]), host.pages[layer, e])
    resident = [host.pages[layer].to(cuda) for layer in range(L)]
    return ly, host, resident


def test_streamed_moe_bit_identical_to_resident(cuda):
    from mrun_b200.moe import PagedInt8ExpertBackend, ResidentInt8ExpertPages, router_topk
    from mrun_b200.streaming import ExpertPageCache

    ly, host, resident = _build(cuda)
    cache = ExpertPageCache(host, budget_bytes=10 * ly.page_stride, device=cuda)
    streamed = PagedInt8ExpertBackend(cache, num_experts=E)
    reference = PagedInt8ExpertBackend(ResidentInt8ExpertPages(ly, resident), num_experts=E)
    rng = np.random.default_rng(5)
    for step in range(3):
        x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(cuda).to(torch.bfloat16)
        routes = [router_topk(torch.from_numpy(rng.standard_normal((T, E)).astype(np.float32)).to(cuda), K)
                  for _ in range(L)]
        hs, hr = x, x
        for layer in range(L):
            if layer + 1 < L:  # predicted next-layer experts (here: the true routes)
                nxt = sorted(set(routes[layer + 1][0].unique().tolist()))
                cache.prefetch(layer + 1, nxt, protect_layer=layer)
            idx, w, _ = routes[layer]
            hs = streamed.moe(layer, hs, idx, w)
            hr = reference.moe(layer, hr, idx, w)
        torch.cuda.synchronize()
        assert torch.equal(hs, hr), f"step {step}"
    st = cache.stats
    assert st.misses > 0 and st.prefetch_hits > 0 and st.evictions > 0
    # pages in the slots are byte-identical to the host tier
    for (layer, e), slot in cache.where.items():
        assert torch.equal(cache.slots[slot].cpu(), host.pages[layer, e])


def test_copy_pages_validates(cuda):
    from mrun_b200 import _lib

    with pytest.raises(ValueError):
        _lib.call("mrb_copy_pages", None, 16, None, 16, None, None, 1, 16, None, None)


@pytest.mark.parametrize("policy,prefill_policy,route_prefetch", [
    ("global-lru-v1", "cache-fill-v1", False),
    ("layer-frequency-lru-v1", "cache-fill-v1", True),
    ("layer-frequency-lru-v1", "transient-frequency-v1", False),
])
def test_policies_bit_identical_and_trace_replays(policy, prefill_policy, route_prefetch, cuda):
    """Every residency policy (prefill from the transient slab included) gives the resident
    outputs bit for bit, slots hold the host pages, and replaying the recorded page trace
    reproduces the live cache's counters (without route prefetch, which replay leaves out)."""
    from mrun_b200.moe import PagedInt8ExpertBackend, ResidentInt8ExpertPages, router_topk
    from mrun_b200.page_policy import replay
    from mrun_b200.streaming import ExpertPageCache

    ly, host, resident = _build(cuda)
    cache = ExpertPageCache(host, budget_bytes=12 * ly.page_stride, device=cuda, cache_policy=policy,
                            prefill_page_policy=prefill_policy, route_prefetch=route_prefetch, page_trace=True)
    streamed = PagedInt8ExpertBackend(cache, num_experts=E)
    reference = PagedInt8ExpertBackend(ResidentInt8ExpertPages(ly, resident), num_experts=E)
    rng = np.random.default_rng(11)
    for step in range(4):
        rows = T if step == 0 else 3  # a prefill pass, then decode steps
        x = torch.from_numpy(rng.standard_normal((rows, H)).astype(np.float32)).to(cuda).to(torch.bfloat16)
        hs, hr = x, x
        for layer in range(L):
            idx, w, _ = router_topk(torch.from_numpy(rng.standard_normal((rows, E)).astype(np.float32)).to(cuda), K)
            hs = streamed.moe(layer, hs, idx, w, prefill=step == 0)
            hr = reference.moe(layer, hr, idx, w, prefill=step == 0)
        torch.cuda.synchronize()
        assert torch.equal(hs, hr), f"step {step}"
    for (layer, e), slot in cache.where.items():
        assert torch.equal(cache.slots[slot].cpu(), host.pages[layer, e])
    report = cache.report()
    assert report["residency"]["page_requests"] > 0 and report["cache_policy"] == policy
    if not route_prefetch:
        got = replay(cache.trace, capacity_pages=cache.capacity, cache_policy=policy,
                     prefill_page_policy=prefill_policy, max_active_pages=cache.max_active_pages)
        live = cache.residency.stats
        for name in ("page_hits", "page_misses", "evictions", "transient_prefill_admitted_pages"):
            assert got[name] == live[name], name
