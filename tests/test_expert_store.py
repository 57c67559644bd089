"""On-disk expert page store: written pages read back bit for bit through the parallel
reader -- whole-file warm-up into the host tier and per-page gathers -- and malformed stores
refused (no GPU)."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch


def _pages(layers, experts, layout, seed=0):
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, (layers, experts, layout.page_stride), dtype=np.uint8)


def test_warm_and_gather_bit_exact(tmp_path):
    from mrun_b200.moe import ExpertPageLayout
    from mrun_b200.streaming import ExpertPageStore, HostPageTier, write_expert_store

    layout = ExpertPageLayout.create(256, 128)
    data = _pages(3, 5, layout)
    write_expert_store(tmp_path / "e", layout, data)
    store = ExpertPageStore(tmp_path / "e")
    assert (store.layers, store.experts, store.layout) == (3, 5, layout)
    tier = HostPageTier.from_store(store, pin=False, threads=4)
    np.testing.assert_array_equal(tier.pages.numpy(), data)
    assert tier.stats["warmed_pages"] == 15
    target = torch.zeros((3, layout.page_stride), dtype=torch.uint8)
    store.gather(2, [4, 0, 3], target)
    np.testing.assert_array_equal(target.numpy(), data[2, [4, 0, 3]])
    with pytest.raises(IndexError):
        store.gather(1, [5], target)
    store.close()


def test_malformed_stores_refused(tmp_path):
    from mrun_b200.moe import ExpertPageLayout
    from mrun_b200.streaming import ExpertPageStore, write_expert_store

    layout = ExpertPageLayout.create(128, 64)
    write_expert_store(tmp_path / "e", layout, _pages(2, 2, layout))
    with (tmp_path / "e" / "expert_pages.u8").open("ab") as f:
        f.write(b"\0" * 16)
    with pytest.raises(ValueError, match="byte length"):
        ExpertPageStore(tmp_path / "e")
    man = json.loads((tmp_path / "e" / "manifest.json").read_text())
    man["layout"]["page_stride"] += 4096
    (tmp_path / "e" / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(ValueError, match="int8 page layout"):
        ExpertPageStore(tmp_path / "e")
    man["schema_version"] = "something-else"
    (tmp_path / "e" / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(ValueError, match="schema"):
        ExpertPageStore(tmp_path / "e")
    with pytest.raises(ValueError, match="uint8"):
        write_expert_store(tmp_path / "f", layout, np.zeros((1, 1, 8), np.float32))


def test_budgeted_host_tier_serves_ram_then_disk(tmp_path):
    """A tier smaller than the store: warm() holds the first pages, gathers of other pages come
    from disk and are admitted until the budget is full; every page is bit-exact."""
    from mrun_b200.moe import ExpertPageLayout
    from mrun_b200.streaming import BudgetedHostPageTier, ExpertPageStore, write_expert_store

    layout = ExpertPageLayout.create(128, 64)
    data = _pages(2, 4, layout, seed=4)
    write_expert_store(tmp_path / "e", layout, data)
    store = ExpertPageStore(tmp_path / "e")
    tier = BudgetedHostPageTier(store, host_cache_mb=3 * layout.page_stride / 1e6, try_pin=False)
    assert tier.capacity == 3
    stats = tier.warm(threads=2)
    assert stats["warmed_pages"] == 3  # pages (0,0), (0,1), (0,2)
    target = torch.zeros((3, layout.page_stride), dtype=torch.uint8)
    tier.gather(0, [2, 3, 1], target)
    np.testing.assert_array_equal(target.numpy(), data[0, [2, 3, 1]])
    assert tier.stats["served_pages"] == 2 and tier.stats["disk_pages"] == 1 and tier.stats["admitted_pages"] == 0
    small = BudgetedHostPageTier(store, host_cache_mb=2 * layout.page_stride / 1e6, try_pin=False)
    small.gather(1, [3, 0], target)  # cold tier: both from disk, both admitted
    small.gather(1, [0, 3, 2], target)
    np.testing.assert_array_equal(target.numpy(), data[1, [0, 3, 2]])
    assert small.stats["admitted_pages"] == 2 and small.stats["served_pages"] == 2 and small.stats["disk_pages"] == 3
    with pytest.raises(ValueError, match="smaller than one expert page"):
        BudgetedHostPageTier(store, host_cache_mb=0.0, try_pin=False)
    store.close()
