"""Host-side pieces of the drop-in boundary that need no GPU: expert page views with the
reference's signature, the W8A8 raw-code reader on a reference-style store, and backend
dispatch of ``open_engine``."""
from __future__ import annotations

import numpy as np
import pytest
import torch


def test_expert_page_views_reference_signature():
    from mrun_b200.moe import DeviceExpertLayer, ExpertPageLayout, expert_page_views, pack_expert_page

    ly = ExpertPageLayout.create(64, 48)
    rng = np.random.default_rng(3)
    raw = torch.zeros(3, ly.page_stride, dtype=torch.uint8)
    parts = []
    for g in range(3):
        gu = torch.from_numpy(rng.integers(-127, 128, (96, 64), dtype=np.int8))
        gus = torch.from_numpy(rng.random(96).astype(np.float32))
        dn = torch.from_numpy(rng.integers(-127, 128, (64, 48), dtype=np.int8))
        dns = torch.from_numpy(rng.random(64).astype(np.float32))
        pack_expert_page(ly, gu, gus, dn, dns, raw[g])
        parts.append((gu, gus, dn, dns))
    views = expert_page_views(raw, ly)
    assert isinstance(views, DeviceExpertLayer)
    assert views.gate_up.shape == (3, 96, 64) and views.down.shape == (3, 64, 48)
    assert views.gate_up_scales.shape == (3, 96) and views.down_scales.shape == (3, 64)
    for g, (gu, gus, dn, dns) in enumerate(parts):
        assert torch.equal(views.gate_up[g], gu) and torch.equal(views.gate_up_scales[g], gus)
        assert torch.equal(views.down[g], dn) and torch.equal(views.down_scales[g], dns)
    assert views.gate_up.data_ptr() == raw.data_ptr()  # views, not copies
    one = expert_page_views(raw[1], ly)
    assert one.gate_up.shape == (1, 96, 64) and torch.equal(one.down[0], parts[1][2])
    with pytest.raises(ValueError):
        expert_page_views(raw.view(torch.int8), ly)


def test_expert_layout_round_trip_and_alignment():
    from mrun_b200.moe import ExpertPageLayout

    ly = ExpertPageLayout.create(2048, 768)
    assert ExpertPageLayout.from_dict(ly.as_dict()) == ly
    bad = dict(ly.as_dict(), down_codes_offset=ly.down_codes_offset + 4)
    with pytest.raises(ValueError, match="16-byte"):
        ExpertPageLayout.from_dict(bad)


def test_raw_qrow_reads_reference_style_store():
    """A store exposing the reference's memory-mapped ``w`` / ``s`` arrays and ``_resolve``
    (no ``page`` method) is read without dequantisation."""
    from mrun_b200.w8a8 import _raw_qrow

    rng = np.random.default_rng(4)
    codes = rng.integers(-127, 128, (6, 32), dtype=np.int8)
    scales = rng.random(6).astype(np.float32)

    class MemmapStore:
        device = "cpu"
        w = np.concatenate([np.zeros(64, np.int8), codes.reshape(-1)])
        s = np.concatenate([np.zeros(3, np.float32), scales])

        def _resolve(self, name):
            assert name == "blk"
            return {"kind": "qrow", "shape": [6, 32], "w_off": 64, "s_off": 12}

    q, sc = _raw_qrow(MemmapStore(), "blk")
    assert q.dtype == torch.int8 and torch.equal(q, torch.from_numpy(codes))
    assert torch.equal(sc, torch.from_numpy(scales))


def test_open_engine_rejects_other_backends(tmp_path):
    from mrun_b200.engine import DENSE_BACKENDS, open_engine

    assert "dense-qstore-cuda" in DENSE_BACKENDS
    with pytest.raises(ValueError, match="not served"):
        open_engine("m", backend="paged", stores_dir=tmp_path)
    with pytest.raises(ValueError, match="stores_dir or store_path"):
        open_engine("m", backend="dense-cuda", fresh=True)


def test_ep_wait_limit_is_validated_on_the_host():
    from mrun_b200 import _lib

    lib = _lib.load()
    assert lib.mrb_ep_set_wait_limit(0) == _lib.MRB_ERR_ARG
    assert lib.mrb_ep_set_wait_limit(1 << 31) == _lib.MRB_ERR_ARG
    assert int(lib.mrb_ep_wait_limit()) == 1 << 22


def test_full_layer_pages_replay_every_shard():
    """The expert-parallel check rebuilds one layer's full expert set on any rank: it equals
    the unsharded model's pages and contains each rank's shard."""
    from mrun_b200.expert_parallel import ExpertShard
    from mrun_b200.moe_engine import MoeConfig, MoeWeights

    cfg = MoeConfig(num_layers=3, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, top_k=2, expert_ffn=128,
                    vocab=300)
    cpu = torch.device("cpu")
    full = MoeWeights.synthetic(cfg, cpu, seed=3)
    shards = [MoeWeights.synthetic(cfg, cpu, seed=3, shard=ExpertShard(4, r, 8)) for r in range(4)]
    for layer in range(3):
        pages = MoeWeights.synthetic_full_layer_pages(cfg, cpu, layer, seed=3)
        assert torch.equal(pages, full.layers[layer].pages)
        for r, sh in enumerate(shards):
            assert torch.equal(pages[2 * r: 2 * r + 2], sh.layers[layer].pages)


def test_expert_page_matrices_view_the_packed_parts():
    """moe.expert_page_matrices: the gate, up and down codes and scales of one slot, as
    views of the packed page (no copies), in the layout pack_expert_page writes."""
    import torch

    from mrun_b200.moe import ExpertPageLayout, expert_page_matrices, pack_expert_page

    h, f = 64, 48
    ly = ExpertPageLayout.create(h, f)
    g = torch.Generator().manual_seed(3)
    pages = torch.zeros((3, ly.page_stride), dtype=torch.uint8)
    parts = []
    for slot in range(3):
        gu = torch.randint(-127, 128, (2 * f, h), dtype=torch.int8, generator=g)
        gus = torch.rand(2 * f, generator=g)
        dn = torch.randint(-127, 128, (h, f), dtype=torch.int8, generator=g)
        dns = torch.rand(h, generator=g)
        pack_expert_page(ly, gu, gus, dn, dns, pages[slot])
        parts.append((gu, gus, dn, dns))
    for slot in range(3):
        gate, gate_s, up, up_s, down, down_s = expert_page_matrices(pages, ly, slot)
        gu, gus, dn, dns = parts[slot]
        assert torch.equal(gate, gu[:f]) and torch.equal(up, gu[f:]) and torch.equal(down, dn)
        assert torch.equal(gate_s, gus[:f]) and torch.equal(up_s, gus[f:]) and torch.equal(down_s, dns)
        assert gate.is_contiguous() and up.is_contiguous() and down.is_contiguous()
        assert gate.data_ptr() == pages[slot].data_ptr() + ly.gate_up_codes_offset  # a view
