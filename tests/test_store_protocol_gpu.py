"""The dense engine's store protocol on the GPU: ``DenseQStore`` pages, projections, head rows,
prebinding and counters; ``enable_w8a8`` on the repo's own stores; the dense engine opened by
backend name decoding the same greedy tokens as the decoder built by hand."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import qrow as oq
from oracle import w8a8 as ow
from oracle.numerics import max_rel_err
from oracle.qstore_files import StoreOracle

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent
GOLDEN = HERE / "golden"


def _small_model(tmp_path):
    sys.path.insert(0, str(HERE))
    from test_dense_loader import _write_store

    hf = {"num_hidden_layers": 2, "hidden_size": 256, "num_attention_heads": 2, "num_key_value_heads": 1,
          "head_dim": 128, "intermediate_size": 256, "vocab_size": 200}
    _write_store(tmp_path / "m", hf, np.random.default_rng(8))
    return tmp_path / "m"


def test_dense_qstore_pages_projections_and_counters(tmp_path, cuda):
    from mrun_b200.dense_qstore_cuda import DenseQStore, load_compact_qrow_page

    path = _small_model(tmp_path)
    oracle = StoreOracle(path)
    qnames = [n for n, b in oracle.blocks.items() if b.get("kind") == "qrow"]  # aliases excluded
    gate, up = "L0.gate", "L0.up"
    x = (torch.randn(3, 256) * 0.5).to(torch.bfloat16)
    xf = x.float().numpy()
    page_bytes = {n: int(np.prod(oracle.blocks[n]["shape"])) + 4 * int(oracle.blocks[n]["shape"][0]) for n in qnames}
    budget_mb = (page_bytes[gate] + page_bytes[up]) / 1e6  # room for exactly the two MLP pages
    with DenseQStore("m", root=tmp_path, device=str(cuda), compact_cache_mb=budget_mb) as store:
        for name in qnames:
            page = store.compact_page(name)
            codes, scales = oracle.qrow(name)
            assert torch.equal(page.codes.cpu(), torch.from_numpy(codes)) and torch.equal(
                page.scales.cpu(), torch.from_numpy(scales))
        # LRU under the byte budget: the last two loaded pages are resident
        assert store.compact_cache_bytes <= store.compact_cache_budget
        y = store.matmul(gate, x.to(cuda))
        assert max_rel_err(y.float().cpu().numpy(), oq.qrow_matmul_w8a16(xf, *oracle.qrow(gate))) < 1e-2
        s, impl = store.fused_swiglu(gate, up, x.to(cuda))
        assert impl.startswith("b200")
        want = oq.swiglu_w8a16(xf, *oracle.qrow(gate), *oracle.qrow(up))
        assert max_rel_err(s.float().cpu().numpy(), want) < 1e-2
        # head rows read alone equal the dequantised rows
        head = "lm_head"  # an alias of the embedding: the physical page is shared
        ids = [5, 0, 199, 5]
        rows = store.selected_rows_fp32(head, ids)
        codes, scales = oracle.qrow(head)
        np.testing.assert_array_equal(rows.cpu().numpy(), codes[ids].astype(np.float32) * scales[ids, None])
        with pytest.raises(IndexError):
            store.selected_rows_fp32(head, [200])
        with pytest.raises(ValueError):
            store.selected_rows_fp32(head, [])
        # prebound pages stay out of the LRU and keep their addresses
        got = store.prebind([gate, up], max_resident_bytes=10 << 20)
        assert got["qrow_pages"] == 2 and got["resident_bytes"] == page_bytes[gate] + page_bytes[up]
        ptr = store.compact_page(gate).codes.data_ptr()
        store.set_compact_cache_budget(0.0)
        assert store.compact_cache_bytes == 0 and store.compact_page(gate).codes.data_ptr() == ptr
        with pytest.raises(MemoryError):
            store.prebind(qnames, max_resident_bytes=1)
        snap = store.stats_snapshot()
        assert snap["paired_swiglu_calls"] == 1 and snap["projection_calls"] == 3
        assert snap["prebound_page_entries"] == 2 and snap["selected_head_rows"] == 4
        assert snap["page_loads"] >= len(qnames) and snap["cache_kind"] == "compact-device-lru"
        part = load_compact_qrow_page(store, gate, start_row=3, end_row=9)
        assert torch.equal(part.codes.cpu(), torch.from_numpy(oracle.qrow(gate)[0][3:9]))
        head32 = store.prepare_resident_exact_head(head, max_resident_bytes=1 << 30)
        np.testing.assert_array_equal(head32.cpu().numpy(), codes.astype(np.float32) * scales[:, None])


@pytest.mark.parametrize("kind", ["qstore", "dense"])
def test_enable_w8a8_on_repo_stores(kind, tmp_path, cuda):
    """enable_w8a8 rebinds matmul on the repo's QStore and DenseQStore: outputs equal the W8A8
    oracle (no protection: bit-exact), fp32 blocks keep the base path, disable restores it."""
    from mrun_b200.dense_qstore_cuda import DenseQStore
    from mrun_b200.qstore import QStore
    from mrun_b200.w8a8 import disable_w8a8, enable_w8a8

    path = _small_model(tmp_path)
    oracle = StoreOracle(path)
    name = "L1.down"
    x = torch.randn(4, int(oracle.blocks[name]["shape"][1])) * 0.7
    cls = QStore if kind == "qstore" else DenseQStore
    with cls("m", root=tmp_path, device=cuda) as store:
        base = store.matmul(name, x.to(cuda).to(torch.bfloat16))
        enable_w8a8(store, protect_k=0)
        y = store.matmul(name, x.to(cuda))
        codes, scales = oracle.qrow(name)
        want = ow.w8a8_matmul(codes, scales, x.numpy())
        np.testing.assert_array_equal(y.cpu().numpy(), want)
        disable_w8a8(store)
        again = store.matmul(name, x.to(cuda).to(torch.bfloat16))
        assert torch.equal(again, base)


def test_open_engine_dense_backend_matches_decoder(tmp_path, cuda):
    """open_engine(backend="dense-qstore-cuda") over a DenseQStore decodes the same greedy tokens
    as a DenseDecoder built from the host-assembled blocks; a second open reuses the pool."""
    from mrun_b200.dense_engine import DenseConfig, DenseDecoder, DenseWeights
    from mrun_b200.engine import close_pooled_engines, open_engine

    path = _small_model(tmp_path)
    oracle = StoreOracle(path)
    cfg = DenseConfig.from_hf_config(oracle.manifest["config"])
    host = DenseWeights.from_blocks(
        cfg, lambda n: tuple(torch.from_numpy(a.copy()).to(cuda) for a in oracle.qrow(n)),
        lambda n: torch.from_numpy(oracle.fp32(n).copy()).to(cuda), lambda n: n in oracle.blocks)
    # distinct lengths: every group is one row, like the one-row reference decoders below
    prompts = [[3, 17, 42, 5, 9], [7, 7, 1, 0], [11, 4]]
    want = []
    for p in prompts:
        dec = DenseDecoder(host, max_batch=1, max_seq_len=64, device=cuda, max_prefill_tokens=16)
        want.append(dec.generate(torch.tensor(p), 6))
    try:
        # max_seq_len 63 gives the engine's decoder the same 64-token KV capacity (and so the
        # same attention split plan) as the decoders above
        opts = dict(stores_dir=tmp_path, device=str(cuda), max_seq_len=63, max_batch=4)
        engine = open_engine("m", backend="dense-qstore-cuda", **opts)
        assert open_engine("m", backend="dense-qstore-cuda", **opts) is engine
        got = engine.generate_batch(prompts, max_new_tokens=6)
        assert got == want
        cut = engine.generate(prompts[0], max_new_tokens=6, eos_token_id=want[0][2])
        assert cut == want[0][:3]
        stats = engine.runtime_stats()
        assert stats["generated_tokens"] >= 18 and stats["store"]["page_loads"] > 0
        with pytest.raises(ValueError, match="not served"):
            open_engine("m", backend="hf", stores_dir=tmp_path)
    finally:
        close_pooled_engines()
