"""On-disk QStore to HBM: pages read directly and through the prefetch ring equal the
reference's outputs bit for bit (byte work); the W8A16 projection on a store page is within
the bf16 tolerance of the oracle."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import qrow as oq
from oracle.numerics import max_rel_err
from oracle.qstore_files import StoreOracle

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("ring", [False, True])
def test_store_matches_reference_outputs(ring, golden, cuda):
    from mrun_b200.qstore import QStore

    g = golden("qstore")
    with QStore("qstore_small", root=GOLDEN, device=cuda, enable_prefetch_ring=ring) as store:
        for _ in range(3):  # the ring learns the order on the first pass, hits afterwards
            for name, block in store.blocks.items():
                key = name.replace(".", "_")
                if block.get("kind") == "fp32":
                    np.testing.assert_array_equal(store.fp32(name).cpu().numpy(), g["fp32__" + key])
                else:
                    np.testing.assert_array_equal(store.weight(name).cpu().numpy(), g["weight__" + key])
        emb = store.embed_rows("model.embed_tokens.weight", g["embed_ids"])
        np.testing.assert_array_equal(emb.cpu().numpy(), g["embed_rows"])
        stats = store.ring_stats()
        if ring:
            assert stats["hits"] + stats["late_hits"] > 0 and stats["staged"] > 0
        else:
            assert stats is None


def test_ring_under_slot_reuse_and_compute(tmp_path, cuda):
    """Many blocks through 3 slots while the consumer runs projections on every page: each
    page is byte-identical to the file, and the projections match the oracle."""
    from mrun_b200.qstore import QStore
    from mrun_b200.qstore_build import write_qstore

    rng = np.random.default_rng(12)
    qrows = {}
    for i in range(12):
        rows = 256 + 64 * (i % 3)
        qrows[f"l{i}"] = (rng.integers(-127, 128, (rows, 1024), dtype=np.int8),
                          (0.001 + 0.01 * rng.random(rows)).astype(np.float32))
    write_qstore(tmp_path / "m", qrows=qrows, fp32={"norm": np.ones(1024, np.float32)})
    oracle = StoreOracle(tmp_path / "m")
    x = (rng.standard_normal((2, 1024)) * 0.5).astype(np.float32)
    x_dev = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    x_bf = x_dev.float().cpu().numpy()
    with QStore("m", root=tmp_path, device=cuda, ring_slots=3, ring_depth=2, read_threads=4) as store:
        for rep in range(3):
            for name in qrows:
                page = store.page(name)
                codes, scales = oracle.qrow(name)
                assert torch.equal(page.codes.cpu(), torch.from_numpy(codes))
                assert torch.equal(page.scales.cpu(), torch.from_numpy(scales))
                out = store.matmul(name, x_dev)
                ref = oq.qrow_matmul_w8a16(x_bf, codes, scales)
                assert max_rel_err(out.float().cpu().numpy(), ref) < 1e-2
        stats = store.ring_stats()
    assert stats["hits"] + stats["late_hits"] >= 12, stats


def test_dense_decoder_from_qstore_matches_host_assembly(tmp_path, cuda):
    """A dense model read from its on-disk QStore (pages through the ring) decodes the same
    greedy tokens as the same blocks assembled from host tensors."""
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from test_dense_loader import _write_store

    from mrun_b200.dense_engine import DenseConfig, DenseDecoder, DenseWeights
    from mrun_b200.qstore import QStore

    hf = {"num_hidden_layers": 2, "hidden_size": 256, "num_attention_heads": 2, "num_key_value_heads": 1,
          "head_dim": 128, "intermediate_size": 256, "vocab_size": 200}
    _write_store(tmp_path / "m", hf, np.random.default_rng(8))
    oracle = StoreOracle(tmp_path / "m")
    cfg = DenseConfig.from_hf_config(oracle.manifest["config"])
    host = DenseWeights.from_blocks(
        cfg, lambda n: tuple(torch.from_numpy(a.copy()).to(cuda) for a in oracle.qrow(n)),
        lambda n: torch.from_numpy(oracle.fp32(n).copy()).to(cuda), lambda n: n in oracle.blocks)
    prompt = torch.tensor([3, 17, 42, 5, 9], dtype=torch.int64)
    want = DenseDecoder(host, max_batch=1, max_seq_len=64, device=cuda, max_prefill_tokens=16).generate(prompt, 6)
    with QStore("m", root=tmp_path, device=cuda) as store:
        loaded = DenseWeights.from_qstore(store)
        got = DenseDecoder(loaded, max_batch=1, max_seq_len=64, device=cuda, max_prefill_tokens=16).generate(prompt, 6)
    assert got == want and len(got) == 6


def test_store_resident_cache_and_row_stable_matmul(tmp_path, cuda):
    """Pages kept resident by the cache are the same bytes; row-stable matmul equals one-row
    calls bit for bit."""
    from mrun_b200.dense_qstore_cuda import qrow_linear
    from mrun_b200.qstore import QStore
    from mrun_b200.qstore_build import write_qstore

    rng = np.random.default_rng(21)
    qrows = {f"l{i}": (rng.integers(-127, 128, (64, 256), dtype=np.int8), rng.random(64).astype(np.float32))
             for i in range(4)}
    write_qstore(tmp_path / "m", qrows=qrows, fp32={"n": np.ones(4, np.float32)})
    x = torch.randn(20, 256, device=cuda).to(torch.bfloat16)
    with QStore("m", root=tmp_path, device=cuda) as store:
        store.set_cache_budget(0.04)  # two of the four 16.6 KB pages
        for _ in range(3):
            for name, (codes, scales) in qrows.items():
                page = store.page(name)
                assert torch.equal(page.codes.cpu(), torch.from_numpy(codes))
                assert torch.equal(page.scales.cpu(), torch.from_numpy(scales))
        stats = store.cache_stats()
        assert stats["admitted"] == 2 and stats["hits"] == 4
        y = store.matmul_row_stable("l1", x)
        page = store.page("l1")
        for i in range(x.shape[0]):
            assert torch.equal(y[i:i + 1], qrow_linear(page.codes, page.scales, x[i:i + 1]))


def test_row_blocks_match_reference_weight(golden, cuda):
    """Row-chunked streaming of a qrow block (uneven last chunk) reassembles the reference's
    fp32 weight bit for bit, also when the chunks come from the resident cache."""
    from mrun_b200.qstore import QStore

    g = golden("qstore")
    want = g["weight__model_embed_tokens_weight"]
    with QStore("qstore_small", root=GOLDEN, device=cuda, enable_prefetch_ring=False) as store:
        store.set_cache_budget(1.0)
        for _ in range(2):
            chunks = list(store.row_blocks("model.embed_tokens.weight", bs=32))
            assert [(s, e) for s, e, _ in chunks] == [(0, 32), (32, 64), (64, 96), (96, 100)]
            np.testing.assert_array_equal(torch.cat([w for _, _, w in chunks]).cpu().numpy(), want)
        assert store.cache_stats()["hits"] == 4
