"""Loading a dense decoder from an on-disk QStore under the reference's canonical block names
(no GPU: the blocks come from the read oracle as host tensors)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.qstore_files import StoreOracle


def _write_store(path, cfg, rng, *, tied=True):
    from mrun_b200.qstore_build import write_qstore

    def q(rows, cols):
        return (rng.integers(-127, 128, (rows, cols), dtype=np.int8), rng.random(rows).astype(np.float32) + 0.01)

    h, hd = cfg["hidden_size"], cfg["head_dim"]
    qd, kd = cfg["num_attention_heads"] * hd, cfg["num_key_value_heads"] * hd
    qrows, fp32 = {"embed": q(cfg["vocab_size"], h)}, {"norm.final": rng.random(h).astype(np.float32)}
    for i in range(cfg["num_hidden_layers"]):
        for name, shape in (("q", (qd, h)), ("k", (kd, h)), ("v", (kd, h)), ("o", (h, qd)),
                            ("gate", (cfg["intermediate_size"], h)), ("up", (cfg["intermediate_size"], h)),
                            ("down", (h, cfg["intermediate_size"]))):
            qrows[f"L{i}.{name}"] = q(*shape)
        for name, n in (("q.bias", qd), ("k.bias", kd), ("v.bias", kd), ("ln1", h), ("ln2", h)):
            fp32[f"L{i}.{name}"] = rng.standard_normal(n).astype(np.float32)
    if not tied:
        qrows["lm_head"] = q(cfg["vocab_size"], h)
    write_qstore(path, qrows=qrows, fp32=fp32, aliases={"lm_head": "embed"} if tied else None, config=cfg)


@pytest.mark.parametrize("tied", [True, False])
def test_dense_weights_from_store_blocks(tmp_path, tied):
    from mrun_b200.dense_engine import DenseConfig, DenseWeights

    hf = {"num_hidden_layers": 2, "hidden_size": 64, "num_attention_heads": 4, "num_key_value_heads": 2,
          "head_dim": 16, "intermediate_size": 96, "vocab_size": 50, "rope_theta": 1e6, "rms_norm_eps": 1e-6}
    _write_store(tmp_path / "m", hf, np.random.default_rng(3), tied=tied)
    oracle = StoreOracle(tmp_path / "m")
    cfg = DenseConfig.from_hf_config(oracle.manifest["config"])
    assert (cfg.num_layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn) == (2, 4, 2, 16, 96)

    def qrow(name):
        codes, scales = oracle.qrow(name)
        return torch.from_numpy(codes.copy()), torch.from_numpy(scales.copy())

    w = DenseWeights.from_blocks(cfg, qrow, lambda n: torch.from_numpy(oracle.fp32(n).copy()),
                                 lambda n: n in oracle.blocks)
    for i, layer in enumerate(w.layers):
        want = np.concatenate([oracle.qrow(f"L{i}.{p}")[0] for p in ("q", "k", "v")])
        np.testing.assert_array_equal(layer.qkv.codes.numpy(), want)
        np.testing.assert_array_equal(layer.qkv.scales.numpy(),
                                      np.concatenate([oracle.qrow(f"L{i}.{p}")[1] for p in ("q", "k", "v")]))
        np.testing.assert_array_equal(layer.qkv_bias.numpy(),
                                      np.concatenate([oracle.fp32(f"L{i}.{p}.bias") for p in ("q", "k", "v")]))
        np.testing.assert_array_equal(layer.down.codes.numpy(), oracle.qrow(f"L{i}.down")[0])
        np.testing.assert_array_equal(layer.ln2.numpy(), oracle.fp32(f"L{i}.ln2"))
    np.testing.assert_array_equal(w.head.codes.numpy(), oracle.qrow("lm_head")[0])
    assert tied == np.array_equal(w.head.codes.numpy(), w.embed.codes.numpy())
    np.testing.assert_array_equal(w.final_norm.numpy(), oracle.fp32("norm.final"))
    # a config that does not match the blocks is refused
    bad = DenseConfig(num_layers=2, hidden=64, heads=8, kv_heads=2, head_dim=16, ffn=96, vocab=50)
    with pytest.raises(ValueError, match="q/k/v blocks"):
        DenseWeights.from_blocks(bad, qrow, lambda n: torch.from_numpy(oracle.fp32(n).copy()),
                                 lambda n: n in oracle.blocks)
