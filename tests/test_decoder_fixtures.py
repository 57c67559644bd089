"""The decoder oracles pinned to the reference's own decoders (no GPU).

Each oracle is scored teacher-forced on the tokens the reference chose: at every step the
oracle's greedy token must equal the reference's unless the reference's own top-1/top-2
margin is below ``NEAR_TIE``, and its top-1 logit must stay within a stated distance of the
reference's. Fixtures: tests/golden/make_decoder_fixtures.py."""
from __future__ import annotations

import numpy as np
import torch

import fixture_models as fm


def _score(step_logits, fixture: dict, *, tol: float) -> int:
    """Walk the fixture's tokens; return how many near-tie steps the oracle picked differently."""
    flips = 0
    for i, logits in enumerate(step_logits):
        order = np.argsort(-logits, kind="stable")
        assert abs(float(logits[order[0]]) - float(fixture["top1"][i])) < tol, i
        if int(order[0]) != int(fixture["tokens"][i]):
            assert float(fixture["margin"][i]) < fm.NEAR_TIE, (i, float(fixture["margin"][i]))
            flips += 1
    return flips


def test_cpu_path_port_matches_paged_forward_kv():
    """The fp32 CPU decode that bench.py times as the CPU baseline equals the reference's
    paged_forward_kv (engine/kernels/paged_forward.py:1016) on the 257-token fixture."""
    from oracle.cpu_path import CpuPathDecoder

    c = fm.dense_config()
    g = fm.load("decoder_fp32")
    torch.set_num_threads(4)
    dec = CpuPathDecoder(num_layers=c["num_hidden_layers"], hidden=c["hidden_size"], heads=c["num_attention_heads"],
                         kv_heads=c["num_key_value_heads"], head_dim=c["head_dim"], ffn=c["intermediate_size"],
                         vocab=c["vocab_size"], weights=fm.dense_oracle_weights())

    def steps():
        logits = dec.forward(g["prompt"])
        yield (logits[-1] if logits.ndim > 1 else logits).numpy()
        for tok in g["tokens"][:-1]:
            logits = dec.forward([int(tok)])
            yield (logits[-1] if logits.ndim > 1 else logits).numpy()

    assert _score(steps(), g, tol=1e-4) == 0
    assert len(g["tokens"]) == 257


def test_dense_oracle_matches_reference_bf16_engine():
    """oracle/decoder.py (the dense CUDA engine's bf16 contract) against DenseQStoreTarget run
    on the CPU (engine/dense_qstore_cuda.py:506): 256 steps after a 32-token prompt."""
    from oracle.decoder import OracleConfig, OracleDecoder

    c = fm.dense_config()
    g = fm.load("decoder_bf16")
    cfg = OracleConfig(c["num_hidden_layers"], c["hidden_size"], c["num_attention_heads"], c["num_key_value_heads"],
                       c["head_dim"], c["intermediate_size"], c["vocab_size"])
    torch.set_num_threads(4)
    dec = OracleDecoder(cfg, fm.dense_oracle_weights())

    def steps():
        yield dec.forward(g["prompt"])[-1].numpy()
        for tok in g["tokens"][:-1]:
            yield dec.forward([int(tok)])[-1].numpy()

    flips = _score(steps(), g, tol=0.03)
    assert flips <= 2


def test_moe_oracle_matches_reference_runtime():
    """oracle/moe_decoder.py against Qwen3MoeDecodeRuntime.forward with a CPU int8 expert
    backend (engine/qwen3_moe_cuda.py:3536): two prompts, 64 steps each, the prompt fed one
    token per step through the decode-step oracle."""
    from oracle.moe_decoder import moe_decode_step

    cfg = fm.moe_config()
    w = fm.moe_host_weights()
    g = fm.load("moe_decode")
    for p in range(2):
        prompt, tokens = g[f"p{p}_prompt"], g[f"p{p}_tokens"]
        fixture = {k: g[f"p{p}_{k}"] for k in ("tokens", "top1", "margin")}
        ks = [np.zeros((0, cfg.kv_heads, cfg.head_dim), np.float32) for _ in range(cfg.num_layers)]
        vs = [k.copy() for k in ks]

        def steps():
            seq = list(prompt) + list(tokens[:-1])
            for t, tok in enumerate(seq):
                new: list = []
                logits, _ = moe_decode_step(w, cfg, [tok], [t], [[k] for k in ks], [[v] for v in vs], new_kv=new)
                for li, (k, v) in enumerate(new):
                    ks[li] = np.concatenate([ks[li], k[:1]])
                    vs[li] = np.concatenate([vs[li], v[:1]])
                if t >= len(prompt) - 1:
                    yield logits[0]

        assert _score(steps(), fixture, tol=0.03) <= 1
