"""End-to-end greedy decode of the dense QStore decoder against the CPU oracle.

The oracle restates the reference's fused-body forward with its bf16 boundaries. Greedy
parity is checked by teacher forcing: for every step, the oracle scores the token the GPU
chose; the GPU's choice must be the oracle's argmax unless the oracle's own top-1/top-2
margin is below the bf16 resolution of the logits (a genuine near-tie), which is reported.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.decoder import OracleConfig, OracleDecoder

pytestmark = pytest.mark.gpu


def _tiny(**kw):
    from mrun_b200.dense_engine import DenseConfig

    base = dict(num_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000)
    base.update(kw)
    return DenseConfig(**base)


def _oracle(cfg, weights, mode="w8a16"):
    ocfg = OracleConfig(cfg.num_layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                        cfg.rope_theta, cfg.eps)
    return OracleDecoder(ocfg, weights.to_host(), mode=mode)


@pytest.mark.parametrize("kw,prompt_len,steps", [
    (dict(), 37, 96),
    (dict(hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=3000, num_layers=3), 100, 256),
])
def test_greedy_decode_matches_oracle(kw, prompt_len, steps, cuda):
    from mrun_b200.dense_engine import DenseDecoder, DenseWeights

    cfg = _tiny(**kw)
    weights = DenseWeights.synthetic(cfg, cuda, seed=1)
    dec = DenseDecoder(weights, max_batch=1, max_seq_len=prompt_len + steps + 16, device=cuda, max_prefill_tokens=256)
    prompt = torch.from_numpy(np.random.default_rng(0).integers(0, cfg.vocab, prompt_len))
    tokens = dec.generate(prompt, steps)
    dec.check_errors()
    assert len(tokens) == steps and all(0 <= t < cfg.vocab for t in tokens)

    oracle = _oracle(cfg, weights)
    picks, gaps, margins = oracle.teacher_forced(prompt.numpy(), tokens)
    # bf16 activations put ~1e-2 absolute noise on O(1) logits; a differing pick must be a
    # near-tie: the GPU's token scores within that noise of the oracle's best.
    tol = 2e-2
    mismatches = [(i, t, p, g, m) for i, (t, p, g, m) in enumerate(zip(tokens, picks, gaps, margins)) if t != p]
    for step, tok, pick, gap, margin in mismatches:
        assert gap <= tol, f"step {step}: gpu {tok} vs oracle {pick}, gap {gap:.4g}, margin {margin:.4g}"
    first = mismatches[0][0] if mismatches else steps
    print(f"greedy parity: {steps - len(mismatches)}/{steps} identical, first near-tie at step {first}, "
          f"near-ties {[(s, round(g, 5)) for s, _, _, g, _ in mismatches]}")
    assert len(mismatches) <= max(3, steps // 10)


def test_graph_replay_matches_eager_and_is_deterministic(cuda):
    from mrun_b200.dense_engine import DenseDecoder, DenseWeights

    cfg = _tiny()
    weights = DenseWeights.synthetic(cfg, cuda, seed=2)
    prompt = torch.arange(20) * 7 % cfg.vocab
    runs = []
    for _ in range(2):
        dec = DenseDecoder(weights, max_batch=1, max_seq_len=128, device=cuda, max_prefill_tokens=64)
        runs.append(dec.generate(prompt, 40))
    assert runs[0] == runs[1]
    # eager: prefill the generated prefix and compare the next token with the graph's. The
    # prefill runs other kernels (tile GEMM, other attention splits), so the two may differ
    # only at a near tie: then both tokens score within bf16 noise in the oracle's logits.
    dec = DenseDecoder(weights, max_batch=1, max_seq_len=128, device=cuda, max_prefill_tokens=128)
    seq = torch.cat([prompt, torch.tensor(runs[0][:-1])])
    nxt = int(dec.prefill(0, seq).item())
    if nxt != runs[0][-1]:
        logits = _oracle(cfg, weights).forward(seq.numpy())[-1]
        gap = abs(float(logits[nxt]) - float(logits[runs[0][-1]]))
        assert gap <= 2e-2, f"graph token {runs[0][-1]} vs eager {nxt}: oracle logit gap {gap:.4g}"
        print(f"graph/eager near tie: tokens {runs[0][-1]} / {nxt}, oracle gap {gap:.4g}")


def test_w8a8_batched_decode_matches_oracle(cuda):
    """W8A8 mode (per-token int8 activations, exact int32 tensor-core accumulation, split-K at
    decode row counts) over ragged prefills then a captured batched decode; each row's tokens
    are scored by the W8A8 oracle teacher-forced, differing only at near-ties."""
    from mrun_b200.dense_engine import DenseDecoder, DenseWeights

    cfg = _tiny(hidden=512, heads=8, kv_heads=2, head_dim=64, ffn=1024, vocab=2000)
    weights = DenseWeights.synthetic(cfg, cuda, seed=3)
    rows, steps = 5, 12
    rng = np.random.default_rng(5)
    prompts = [torch.from_numpy(rng.integers(0, cfg.vocab, int(n))) for n in rng.integers(3, 60, rows)]
    dec = DenseDecoder(weights, max_batch=rows, max_seq_len=128, device=cuda, max_prefill_tokens=64, mode="w8a8")
    firsts = [int(dec.prefill(i, p).item()) for i, p in enumerate(prompts)]
    lengths = [dec.kv.lengths[i] for i in range(rows)]
    for i in range(rows):
        dec.kv.reserve(i, lengths[i] + steps)
    dec.begin_decode(rows, torch.tensor(firsts), lengths)
    dec.capture(rows)
    out = [[f] for f in firsts]
    for _ in range(steps - 1):
        dec.step()
        ids = dec.next_ids[:rows].cpu().tolist()
        for i in range(rows):
            out[i].append(int(ids[i]))
    dec.check_errors()
    oracle = _oracle(cfg, weights, mode="w8a8")
    total = 0
    for i in range(rows):
        picks, gaps, margins = oracle.teacher_forced(prompts[i].numpy(), out[i])
        for step, (tok, pick, gap) in enumerate(zip(out[i], picks, gaps)):
            if tok != pick:
                total += 1
                assert gap <= 2e-2, f"row {i} step {step}: gpu {tok} vs oracle {pick}, gap {gap:.4g}"
    assert total <= max(3, rows * steps // 10)


@pytest.mark.slow
def test_qwen25_7b_shape_decode_smoke(cuda):
    """Full Qwen2.5-7B shapes (28 layers, hidden 3584, vocab 152064): prefill 512 random ids, 32 greedy steps, twice."""
    from mrun_b200.dense_engine import DenseConfig, DenseDecoder, DenseWeights

    cfg = DenseConfig.qwen25_7b()
    weights = DenseWeights.synthetic(cfg, cuda, seed=0)
    prompt = torch.from_numpy(np.random.default_rng(0).integers(0, cfg.vocab, 512))
    dec = DenseDecoder(weights, max_batch=1, max_seq_len=512 + 256, device=cuda, max_prefill_tokens=512)
    a = dec.generate(prompt, 32)
    dec.check_errors()
    dec2 = DenseDecoder(weights, max_batch=1, max_seq_len=512 + 256, device=cuda, max_prefill_tokens=512)
    b = dec2.generate(prompt, 32)
    assert a == b and all(0 <= t < cfg.vocab for t in a)
