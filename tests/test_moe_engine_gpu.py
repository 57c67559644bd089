"""Ragged MoE decode steps (Qwen3-MoE family) against the CPU step oracle.

Each step is checked on its own: the oracle gets the same committed K/V the device step saw
(gathered from the paged cache) and recomputes the step with the reference's bf16
boundaries (engine/qwen3_moe_cuda.py:3790-3960). The device's greedy token must be the
oracle's argmax unless the oracle's logits put it within bf16 noise of the best (a near
tie), and the device's chosen-logit value must track the oracle's. Routes (top-k expert
indices) must match wherever the oracle's k-th/k+1-th router margin is not a near tie.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.moe_decoder import moe_decode_step

pytestmark = pytest.mark.gpu

LOGIT_GAP_TOL = 2e-2


def _tiny():
    from mrun_b200.moe_engine import MoeConfig

    return MoeConfig(num_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, top_k=2,
                     expert_ffn=128, vocab=500)


@pytest.mark.parametrize("graph", [False, True, "streamed"])
def test_moe_decode_steps_match_oracle(graph, cuda):
    """graph False / True: the Qwen3 form, eager and captured. "streamed": the Mixtral form (no
    q/k norm) with the expert pages in a pinned host tier behind an HBM slot cache of 10 of the
    16 pages (a layer may route to all 8 experts, so a slot cache holds at least 8; eager)."""
    from dataclasses import replace

    from mrun_b200.moe_engine import MoeDecoder, MoeWeights

    cfg = _tiny()
    streamed = graph == "streamed"
    if streamed:
        cfg = replace(cfg, qk_norm=False)
        graph = False
    w = MoeWeights.synthetic(cfg, cuda, seed=3, host_experts=streamed)
    lengths = [5, 17, 33, 1, 64]
    rows = len(lengths)
    steps = 4
    dec = MoeDecoder(w, max_rows=8, max_seq_len=96, device=cuda,
                     expert_cache_bytes=10 * w.layout.page_stride if streamed else None)
    assert dec.streamed == streamed
    first = torch.tensor([7, 123, 42, 499, 0])
    dec.load_synthetic_context(lengths, first, steps=steps, seed=1)
    host = w.to_host()
    if graph:
        dec.capture(rows)
    ids = first.numpy()
    pos = np.array(lengths)
    near_ties = 0
    for _ in range(steps):
        ctx_k = [[dec.gather_kv(li, r, int(pos[r]))[0] for r in range(rows)] for li in range(cfg.num_layers)]
        ctx_v = [[dec.gather_kv(li, r, int(pos[r]))[1] for r in range(rows)] for li in range(cfg.num_layers)]
        logits, _ = moe_decode_step(host, cfg, ids, pos, ctx_k, ctx_v)
        dec.routes = []
        if graph:
            dec.routes = None
        dec.step(rows)
        torch.cuda.synchronize()
        got = dec.next_ids[:rows].cpu().numpy()
        val = dec.next_val[:rows].cpu().numpy()
        for r in range(rows):
            best = float(logits[r].max())
            gap = best - float(logits[r, got[r]])
            assert gap <= LOGIT_GAP_TOL, f"row {r}: token {got[r]} is {gap:.4g} below the oracle's best"
            near_ties += int(got[r] != int(np.argmax(logits[r])))
            assert abs(val[r] - float(logits[r, got[r]])) <= LOGIT_GAP_TOL + 1e-2 * abs(best)
        ids = got
        pos = pos + 1
    dec.check_errors()
    assert near_ties <= 2
    if streamed:
        st = dec.expert_cache.stats
        assert st.misses > 0 and st.evictions > 0 and dec.expert_cache.capacity == 10


def test_streamed_experts_decode_like_resident_pages(cuda):
    """Continuous batching over the Mixtral form: the decoder whose expert pages stream from a
    pinned host tier through an HBM slot cache (10 of the 24 pages under global LRU; 20 under
    the resident-prefix rule, 4 of them held for good) generates, for
    every request, the tokens of the decoder holding every page in HBM (both eager over the
    same rows, so every kernel sees the same inputs; the pages are the same bytes)."""
    from mrun_b200.continuous import MoeContinuousBatcher
    from mrun_b200.moe_engine import MoeConfig, MoeDecoder, MoeWeights

    cfg = MoeConfig(num_layers=3, hidden=256, heads=4, kv_heads=2, head_dim=64, experts=8, top_k=2,
                    expert_ffn=384, vocab=500, qk_norm=False)
    resident = MoeWeights.synthetic(cfg, cuda, seed=5)
    host = MoeWeights.synthetic(cfg, cuda, seed=5, host_experts=True)
    for i, layer in enumerate(resident.layers):
        assert torch.equal(host.host.pages[i].to(cuda), layer.pages)
    prompts = [([1, 2, 3], 10), ([7], 20), ([9, 9, 9, 9, 9], 6), ([4, 5], 12), ([300], 8), ([11, 12], 5)]
    outs, decs = [], []
    for w, policy in ((resident, None), (host, "global-lru-v1"), (host, "resident-prefix-v1")):
        dec = MoeDecoder(w, max_rows=4, max_seq_len=64, device=cuda, cache_policy=policy,
                         expert_cache_bytes=(20 if policy == "resident-prefix-v1" else 10) * w.layout.page_stride
                         if w.host is not None else None)
        bat = MoeContinuousBatcher(dec, max_context_tokens=64, graph=False)
        ids = [bat.submit(p, max_new_tokens=n) for p, n in prompts]
        out = bat.run()
        outs.append([out[i] for i in ids])
        decs.append(dec)
        assert bat.pool.telemetry().slot_reuses == 2
    assert outs[0] == outs[1] == outs[2]
    assert [len(o) for o in outs[1]] == [n for _, n in prompts]
    for dec in decs[1:]:
        st = dec.expert_cache.stats
        assert st.misses > 0 and st.evictions > 0 and st.bytes_h2d > 0
    assert decs[2].expert_cache.residency.prefix_pages == 4  # 20 slots - 2 x 8 active


def test_moe_routes_match_oracle_first_layer(cuda):
    """Layer-0 top-k expert indices equal the oracle's wherever the router margin is clear."""
    from mrun_b200.moe_engine import MoeDecoder, MoeWeights
    from oracle.moe import softmax_f32

    cfg = _tiny()
    w = MoeWeights.synthetic(cfg, cuda, seed=5)
    lengths = [3, 9, 20]
    dec = MoeDecoder(w, max_rows=4, max_seq_len=40, device=cuda)
    first = torch.tensor([1, 2, 3])
    dec.load_synthetic_context(lengths, first, steps=1, seed=2)
    host = w.to_host()
    ctx_k = [[dec.gather_kv(li, r, lengths[r])[0] for r in range(3)] for li in range(cfg.num_layers)]
    ctx_v = [[dec.gather_kv(li, r, lengths[r])[1] for r in range(3)] for li in range(cfg.num_layers)]
    _, routes = moe_decode_step(host, cfg, first.numpy(), np.array(lengths), ctx_k, ctx_v)
    dec.routes = []
    dec.step(3)
    got = dec.routes[0].cpu().numpy()
    assert np.array_equal(np.sort(got, axis=1), np.sort(routes[0], axis=1))


def test_expert_parallel_shards_hold_the_same_experts(cuda):
    """A sharded model materialises exactly the unsharded model's experts."""
    from mrun_b200.expert_parallel import ExpertShard
    from mrun_b200.moe_engine import MoeWeights

    cfg = _tiny()
    full = MoeWeights.synthetic(cfg, cuda, seed=9)
    part = MoeWeights.synthetic(cfg, cuda, seed=9, shard=ExpertShard(4, 2, cfg.experts))
    for a, b in zip(full.layers, part.layers):
        assert torch.equal(a.pages[4:6], b.pages)
        assert torch.equal(a.qkv.codes, b.qkv.codes)
