"""The B200 decoders free-running against the reference's own greedy decodes.

Dense: the fixture model is written as an on-disk QStore, loaded through ``DenseQStore`` and
decoded by ``DenseDecoder`` (flash prefill, then the captured CUDA-graph step) for 256 greedy
steps after a 32-token prompt, against ``DenseQStoreTarget`` (the reference dense engine's
bf16 contract, run on the CPU). MoE: ``MoeDecoder`` (captured step) against
``Qwen3MoeDecodeRuntime`` with a CPU int8 expert backend, 64 steps after each prompt.

The GPU decodes on its own tokens. A step whose token differs from the reference's is allowed
only where the reference's top-1/top-2 margin is below ``NEAR_TIE``; the test then feeds the
reference's token (re-sync) and continues, and it bounds how many such steps there are. The
head's top-1 logit is compared with the reference's at every step."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import fixture_models as fm

pytestmark = pytest.mark.gpu


def _compare(i, got, got_val, fixture, flips, *, tol):
    want = int(fixture["tokens"][i])
    assert abs(got_val - float(fixture["top1"][i])) < tol, (i, got_val, float(fixture["top1"][i]))
    if got == want:
        return False
    margin = float(fixture["margin"][i])
    assert margin < fm.NEAR_TIE, f"step {i}: token {got} != reference {want} with margin {margin:.4f}"
    flips.append((i, margin))
    return True


def test_dense_decoder_free_running_matches_reference_engine(tmp_path, cuda):
    from mrun_b200.dense_engine import DenseDecoder, DenseWeights
    from mrun_b200.dense_qstore_cuda import DenseQStore

    fm.mdf.build_dense_store(tmp_path / "dense_small")
    g = fm.load("decoder_bf16")
    steps = len(g["tokens"]) - 1
    prompt = torch.from_numpy(g["prompt"])
    flips: list = []
    with DenseQStore("dense_small", root=tmp_path, device=str(cuda)) as store:
        dec = DenseDecoder(DenseWeights.from_qstore(store), max_batch=1, max_seq_len=len(prompt) + steps + 16,
                           device=cuda, max_prefill_tokens=64)
        first = int(dec.prefill(0, prompt))
        if _compare(0, first, float(dec.next_val[0]), g, flips, tol=0.05):
            first = int(g["tokens"][0])
        length = dec.kv.lengths[0]
        dec.kv.reserve(0, length + steps + 1)
        dec.begin_decode(1, torch.tensor([first]), [length])
        dec.capture(1)
        for i in range(1, steps + 1):
            dec.step()
            got, val = int(dec.next_ids[0]), float(dec.next_val[0])
            if _compare(i, got, val, g, flips, tol=0.05):
                dec.in_ids[0] = int(g["tokens"][i])  # re-sync on the reference's token
        dec.check_errors()
    print(f"dense: {steps + 1} tokens, near-tie steps that differed: {flips}")
    assert len(flips) <= 3


def test_moe_decoder_free_running_matches_reference_runtime(cuda):
    from mrun_b200.moe_engine import MoeDecoder

    g = fm.load("moe_decode")
    weights = fm.moe_device_weights(cuda)
    for p in range(2):
        prompt, tokens = g[f"p{p}_prompt"], g[f"p{p}_tokens"]
        fixture = {k: g[f"p{p}_{k}"] for k in ("tokens", "top1", "margin")}
        total = len(prompt) + len(tokens)
        dec = MoeDecoder(weights, max_rows=1, max_seq_len=total + 16, device=cuda)
        dec.kv.release(0)
        dec.kv.reserve(0, total + 1)
        dec.in_ids[0] = int(prompt[0])
        dec.positions[0] = 0
        dec.row_len[0] = 1
        dec.capture(1)
        # the prompt goes through the decode step one token at a time (teacher-forced)
        for t in range(1, len(prompt)):
            dec.step(1)
            dec.in_ids[0] = int(prompt[t])
        flips: list = []
        for i in range(len(tokens)):
            dec.step(1)
            got, val = int(dec.next_ids[0]), float(dec.next_val[0])
            if _compare(i, got, val, fixture, flips, tol=0.05):
                dec.in_ids[0] = int(tokens[i])
        dec.check_errors()
        dec.close()
        print(f"moe prompt {p}: {len(tokens)} tokens, near-tie steps that differed: {flips}")
        assert len(flips) <= 2


def _agrees_until_near_tie(got, fixture):
    """The generated tokens equal the reference's until the end or until a step whose
    reference top-1/top-2 margin is below NEAR_TIE (after which the decodes may part)."""
    want, margin = fixture["tokens"], fixture["margin"]
    for i, (a, b) in enumerate(zip(got, want)):
        if int(a) != int(b):
            assert float(margin[i]) < fm.NEAR_TIE, f"step {i}: token {a} != reference {b} (margin {margin[i]:.4f})"
            return i
        if float(margin[i]) < fm.NEAR_TIE:
            return i
    return len(got)


def test_moe_continuous_batcher_matches_reference_runtime(cuda):
    """MoeContinuousBatcher over a 4-slot captured step: both fixture prompts, each twice, one
    copy arriving while the others decode and one waiting for a retired slot; every request
    follows the reference's greedy decode until its first near-tie step, whatever slot and
    companions it had."""
    from mrun_b200.continuous import MoeContinuousBatcher
    from mrun_b200.moe_engine import MoeDecoder

    g = fm.load("moe_decode")
    weights = fm.moe_device_weights(cuda)
    fixtures = [{k: g[f"p{p}_{k}"] for k in ("prompt", "tokens", "margin")} for p in range(2)]
    steps = len(fixtures[0]["tokens"])
    ctx = max(len(f["prompt"]) for f in fixtures) + steps + 1
    dec = MoeDecoder(weights, max_rows=4, max_seq_len=ctx, device=cuda)
    bat = MoeContinuousBatcher(dec, max_context_tokens=ctx)
    ids = {bat.submit(fixtures[0]["prompt"], max_new_tokens=steps): 0,
           bat.submit(fixtures[1]["prompt"], max_new_tokens=steps): 1,
           bat.submit(fixtures[1]["prompt"], max_new_tokens=24): 1}
    results = {}
    for _ in range(7):
        results.update(bat.step())
    ids[bat.submit(fixtures[0]["prompt"], max_new_tokens=steps)] = 0  # joins mid-decode
    ids[bat.submit(fixtures[0]["prompt"], max_new_tokens=16)] = 0     # waits for a slot
    results.update(bat.run())
    assert set(results) == set(ids)
    agreed = []
    for rid, p in ids.items():
        assert len(results[rid]) == (steps if rid not in (2, 4) else (24 if rid == 2 else 16))
        agreed.append(_agrees_until_near_tie(results[rid], fixtures[p]))
    t = bat.pool.telemetry()
    assert t.allocations == 5 and t.releases == 5 and t.peak_active_slots == 4 and t.slot_reuses >= 1
    bat.close()
    dec.close()
    print(f"continuous: tokens agreeing with the reference before a near tie: {agreed}")
    # the first near-tie steps of the two prompts are 9 and 17
    assert min(agreed) >= 9
