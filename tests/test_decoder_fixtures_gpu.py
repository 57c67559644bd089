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
