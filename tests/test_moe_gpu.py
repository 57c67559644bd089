"""Routed-MoE chain parity: router indices/weights, route plans (counts, starts, token order,
coefficients, inverse) and the stable combine bit-exact against the reference's golden
vectors; grouped int8 expert projections within the bf16 tolerance of the oracle, and
bit-identical per row whatever the group composition (the property expert parallelism
relies on)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe as omoe
from oracle import qrow as oq
from oracle.numerics import bf16_round, max_rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2


def test_router_topk_golden(golden, cuda):
    from mrun_b200.moe import router_topk

    g = golden("moe")
    idx, w16, _ = router_topk(torch.from_numpy(g["router_logits"]).to(cuda), 8, renorm=True)
    np.testing.assert_array_equal(idx.cpu().numpy(), g["router_idx"])
    np.testing.assert_array_equal(w16.float().cpu().numpy(), g["router_w"])


def test_route_compile_golden_and_kat(golden, cuda):
    from mrun_b200.moe import grouped_route_tensors, grouped_route_tensors_with_inverse

    g = golden("moe")
    tok, coef, starts, counts, inv, _ = grouped_route_tensors_with_inverse(
        torch.from_numpy(g["router_idx"]).to(cuda), torch.from_numpy(g["router_w"]).to(cuda), num_experts=128)
    np.testing.assert_array_equal(tok.cpu().numpy(), g["route_tok"])
    np.testing.assert_array_equal(coef.cpu().numpy(), g["route_coef"])
    np.testing.assert_array_equal(starts.cpu().numpy(), g["route_starts"])
    np.testing.assert_array_equal(counts.cpu().numpy(), g["route_counts"])
    np.testing.assert_array_equal(inv.cpu().numpy(), g["route_inv"])
    # tests/test_olmoe_cuda.py:73-90 of the reference
    idx = torch.tensor([[3, 1], [1, 2], [3, 2]], device=cuda)
    w = torch.tensor([[0.7, 0.3], [0.6, 0.4], [0.8, 0.2]], device=cuda)
    tok, coef, starts, counts, _ = grouped_route_tensors(idx, w, num_experts=5)
    assert counts.tolist() == [0, 2, 2, 2, 0]
    assert starts.tolist() == [0, 0, 2, 4, 6]
    assert tok.tolist() == [0, 1, 1, 2, 0, 2]
    torch.testing.assert_close(coef, torch.tensor([0.3, 0.6, 0.4, 0.2, 0.7, 0.8], device=cuda))


@pytest.mark.parametrize("tokens,k,experts", [(32, 8, 128), (2048, 8, 128), (256, 2, 8), (5000, 4, 64)])
def test_route_compile_random_bit_exact(tokens, k, experts, cuda):
    from mrun_b200.moe import grouped_route_tensors_with_inverse

    rng = np.random.default_rng(tokens)
    idx = np.stack([rng.permutation(experts)[:k] for _ in range(tokens)]).astype(np.int64)
    w = rng.random((tokens, k)).astype(np.float32)
    got = grouped_route_tensors_with_inverse(torch.from_numpy(idx).to(cuda), torch.from_numpy(w).to(cuda),
                                             num_experts=experts)
    ref = omoe.route_tensors(idx, w, experts)
    for a, b in zip(got[:5], (ref[0], ref[1], ref[2], ref[3], ref[4])):
        np.testing.assert_array_equal(a.cpu().numpy(), b)


def test_stable_reduce_golden(golden, cuda):
    from mrun_b200.moe import stable_route_reduce

    g = golden("moe")
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    out = stable_route_reduce(dev(g["reduce_eo"]).to(torch.bfloat16), dev(g["route_coef"]), dev(g["route_tok"]),
                              dev(g["route_counts"]), dev(g["router_idx"]), torch.arange(128, device=cuda),
                              inverse_assignments=dev(g["route_inv"]))
    np.testing.assert_array_equal(out.cpu().numpy(), g["reduce_out"])


def _expert_pages(rng, experts, hidden, ffn, dev):
    from mrun_b200.moe import ExpertPageLayout, pack_expert_page

    ly = ExpertPageLayout.create(hidden, ffn)
    pages = torch.zeros((experts, ly.page_stride), dtype=torch.uint8, device=dev)
    host = []
    for e in range(experts):
        gu_q, gu_s = oq.quant_row_int8((rng.standard_normal((2 * ffn, hidden)) * 0.02).astype(np.float32))
        dn_q, dn_s = oq.quant_row_int8((rng.standard_normal((hidden, ffn)) * 0.02).astype(np.float32))
        pack_expert_page(ly, torch.from_numpy(gu_q), torch.from_numpy(gu_s), torch.from_numpy(dn_q),
                         torch.from_numpy(dn_s), pages[e])
        host.append((gu_q, gu_s, dn_q, dn_s))
    return ly, pages, host


@pytest.mark.parametrize("tokens,k,experts,hidden,ffn", [
    (32, 8, 16, 256, 128), (7, 2, 8, 512, 384), (64, 4, 8, 2048, 768),
    # Mixtral's expert ffn: the down projection's 14336 in_features stage 4 rows per pass
    (24, 2, 2, 1024, 14336),
])
def test_moe_backend_vs_oracle_and_row_independence(tokens, k, experts, hidden, ffn, cuda):
    from mrun_b200.moe import PagedInt8ExpertBackend, ResidentInt8ExpertPages, router_topk

    rng = np.random.default_rng(tokens + experts)
    ly, pages, host = _expert_pages(rng, experts, hidden, ffn, cuda)
    backend = PagedInt8ExpertBackend(ResidentInt8ExpertPages(ly, [pages]), num_experts=experts)
    x = torch.from_numpy(bf16_round(rng.standard_normal((tokens, hidden)).astype(np.float32))).to(cuda).to(torch.bfloat16)
    logits = torch.from_numpy(rng.standard_normal((tokens, experts)).astype(np.float32)).to(cuda)
    idx, w16, _ = router_topk(logits, k)
    out = backend.moe(0, x, idx, w16)
    # oracle: route, per-expert exact projections with the same bf16 boundaries, stable combine
    idx_np, w_np = idx.cpu().numpy(), w16.float().cpu().numpy()
    tok, coef, starts, counts, inv = omoe.route_tensors(idx_np, w_np, experts)
    xf = x.float().cpu().numpy()
    eo = np.zeros((tok.size, hidden), np.float32)
    for e in range(experts):
        s, c = int(starts[e]), int(counts[e])
        if c:
            eo[s:s + c] = omoe.expert_swiglu_exact(xf[tok[s:s + c]], *host[e])
    ref = bf16_round(omoe.stable_route_reduce(eo, coef, inv, tokens, k))
    assert max_rel_err(out.float().cpu().numpy(), ref) < TOL
    # each token's result is independent of which other tokens share its experts
    single = torch.stack([backend.moe(0, x[i:i + 1], idx[i:i + 1], w16[i:i + 1])[0] for i in range(min(tokens, 6))])
    assert torch.equal(single, out[: single.shape[0]])


@pytest.mark.parametrize("t,e,k,h", [(32, 128, 8, 2048), (5, 8, 2, 4096), (64, 60, 4, 512), (1, 256, 16, 256),
                                     (97, 200, 8, 1032)])
def test_fused_router_matches_projection_and_selection(t, e, k, h, cuda):
    """mrb_router_qrow_topk: logits within one bf16 rounding of the exact int8 x bf16 product;
    the selection bit-identical to router_topk on those same logits (indices, bf16 weights);
    coefficients are the bf16 weights as fp32."""
    from mrun_b200.moe import router_qrow_topk, router_topk

    gen = torch.Generator(device="cpu").manual_seed(t * 1000 + e)
    codes = torch.randint(-127, 128, (e, h), generator=gen, dtype=torch.int8)
    scales = torch.rand(e, generator=gen) * 1e-3 + 1e-4
    x = torch.randn(t, h, generator=gen).to(torch.bfloat16)
    logits = torch.empty(t, e, dtype=torch.bfloat16, device=cuda)
    idx, w16, coef = router_qrow_topk(x.to(cuda), codes.to(cuda), scales.to(cuda), k, logits=logits)
    exact = (x.double() @ codes.double().T) * scales.double()[None, :]
    got = logits.double().cpu()
    # per element: one bf16 rounding (2^-9 relative) plus fp32 summation error, measured
    # against the row's largest logit so that near-zero logits do not divide by ~0
    rowmax = exact.abs().amax(dim=1, keepdim=True)
    assert float(((got - exact).abs() / rowmax).max()) <= 2.0 ** -8
    ridx, rw16, _ = router_topk(logits, k, renorm=True)
    assert torch.equal(idx, ridx) and torch.equal(w16, rw16)
    assert torch.equal(coef, w16.float())
    # deterministic
    for _ in range(3):
        idx2, w2, _ = router_qrow_topk(x.to(cuda), codes.to(cuda), scales.to(cuda), k)
        assert torch.equal(idx2, idx) and torch.equal(w2, w16)


@pytest.mark.parametrize("tokens,k,experts,hidden,ffn", [(64, 4, 32, 512, 384), (32, 8, 128, 2048, 768),
                                                         (16, 2, 8, 1024, 14336)])
def test_overlapped_expert_mlp_matches_separate_launches(tokens, k, experts, hidden, ffn, cuda):
    """mrb_grouped_expert_mlp (the down launch starting on each expert as its gate/up work is
    stored) gives the bits of the two lone grouped launches, and leaves its counters at zero
    call after call."""
    from mrun_b200 import _lib
    from mrun_b200.moe import expert_mlp_sync, grouped_expert_mlp, grouped_route_tensors_with_inverse, router_topk

    rng = np.random.default_rng(tokens * experts)
    ly, pages, _ = _expert_pages(rng, experts, hidden, ffn, cuda)
    x = torch.from_numpy(bf16_round(rng.standard_normal((tokens, hidden)).astype(np.float32))).to(cuda).to(torch.bfloat16)
    idx, w16, _ = router_topk(torch.from_numpy(rng.standard_normal((tokens, experts)).astype(np.float32)).to(cuda), k)
    token_ids, _, starts, counts, _, _ = grouped_route_tensors_with_inverse(idx, w16, num_experts=experts)
    a = int(token_ids.numel())
    act = torch.empty(a, ffn, dtype=torch.bfloat16, device=cuda)
    ref = torch.empty(a, hidden, dtype=torch.bfloat16, device=cuda)
    base, stride, stream = pages.data_ptr(), ly.page_stride, _lib.stream_handle(cuda)
    _lib.call("mrb_grouped_qrow", x.data_ptr(), token_ids.data_ptr(), starts.data_ptr(), counts.data_ptr(), experts,
              base + ly.gate_up_codes_offset, stride, base + ly.gate_up_scales_offset, stride // 4, None, ffn, hidden,
              ffn, 1, a, act.data_ptr(), stream)
    _lib.call("mrb_grouped_qrow", act.data_ptr(), None, starts.data_ptr(), counts.data_ptr(), experts,
              base + ly.down_codes_offset, stride, base + ly.down_scales_offset, stride // 4, None, hidden, ffn, 0, 0,
              a, ref.data_ptr(), stream)
    sync = expert_mlp_sync(experts, cuda)
    for _ in range(3):
        y = grouped_expert_mlp(x, token_ids, starts, counts, pages, ly, sync=sync)
        assert torch.equal(y, ref)
    assert not sync.any()


def test_large_expert_counts_on_the_gemms_match_the_grouped_kernel(cuda):
    """expert_mlp_large_counts: experts with at least 64 routed rows run on the tcgen05 GEMMs
    (rows within the bf16 tolerance of the grouped kernel's); the others stay on the grouped
    kernel, bit-identical to it."""
    from mrun_b200.moe import (expert_mlp_large_counts, expert_mlp_sync, grouped_expert_mlp,
                               grouped_route_tensors_with_inverse)

    tokens, k, experts, hidden, ffn = 200, 2, 8, 1024, 2048
    rng = np.random.default_rng(9)
    ly, pages, _ = _expert_pages(rng, experts, hidden, ffn, cuda)
    x = torch.from_numpy(bf16_round(rng.standard_normal((tokens, hidden)).astype(np.float32))).to(cuda).to(torch.bfloat16)
    # skewed routing: experts 0 and 1 take most rows, the rest a few each
    logits = rng.standard_normal((tokens, experts)).astype(np.float32)
    logits[:, :2] += 3.0
    idx = torch.from_numpy(np.argsort(-logits, axis=1)[:, :k].copy()).to(cuda)
    w = torch.full((tokens, k), 0.5, device=cuda)
    token_ids, _, starts, counts, _, _ = grouped_route_tensors_with_inverse(idx, w, num_experts=experts)
    c = counts.cpu().tolist()
    assert c[0] >= 64 and c[1] >= 64 and min(c[2:]) < 64
    sync = expert_mlp_sync(experts, cuda)
    ref = grouped_expert_mlp(x, token_ids, starts, counts, pages, ly, sync=sync)
    for _ in range(2):
        got = expert_mlp_large_counts(x, token_ids, starts, counts, pages, ly, sync=sync)
        big = int(starts[2].item())  # experts 0 and 1 fill rows [0, big)
        assert max_rel_err(got[:big].float().cpu().numpy(), ref[:big].float().cpu().numpy()) < TOL
        assert torch.equal(got[big:], ref[big:])
    assert not sync.any()
