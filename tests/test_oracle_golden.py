"""Pin the CPU oracle to the reference: golden vectors made by the reference itself
(tests/golden/make_golden.py) and the reference's own known-answer tests."""
from __future__ import annotations

import hashlib

import numpy as np
import torch

from oracle import attention as oatt
from oracle import moe as omoe
from oracle import qrow as oq
from oracle import w8a8 as ow8
from oracle.numerics import bf16_round, max_rel_err


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---------------------------------------------------------------- quantiser KATs
# tests/test_paged_parity.py:18-33 of the reference


def test_quant_row_int8_roundtrip_is_per_row_symmetric():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((8, 16)).astype(np.float32)
    q, scale = oq.quant_row_int8(w)
    assert q.dtype == np.int8 and q.shape == w.shape and scale.shape == (8,)
    deq = q.astype(np.float32) * scale[:, None]
    step = np.abs(w).max(axis=1) / 127.0
    assert np.all(np.abs(w - deq) <= step[:, None] + 1e-6)


def test_quant_row_int8_zero_row_uses_unit_scale():
    q, scale = oq.quant_row_int8(np.zeros((2, 4), np.float32))
    assert np.all(q == 0) and np.all(scale == 1.0)


def test_quant_matches_reference_bitwise(golden):
    g = golden("qrow")
    q, s = oq.quant_row_int8(g["quant_w"])
    np.testing.assert_array_equal(q, g["quant_q"])
    np.testing.assert_array_equal(s, g["quant_s"])


def test_config1_quantiser_and_outputs_match_reference(golden):
    g = golden("config1")
    torch.manual_seed(0)
    x = torch.randn(8, 2048).numpy()
    w = (torch.randn(2048, 2048) * 0.02).numpy()
    q, s = oq.quant_row_int8(w)
    assert _sha(q) == str(g["codes_sha"])
    assert _sha(s) == str(g["scales_sha"])
    y = oq.qrow_matmul_fp32(x, q, s)
    assert max_rel_err(y, g["y_w8a16"]) < 1e-5
    qx, act = ow8.quantize_activations(x)
    np.testing.assert_array_equal(qx, g["qx"])
    np.testing.assert_array_equal(act, g["act_scale"])
    acc = ow8.int8_gemm(qx, q)
    assert _sha(acc) == str(g["acc_sha"])
    y8 = ow8.w8a8_matmul(q, s, x)
    np.testing.assert_array_equal(y8, g["y_w8a8"])


# ---------------------------------------------------------------- linear contracts


def test_fp32_matmul_matches_reference(golden):
    g = golden("qrow")
    y = oq.qrow_matmul_fp32(g["mm32_x"], g["quant_q"], g["quant_s"])
    assert max_rel_err(y, g["mm32_y"]) < 1e-6


def test_w8a16_contract_matches_reference(golden):
    g = golden("qrow")
    y = oq.qrow_matmul_w8a16(g["w16_x"], g["w16_q"], g["w16_s"])
    # bf16 outputs: allow one bf16 ulp where fp32 summation order differs
    assert max_rel_err(y, g["w16_y"]) < 1e-2
    assert np.mean(y == g["w16_y"]) > 0.95


def test_swiglu_matches_reference(golden):
    g = golden("qrow")
    y = oq.swiglu_w8a16(g["sw_x"], g["sw_gq"], g["sw_gs"], g["sw_uq"], g["sw_us"])
    assert max_rel_err(y, g["sw_y"]) < 1e-2
    assert np.mean(y == g["sw_y"]) > 0.9


def test_residual_rms_norm_matches_reference(golden):
    g = golden("qrow")
    r, n = oq.residual_rms_norm(g["rr_res"], g["rr_upd"], g["rr_w"], 1e-6)
    np.testing.assert_array_equal(r, g["rr_r"])
    assert max_rel_err(n, g["rr_n"]) < 1e-2
    assert np.mean(n == g["rr_n"]) > 0.98


def test_rms_norm_matches_reference(golden):
    g = golden("qrow")
    y = oq.rms_norm(g["rn_x"], g["rr_w"], 1e-6, out_bf16=True)
    assert max_rel_err(y, g["rn_y"]) < 1e-2
    assert np.mean(y == g["rn_y"]) > 0.98


def test_exact_head_matches_reference_rerank(golden):
    g = golden("qrow")
    x = g["hd_x"]
    best, logits = oq.exact_head_argmax(x, g["hd_q"], g["hd_s"], semantic_rows=290)
    # the reference's top-2 shortlist + fp32 rerank equals the exact argmax here
    np.testing.assert_array_equal(best, g["hd_best"])
    for row in range(x.shape[0]):
        top2 = np.argsort(-logits[row, :290], kind="stable")[:2]
        assert set(top2.tolist()) == set(g["hd_top2"][row].tolist())


# ---------------------------------------------------------------- W8A8


def test_w8a8_matches_reference(golden):
    g = golden("w8a8")
    y0 = ow8.w8a8_matmul(g["q_w"], g["sc_w"], g["x"], protect_k=0)
    np.testing.assert_array_equal(y0, g["y_k0"])
    y4 = ow8.w8a8_matmul(g["q_w"], g["sc_w"], g["x"], protect_k=4)
    assert max_rel_err(y4, g["y_k4"]) < 1e-5
    np.testing.assert_array_equal(ow8.int8_gemm(g["gemm_qx"], g["q_w"]), g["gemm_acc"])


def test_w8a8_outlier_protection_kat(golden):
    """tests/test_w8a8.py:34-44 of the reference, on the oracle."""
    g = golden("w8a8")
    ref = g["x"] @ (g["q_w"].astype(np.float32) * g["sc_w"][:, None]).T
    d0 = np.abs(ow8.w8a8_matmul(g["q_w"], g["sc_w"], g["x"], protect_k=0) - ref).max()
    d = np.abs(ow8.w8a8_matmul(g["q_w"], g["sc_w"], g["x"], protect_k=4) - ref).max()
    assert d0 > 20.0 and d < 0.5 and d < d0 / 20


# ---------------------------------------------------------------- attention


def test_segmented_decode_attention_matches_reference(golden):
    g = golden("attention")
    y = oatt.segmented_decode_attention(g["seg_q"], g["seg_ck"], g["seg_cv"], g["seg_kn"], g["seg_vn"], g["seg_len"])
    assert max_rel_err(y, g["seg_out"]) < 1e-2


def test_segmented_gqa_decode_matches_reference(golden):
    g = golden("attention")
    y = oatt.segmented_gqa_decode(g["gqa_q"], g["gqa_kc"], g["gqa_vc"], g["gqa_slots"], g["gqa_len"])
    assert max_rel_err(y, g["gqa_out"]) < 1e-2


def test_paged_gather_is_exact_and_matches_contiguous():
    rng = np.random.default_rng(0)
    hkv, d, length = 2, 8, 37
    contiguous = rng.standard_normal((length, hkv, d)).astype(np.float32)
    pages_needed = (length + 15) // 16
    table = rng.permutation(10)[:pages_needed]
    pages = np.zeros((10, hkv, 16, d), np.float32)
    for t in range(length):
        pages[table[t // 16], :, t % 16] = contiguous[t]
    np.testing.assert_array_equal(oatt.paged_gather(pages, table, length), contiguous)


# ---------------------------------------------------------------- MoE


def test_router_topk_matches_reference(golden):
    g = golden("moe")
    idx, _, w = omoe.router_topk(g["router_logits"], 8, renorm=True)
    np.testing.assert_array_equal(idx, g["router_idx"])
    np.testing.assert_array_equal(w, g["router_w"])


def test_route_tensors_match_reference_bitwise(golden):
    g = golden("moe")
    tok, coef, starts, counts, inv = omoe.route_tensors(g["router_idx"], g["router_w"], 128)
    np.testing.assert_array_equal(tok, g["route_tok"])
    np.testing.assert_array_equal(coef, g["route_coef"])
    np.testing.assert_array_equal(starts, g["route_starts"])
    np.testing.assert_array_equal(counts, g["route_counts"])
    np.testing.assert_array_equal(inv, g["route_inv"])


def test_route_tensors_reference_kat():
    """tests/test_olmoe_cuda.py:73-90 of the reference."""
    idx = np.array([[3, 1], [1, 2], [3, 2]])
    w = np.array([[0.7, 0.3], [0.6, 0.4], [0.8, 0.2]], np.float32)
    tok, coef, starts, counts, inv = omoe.route_tensors(idx, w, 5)
    assert counts.tolist() == [0, 2, 2, 2, 0]
    assert starts.tolist() == [0, 0, 2, 4, 6]
    assert tok.tolist() == [0, 1, 1, 2, 0, 2]
    np.testing.assert_allclose(coef, [0.3, 0.6, 0.4, 0.2, 0.7, 0.8])
    assert sorted(inv.tolist()) == list(range(6))


def test_stable_reduce_matches_reference_bitwise(golden):
    g = golden("moe")
    out = omoe.stable_route_reduce(g["reduce_eo"], g["route_coef"], g["route_inv"], 32, 8)
    np.testing.assert_array_equal(out, g["reduce_out"])


def test_bf16_round_is_rne():
    vals = np.array([1.0, 1.00390625, 1.01171875, -3.3, 65504.0], np.float32)
    expected = torch.tensor(vals).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(bf16_round(vals), expected)
