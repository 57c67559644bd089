"""Parity of the B200 int8 QStore linear kernels against the CPU oracle and the reference's
golden vectors. Tolerances: fp32 outputs max relative error 1e-4, bf16 outputs 1e-2
(norm-wise: max|a-b| / max|b|); integer results bit-exact."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from oracle import qrow as oq
from oracle.numerics import bf16_round, max_rel_err

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2
FP32_TOL = 1e-4


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _dev(a, dtype=None, device="cuda"):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return t if dtype is None else t.to(dtype)


def test_quantiser_bit_exact(golden, cuda):
    from mrun_b200.qstore_build import quant_row_int8

    g = golden("qrow")
    q, s = quant_row_int8(_dev(g["quant_w"]))
    np.testing.assert_array_equal(q.cpu().numpy(), g["quant_q"])
    np.testing.assert_array_equal(s.cpu().numpy(), g["quant_s"])


def test_config1_w8a16_fp32_against_reference(golden, cuda):
    from mrun_b200.dense_qstore_cuda import qrow_linear
    from mrun_b200.qstore_build import quant_row_int8

    g = golden("config1")
    torch.manual_seed(0)
    x = torch.randn(8, 2048)
    w = torch.randn(2048, 2048) * 0.02
    q, s = quant_row_int8(w.to(cuda))
    assert _sha(q.cpu().numpy()) == str(g["codes_sha"])
    assert _sha(s.cpu().numpy()) == str(g["scales_sha"])
    y = qrow_linear(q, s, x.to(cuda))
    assert y.dtype == torch.float32
    assert max_rel_err(y.cpu().numpy(), g["y_w8a16"]) < FP32_TOL


def test_fp32_rows_against_golden(golden, cuda):
    from mrun_b200.dense_qstore_cuda import qrow_linear

    g = golden("qrow")
    y = qrow_linear(_dev(g["quant_q"]), _dev(g["quant_s"]), _dev(g["mm32_x"]))
    assert max_rel_err(y.cpu().numpy(), g["mm32_y"]) < FP32_TOL


def test_w8a16_bf16_against_golden(golden, cuda):
    from mrun_b200.dense_qstore_cuda import CompactQRowPage, fused_qrow_matmul

    g = golden("qrow")
    page = CompactQRowPage("p", 0, 96, 256, _dev(g["w16_q"]), _dev(g["w16_s"]))
    y, impl = fused_qrow_matmul(page, _dev(g["w16_x"], torch.bfloat16))
    assert impl.startswith("b200-")
    assert y.dtype == torch.bfloat16
    assert max_rel_err(y.float().cpu().numpy(), g["w16_y"]) < BF16_TOL


@pytest.mark.parametrize("m", [1, 2, 3, 8, 9, 16])
@pytest.mark.parametrize("n,k", [(1, 16), (17, 80), (512, 3584), (4608, 3584), (96, 18944)])
def test_w8a16_shapes(m, n, k, cuda):
    from mrun_b200.dense_qstore_cuda import qrow_linear
    from mrun_b200.qstore_build import quant_row_int8

    gen = torch.Generator(device="cpu").manual_seed(m * 1000 + n + k)
    w = torch.randn(n, k, generator=gen) * 0.02
    x = (torch.randn(m, k, generator=gen) * 3).to(torch.bfloat16)
    q, s = quant_row_int8(w.to(cuda))
    y = qrow_linear(q, s, x.to(cuda)).float().cpu().numpy()
    exact = oq.qrow_matmul_exact(x.float().numpy(), q.cpu().numpy(), s.cpu().numpy())
    assert max_rel_err(y, exact) < 4e-3  # one bf16 rounding of the output
    ref = oq.qrow_matmul_w8a16(x.float().numpy(), q.cpu().numpy(), s.cpu().numpy())
    assert max_rel_err(y, ref) < BF16_TOL


@pytest.mark.parametrize("m", [1, 4, 5, 8])
def test_fp32_rows_shapes(m, cuda):
    from mrun_b200.dense_qstore_cuda import qrow_linear

    gen = torch.Generator(device="cpu").manual_seed(m)
    q = torch.randint(-127, 128, (300, 1024), generator=gen, dtype=torch.int8)
    s = torch.rand(300, generator=gen) * 0.01 + 1e-4
    x = torch.randn(m, 1024, generator=gen) * torch.logspace(-3, 3, 1024)[None, :]
    y = qrow_linear(q.to(cuda), s.to(cuda), x.to(cuda)).cpu().numpy()
    exact = oq.qrow_matmul_exact(x.numpy(), q.numpy(), s.numpy())
    assert max_rel_err(y, exact) < 1e-5


def test_bias_added_in_compute_dtype(cuda):
    from mrun_b200.dense_qstore_cuda import qrow_linear

    gen = torch.Generator(device="cpu").manual_seed(11)
    q = torch.randint(-127, 128, (64, 128), generator=gen, dtype=torch.int8)
    s = torch.rand(64, generator=gen) * 0.01
    x = torch.randn(2, 128, generator=gen).to(torch.bfloat16)
    bias = torch.randn(64, generator=gen)
    y = qrow_linear(q.to(cuda), s.to(cuda), x.to(cuda), bias=bias.to(cuda)).float().cpu().numpy()
    base = bf16_round(oq.qrow_matmul_exact(x.float().numpy(), q.numpy(), s.numpy()))
    expected = bf16_round(base + bf16_round(bias.numpy())[None, :])
    assert max_rel_err(y, expected) < BF16_TOL


def test_swiglu_against_golden_and_oracle(golden, cuda):
    from mrun_b200.dense_qstore_cuda import CompactQRowPage, fused_qrow_swiglu

    g = golden("qrow")
    gp = CompactQRowPage("g", 0, 64, 128, _dev(g["sw_gq"]), _dev(g["sw_gs"]))
    up = CompactQRowPage("u", 0, 64, 128, _dev(g["sw_uq"]), _dev(g["sw_us"]))
    y, _ = fused_qrow_swiglu(gp, up, _dev(g["sw_x"], torch.bfloat16))
    assert max_rel_err(y.float().cpu().numpy(), g["sw_y"]) < BF16_TOL
    # larger shape against the oracle
    gen = torch.Generator(device="cpu").manual_seed(3)
    x = torch.randn(1, 3584, generator=gen).to(torch.bfloat16)
    wg = torch.randn(1000, 3584, generator=gen) * 0.02
    wu = torch.randn(1000, 3584, generator=gen) * 0.02
    gq, gs = oq.quant_row_int8(wg.numpy())
    uq, us = oq.quant_row_int8(wu.numpy())
    gp = CompactQRowPage("g", 0, 1000, 3584, _dev(gq), _dev(gs))
    up = CompactQRowPage("u", 0, 1000, 3584, _dev(uq), _dev(us))
    y, _ = fused_qrow_swiglu(gp, up, x.to(cuda))
    ref = oq.swiglu_w8a16(x.float().numpy(), gq, gs, uq, us)
    assert max_rel_err(y.float().cpu().numpy(), ref) < BF16_TOL


def test_residual_rms_norm_against_golden(golden, cuda):
    from mrun_b200.dense_qstore_cuda import fused_residual_rms_norm

    g = golden("qrow")
    r, n, _ = fused_residual_rms_norm(_dev(g["rr_res"], torch.bfloat16), _dev(g["rr_upd"], torch.bfloat16),
                                      _dev(g["rr_w"]), 1e-6)
    np.testing.assert_array_equal(r.float().cpu().numpy(), g["rr_r"])
    assert max_rel_err(n.float().cpu().numpy(), g["rr_n"]) < BF16_TOL


def test_rms_norm_against_golden(golden, cuda):
    from mrun_b200.dense_qstore_cuda import stable_rms_norm

    g = golden("qrow")
    y, _ = stable_rms_norm(_dev(g["rn_x"], torch.bfloat16), _dev(g["rr_w"]), 1e-6)
    assert max_rel_err(y.float().cpu().numpy(), g["rn_y"]) < BF16_TOL


def test_exact_argmax_head(golden, cuda):
    from mrun_b200.dense_qstore_cuda import CompactQRowPage, fused_qrow_exact_argmax

    g = golden("qrow")
    page = CompactQRowPage("lm_head", 0, 300, 64, _dev(g["hd_q"]), _dev(g["hd_s"]))
    best, val, _ = fused_qrow_exact_argmax(page, _dev(g["hd_x"], torch.bfloat16), semantic_row_count=290)
    np.testing.assert_array_equal(best.cpu().numpy(), g["hd_best"])


def test_argmax_ties_pick_lowest_index(cuda):
    from mrun_b200.dense_qstore_cuda import qrow_argmax

    q = torch.zeros(4000, 64, dtype=torch.int8)
    q[[7, 1234, 3999], 0] = 100  # three identical maximal rows
    s = torch.ones(4000)
    x = torch.zeros(2, 64, dtype=torch.bfloat16)
    x[:, 0] = 1.0
    idx, val, _ = qrow_argmax(q.to(cuda), s.to(cuda), x.to(cuda))
    assert idx.cpu().tolist() == [7, 7]
    idx, _, _ = qrow_argmax(q.to(cuda), s.to(cuda), x.to(cuda), semantic_rows=5)
    assert idx.cpu().tolist() == [0, 0]


@pytest.mark.parametrize("m,n,k,semantic", [(64, 152064, 512, 152000), (40, 3001, 256, 3001), (300, 9000, 128, 8999),
                                             (32, 151936, 256, 151936)])
def test_greedy_head_many_rows(m, n, k, semantic, cuda):
    """Above 16 rows the greedy head runs on the tcgen05 W8A16 GEMM with the argmax fused
    into its epilogue: fp32 logits within 1e-4 of the float64 product and every pick the
    float64 argmax unless the top two are within that error (reported near-tie)."""
    from mrun_b200.dense_qstore_cuda import qrow_argmax

    gen = torch.Generator(device="cpu").manual_seed(m + n)
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    s = torch.rand(n, generator=gen) * 1e-3 + 1e-4
    x = torch.randn(m, k, generator=gen).to(torch.bfloat16)
    idx, val, logits = qrow_argmax(q.to(cuda), s.to(cuda), x.to(cuda), semantic_rows=semantic)
    exact = oq.qrow_matmul_exact(x.float().numpy(), q.numpy(), s.numpy())
    got = logits.cpu().numpy()
    assert max_rel_err(got, exact) < FP32_TOL
    e = exact[:, :semantic]
    best = e.argmax(axis=1)
    picks = idx.cpu().numpy()
    for r in range(m):
        if picks[r] != best[r]:
            assert e[r, best[r]] - e[r, picks[r]] <= 1e-4 * np.abs(e[r]).max(), (r, picks[r], best[r])
    np.testing.assert_array_equal(val.cpu().numpy(), got[np.arange(m), picks])
    assert _tc_timeouts() == 0


def test_embed_rows_bit_exact(cuda):
    from mrun_b200.qstore_build import embed_rows

    gen = torch.Generator(device="cpu").manual_seed(5)
    q = torch.randint(-127, 128, (500, 256), generator=gen, dtype=torch.int8)
    s = torch.rand(500, generator=gen) * 0.02
    ids = torch.tensor([0, 499, 17, 17, 250])
    out = embed_rows(q.to(cuda), s.to(cuda), ids.to(cuda), dtype=torch.float32).cpu().numpy()
    np.testing.assert_array_equal(out, oq.embed_rows(q.numpy(), s.numpy(), ids.numpy()))
    bad = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = embed_rows(q.to(cuda), s.to(cuda), torch.tensor([3, 600], device=cuda), bad_ids=bad)
    assert int(bad.item()) == 1 and float(out[1].abs().sum()) == 0.0


def test_edge_cases(cuda):
    from mrun_b200.dense_qstore_cuda import qrow_linear

    q = torch.ones(32, 64, dtype=torch.int8, device=cuda)
    s = torch.ones(32, device=cuda)
    empty = qrow_linear(q, s, torch.empty(0, 64, dtype=torch.bfloat16, device=cuda))
    assert empty.shape == (0, 32)
    with pytest.raises(RuntimeError, match="multiple of 16"):
        qrow_linear(torch.ones(8, 24, dtype=torch.int8, device=cuda), torch.ones(8, device=cuda),
                    torch.ones(1, 24, dtype=torch.bfloat16, device=cuda))
    with pytest.raises(ValueError):
        qrow_linear(q, s, torch.ones(1, 32, dtype=torch.bfloat16, device=cuda))


@pytest.mark.parametrize("m,n,k", [(17, 64, 128), (100, 300, 512), (512, 512, 3584), (130, 200, 80)])
def test_w8a16_gemm_path(m, n, k, cuda):
    """Prefill-size rows take the tensor-core GEMM; same contract as the GEMV."""
    from mrun_b200.dense_qstore_cuda import qrow_linear

    gen = torch.Generator(device="cpu").manual_seed(m + n + k)
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    s = torch.rand(n, generator=gen) * 0.01 + 1e-4
    x = (torch.randn(m, k, generator=gen) * 2).to(torch.bfloat16)
    bias = torch.randn(n, generator=gen)
    y = qrow_linear(q.to(cuda), s.to(cuda), x.to(cuda)).float().cpu().numpy()
    exact = oq.qrow_matmul_exact(x.float().numpy(), q.numpy(), s.numpy())
    assert max_rel_err(y, exact) < 4e-3
    yb = qrow_linear(q.to(cuda), s.to(cuda), x.to(cuda), bias=bias.to(cuda)).float().cpu().numpy()
    expected = bf16_round(bf16_round(exact) + bf16_round(bias.numpy())[None, :])
    assert max_rel_err(yb, expected) < BF16_TOL


@pytest.mark.parametrize("m,n,k", [(17, 64, 128), (200, 300, 512), (512, 256, 3584)])
def test_swiglu_gemm_path(m, n, k, cuda):
    from mrun_b200.dense_qstore_cuda import qrow_swiglu

    gen = torch.Generator(device="cpu").manual_seed(m * 7 + n)
    gq = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    uq = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    gs = torch.rand(n, generator=gen) * 0.002
    us = torch.rand(n, generator=gen) * 0.002
    x = torch.randn(m, k, generator=gen).to(torch.bfloat16)
    y = qrow_swiglu(gq.to(cuda), gs.to(cuda), uq.to(cuda), us.to(cuda), x.to(cuda)).float().cpu().numpy()
    ref = oq.swiglu_w8a16(x.float().numpy(), gq.numpy(), gs.numpy(), uq.numpy(), us.numpy())
    assert max_rel_err(y, ref) < BF16_TOL
    # the GEMV and GEMM paths agree on the rows they share
    y_small = qrow_swiglu(gq.to(cuda), gs.to(cuda), uq.to(cuda), us.to(cuda), x[:4].to(cuda)).float().cpu().numpy()
    assert max_rel_err(y_small, y[:4]) < BF16_TOL


def _tc_timeouts() -> int:
    import ctypes

    from mrun_b200 import _lib

    out = ctypes.c_uint(0)
    _lib.call("mrb_tc_status", ctypes.addressof(out))
    return out.value


@pytest.mark.parametrize("m,n,k", [
    (64, 300, 512),      # 128 x 128 tiles, one k tail-free tile row
    (300, 1001, 80),     # ragged rows / columns (scalar stores), k tail inside a 64-wide stage
    (1024, 4736, 512),   # 128 x 256 double-buffered tiles
    (4096, 9472, 64),    # 256 x 256 tiles (two accumulator halves), one k stage
    (33, 4096, 3584),
    # 17-32 rows: k split over a thread-block cluster, partials reduced through distributed
    # shared memory (config-4 o, qkv and router shapes)
    (32, 2048, 4096),
    (32, 5120, 2048),
    (17, 128, 2048),
    (24, 1000, 1024),
])
def test_tcgen05_w8a16_gemm(m, n, k, cuda):
    """The tcgen05 W8A16 GEMM (int8 weights converted to bf16 in shared memory, fp32 TMEM
    accumulators) against the float64 product, plus the bias epilogue; no wait timed out."""
    from mrun_b200.dense_qstore_cuda import qrow_linear

    gen = torch.Generator(device="cpu").manual_seed(m * 3 + n + k)
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    s = torch.rand(n, generator=gen) * 0.01 + 1e-4
    x = torch.randn(m, k, generator=gen).to(torch.bfloat16)
    y = qrow_linear(q.to(cuda), s.to(cuda), x.to(cuda)).float().cpu().numpy()
    exact = oq.qrow_matmul_exact(x.float().numpy(), q.numpy(), s.numpy())
    # fp32 accumulation of exact bf16 products, one bf16 rounding at the end
    assert max_rel_err(y, exact) < 4e-3
    bias = torch.randn(n, generator=gen)
    yb = qrow_linear(q.to(cuda), s.to(cuda), x.to(cuda), bias=bias.to(cuda)).float().cpu().numpy()
    assert max_rel_err(yb, bf16_round(bf16_round(exact) + bf16_round(bias.numpy())[None, :])) < BF16_TOL
    # deterministic
    y2 = qrow_linear(q.to(cuda), s.to(cuda), x.to(cuda)).float().cpu().numpy()
    assert np.array_equal(y, y2)
    assert _tc_timeouts() == 0


@pytest.mark.parametrize("m,n,k", [(512, 18944, 512), (100, 700, 256), (1024, 2368, 128), (32, 700, 1024)])
def test_tcgen05_w8a16_swiglu(m, n, k, cuda):
    """Paired gate/up tiles (gate rows then up rows in one B operand) with the SwiGLU epilogue."""
    from mrun_b200.dense_qstore_cuda import qrow_swiglu

    gen = torch.Generator(device="cpu").manual_seed(m + 5 * n + k)
    gq = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    uq = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    gs = torch.rand(n, generator=gen) * 0.004
    us = torch.rand(n, generator=gen) * 0.004
    x = torch.randn(m, k, generator=gen).to(torch.bfloat16)
    y = qrow_swiglu(gq.to(cuda), gs.to(cuda), uq.to(cuda), us.to(cuda), x.to(cuda)).float().cpu().numpy()
    ref = oq.swiglu_w8a16(x.float().numpy(), gq.numpy(), gs.numpy(), uq.numpy(), us.numpy())
    assert max_rel_err(y, ref) < BF16_TOL
    assert _tc_timeouts() == 0


def _abi_matmul(x, q, s, workspace):
    """mrb_qrow_matmul through the C ABI with an explicit workspace (None: whole tiles)."""
    from mrun_b200 import _lib

    m, k = x.shape
    n = q.shape[0]
    y = torch.empty((m, n), dtype=x.dtype, device=x.device)
    code = _lib.dtype_code(x.dtype)
    _lib.call("mrb_qrow_matmul", x.data_ptr(), code, m, k, q.data_ptr(), s.data_ptr(), n, None, y.data_ptr(), code,
              _lib.ptr(workspace), 0 if workspace is None else workspace.numel(), _lib.stream_handle(x.device))
    return y


@pytest.mark.parametrize("m,n,k,dtype", [
    (1, 3584, 3584, torch.bfloat16),    # 224 tiles on 296 CTA slots: tiles split along k
    (1, 3584, 18944, torch.bfloat16),
    (3, 3584, 128, torch.bfloat16),     # 2 k blocks per tile: CTAs of 1 or 2 units
    (16, 3584, 3584, torch.bfloat16),
    (2, 200, 1024, torch.float16),      # 13 tiles over many CTAs: every tile split
    (4, 3584, 1024, torch.float32),     # fp32 rows (hi/lo split columns)
])
def test_stream_k_matches_whole_tiles_and_oracle(m, n, k, dtype, cuda):
    from mrun_b200.dense_qstore_cuda import qrow_workspace_bytes

    gen = torch.Generator(device="cpu").manual_seed(n + k + m)
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    s = torch.rand(n, generator=gen) * 0.01 + 1e-4
    x = (torch.randn(m, k, generator=gen) * 2).to(dtype)
    qd, sd, xd = q.to(cuda), s.to(cuda), x.to(cuda)
    ws = torch.zeros(qrow_workspace_bytes(xd.device, n), dtype=torch.uint8, device=cuda)
    split = _abi_matmul(xd, qd, sd, ws)
    again = _abi_matmul(xd, qd, sd, ws)  # counters reset themselves: same bits on reuse
    whole = _abi_matmul(xd, qd, sd, None)
    torch.testing.assert_close(split, again, rtol=0, atol=0)
    exact = oq.qrow_matmul_exact(x.float().numpy(), q.numpy(), s.numpy())
    tol = FP32_TOL if dtype is torch.float32 else 4e-3
    assert max_rel_err(split.float().cpu().numpy(), exact) < tol
    assert max_rel_err(whole.float().cpu().numpy(), exact) < tol


def test_stream_k_swiglu_matches_oracle(cuda):
    from mrun_b200.dense_qstore_cuda import qrow_swiglu, qrow_workspace_bytes

    n, k = 3584, 2048  # 224 tiles: the stream-K schedule
    gen = torch.Generator(device="cpu").manual_seed(7)
    qg = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    qu = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    sg = torch.rand(n, generator=gen) * 0.002
    su = torch.rand(n, generator=gen) * 0.002
    x = torch.randn(2, k, generator=gen).to(torch.bfloat16)
    ws = torch.zeros(qrow_workspace_bytes(torch.device(cuda), n), dtype=torch.uint8, device=cuda)
    y = qrow_swiglu(qg.to(cuda), sg.to(cuda), qu.to(cuda), su.to(cuda), x.to(cuda), workspace=ws)
    ref = oq.swiglu_w8a16(x.float().numpy(), qg.numpy(), sg.numpy(), qu.numpy(), su.numpy())
    assert max_rel_err(y.float().cpu().numpy(), ref) < BF16_TOL


def test_stream_k_workspace_shared_across_widths(cuda):
    """One workspace serves a chain of projections of different widths (the decoder's
    qkv -> o -> down order); every call must equal the same call on a fresh workspace."""
    from mrun_b200.dense_qstore_cuda import qrow_workspace_bytes

    gen = torch.Generator(device="cpu").manual_seed(11)
    shapes = [(1536, 512), (512, 1024), (1024, 512), (512, 1024), (1536, 512)]
    size = max(qrow_workspace_bytes(torch.device(cuda), n) for n, _ in shapes)
    shared = torch.zeros(size, dtype=torch.uint8, device=cuda)
    for n, k in shapes * 2:
        q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8).to(cuda)
        s = (torch.rand(n, generator=gen) * 0.01).to(cuda)
        x = torch.randn(1, k, generator=gen).to(torch.bfloat16).to(cuda)
        fresh = torch.zeros(size, dtype=torch.uint8, device=cuda)
        torch.testing.assert_close(_abi_matmul(x, q, s, shared), _abi_matmul(x, q, s, fresh), rtol=0, atol=0)
