"""W8A8 parity: int32 accumulators and activation codes bit-exact, outputs bit-identical to
the reference (no protected columns) and within 1e-4 (fp32) with protected columns."""
from __future__ import annotations

import ctypes
import hashlib

import numpy as np
import pytest
import torch

from oracle import qrow as oq
from oracle import w8a8 as ow8
from oracle.numerics import bf16_round, max_rel_err

pytestmark = pytest.mark.gpu


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_config1_w8a8_bit_exact(golden, cuda):
    from mrun_b200.qstore_build import quant_row_int8
    from mrun_b200.w8a8 import quantize_activations, w8a8_matmul

    g = golden("config1")
    torch.manual_seed(0)
    x = torch.randn(8, 2048)
    w = torch.randn(2048, 2048) * 0.02
    q, s = quant_row_int8(w.to(cuda))
    qx, scale = quantize_activations(x.to(cuda))
    np.testing.assert_array_equal(qx.cpu().numpy(), g["qx"])
    np.testing.assert_array_equal(scale.cpu().numpy(), g["act_scale"])
    acc = torch.empty(8, 2048, dtype=torch.int32, device=cuda)
    y = w8a8_matmul(q, s, x.to(cuda), acc_out=acc)
    assert _sha(acc.cpu().numpy()) == str(g["acc_sha"])
    np.testing.assert_array_equal(y.cpu().numpy(), g["y_w8a8"])


def test_reference_w8a8_fixture(golden, cuda):
    from mrun_b200.w8a8 import _int8_gemm, w8a8_matmul

    g = golden("w8a8")
    qw = torch.from_numpy(g["q_w"]).to(cuda)
    sw = torch.from_numpy(g["sc_w"]).to(cuda)
    x = torch.from_numpy(g["x"]).to(cuda)
    np.testing.assert_array_equal(w8a8_matmul(qw, sw, x, protect_k=0).cpu().numpy(), g["y_k0"])
    y4 = w8a8_matmul(qw, sw, x, protect_k=4).cpu().numpy()
    assert max_rel_err(y4, g["y_k4"]) < 1e-4
    np.testing.assert_array_equal(_int8_gemm(torch.from_numpy(g["gemm_qx"]).to(cuda), qw).cpu().numpy(), g["gemm_acc"])


@pytest.mark.parametrize("m", [1, 5, 16, 17, 64, 300])
@pytest.mark.parametrize("n,k", [(512, 3584), (4608, 3584), (3584, 18944)])
def test_w8a8_gemv_and_gemm_bit_exact(m, n, k, cuda):
    from mrun_b200.w8a8 import w8a8_matmul

    if m == 300 and k == 18944:
        pytest.skip("oracle int64 matmul too slow at this size")
    gen = torch.Generator().manual_seed(m + n + k)
    qw = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    sw = torch.rand(n, generator=gen) * 0.01
    x = torch.randn(m, k, generator=gen).to(torch.bfloat16)
    acc = torch.empty(m, n, dtype=torch.int32, device=cuda)
    y = w8a8_matmul(qw.to(cuda), sw.to(cuda), x.to(cuda), acc_out=acc).cpu().numpy()
    xf = x.float().numpy()
    qx, act = ow8.quantize_activations(xf)
    ref_acc = ow8.int8_gemm(qx, qw.numpy())
    np.testing.assert_array_equal(acc.cpu().numpy(), ref_acc)
    np.testing.assert_array_equal(y, ow8.w8a8_matmul(qw.numpy(), sw.numpy(), xf))


def test_protect_topk_matches_oracle(cuda):
    from mrun_b200.w8a8 import w8a8_matmul

    gen = torch.Generator().manual_seed(9)
    qw = torch.randint(-127, 128, (128, 256), generator=gen, dtype=torch.int8)
    sw = torch.rand(128, generator=gen) * 0.02 + 1e-3
    x = torch.randn(8, 256, generator=gen)
    x[:, torch.randperm(256, generator=gen)[:4]] *= 300.0
    y = w8a8_matmul(qw.to(cuda), sw.to(cuda), x.to(cuda), protect_k=8).cpu().numpy()
    ref = ow8.w8a8_matmul(qw.numpy(), sw.numpy(), x.numpy(), protect_k=8)
    assert max_rel_err(y, ref) < 1e-5
    exact = x.numpy().astype(np.float64) @ (qw.numpy().astype(np.float64) * sw.numpy()[:, None]).T
    assert np.array_equal(y.argmax(-1), exact.argmax(-1))


@pytest.mark.parametrize("m,n,k", [
    (1, 256, 64),        # single row, one tile, k inside one 128-byte stage
    (17, 300, 160),      # ragged m, n and k (zero-filled tile edges)
    (128, 256, 128),     # exactly one tile and one stage
    (200, 700, 1040),
    (512, 3584, 3584),   # config-2 prefill o projection (128 x 128 tiles)
    (2048, 4096, 256),   # 128 x 256 tiles, double-buffered accumulators
    (4100, 8200, 272),   # 256 x 256 tiles (two halves), ragged last tile with an empty half
])
def test_tensor_core_int8_gemm_exact(m, n, k, cuda):
    """The tcgen05 int8 GEMM (TMA + TMEM accumulators) equals exact integer matmul."""
    from mrun_b200.w8a8 import _int8_gemm

    gen = torch.Generator(device="cpu").manual_seed(m * 7 + n + k)
    qx = torch.randint(-127, 128, (m, k), generator=gen, dtype=torch.int8)
    qw = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    acc = _int8_gemm(qx.to(cuda), qw.to(cuda)).cpu().numpy()
    # float64 products and sums are exact here (|acc| <= 127^2 k < 2^53)
    exact = qx.numpy().astype(np.float64) @ qw.numpy().astype(np.float64).T
    np.testing.assert_array_equal(acc.astype(np.float64), exact)


def test_tensor_core_waits_never_timed_out(cuda):
    import ctypes

    from mrun_b200 import _lib

    count = ctypes.c_uint(99)
    _lib.call("mrb_tc_status", ctypes.addressof(count))
    assert count.value == 0


@pytest.mark.parametrize("m,n,k,paired,with_bias", [
    (64, 3584, 3584, False, False),    # o projection at 64 decode rows: k split over a cluster
    (64, 4608, 3584, False, True),     # qkv with bias, split
    (64, 3584, 18944, False, False),   # down projection, split
    (64, 18944, 3584, True, False),    # paired gate/up, 296 tiles: no split
    (64, 1000, 1024, True, False),     # paired, split, ragged output columns
    (100, 1000, 512, False, True),     # split with a ragged row tile
    (300, 1000, 512, False, True),     # several row tiles
    (1, 256, 128, False, False),
])
def test_w8a8_linear_bf16_exact_and_split_invariant(m, n, k, paired, with_bias, cuda):
    """bf16 W8A8 projection: int32 accumulation is exact, so rows computed in a skinny batch
    (k split over a cluster) equal the same rows computed inside a tall batch (no split) bit
    for bit, and the plain epilogue equals the oracle's fp32 rescale rounded once to bf16."""
    from mrun_b200.w8a8 import w8a8_linear_bf16

    gen = torch.Generator(device="cpu").manual_seed(m + n + k)
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    s = torch.rand(n, generator=gen) * 1e-3 + 1e-5
    qu = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    su = torch.rand(n, generator=gen) * 1e-3 + 1e-5
    tall = 2048  # enough 128-row tiles that nothing splits
    x_all = torch.randn(tall, k, generator=gen).to(torch.bfloat16)
    x = x_all[:m].contiguous()
    bias = torch.randn(n, generator=gen) * 0.1 if with_bias else None
    dev = lambda t: None if t is None else t.to(cuda)  # noqa: E731
    up = (dev(qu), dev(su)) if paired else None
    y = w8a8_linear_bf16(dev(q), dev(s), dev(x), bias=dev(bias), up=up)
    y_again = w8a8_linear_bf16(dev(q), dev(s), dev(x), bias=dev(bias), up=up)
    y_tall = w8a8_linear_bf16(dev(q), dev(s), dev(x_all), bias=dev(bias), up=up)
    assert torch.equal(y, y_again) and torch.equal(y, y_tall[:m])

    qx, sx = ow8.quantize_activations(x.float().numpy())
    acc = ow8.int8_gemm(qx, q.numpy())
    g = (acc.astype(np.float32) * sx).astype(np.float32) * s.numpy()[None, :]
    if paired:
        u = (ow8.int8_gemm(qx, qu.numpy()).astype(np.float32) * sx).astype(np.float32) * su.numpy()[None, :]
        gv, uv = bf16_round(g), bf16_round(u)
        ref = bf16_round(bf16_round(gv * oq.sigmoid_f32(gv)) * uv)
        assert max_rel_err(y.float().cpu().numpy(), ref) < 1e-2
    else:
        if bias is not None:
            g = (g + bias.numpy()[None, :]).astype(np.float32)
        np.testing.assert_array_equal(y.float().cpu().numpy(), bf16_round(g))
    out = ctypes.c_uint(0)
    from mrun_b200 import _lib

    _lib.call("mrb_tc_status", ctypes.addressof(out))
    assert out.value == 0


@pytest.mark.parametrize("m,k", [(64, 3584), (3, 18944), (5, 20480), (2, 20496), (7, 40)])
def test_bf16_activation_quantiser_bit_exact(m, k, cuda):
    """bf16 rows (the vector path up to 20480 columns, the generic one beyond): codes and
    scales bit-identical to the oracle quantiser."""
    from mrun_b200.w8a8 import quantize_activations

    gen = torch.Generator(device="cpu").manual_seed(m * k)
    x = (torch.randn(m, k, generator=gen) * 3).to(torch.bfloat16)
    x[0, 5] = 0.0
    if m > 2:
        x[2] = 0.0  # an all-zero row takes scale 1
    qx, sx = quantize_activations(x.to(cuda))
    rq, rs = ow8.quantize_activations(x.float().numpy())
    np.testing.assert_array_equal(qx.cpu().numpy(), rq)
    np.testing.assert_array_equal(sx.cpu().numpy().reshape(-1), rs.reshape(-1))
