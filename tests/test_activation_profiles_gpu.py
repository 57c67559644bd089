"""W8A16 projections with the activation profiles real decoders produce, not only N(0, 1).

RMSNorm outputs are often all of one sign or carry a few outlier channels. The 16-row GEMV
feeds biased codes (q + 1152) through the fp32 mma and removes 1152 * sum(x) after the k sum,
so a row whose sum(x) is large against sum(q * x) is the hard case for its fp32 accumulation;
the tensor-core GEMM (above 16 rows) converts codes exactly. Every path is checked
against the float64 product of the same bf16 activations and codes (norm-wise max relative
error: 4e-3 for bf16 outputs, 1e-4 for fp32 head logits), plus row independence (a row's bits
do not depend on the other rows of its batch) and determinism."""
from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

from oracle import qrow as oq
from oracle.numerics import bf16_round, max_rel_err

pytestmark = pytest.mark.gpu

BF16_OUT_TOL = 4e-3  # one bf16 rounding of an fp32-accumulated exact-product sum
FP32_TOL = 1e-4


def _seed(*parts) -> int:
    return zlib.crc32(repr(parts).encode())


def _activations(kind: str, m: int, k: int, gen: torch.Generator) -> torch.Tensor:
    x = torch.randn(m, k, generator=gen)
    if kind == "positive":      # all of one sign: |N(0,1)| + 1
        x = x.abs() + 1.0
    elif kind == "negative":
        x = -(x.abs() + 0.5)
    elif kind == "outlier":     # one channel 50x the rest, as RMSNorm outputs of real models have
        x[:, k // 3] *= 50.0
    elif kind == "offset":      # mean far from zero with small spread
        x = 4.0 + 0.1 * x
    return x.to(torch.bfloat16)


KINDS = ["normal", "positive", "negative", "outlier", "offset"]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("m,n,k", [(1, 4608, 3584), (16, 2048, 4096), (7, 300, 1024),  # 16-row GEMV
                                   (17, 64, 128), (24, 1000, 1024), (32, 2048, 4096), (32, 5120, 2048),
                                   (20, 333, 80),  # decode batches of 17-32 rows, including a k tail
                                   (64, 512, 3584), (200, 300, 512)])  # tensor-core GEMM
def test_projection_activation_profiles(kind, m, n, k, cuda):
    from mrun_b200.dense_qstore_cuda import qrow_linear

    gen = torch.Generator(device="cpu").manual_seed(_seed(kind, m, n, k))
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    s = torch.rand(n, generator=gen) * 0.01 + 1e-4
    x = _activations(kind, m, k, gen)
    qd, sd, xd = q.to(cuda), s.to(cuda), x.to(cuda)
    y = qrow_linear(qd, sd, xd)
    exact = oq.qrow_matmul_exact(x.float().numpy(), q.numpy(), s.numpy())
    assert max_rel_err(y.float().cpu().numpy(), exact) < BF16_OUT_TOL, kind
    assert torch.equal(y, qrow_linear(qd, sd, xd))  # deterministic
    if 16 < m <= 32:  # rows are independent of the batch they come in (one split plan up to 128 rows)
        extra = _activations(kind, 32 - m + 5, k, gen)[: 32 - m]
        wider = qrow_linear(qd, sd, torch.cat([x, extra]).to(cuda)) if m < 32 else y
        assert torch.equal(wider[:m], y)
        if m > 17:
            assert torch.equal(qrow_linear(qd, sd, xd[:17].contiguous()), y[:17])
    bias = torch.randn(n, generator=gen)
    yb = qrow_linear(qd, sd, xd, bias=bias.to(cuda)).float().cpu().numpy()
    assert max_rel_err(yb, bf16_round(bf16_round(exact) + bf16_round(bias.numpy())[None, :])) < 1e-2


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("m,n,k", [(1, 18944, 3584), (9, 700, 1024), (32, 768, 2048), (20, 333, 80), (64, 256, 512)])
def test_swiglu_activation_profiles(kind, m, n, k, cuda):
    from mrun_b200.dense_qstore_cuda import qrow_swiglu

    gen = torch.Generator(device="cpu").manual_seed(_seed(kind, m, n, k, "s"))
    gq = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    uq = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    gs = torch.rand(n, generator=gen) * 0.002
    us = torch.rand(n, generator=gen) * 0.002
    x = _activations(kind, m, k, gen)
    y = qrow_swiglu(gq.to(cuda), gs.to(cuda), uq.to(cuda), us.to(cuda), x.to(cuda)).float().cpu().numpy()
    # the SwiGLU boundaries (bf16 g and u, bf16 silu(g), bf16 product) over the exact
    # projections; the reference's contract also rounds each weight to bf16 first, which with
    # same-sign activations adds up coherently (about 1.5 % here) -- the kernels multiply the
    # exact codes and apply the row scale once
    xf = x.float().numpy()
    g = bf16_round(oq.qrow_matmul_exact(xf, gq.numpy(), gs.numpy()))
    u = bf16_round(oq.qrow_matmul_exact(xf, uq.numpy(), us.numpy()))
    ref = bf16_round(bf16_round(g * oq.sigmoid_f32(g)) * u)
    assert max_rel_err(y, ref) < 1e-2, kind
    contract = oq.swiglu_w8a16(xf, gq.numpy(), gs.numpy(), uq.numpy(), us.numpy())
    assert max_rel_err(y, contract) < 3e-2, kind


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("m", [1, 12, 32, 48])
def test_greedy_head_activation_profiles(kind, m, cuda):
    """The fused argmax head (GEMV up to 16 rows, tensor-core GEMM above): fp32 logits within
    1e-4 of the float64 product; a pick may differ from the float64 argmax only where the top
    two are within that error."""
    from mrun_b200.dense_qstore_cuda import qrow_argmax

    n, k = 32000, 1024
    gen = torch.Generator(device="cpu").manual_seed(_seed(kind, m, "head"))
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
    s = torch.rand(n, generator=gen) * 1e-3 + 1e-4
    x = _activations(kind, m, k, gen)
    idx, val, logits = qrow_argmax(q.to(cuda), s.to(cuda), x.to(cuda))
    exact = oq.qrow_matmul_exact(x.float().numpy(), q.numpy(), s.numpy())
    got = logits.cpu().numpy()
    assert max_rel_err(got, exact) < FP32_TOL, kind
    picks = idx.cpu().numpy()
    best = exact.argmax(axis=1)
    for r in range(m):
        if picks[r] != best[r]:
            assert exact[r, best[r]] - exact[r, picks[r]] <= FP32_TOL * np.abs(exact[r]).max(), (kind, r)
