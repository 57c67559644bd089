"""The allocation-free attention entry point against the workspace entry point.

mrb_paged_attention_static exists for callers that cannot allocate device memory (a host
that pre-reserves all GPU memory, a latency-critical path where cudaMalloc could
synchronise, a binding that only holds raw pointers): it keeps its split-K scratch in a
static device array. This test calls both entry points through the C ABI on the same
inputs, twice in a row (the second call checks that the shared scratch is left clean), and
compares them within the bf16 tolerance used by the attention tests. The file sorts last so
a failure here does not hide the rest of the suite.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle.numerics import bf16_round, max_rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _case(rows, hq, hkv, lengths, seed, dev):
    d = 128
    rng = np.random.default_rng(seed)
    total_pages = sum((n + 15) // 16 for n in lengths) + 2
    pk = bf16_round(rng.standard_normal((total_pages, hkv, 16, d)).astype(np.float32))
    pv = bf16_round(rng.standard_normal((total_pages, hkv, 16, d)).astype(np.float32))
    maxp = max((n + 15) // 16 for n in lengths) + 1
    table = np.full((rows, maxp), -1, np.int32)
    perm = rng.permutation(total_pages)
    used = 0
    for r, n in enumerate(lengths):
        need = (n + 15) // 16
        table[r, :need] = perm[used:used + need]
        used += need
    q = bf16_round(rng.standard_normal((rows, hq, d)).astype(np.float32))

    def bf(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(torch.bfloat16)

    return dict(q=bf(q), k=bf(pk), v=bf(pv), table=torch.from_numpy(table).to(dev),
                lens=torch.tensor(lengths, dtype=torch.int32, device=dev), d=d, hq=hq, hkv=hkv,
                np=(q, pk, pv, table))


def _args(c, out, max_total):
    from mrun_b200 import _lib

    d, hq, hkv = c["d"], c["hq"], c["hkv"]
    return [c["q"].data_ptr(), c["q"].shape[0], hq, hkv, d, c["k"].data_ptr(), c["v"].data_ptr(),
            hkv * 16 * d, 16 * d, d, 16, c["table"].data_ptr(), c["table"].stride(0), None, c["lens"].data_ptr(),
            None, None, 1.0 / np.sqrt(d), max_total, out.data_ptr()], _lib


@pytest.mark.parametrize("rows,hq,hkv,lengths,max_total", [
    (1, 28, 4, [700], 1024),          # decode shape: split-K with a cross-split merge
    (3, 32, 4, [17, 256, 1500], 2048),
    (2, 8, 8, [33, 300], 512),
    (4, 8, 4, [100, 1000, 2500, 4000], 4096),  # long contexts: the tensor-core kernel
])
def test_static_scratch_matches_workspace_entry_point(rows, hq, hkv, lengths, max_total, cuda):
    c = _case(rows, hq, hkv, lengths, rows * 7 + hq, cuda)
    from mrun_b200 import _lib

    need = int(_lib.load().mrb_paged_attention_workspace(rows, hq, hkv, c["d"], max_total))
    assert need > 0, "case must exercise the split-K scratch"
    assert need <= int(_lib.load().mrb_paged_attention_static_capacity())
    workspace = torch.zeros(need, dtype=torch.uint8, device=cuda)
    ref = torch.empty_like(c["q"])
    args, lib = _args(c, ref, max_total)
    stream = _lib.stream_handle(cuda)
    _lib.call("mrb_paged_attention", *args, workspace.data_ptr(), need, stream)
    outs = []
    for _ in range(2):  # two calls in a row share the static scratch
        out = torch.empty_like(c["q"])
        args, _ = _args(c, out, max_total)
        _lib.call("mrb_paged_attention_static", *args, stream)
        outs.append(out)
    torch.cuda.synchronize()
    oracle = oatt.paged_gqa_decode(*c["np"][:3], c["np"][3], lengths)
    for out in outs:
        assert max_rel_err(out.float().cpu().numpy(), ref.float().cpu().numpy()) < TOL
        assert max_rel_err(out.float().cpu().numpy(), oracle) < TOL


def test_static_scratch_rejects_oversized_plans(cuda):
    from mrun_b200 import _lib

    cap = int(_lib.load().mrb_paged_attention_static_capacity())
    # 16-way query groups over 8 KV heads and a long context need more scratch than the array
    # in either schedule: 128 (row, head) groups leave no room for a wave of balanced CTAs
    # (one partial slot per CTA and per group), and the fixed splits need several per group
    rows, hq, hkv, max_total = 16, 128, 8, 1 << 20
    need = int(_lib.load().mrb_paged_attention_workspace(rows, hq, hkv, 128, max_total))
    assert need > cap
    # every row maps to one real page and holds one token, so even a launch that the size
    # check failed to stop would stay inside these buffers
    k = torch.zeros(1, hkv, 16, 128, dtype=torch.bfloat16, device=cuda)
    v = torch.zeros_like(k)
    table = torch.zeros(rows, 1, dtype=torch.int32, device=cuda)
    row_len = torch.ones(rows, dtype=torch.int32, device=cuda)
    out = torch.empty(rows, hq, 128, dtype=torch.bfloat16, device=cuda)
    q = torch.zeros(rows, hq, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError, match="bytes of scratch"):
        _lib.call("mrb_paged_attention_static", q.data_ptr(), rows, hq, hkv, 128, k.data_ptr(), v.data_ptr(),
                  hkv * 16 * 128, 16 * 128, 128, 16, table.data_ptr(), 1, None, row_len.data_ptr(), None, None,
                  0.088, max_total,
                  out.data_ptr(), _lib.stream_handle(cuda))


def test_static_scratch_balanced_schedule_under_the_cap(cuda):
    """The routed-MoE decode shape (32 ragged rows, 32/4 heads): the workspace entry point
    plans one wave of balanced CTAs whose partial slots exceed the static array; the static
    entry point plans fewer CTAs to fit and still matches the oracle."""
    from mrun_b200 import _lib

    rng = np.random.default_rng(44)
    rows, hq, hkv = 32, 32, 4
    lengths = rng.integers(256, 4097, rows).tolist()
    max_total = 4096
    c = _case(rows, hq, hkv, lengths, 44, cuda)
    need = int(_lib.load().mrb_paged_attention_workspace(rows, hq, hkv, c["d"], max_total))
    assert need > int(_lib.load().mrb_paged_attention_static_capacity())
    out = torch.empty_like(c["q"])
    args, _ = _args(c, out, max_total)
    _lib.call("mrb_paged_attention_static", *args, _lib.stream_handle(cuda))
    torch.cuda.synchronize()
    oracle = oatt.paged_gqa_decode(*c["np"][:3], c["np"][3], lengths)
    assert max_rel_err(out.float().cpu().numpy(), oracle) < TOL
