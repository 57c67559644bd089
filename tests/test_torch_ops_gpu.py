"""torch.ops.mrun_b200.* (the PyTorch operator library over the C ABI) against the same entry
points called through ctypes: bit-identical outputs, the current stream honoured, and the
operators captured and replayed in a CUDA graph."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand(*shape, gen, dtype=torch.bfloat16, device="cuda"):
    return torch.randn(*shape, generator=gen, device=device).to(dtype)


def test_qrow_ops_match_the_c_abi(cuda):
    from mrun_b200 import _lib

    gen = torch.Generator(device=cuda).manual_seed(11)
    for m, k, n in ((1, 2048, 4096), (24, 1024, 768), (96, 512, 1536)):
        codes = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=cuda, generator=gen)
        scales = torch.rand(n, device=cuda, generator=gen) * 1e-2
        x = _rand(m, k, gen=gen)
        y_ops = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        _lib.ops().qrow_linear(x, codes, scales, None, y_ops, None)
        y_abi = torch.empty_like(y_ops)
        _lib.call("mrb_qrow_matmul", x.data_ptr(), _lib.MRB_BF16, m, k, codes.data_ptr(), scales.data_ptr(), n, None,
                  y_abi.data_ptr(), _lib.MRB_BF16, None, 0, _lib.stream_handle(cuda))
        assert torch.equal(y_ops, y_abi)
        s_ops = torch.empty_like(y_ops)
        _lib.ops().qrow_swiglu(x, codes, scales, codes, scales, s_ops, None)
        s_abi = torch.empty_like(y_ops)
        _lib.call("mrb_qrow_swiglu", x.data_ptr(), m, k, codes.data_ptr(), scales.data_ptr(), codes.data_ptr(),
                  scales.data_ptr(), n, s_abi.data_ptr(), None, 0, _lib.stream_handle(cuda))
        assert torch.equal(s_ops, s_abi)
    w = torch.randn(64, 256, device=cuda, generator=gen)
    q, s = torch.empty(64, 256, dtype=torch.int8, device=cuda), torch.empty(64, device=cuda)
    _lib.ops().quant_row_int8(w, q, s)
    q2, s2 = torch.empty_like(q), torch.empty_like(s)
    _lib.call("mrb_quant_row_int8", w.data_ptr(), 64, 256, q2.data_ptr(), s2.data_ptr(), _lib.stream_handle(cuda))
    assert torch.equal(q, q2) and torch.equal(s, s2)


def test_moe_ops_match_the_c_abi(cuda):
    from mrun_b200 import _lib
    from mrun_b200.moe import ExpertPageLayout, expert_mlp_sync

    gen = torch.Generator(device=cuda).manual_seed(5)
    t, e, k, h, f = 40, 16, 4, 512, 256
    logits = torch.randn(t, e, device=cuda, generator=gen)
    idx, w32, w16 = (torch.empty(t, k, dtype=d, device=cuda) for d in (torch.int64, torch.float32, torch.bfloat16))
    _lib.ops().router_topk(logits, k, True, idx, w32, w16)
    idx2, w32b, w16b = (torch.empty_like(v) for v in (idx, w32, w16))
    _lib.call("mrb_router_topk", logits.data_ptr(), _lib.MRB_F32, t, e, k, 1, idx2.data_ptr(), w32b.data_ptr(),
              w16b.data_ptr(), _lib.stream_handle(cuda))
    assert torch.equal(idx, idx2) and torch.equal(w32, w32b) and torch.equal(w16, w16b)
    a = t * k
    coef_in = w16.float().reshape(-1).contiguous()
    plan = [torch.empty(e, dtype=torch.int32, device=cuda), torch.empty(e, dtype=torch.int32, device=cuda),
            torch.empty(a, dtype=torch.int64, device=cuda), torch.empty(a, device=cuda),
            torch.empty(a, dtype=torch.int64, device=cuda)]
    _lib.ops().route_compile(idx, coef_in, e, *plan)
    plan2 = [torch.empty_like(v) for v in plan]
    _lib.call("mrb_route_compile", idx.data_ptr(), coef_in.data_ptr(), t, k, e, *(v.data_ptr() for v in plan2), None,
              _lib.stream_handle(cuda))
    assert all(torch.equal(u, v) for u, v in zip(plan, plan2))
    counts, starts, token_ids, coef, inverse = plan
    ly = ExpertPageLayout.create(h, f)
    pages = torch.randint(0, 256, (e, ly.page_stride), dtype=torch.uint8, device=cuda, generator=gen)
    for off, nbytes in ((ly.gate_up_scales_offset, ly.gate_up_scales_bytes), (ly.down_scales_offset, ly.down_scales_bytes)):
        pages[:, off:off + nbytes] = torch.full((e, nbytes // 4), 1e-3, device=cuda).view(torch.uint8)
    x = _rand(t, h, gen=gen)
    act, y = torch.empty(a, f, dtype=torch.bfloat16, device=cuda), torch.empty(a, h, dtype=torch.bfloat16, device=cuda)
    sync = expert_mlp_sync(e, cuda)
    _lib.ops().grouped_expert_mlp(x, token_ids, starts, counts, pages, ly.page_stride, ly.gate_up_codes_offset,
                                  ly.gate_up_scales_offset, ly.down_codes_offset, ly.down_scales_offset, None, act, y,
                                  sync)
    act2, y2 = torch.empty_like(act), torch.empty_like(y)
    _lib.call("mrb_grouped_expert_mlp", x.data_ptr(), token_ids.data_ptr(), starts.data_ptr(), counts.data_ptr(), e,
              pages.data_ptr(), ly.page_stride, ly.gate_up_codes_offset, ly.gate_up_scales_offset,
              ly.down_codes_offset, ly.down_scales_offset, None, h, f, a, act2.data_ptr(), y2.data_ptr(),
              sync.data_ptr(), _lib.stream_handle(cuda))
    assert torch.equal(y, y2) and torch.equal(act, act2) and not sync.any()
    out, out16 = torch.empty(t, h, device=cuda), torch.empty(t, h, dtype=torch.bfloat16, device=cuda)
    _lib.ops().stable_route_reduce(y, coef, inverse, t, k, out, out16)
    out2 = torch.empty_like(out)
    _lib.call("mrb_stable_route_reduce", y.data_ptr(), coef.data_ptr(), inverse.data_ptr(), t, k, h, out2.data_ptr(),
              None, _lib.stream_handle(cuda))
    assert torch.equal(out, out2) and torch.equal(out16, out2.to(torch.bfloat16))


def test_ops_follow_the_current_stream_and_capture_in_a_graph(cuda):
    from mrun_b200 import _lib

    gen = torch.Generator(device=cuda).manual_seed(2)
    codes = torch.randint(-127, 128, (2048, 1024), dtype=torch.int8, device=cuda, generator=gen)
    scales = torch.rand(2048, device=cuda, generator=gen) * 1e-2
    x = _rand(4, 1024, gen=gen)
    ref = torch.empty(4, 2048, dtype=torch.bfloat16, device=cuda)
    _lib.ops().qrow_linear(x, codes, scales, None, ref, None)
    side = torch.cuda.Stream(cuda)
    side.wait_stream(torch.cuda.current_stream(cuda))
    y = torch.zeros_like(ref)
    with torch.cuda.stream(side):
        _lib.ops().qrow_linear(x, codes, scales, None, y, None)
    torch.cuda.current_stream(cuda).wait_stream(side)
    torch.cuda.synchronize(cuda)
    assert torch.equal(y, ref)
    graph = torch.cuda.CUDAGraph()
    g_out = torch.zeros_like(ref)
    with torch.cuda.graph(graph, stream=side):
        _lib.ops().qrow_linear(x, codes, scales, None, g_out, None)
    graph.replay()
    torch.cuda.synchronize(cuda)
    assert torch.equal(g_out, ref)
    with pytest.raises(ValueError, match="contiguous"):
        _lib.ops().qrow_linear(x, codes.t(), scales, None, ref, None)
