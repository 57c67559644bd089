"""Parity of the B200 paged decode attention and RoPE/KV-append kernels against the CPU
oracle and the reference's golden vectors. bf16 outputs: max relative error 1e-2
(norm-wise); page gathers and KV appends are bit-exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle.numerics import bf16_round, max_rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _bf(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)


def test_segmented_decode_attention_golden(golden, cuda):
    from mrun_b200.segmented_gqa_decode import segmented_decode_attention

    g = golden("attention")
    out, impl = segmented_decode_attention(
        _bf(g["seg_q"], cuda), _bf(g["seg_ck"], cuda), _bf(g["seg_cv"], cuda), _bf(g["seg_kn"], cuda),
        _bf(g["seg_vn"], cuda), torch.from_numpy(g["seg_len"]).to(cuda),
    )
    assert impl.startswith("b200-")
    assert max_rel_err(out.float().cpu().numpy(), g["seg_out"]) < TOL


def test_segmented_gqa_decode_golden(golden, cuda):
    from mrun_b200.segmented_gqa_decode import segmented_gqa_decode

    g = golden("attention")
    out = segmented_gqa_decode(
        _bf(g["gqa_q"], cuda), _bf(g["gqa_kc"], cuda), _bf(g["gqa_vc"], cuda),
        torch.from_numpy(g["gqa_slots"]).to(cuda), torch.from_numpy(g["gqa_len"]).to(cuda),
        max_sequence_length=48,
    )
    assert max_rel_err(out.float().cpu().numpy(), g["gqa_out"]) < TOL


def _random_paged(rng, rows, hkv, d, lengths, num_pages):
    pages_k = bf16_round(rng.standard_normal((num_pages, hkv, 16, d)).astype(np.float32))
    pages_v = bf16_round(rng.standard_normal((num_pages, hkv, 16, d)).astype(np.float32))
    maxp = max((n + 15) // 16 for n in lengths)
    perm = rng.permutation(num_pages)
    table = np.full((rows, maxp + 2), -1, np.int32)
    used = 0
    for r, n in enumerate(lengths):
        need = (n + 15) // 16
        table[r, :need] = perm[used:used + need]
        used += need
    return pages_k, pages_v, table


@pytest.mark.parametrize("rows,hq,hkv,lengths", [
    (1, 28, 4, [768]),
    (1, 28, 4, [1]),
    (3, 32, 4, [17, 256, 4096]),
    (4, 8, 8, [16, 15, 33, 100]),
    (2, 32, 8, [1024, 2047]),
    # (row, head) groups x context tiles >= 4096: the tensor-core kernel, ragged lengths,
    # query groups of 8 and 7
    (8, 32, 4, [1, 300, 777, 1024, 1500, 1999, 2048, 64]),
    (6, 28, 4, [4000, 3333, 2500, 17, 1024, 3100]),
    # tensor-core kernel with a 16-head group (both 8-row halves of the mma tile in use)
    (4, 64, 4, [3000, 100, 2048, 4096]),
])
def test_paged_attention_vs_oracle(rows, hq, hkv, lengths, cuda):
    from mrun_b200.segmented_gqa_decode import paged_attention

    rng = np.random.default_rng(rows * 100 + hq)
    d = 128
    total_pages = sum((n + 15) // 16 for n in lengths) + 3
    pk, pv, table = _random_paged(rng, rows, hkv, d, lengths, total_pages)
    q = bf16_round(rng.standard_normal((rows, hq, d)).astype(np.float32))
    out = paged_attention(
        _bf(q, cuda), _bf(pk, cuda), _bf(pv, cuda), strides=(hkv * 16 * d, 16 * d, d), page_size=16,
        block_table=torch.from_numpy(table).to(cuda), row_len=torch.tensor(lengths, dtype=torch.int32, device=cuda),
        max_total_tokens=max(lengths),
    )
    ref = oatt.paged_gqa_decode(q, pk, pv, table, lengths)
    assert max_rel_err(out.float().cpu().numpy(), ref) < TOL
    # deterministic: same inputs give identical bits
    out2 = paged_attention(
        _bf(q, cuda), _bf(pk, cuda), _bf(pv, cuda), strides=(hkv * 16 * d, 16 * d, d), page_size=16,
        block_table=torch.from_numpy(table).to(cuda), row_len=torch.tensor(lengths, dtype=torch.int32, device=cuda),
        max_total_tokens=max(lengths),
    )
    assert torch.equal(out, out2)


def test_rope_kv_append_bit_exact_and_gather(cuda):
    from mrun_b200.paged_kv import PagedKVCache

    rng = np.random.default_rng(7)
    hq, hkv, d, tokens = 28, 4, 128, 40
    cache = PagedKVCache(num_layers=2, num_pages=16, kv_heads=hkv, head_dim=d, max_seqs=2, max_pages_per_seq=8,
                         device=cuda)
    cache.reserve(1, tokens)
    positions = np.arange(tokens, dtype=np.int32)
    cos, sin = oatt.rope_tables(d, 1e6, np.arange(256))
    qkv = bf16_round(rng.standard_normal((tokens, (hq + 2 * hkv) * d)).astype(np.float32))
    qkv_dev = _bf(qkv, cuda)
    q_out = torch.empty(tokens, hq, d, dtype=torch.bfloat16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    cache.append(
        1, qkv_dev[:, hq * d:], qkv_dev[:, (hq + hkv) * d:], torch.from_numpy(positions).to(cuda),
        torch.ones(tokens, dtype=torch.int32, device=cuda), q_rows=qkv_dev, q_out=q_out,
        rope=(torch.from_numpy(cos[:, : d // 2].copy()).to(cuda), torch.from_numpy(sin[:, : d // 2].copy()).to(cuda)), in_row_stride=(hq + 2 * hkv) * d,
        num_heads=hq, error_flag=err,
    )
    assert int(err.item()) == 0
    c, s = cos[positions], sin[positions]
    q_ref = oatt.rope(qkv[:, : hq * d].reshape(tokens, hq, d), c, s)
    k_ref = oatt.rope(qkv[:, hq * d:(hq + hkv) * d].reshape(tokens, hkv, d), c, s)
    v_ref = qkv[:, (hq + hkv) * d:].reshape(tokens, hkv, d)
    np.testing.assert_array_equal(q_out.float().cpu().numpy(), q_ref)
    table = cache.pages_of(1)
    k_pages = cache.k[1].float().cpu().numpy()
    v_pages = cache.v[1].float().cpu().numpy()
    np.testing.assert_array_equal(oatt.paged_gather(k_pages, table, tokens), k_ref)
    np.testing.assert_array_equal(oatt.paged_gather(v_pages, table, tokens), v_ref)
    # out-of-range position sets the error flag and writes nothing
    cache.append(0, qkv_dev[:1, hq * d:], qkv_dev[:1, (hq + hkv) * d:], torch.tensor([999], dtype=torch.int32, device=cuda),
                 torch.zeros(1, dtype=torch.int32, device=cuda), in_row_stride=(hq + 2 * hkv) * d, error_flag=err)
    assert int(err.item()) == 1


def test_scatter_segmented_decode_kv(cuda):
    from mrun_b200.segmented_gqa_decode import scatter_segmented_decode_kv

    rng = np.random.default_rng(3)
    kc = torch.zeros(4, 2, 32, 64, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    k = _bf(rng.standard_normal((3, 2, 64)), cuda)
    v = _bf(rng.standard_normal((3, 2, 64)), cuda)
    slots = torch.tensor([2, 0, 3], device=cuda)
    parents = torch.tensor([0, 5, 31], device=cuda)
    scatter_segmented_decode_kv(k, v, kc, vc, slots, parents)
    for row, (slot, pos) in enumerate([(2, 0), (0, 5), (3, 31)]):
        assert torch.equal(kc[slot, :, pos], k[row])
        assert torch.equal(vc[slot, :, pos], v[row])
    assert int((kc != 0).any(dim=-1).sum()) == 6


def _qk_rms(x, w, eps):
    from oracle.moe_decoder import _rms

    return _rms(x, w, eps)


@pytest.mark.parametrize("rows,hq,hkv,d,positions,max_total,use_rope,qk_norm", [
    (1, 28, 4, 128, [520], 960, True, False),        # config-2 shape: 16-CTA clusters
    (1, 28, 4, 128, [0], 16, True, False),           # first token: one CTA, no cluster
    (3, 32, 4, 128, [15, 16, 255], 300, True, True),  # page edges, Qwen3 q/k norm
    (2, 8, 8, 64, [31, 100], 128, True, False),      # head_dim 64, group 1
    (8, 28, 4, 128, [1, 17, 300, 511, 64, 5, 1000, 47], 1024, True, False),  # 9-CTA clusters, ragged
    (1, 64, 4, 128, [3000], 4096, True, False),      # 16-head group
    (2, 28, 4, 128, [40, 7], 64, False, False),      # no rotation (plain append)
])
def test_rope_append_attention_vs_separate_and_oracle(rows, hq, hkv, d, positions, max_total, use_rope, qk_norm,
                                                      cuda):
    from mrun_b200.paged_kv import PagedKVCache
    from mrun_b200.segmented_gqa_decode import rope_append_attention_cluster

    rng = np.random.default_rng(sum(positions) + hq)
    seqs = list(range(rows))[::-1]  # row r continues sequence rows-1-r
    pages_per_seq = (max_total + 15) // 16
    cache = PagedKVCache(num_layers=1, num_pages=rows * pages_per_seq + 2, kv_heads=hkv, head_dim=d,
                         max_seqs=rows, max_pages_per_seq=pages_per_seq, device=cuda)
    for r, p in enumerate(positions):
        cache.reserve(seqs[r], p + 1)
    # the cached prefix: random bf16 K/V in every mapped page
    cache.k.copy_(_bf(rng.standard_normal(tuple(cache.k.shape)), cuda))
    cache.v.copy_(_bf(rng.standard_normal(tuple(cache.v.shape)), cuda))
    width = (hq + 2 * hkv) * d
    qkv = bf16_round(rng.standard_normal((rows, width)).astype(np.float32))
    qkv_dev = _bf(qkv, cuda)
    pos_dev = torch.tensor(positions, dtype=torch.int32, device=cuda)
    seq_dev = torch.tensor(seqs, dtype=torch.int32, device=cuda)
    cos, sin = oatt.rope_tables(d, 1e6, np.arange(max_total))
    rope = (torch.from_numpy(cos[:, : d // 2].copy()).to(cuda), torch.from_numpy(sin[:, : d // 2].copy()).to(cuda)) \
        if use_rope else None
    norms = None
    if qk_norm:
        qw = bf16_round(1.0 + 0.1 * rng.standard_normal(d).astype(np.float32))
        kw = bf16_round(1.0 + 0.1 * rng.standard_normal(d).astype(np.float32))
        norms = (_bf(qw, cuda), _bf(kw, cuda))
    k0, v0 = cache.k.clone(), cache.v.clone()

    # separate launches: rope_kv_append + paged_attention
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    q_rot = torch.empty(rows, hq, d, dtype=torch.bfloat16, device=cuda)
    cache.append(0, qkv_dev[:, hq * d:], qkv_dev[:, (hq + hkv) * d:], pos_dev, seq_dev, q_rows=qkv_dev, q_out=q_rot,
                 rope=rope, in_row_stride=width, num_heads=hq, error_flag=err, qk_norm=norms)
    sep = cache.attend(0, q_rot, pos_dev + 1, max_total_tokens=max_total, row_seq=seq_dev)
    k_sep, v_sep = cache.k.clone(), cache.v.clone()
    # fused launch on the original cache
    cache.k.copy_(k0)
    cache.v.copy_(v0)
    fused = cache.append_attend(0, qkv_dev, qkv_dev[:, hq * d:], qkv_dev[:, (hq + hkv) * d:], pos_dev, seq_dev,
                                num_heads=hq, max_total_tokens=max_total, in_row_stride=width, rope=rope,
                                qk_norm=norms, error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert rope_append_attention_cluster(rows, hq, hkv, d, max_total) >= 1
    # the append is bit-exact with the separate kernel
    assert torch.equal(cache.k, k_sep) and torch.equal(cache.v, v_sep)
    # attention against the oracle over the gathered cache (the new token included)
    k_pages = cache.k[0].float().cpu().numpy()
    v_pages = cache.v[0].float().cpu().numpy()
    q = qkv[:, : hq * d].reshape(rows, hq, d)
    k_new = qkv[:, hq * d:(hq + hkv) * d].reshape(rows, hkv, d)
    if qk_norm:
        q = _qk_rms(q, qw, 1e-6)
        k_new = _qk_rms(k_new, kw, 1e-6)
    if use_rope:
        q = np.stack([oatt.rope(q[r:r + 1], cos[p:p + 1], sin[p:p + 1])[0] for r, p in enumerate(positions)])
        k_new = np.stack([oatt.rope(k_new[r:r + 1], cos[p:p + 1], sin[p:p + 1])[0] for r, p in enumerate(positions)])
    keys = [oatt.paged_gather(k_pages, cache.pages_of(seqs[r]), p + 1) for r, p in enumerate(positions)]
    vals = [oatt.paged_gather(v_pages, cache.pages_of(seqs[r]), p + 1) for r, p in enumerate(positions)]
    for r, p in enumerate(positions):
        if qk_norm:  # fp32 rsqrt in the kernel vs float64 here: equal up to bf16 rounding ties
            assert max_rel_err(keys[r][p], k_new[r]) < TOL
        else:
            np.testing.assert_array_equal(keys[r][p], k_new[r])
        np.testing.assert_array_equal(vals[r][p], qkv[r, (hq + hkv) * d:].reshape(hkv, d))
    ref = bf16_round(oatt.gqa_decode_rows(q, keys, vals))
    assert max_rel_err(fused.float().cpu().numpy(), ref) < TOL
    assert max_rel_err(fused.float().cpu().numpy(), sep.float().cpu().numpy()) < TOL
    # deterministic: a second run on the same inputs gives identical bits, also when the step
    # state is read before the dependency wait (state_ready: nothing in flight writes it)
    cache.k.copy_(k0)
    cache.v.copy_(v0)
    torch.cuda.synchronize()
    again = cache.append_attend(0, qkv_dev, qkv_dev[:, hq * d:], qkv_dev[:, (hq + hkv) * d:], pos_dev, seq_dev,
                                num_heads=hq, max_total_tokens=max_total, in_row_stride=width, rope=rope,
                                qk_norm=norms, error_flag=err, state_ready=True)
    assert torch.equal(again, fused)
    assert torch.equal(cache.k, k_sep) and torch.equal(cache.v, v_sep)


def test_rope_append_attention_bad_position_flags_and_zeroes(cuda):
    from mrun_b200.paged_kv import PagedKVCache

    rng = np.random.default_rng(11)
    hq, hkv, d = 8, 2, 128
    cache = PagedKVCache(num_layers=1, num_pages=8, kv_heads=hkv, head_dim=d, max_seqs=2, max_pages_per_seq=4,
                         device=cuda)
    cache.reserve(0, 20)
    cache.reserve(1, 20)
    width = (hq + 2 * hkv) * d
    qkv = _bf(rng.standard_normal((2, width)), cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    # row 1's position lies on an unmapped page (the table row maps 2 pages = 32 tokens)
    pos = torch.tensor([19, 40], dtype=torch.int32, device=cuda)
    out = cache.append_attend(0, qkv, qkv[:, hq * d:], qkv[:, (hq + hkv) * d:], pos,
                              torch.tensor([0, 1], dtype=torch.int32, device=cuda), num_heads=hq,
                              max_total_tokens=64, in_row_stride=width, error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    assert not bool(out[1].any())
    assert bool(out[0].any())
    assert bool(torch.isfinite(out[0].float()).all())


@pytest.mark.parametrize("n,start,hq,hkv", [(512, 0, 28, 4), (37, 0, 32, 4), (100, 250, 28, 4), (1, 77, 8, 8),
                                            (64, 16, 64, 4), (200, 3, 16, 2)])
def test_paged_prefill_attention_vs_oracle(n, start, hq, hkv, cuda):
    """Causal prefill attention (query blocks of 16 tokens, the whole K/V prefix per block)
    against the oracle's per-token attention over the gathered pages; deterministic."""
    from mrun_b200.paged_kv import PagedKVCache

    rng = np.random.default_rng(n + start + hq)
    d = 128
    total = start + n
    cache = PagedKVCache(num_layers=1, num_pages=(total + 15) // 16 + 5, kv_heads=hkv, head_dim=d, max_seqs=2,
                         max_pages_per_seq=(total + 15) // 16 + 1, device=cuda)
    cache.reserve(0, 5)  # another sequence's pages first, so the block table is not the identity
    cache.reserve(1, total)
    cache.k.copy_(_bf(rng.standard_normal(tuple(cache.k.shape)), cuda))
    cache.v.copy_(_bf(rng.standard_normal(tuple(cache.v.shape)), cuda))
    q = bf16_round(rng.standard_normal((n, hq, d)).astype(np.float32))
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = cache.attend_prefill(0, _bf(q, cuda), 1, start, error_flag=err)
    again = cache.attend_prefill(0, _bf(q, cuda), 1, start)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out, again)
    pages = cache.pages_of(1)
    kp, vp = cache.k[0].float().cpu().numpy(), cache.v[0].float().cpu().numpy()
    keys = [oatt.paged_gather(kp, pages, start + i + 1) for i in range(n)]
    vals = [oatt.paged_gather(vp, pages, start + i + 1) for i in range(n)]
    ref = bf16_round(oatt.gqa_decode_rows(q, keys, vals))
    assert max_rel_err(out.float().cpu().numpy(), ref) < TOL
    # the split-K decode kernel over the same rows (one query row per token) agrees
    rows_len = torch.arange(start + 1, start + n + 1, dtype=torch.int32, device=cuda)
    dec = cache.attend(0, _bf(q, cuda), rows_len, max_total_tokens=total,
                       row_seq=torch.ones(n, dtype=torch.int32, device=cuda))
    assert max_rel_err(out.float().cpu().numpy(), dec.float().cpu().numpy()) < TOL


def _paged_call(cuda, q, pk, pv, table, lengths, max_total, **kw):
    from mrun_b200.segmented_gqa_decode import paged_attention

    hkv, d = pk.shape[1], pk.shape[3]
    return paged_attention(
        _bf(q, cuda), _bf(pk, cuda), _bf(pv, cuda), strides=(hkv * 16 * d, 16 * d, d), page_size=16,
        block_table=torch.from_numpy(table).to(cuda),
        row_len=torch.tensor(lengths, dtype=torch.int32, device=cuda), max_total_tokens=max_total, **kw)


@pytest.mark.parametrize("rows,hq,hkv,lengths,max_total", [
    # 32 ragged rows of the routed-MoE decode shape: the tiles of all (row, head) groups
    # shared by one wave of CTAs, groups cut across CTAs
    (32, 32, 4, "u256-4096", None),
    # actual lengths far below the bound: fewer tiles than CTAs (most CTAs have nothing)
    (4, 32, 4, [1, 5, 16, 33], 8192),
    # many short groups per CTA (whole groups written directly) next to long ones
    (96, 32, 8, "u1-200", 4096),
])
def test_paged_attention_balanced_schedule(rows, hq, hkv, lengths, max_total, cuda):
    rng = np.random.default_rng(rows + hq + hkv)
    if lengths == "u256-4096":
        lengths = rng.integers(256, 4097, rows).tolist()
    elif lengths == "u1-200":
        lengths = rng.integers(1, 201, rows).tolist()
        lengths[5] = 4000
    d = 128
    max_total = max_total or max(lengths)
    pk, pv, table = _random_paged(rng, rows, hkv, d, lengths, sum((n + 15) // 16 for n in lengths) + 3)
    q = bf16_round(rng.standard_normal((rows, hq, d)).astype(np.float32))
    out = _paged_call(cuda, q, pk, pv, table, lengths, max_total)
    ref = oatt.paged_gqa_decode(q, pk, pv, table, lengths)
    assert max_rel_err(out.float().cpu().numpy(), ref) < TOL
    again = _paged_call(cuda, q, pk, pv, table, lengths, max_total)
    assert torch.equal(out, again)  # merge counters were left at zero; same plan, same bits
    from mrun_b200 import _lib

    assert int(_lib.load().mrb_paged_attention_timeouts()) == 0  # every bounded stage wait completed


def test_paged_attention_empty_row_writes_zeros(cuda):
    rng = np.random.default_rng(11)
    rows, hq, hkv, d = 3, 32, 4, 128
    lengths = [0, 40, 7]
    pk, pv, table = _random_paged(rng, rows, hkv, d, [max(n, 1) for n in lengths], 8)
    q = bf16_round(rng.standard_normal((rows, hq, d)).astype(np.float32))
    out = _paged_call(cuda, q, pk, pv, table, lengths, 8192).float().cpu().numpy()
    assert not out[0].any()
    ref = oatt.paged_gqa_decode(q[1:], pk, pv, table[1:], lengths[1:])
    assert max_rel_err(out[1:], ref) < TOL


def test_paged_attention_graph_follows_lengths(cuda):
    """A captured launch re-plans from row_len on every replay: lengths changed on the device
    between replays are attended in full, and the merge counters stay consistent."""
    from mrun_b200.segmented_gqa_decode import paged_attention, paged_attention_workspace_bytes

    rng = np.random.default_rng(5)
    rows, hq, hkv, d, cap = 16, 32, 4, 128, 2048
    pk, pv, table = _random_paged(rng, rows, hkv, d, [cap] * rows, rows * cap // 16 + 3)
    q = _bf(bf16_round(rng.standard_normal((rows, hq, d)).astype(np.float32)), cuda)
    kd, vd, td = _bf(pk, cuda), _bf(pv, cuda), torch.from_numpy(table).to(cuda)
    row_len = torch.full((rows,), 16, dtype=torch.int32, device=cuda)
    out = torch.empty_like(q)
    ws = torch.zeros(paged_attention_workspace_bytes(rows, hq, hkv, d, cap), dtype=torch.uint8, device=cuda)
    kw = dict(strides=(hkv * 16 * d, 16 * d, d), page_size=16, block_table=td, row_len=row_len, max_total_tokens=cap,
              out=out, workspace=ws)
    stream = torch.cuda.Stream(cuda)
    stream.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(stream):
        paged_attention(q, kd, vd, **kw)
    torch.cuda.synchronize(cuda)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        paged_attention(q, kd, vd, **kw)
    qn = q.float().cpu().numpy()
    for step in range(4):
        lengths = rng.integers(1, cap + 1, rows).tolist()
        row_len.copy_(torch.tensor(lengths, dtype=torch.int32))
        graph.replay()
        torch.cuda.synchronize(cuda)
        ref = oatt.paged_gqa_decode(qn, pk, pv, table, lengths)
        assert max_rel_err(out.float().cpu().numpy(), ref) < TOL, step


@pytest.mark.parametrize("lengths", [[1000, 2047, 3000, 15, 16, 31, 32, 2500], [0, 4095, 17, 1023]])
def test_paged_attention_provisional_token(lengths, cuda):
    """k_new / v_new: the token at position row_len, held outside the pool, is attended as the
    last token (tiles that hold only it, tiles it ends), on the tensor-core path."""
    from mrun_b200.segmented_gqa_decode import paged_attention

    rng = np.random.default_rng(len(lengths))
    rows, hq, hkv, d = len(lengths), 32, 4, 128
    pk, pv, table = _random_paged(rng, rows, hkv, d, [max(n, 1) for n in lengths],
                                  sum((max(n, 1) + 15) // 16 for n in lengths) + 3)
    q = bf16_round(rng.standard_normal((rows, hq, d)).astype(np.float32))
    kn = bf16_round(rng.standard_normal((rows, hkv, d)).astype(np.float32))
    vn = bf16_round(rng.standard_normal((rows, hkv, d)).astype(np.float32))
    out = paged_attention(
        _bf(q, cuda), _bf(pk, cuda), _bf(pv, cuda), strides=(hkv * 16 * d, 16 * d, d), page_size=16,
        block_table=torch.from_numpy(table).to(cuda), row_len=torch.tensor(lengths, dtype=torch.int32, device=cuda),
        k_new=_bf(kn, cuda), v_new=_bf(vn, cuda), max_total_tokens=max(lengths) + 1)
    keys = [np.concatenate([oatt.paged_gather(pk, table[r], n), kn[r][None]]) for r, n in enumerate(lengths)]
    vals = [np.concatenate([oatt.paged_gather(pv, table[r], n), vn[r][None]]) for r, n in enumerate(lengths)]
    ref = bf16_round(oatt.gqa_decode_rows(q, keys, vals, None))
    assert max_rel_err(out.float().cpu().numpy(), ref) < TOL
