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
