"""Continuous batching, host side: the K/V slot-lease contract of the reference's
``Qwen3MoeKVSlotPool`` (runtime/qwen3_moe_continuous.py:127-281 -- heap-ordered slots,
per-slot generations, stale-authority errors, telemetry, close refused while rows live, the
same exception types and messages) over the paged K/V pool, and the batcher's admission,
prompt feeding, retirement and slot reuse against a fake decoder on the CPU."""
from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from mrun_b200.continuous import (MoeContinuousBatcher, Qwen3MoeContinuousRuntimeError, Qwen3MoeKVPoolTelemetry,
                                  Qwen3MoeKVSlotPool)
from mrun_b200.paged_kv import PagedKVCache


def _kv(slots=4, max_seq=256, layers=2):
    pps = (max_seq + 15) // 16
    return PagedKVCache(num_layers=layers, num_pages=slots * pps, kv_heads=2, head_dim=16, max_seqs=slots,
                        max_pages_per_seq=pps, device=torch.device("cpu"))


def _pool(slots=4, max_ctx=256, **kw):
    return Qwen3MoeKVSlotPool(SimpleNamespace(kv=_kv(slots, max_ctx)), max_slots=slots, max_context_tokens=max_ctx,
                              **kw)


@pytest.mark.parametrize("bad", [0, -1, True, 2.0, "3", None])
def test_pool_rejects_non_positive_integers(bad):
    with pytest.raises(ValueError, match="max_slots must be a positive integer"):
        _pool_kw = dict(max_slots=bad, max_context_tokens=64)
        Qwen3MoeKVSlotPool(SimpleNamespace(kv=_kv()), **_pool_kw)
    with pytest.raises(ValueError, match="max_context_tokens must be a positive integer"):
        Qwen3MoeKVSlotPool(SimpleNamespace(kv=_kv()), max_slots=2, max_context_tokens=bad)
    pool = _pool()
    with pytest.raises(ValueError, match="capacity must be a positive integer"):
        pool.acquire("a", bad)


def test_pool_arena_shape_and_bytes_checks():
    with pytest.raises(TypeError):
        Qwen3MoeKVSlotPool(SimpleNamespace(), max_slots=2, max_context_tokens=64)
    with pytest.raises(Qwen3MoeContinuousRuntimeError, match="wrong fixed arena shape"):
        Qwen3MoeKVSlotPool(SimpleNamespace(kv=_kv(slots=2)), max_slots=4, max_context_tokens=64)
    with pytest.raises(Qwen3MoeContinuousRuntimeError, match="wrong fixed arena shape"):
        Qwen3MoeKVSlotPool(SimpleNamespace(kv=_kv(max_seq=64)), max_slots=4, max_context_tokens=65)
    kv = _kv()
    with pytest.raises(ValueError, match="disagrees with the physical Qwen K/V allocation"):
        Qwen3MoeKVSlotPool(SimpleNamespace(kv=kv), max_slots=4, max_context_tokens=64,
                           kv_bytes_per_token=kv.bytes_per_token + 2)
    pool = Qwen3MoeKVSlotPool(SimpleNamespace(kv=kv), max_slots=4, max_context_tokens=64,
                              kv_bytes_per_token=kv.bytes_per_token)
    assert pool.kv_bytes_per_token == 2 * 2 * 2 * 16 * 2
    assert pool.device_bytes == 2 * kv.k.numel() * 2
    assert pool.cache is kv


def test_pool_lease_contract_and_telemetry():
    pool = _pool(slots=3, max_ctx=128)
    kv = pool.cache
    # every idle slot parks exactly one page
    assert all(len(kv.pages_of(s)) == 1 for s in range(3))
    a = pool.acquire("a", 40)
    b = pool.acquire("b", 17)
    c = pool.acquire("c", 128)
    assert [a[0], b[0], c[0]] == [0, 1, 2] and [a[1], b[1], c[1]] == [1, 1, 1]
    assert len(a[2].pages) == 3 and len(b[2].pages) == 2 and len(c[2].pages) == 8
    assert a[2].block_table_row.tolist()[:3] == list(a[2].pages)
    assert len(set(a[2].pages) | set(b[2].pages) | set(c[2].pages)) == 13
    with pytest.raises(Qwen3MoeContinuousRuntimeError, match="Qwen K/V slot pool is exhausted"):
        pool.acquire("d", 8)
    with pytest.raises(OverflowError, match="requested Qwen K/V capacity exceeds the fixed slot arena"):
        pool.acquire("d", 129)
    pool.assert_binding(state_id="b", slot=1, storage_generation=1)
    with pytest.raises(Qwen3MoeContinuousRuntimeError, match="Qwen K/V slot authority is stale"):
        pool.release(state_id="x", slot=1, storage_generation=1)
    with pytest.raises(Qwen3MoeContinuousRuntimeError, match="Qwen K/V slot generation is stale"):
        pool.release(state_id="b", slot=1, storage_generation=2)
    pool.release(state_id="b", slot=1, storage_generation=1)
    assert len(kv.pages_of(1)) == 1  # parked again
    with pytest.raises(Qwen3MoeContinuousRuntimeError, match="Qwen K/V row no longer owns its slot"):
        pool.assert_binding(state_id="b", slot=1, storage_generation=1)
    # the lowest free slot comes back with the next generation
    d = pool.acquire("d", 64)
    assert d[0] == 1 and d[1] == 2
    with pytest.raises(Qwen3MoeContinuousRuntimeError, match="Qwen K/V row no longer owns its slot"):
        pool.assert_binding(state_id="d", slot=1, storage_generation=1)
    t = pool.telemetry()
    assert isinstance(t, Qwen3MoeKVPoolTelemetry)
    assert (t.max_slots, t.max_context_tokens, t.active_slots, t.peak_active_slots) == (3, 128, 3, 3)
    assert (t.allocations, t.releases, t.slot_reuses) == (4, 1, 1)
    assert t.kv_resident_bytes == pool.device_bytes
    with pytest.raises(Qwen3MoeContinuousRuntimeError, match="cannot close the Qwen K/V pool with live row"):
        pool.close()
    for sid, (slot, gen, _) in (("a", a), ("c", c), ("d", d)):
        pool.release(state_id=sid, slot=slot, storage_generation=gen)
    pool.close()
    with pytest.raises(Qwen3MoeContinuousRuntimeError, match="Qwen K/V slot pool is closed"):
        pool.acquire("e", 8)
    # a failed page mapping leaves the slot free and parked
    assert kv.free_pages() == 3 * 8 - 3


def test_pool_pages_exhausted_keeps_slot_free():
    kv = _kv(slots=2, max_seq=64)
    kv._free = kv._free[-6:]  # a pool smaller than the arena: 6 pages left
    pool = Qwen3MoeKVSlotPool(SimpleNamespace(kv=kv), max_slots=2, max_context_tokens=64)
    s0 = pool.acquire("a", 64)
    with pytest.raises(MemoryError):
        pool.acquire("b", 64)
    assert pool.telemetry().active_slots == 1 and len(kv.pages_of(1)) == 1
    s1 = pool.acquire("b", 16)
    assert s1[0] == 1
    pool.release(state_id="a", slot=s0[0], storage_generation=s0[1])


class _FakeDecoder:
    """The decoder surface the batcher drives, on the CPU: step(rows) turns (in_id, position)
    into next_id with a fixed hash, then advances the state like mrb_decode_advance."""

    VOCAB = 97

    def __init__(self, rows, max_seq):
        self.device = torch.device("cpu")
        self.max_rows = rows
        self.kv = _kv(rows, max_seq)
        self.in_ids = torch.zeros(rows, dtype=torch.int64)
        self.positions = torch.zeros(rows, dtype=torch.int32)
        self.row_len = torch.zeros(rows, dtype=torch.int32)
        self.next_ids = torch.zeros(rows, dtype=torch.int64)
        self.ep = None
        self.backend = object()
        self.captured = None
        self.history = [[] for _ in range(rows)]

    @staticmethod
    def next_token(context):
        return (sum((t + 1) * (i + 3) for i, t in enumerate(context)) * 31 + len(context)) % _FakeDecoder.VOCAB

    def capture(self, rows):
        self.captured = rows

    def step(self, rows):
        assert rows == self.captured
        for r in range(rows):
            pos = int(self.positions[r])
            assert int(self.row_len[r]) == pos + 1
            assert pos < len(self.kv.pages_of(r)) * 16, "a step wrote past the slot's pages"
            self.history[r] = self.history[r][:pos] + [int(self.in_ids[r])]
            self.next_ids[r] = self.next_token(self.history[r])
        self.in_ids[:rows] = self.next_ids[:rows]
        self.positions[:rows] += 1
        self.row_len[:rows] += 1

    def check_errors(self):
        pass


def _alone(prompt, n, eos=None):
    ctx, out = list(prompt), []
    while len(out) < n:
        t = _FakeDecoder.next_token(ctx)
        out.append(t)
        ctx.append(t)
        if eos is not None and t == eos:
            break
    return out


def test_batcher_admits_feeds_retires_and_reuses_slots():
    dec = _FakeDecoder(rows=3, max_seq=128)
    bat = MoeContinuousBatcher(dec, max_context_tokens=128)
    assert dec.captured == 3
    g = torch.Generator().manual_seed(0)
    reqs = {}
    for i in range(7):  # more requests than slots: the rest wait for a retirement
        prompt = torch.randint(0, 97, (int(torch.randint(1, 20, (1,), generator=g)),), generator=g).tolist()
        n = int(torch.randint(1, 30, (1,), generator=g))
        reqs[bat.submit(prompt, max_new_tokens=n)] = (prompt, n)
    results = {}
    for _ in range(3):  # a late arrival while others decode
        results.update(bat.step())
    reqs[bat.submit([5, 6, 7], max_new_tokens=9)] = ([5, 6, 7], 9)
    results.update(bat.run())
    assert set(results) == set(reqs)
    for rid, (prompt, n) in reqs.items():
        assert results[rid] == _alone(prompt, n), rid
    t = bat.pool.telemetry()
    assert t.allocations == 8 and t.releases == 8 and t.active_slots == 0 and t.peak_active_slots == 3
    assert t.slot_reuses == 5
    # idle slots are parked at position 0
    assert dec.positions.tolist() == [0, 0, 0] and dec.row_len.tolist() == [1, 1, 1]
    bat.close()


def test_batcher_eos_and_limits():
    dec = _FakeDecoder(rows=2, max_seq=64)
    bat = MoeContinuousBatcher(dec, max_context_tokens=64)
    ref = _alone([1, 2, 3], 40)
    eos = ref[4]
    rid = bat.submit([1, 2, 3], max_new_tokens=40, eos=eos)
    out = bat.run()[rid]
    assert out == ref[: ref.index(eos) + 1]
    with pytest.raises(ValueError, match="prompt must hold at least one token"):
        bat.submit([], max_new_tokens=4)
    with pytest.raises(ValueError, match="max_new_tokens must be a positive integer"):
        bat.submit([1], max_new_tokens=0)
    with pytest.raises(OverflowError):
        bat.submit([1] * 61, max_new_tokens=4)
    assert bat.step() == {} and bat.pending == 0


class _FakeStreamedDecoder(_FakeDecoder):
    """A decoder that cannot be captured (host-tier experts): the batcher steps it eagerly
    over the live prefix of its slots."""

    streamed = True

    def capture(self, rows):
        raise AssertionError("a streamed decoder is never captured")

    def step_eager(self, rows):
        self.rows_seen.append(rows)
        self.captured = rows
        self.step(rows)


def test_batcher_eager_prefix_and_prefilled_context():
    dec = _FakeStreamedDecoder(rows=4, max_seq=128)
    dec.rows_seen = []
    bat = MoeContinuousBatcher(dec, max_context_tokens=128)
    leases = []
    # a request whose first 20 positions are committed at admission (its prefill callback sees
    # the lease), then two plain prompts
    r0 = bat.submit_with_context(11, 20, max_new_tokens=5, prefill=leases.append)
    r1 = bat.submit([3, 4], max_new_tokens=3)
    r2 = bat.submit([9], max_new_tokens=8)
    first = bat.step()
    assert first == {} and dec.rows_seen == [3]
    assert len(leases) == 1 and leases[0].slot == 0 and leases[0].capacity == 26
    assert dec.positions[0] == 21  # the prefilled row decoded its first token at position 20
    out = {**first, **bat.run()}
    assert out[r1] == _alone([3, 4], 3) and out[r2] == _alone([9], 8)
    assert len(out[r0]) == 5
    # rows stepped never exceed the highest leased slot + 1
    assert max(dec.rows_seen) == 3
    with pytest.raises(ValueError, match="context_tokens must be a positive integer"):
        bat.submit_with_context(1, 0, max_new_tokens=2)
    with pytest.raises(OverflowError):
        bat.submit_with_context(1, 120, max_new_tokens=8)
