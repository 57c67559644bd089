"""Continuous batching over the routed-MoE decoder.

``Qwen3MoeKVSlotPool`` keeps the reference's K/V slot-lease contract
(runtime/qwen3_moe_continuous.py:127-281): one fixed physical K/V allocation leased as
independently versioned rows -- ``acquire(state_id, capacity)`` -> (slot, generation, row
view), ``release``/``assert_binding`` checked against the holder's id and the slot's
generation, telemetry, ``close`` refused while rows are live -- with the reference's
exception types and messages. Here the allocation is the decoder's paged K/V pool: a lease
maps the pages its capacity needs into the slot's block-table row, and a released slot keeps
one parked page (the captured step still runs every slot; an idle slot rewrites position 0).

``MoeContinuousBatcher`` admits requests into free slots while others decode: each step runs
the decoder once over every slot (a CUDA-graph replay when the decoder's experts are
resident, eager when they stream from the host tier), feeds prompt tokens one per step,
collects greedy tokens, retires finished requests and reuses their slots at the next step.
"""
from __future__ import annotations

import heapq
import threading
from collections import deque
from dataclasses import dataclass, field
from typing import Any

import torch


class Qwen3MoeContinuousRuntimeError(RuntimeError):
    """A continuous-batching contract was violated (stale lease, exhausted or closed pool)."""


def _strict_positive_int(value: int, field_name: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
        raise ValueError(f"{field_name} must be a positive integer")
    return int(value)


@dataclass(frozen=True, slots=True)
class Qwen3MoeKVPoolTelemetry:
    max_slots: int
    max_context_tokens: int
    active_slots: int
    peak_active_slots: int
    allocations: int
    releases: int
    slot_reuses: int
    kv_resident_bytes: int


@dataclass(frozen=True)
class KVRowLease:
    """One slot of the paged pool: its capacity in tokens and its block-table row (a device
    view: page numbers of positions [16j, 16j + 16) at entry j)."""

    slot: int
    capacity: int
    block_table_row: torch.Tensor
    pages: tuple[int, ...]


class Qwen3MoeKVSlotPool:
    """One fixed physical K/V allocation (the decoder's paged pool) leased as independently
    versioned rows."""

    def __init__(self, decoder: Any, *, max_slots: int = 8, max_context_tokens: int,
                 kv_bytes_per_token: int | None = None) -> None:
        self.max_slots = _strict_positive_int(max_slots, "max_slots")
        self.max_context_tokens = _strict_positive_int(max_context_tokens, "max_context_tokens")
        kv = getattr(decoder, "kv", None)
        if kv is None or not hasattr(kv, "reserve") or not hasattr(kv, "release"):
            raise TypeError("the decoder must expose its paged K/V pool as .kv")
        if int(kv.max_seqs) < self.max_slots:
            raise Qwen3MoeContinuousRuntimeError("Qwen K/V factory returned a cache with the wrong fixed arena shape")
        if self.max_context_tokens > int(kv.max_pages_per_seq) * int(kv.page_size):
            raise Qwen3MoeContinuousRuntimeError("Qwen K/V factory returned a cache with the wrong fixed arena shape")
        self._decoder = decoder
        self._kv = kv
        self._lock = threading.RLock()
        self._free = list(range(self.max_slots))
        heapq.heapify(self._free)
        self._slot_generations = [0] * self.max_slots
        self._active: dict[int, str] = {}
        self._allocations = 0
        self._releases = 0
        self._slot_reuses = 0
        self._peak_active = 0
        self._closed = False
        inferred = int(kv.bytes_per_token)
        if kv_bytes_per_token is None:
            self.kv_bytes_per_token = inferred
        else:
            self.kv_bytes_per_token = _strict_positive_int(kv_bytes_per_token, "kv_bytes_per_token")
            if self.kv_bytes_per_token != inferred:
                raise ValueError("kv_bytes_per_token disagrees with the physical Qwen K/V allocation")
        for slot in range(self.max_slots):  # every idle slot parks one page
            kv.release(slot)
            kv.reserve(slot, 1)

    @property
    def cache(self) -> Any:
        """The full fixed arena; only the bound decoder consumes it."""
        return self._kv

    @property
    def device_bytes(self) -> int:
        return int(self._kv.k.numel() + self._kv.v.numel()) * int(self._kv.k.element_size())

    def acquire(self, state_id: str, capacity: int) -> tuple[int, int, KVRowLease]:
        capacity = _strict_positive_int(capacity, "capacity")
        if capacity > self.max_context_tokens:
            raise OverflowError("requested Qwen K/V capacity exceeds the fixed slot arena")
        with self._lock:
            if self._closed:
                raise Qwen3MoeContinuousRuntimeError("Qwen K/V slot pool is closed")
            if not self._free:
                raise Qwen3MoeContinuousRuntimeError("Qwen K/V slot pool is exhausted")
            slot = heapq.heappop(self._free)
            try:
                self._kv.release(slot)
                self._kv.reserve(slot, capacity)
            except Exception:
                self._kv.reserve(slot, 1)
                heapq.heappush(self._free, slot)
                raise
            generation = self._slot_generations[slot] + 1
            if generation > 1:
                self._slot_reuses += 1
            self._slot_generations[slot] = generation
            self._active[slot] = state_id
            self._allocations += 1
            self._peak_active = max(self._peak_active, len(self._active))
            lease = KVRowLease(slot=slot, capacity=capacity, block_table_row=self._kv.block_table[slot],
                               pages=tuple(self._kv.pages_of(slot)))
        return slot, generation, lease

    def release(self, *, state_id: str, slot: int, storage_generation: int) -> None:
        with self._lock:
            if self._active.get(slot) != state_id:
                raise Qwen3MoeContinuousRuntimeError("Qwen K/V slot authority is stale")
            if self._slot_generations[slot] != storage_generation:
                raise Qwen3MoeContinuousRuntimeError("Qwen K/V slot generation is stale")
            del self._active[slot]
            self._kv.release(slot)
            self._kv.reserve(slot, 1)  # parked
            heapq.heappush(self._free, slot)
            self._releases += 1

    def assert_binding(self, *, state_id: str, slot: int, storage_generation: int) -> None:
        with self._lock:
            if self._active.get(slot) != state_id or self._slot_generations[slot] != storage_generation:
                raise Qwen3MoeContinuousRuntimeError("Qwen K/V row no longer owns its slot")

    def telemetry(self) -> Qwen3MoeKVPoolTelemetry:
        with self._lock:
            return Qwen3MoeKVPoolTelemetry(
                max_slots=self.max_slots,
                max_context_tokens=self.max_context_tokens,
                active_slots=len(self._active),
                peak_active_slots=self._peak_active,
                allocations=self._allocations,
                releases=self._releases,
                slot_reuses=self._slot_reuses,
                kv_resident_bytes=self.device_bytes,
            )

    def close(self) -> None:
        with self._lock:
            if self._active:
                raise Qwen3MoeContinuousRuntimeError("cannot close the Qwen K/V pool with live row authorities")
            self._closed = True


@dataclass
class _Request:
    request_id: int
    prompt: list[int]
    max_new_tokens: int
    eos: int | None
    context: int = 0  # positions already committed in the slot's K/V at admission
    prefill: Any = None
    state_id: str = ""
    slot: int = -1
    generation: int = 0
    fed: int = 0
    tokens: list[int] = field(default_factory=list)


class MoeContinuousBatcher:
    """Requests in, greedy tokens out, over one ``MoeDecoder`` whose slots are leased from a
    ``Qwen3MoeKVSlotPool``. ``submit`` queues a prompt; ``step`` admits queued requests into
    free slots, runs the decoder once over every slot and returns the requests that finished
    (id -> generated tokens); ``run`` steps until everything submitted is done. With expert
    parallelism every rank runs its own batcher and calls ``step`` the same number of times
    (an idle rank still steps, so the exchanges stay in lockstep)."""

    def __init__(self, decoder: Any, *, max_context_tokens: int, graph: bool = True) -> None:
        self.decoder = decoder
        self.slots = int(decoder.max_rows)
        self.pool = Qwen3MoeKVSlotPool(decoder, max_slots=self.slots, max_context_tokens=max_context_tokens)
        self._queue: deque[_Request] = deque()
        self._active: dict[int, _Request] = {}
        self._next_id = 0
        self.steps = 0
        self.generated = 0
        self.rows_stepped = 0
        dev = decoder.device
        # every slot starts parked: token 0 at position 0
        decoder.in_ids[: self.slots].zero_()
        decoder.positions[: self.slots].zero_()
        decoder.row_len[: self.slots].fill_(1)
        self._graph = bool(graph) and decoder.ep is None and not getattr(decoder, "streamed", False)
        if self._graph:
            decoder.capture(self.slots)
        self._dev = dev

    def submit(self, prompt: list[int] | torch.Tensor, *, max_new_tokens: int, eos: int | None = None) -> int:
        prompt = [int(t) for t in (prompt.tolist() if isinstance(prompt, torch.Tensor) else prompt)]
        if not prompt:
            raise ValueError("prompt must hold at least one token")
        _strict_positive_int(max_new_tokens, "max_new_tokens")
        if len(prompt) + max_new_tokens > self.pool.max_context_tokens:
            raise OverflowError("requested Qwen K/V capacity exceeds the fixed slot arena")
        req = _Request(self._next_id, prompt, int(max_new_tokens), eos)
        self._next_id += 1
        self._queue.append(req)
        return req.request_id

    def submit_with_context(self, first_token: int, context_tokens: int, *, max_new_tokens: int,
                            eos: int | None = None, prefill: Any = None) -> int:
        """Queue a request whose first ``context_tokens`` positions are committed in its K/V
        pages at admission and whose next input is ``first_token``: ``prefill(lease)`` is
        called when the slot is leased and writes those pages (a prefill engine; left None,
        the pages keep what they hold, which the synthetic benchmarks fill with random K/V)."""
        context_tokens = _strict_positive_int(context_tokens, "context_tokens")
        _strict_positive_int(max_new_tokens, "max_new_tokens")
        if context_tokens + 1 + max_new_tokens > self.pool.max_context_tokens:
            raise OverflowError("requested Qwen K/V capacity exceeds the fixed slot arena")
        req = _Request(self._next_id, [int(first_token)], int(max_new_tokens), eos, context=context_tokens,
                       prefill=prefill)
        self._next_id += 1
        self._queue.append(req)
        return req.request_id

    @property
    def pending(self) -> int:
        return len(self._queue) + len(self._active)

    def _write(self, tensor: torch.Tensor, slots: list[int], values: list[int]) -> None:
        if slots:
            idx = torch.tensor(slots, dtype=torch.int64, device=self._dev)
            tensor.index_copy_(0, idx, torch.tensor(values, dtype=tensor.dtype, device=self._dev))

    def _admit(self) -> None:
        slots, ids, pos, lens = [], [], [], []
        while self._queue and len(self._active) < self.slots:
            req = self._queue[0]
            req.state_id = f"moe-request-{req.request_id}"
            # the last generated token is never fed back: positions end at
            # context + len(prompt) + max_new_tokens - 2
            req.slot, req.generation, lease = self.pool.acquire(
                req.state_id, req.context + len(req.prompt) + req.max_new_tokens)
            self._queue.popleft()
            if req.prefill is not None:
                req.prefill(lease)
            req.fed = 1
            self._active[req.slot] = req
            slots.append(req.slot)
            ids.append(req.prompt[0])
            pos.append(req.context)
            lens.append(req.context + 1)
        self._write(self.decoder.in_ids, slots, ids)
        self._write(self.decoder.positions, slots, pos)
        self._write(self.decoder.row_len, slots, lens)

    def step(self) -> dict[int, list[int]]:
        self._admit()
        dec = self.decoder
        if not self._active and dec.ep is None:
            return {}
        # a captured step runs every slot; an eager one only up to the highest leased slot
        # (slots are leased lowest first, so the live rows stay packed at the front)
        rows = self.slots if self._graph or not self._active else max(self._active) + 1
        if self._graph:
            dec.step(rows)
        else:
            dec.step_eager(rows)
        self.steps += 1
        self.rows_stepped += rows
        out = dec.next_ids[:rows].cpu().tolist()
        done: dict[int, list[int]] = {}
        feed_s, feed_v = [], []
        for slot, req in list(self._active.items()):
            self.pool.assert_binding(state_id=req.state_id, slot=slot, storage_generation=req.generation)
            if req.fed < len(req.prompt):  # still reading the prompt: feed the next token
                feed_s.append(slot)
                feed_v.append(req.prompt[req.fed])
                req.fed += 1
                continue
            tok = int(out[slot])
            req.tokens.append(tok)
            self.generated += 1
            if len(req.tokens) >= req.max_new_tokens or (req.eos is not None and tok == req.eos):
                done[req.request_id] = req.tokens
                self.pool.release(state_id=req.state_id, slot=slot, storage_generation=req.generation)
                del self._active[slot]
        idle = [s for s in range(self.slots) if s not in self._active]
        self._write(dec.in_ids, feed_s, feed_v)
        # idle slots rewrite position 0 of their parked page every step
        self._write(dec.in_ids, idle, [0] * len(idle))
        self._write(dec.positions, idle, [0] * len(idle))
        self._write(dec.row_len, idle, [1] * len(idle))
        return done

    def run(self) -> dict[int, list[int]]:
        results: dict[int, list[int]] = {}
        while self.pending:
            results.update(self.step())
        self.decoder.check_errors()
        return results

    def close(self) -> None:
        self.pool.close()


__all__ = [
    "KVRowLease",
    "MoeContinuousBatcher",
    "Qwen3MoeContinuousRuntimeError",
    "Qwen3MoeKVPoolTelemetry",
    "Qwen3MoeKVSlotPool",
]
