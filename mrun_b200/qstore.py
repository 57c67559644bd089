"""On-disk QStore reader: int8 row-quantised pages from disk to HBM through pinned staging.

Reads the reference's paged store directory (engine/kernels/qstore.py:662-1128): a
``manifest.json`` whose ``blocks`` table maps each name to a ``qrow`` block (int8 codes
``[out, in]`` at ``w_off`` in ``weights.i8`` plus fp32 row scales at ``s_off`` in
``scales.f32``), an ``fp32`` block (at ``e_off`` in ``extras.f32``) or an ``alias`` of another
name. Bytes come off disk through the library's parallel ``pread`` reader
(``mrb_store_file_read``) straight into pinned host buffers, then one asynchronous copy puts
them in HBM, where the B200 kernels consume the codes as they are (no fp32 weight copy).

``_PageRing`` is the B200 counterpart of the reference's successor-oracle ``_RingPrefetch``
(engine/kernels/qstore.py:459-660): it learns which block follows which, stages the predicted
next blocks into reusable pinned slots on a worker thread (the reads release the GIL) and
issues their host-to-device copies on a dedicated stream, so a decode loop's disk and PCIe
traffic overlaps its kernels. A hit returns the same bytes as a direct read.

The manifest's content-identity and provenance digests are not verified here (the
reference's identity layer is outside this path); the block layout is validated as the
reference validates it (engine/kernels/qstore.py:124-219).
"""
from __future__ import annotations

import ctypes
import json
import math
import os
import threading
from collections import OrderedDict
from collections.abc import Mapping
from concurrent.futures import Future, ThreadPoolExecutor
from pathlib import Path
from typing import Any

import numpy as np
import torch

from . import _lib
from .dense_qstore_cuda import CompactQRowPage, qrow_linear

QSTORE_FILES = ("weights.i8", "scales.f32", "extras.f32")
# parallel pread calls per block read: one per host core up to 32 (measured on a 16-core B200
# host, page cache to pinned memory: 8.0 GB/s with 1 thread, 36.6 with 8, 45.7 with 16)
DEFAULT_READ_THREADS = max(4, min(32, os.cpu_count() or 8))


def store_options_from_env(*, ring: bool = True, ring_slots: int = 3, cache_policy: str | None = None,
                           environ=None) -> dict:
    """The reference's QStore switches (engine/kernels/qstore.py:756-772, 948-973):
    MRUN_PAGED_RING = "0" turns the prefetch ring off and an integer above 1 sets its slot
    count; MRUN_QSTORE_CACHE_POLICY picks the resident cache policy when none is given
    (pin-fill by default and for an unknown name, which is reported)."""
    env = os.environ if environ is None else environ
    ring_env = env.get("MRUN_PAGED_RING", "").strip()
    if ring_env == "0":
        ring = False
    elif ring_env.isdigit() and int(ring_env) > 1:
        ring_slots = int(ring_env)
    policy = cache_policy
    if policy is None:
        policy = env.get("MRUN_QSTORE_CACHE_POLICY", "pin-fill").strip().lower() or "pin-fill"
        if policy not in ResidentPageCache.POLICIES:
            import warnings

            warnings.warn(f"MRUN_QSTORE_CACHE_POLICY={policy!r} unknown -> pin-fill (want pin-fill|lru)")
            policy = "pin-fill"
    return {"ring": ring, "ring_slots": int(ring_slots), "cache_policy": policy}


# ------------------------------------------------------------------ native file reader


class StoreFile:
    """One store file opened for parallel positional reads (``mrb_store_file_*``)."""

    def __init__(self, path: str | Path) -> None:
        self.path = Path(path)
        handle = ctypes.c_void_p()
        size = ctypes.c_uint64()
        _lib.call("mrb_store_file_open", str(self.path).encode(), ctypes.byref(handle), ctypes.byref(size))
        self._handle = handle.value
        self.size = int(size.value)
        self._lock = threading.Lock()

    def read_into(self, offset: int, nbytes: int, dst: np.ndarray | torch.Tensor, *, threads: int = 1,
                  drop_after: bool = False) -> None:
        """Copy file bytes [offset, offset + nbytes) into the start of host buffer ``dst``."""
        if isinstance(dst, torch.Tensor):
            if dst.is_cuda or not dst.is_contiguous():
                raise ValueError("destination must be a contiguous host tensor")
            capacity, address = dst.numel() * dst.element_size(), dst.data_ptr()
        else:
            if not dst.flags["C_CONTIGUOUS"] or not dst.flags["WRITEABLE"]:
                raise ValueError("destination must be a writable contiguous array")
            capacity, address = dst.nbytes, dst.ctypes.data
        if nbytes > capacity:
            raise ValueError(f"destination holds {capacity} bytes, {nbytes} requested")
        if self._handle is None:
            raise ValueError(f"{self.path} is closed")
        _lib.call("mrb_store_file_read", self._handle, int(offset), int(nbytes), address, int(threads),
                  1 if drop_after else 0)

    def advise(self, offset: int, nbytes: int, *, will_need: bool = True) -> None:
        if self._handle is not None:
            _lib.call("mrb_store_file_advise", self._handle, int(offset), int(nbytes), 1 if will_need else 0)

    def close(self) -> None:
        with self._lock:
            handle, self._handle = self._handle, None
        if handle is not None:
            _lib.call("mrb_store_file_close", handle)

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order varies
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ manifest


class QStoreLayoutError(RuntimeError):
    """A store directory whose block table does not describe its files.

    ``reason`` names the broken rule (one of ``LAYOUT_REASONS``) and ``subject`` the block or
    file it was found on, so callers can branch without parsing the message."""

    def __init__(self, reason: str, subject: str | None, message: str) -> None:
        super().__init__(message)
        self.reason = reason
        self.subject = subject


LAYOUT_REASONS = ("header", "kinds", "field", "shape", "length", "kind", "alias-target", "alias-cycle",
                  "missing-file", "bounds", "overlap", "gap", "tail")

# For each data kind: the file ranges a block of that kind owns, as (file, offset field,
# length field, bytes per element, element count from the shape). Aliases own no bytes.
_KIND_SPANS = {
    "qrow": (("weights.i8", "w_off", "w_len", 1, lambda shape: shape[0] * shape[1]),
             ("scales.f32", "s_off", "s_len", 4, lambda shape: shape[0])),
    "fp32": (("extras.f32", "e_off", "e_len", 4, math.prod),),
}
_KIND_DIMS = {"qrow": 2, "fp32": None}


def _layout_error(reason: str, subject: str | None, text: str) -> QStoreLayoutError:
    return QStoreLayoutError(reason, subject, f"QStore layout ({reason}): {text}")


def _count(block: Mapping[str, Any], field: str, name: str, *, least: int) -> int:
    """A byte offset (least 0) or length (least 1) read from a block descriptor."""
    value = block.get(field)
    if type(value) is not int:  # bool is an int subclass and is refused too
        raise _layout_error("field", name, f"block {name!r} field {field!r} is {value!r}, not an integer")
    if value < least:
        raise _layout_error("field", name, f"block {name!r} field {field!r} = {value} is below {least}")
    return value


def _dims(block: Mapping[str, Any], name: str, rank: int | None) -> tuple[int, ...]:
    shape = block.get("shape")
    ok = isinstance(shape, list) and len(shape) > 0 and all(type(v) is int and v > 0 for v in shape)
    if not ok or (rank is not None and len(shape) != rank):
        want = f"{rank} positive integers" if rank else "a non-empty list of positive integers"
        raise _layout_error("shape", name, f"block {name!r} shape {shape!r} is not {want}")
    return tuple(shape)


def _block_spans(name: str, block: Mapping[str, Any]) -> list[tuple[str, int, int]]:
    """The (file, start, end) byte ranges a data block occupies, checked against its shape."""
    kind = block.get("kind")
    if kind not in _KIND_SPANS:
        raise _layout_error("kind", name, f"block {name!r} has kind {kind!r}; only 'qrow' and 'fp32' are stored")
    shape = _dims(block, name, _KIND_DIMS[kind])
    spans = []
    for filename, off_field, len_field, width, elements in _KIND_SPANS[kind]:
        start = _count(block, off_field, name, least=0)
        length = _count(block, len_field, name, least=1)
        if length != elements(shape) * width or start % width:
            raise _layout_error("length", name, f"block {name!r} range {start}+{length} in {filename} does not "
                                f"hold {elements(shape)} elements of {width} byte(s) for shape {list(shape)}")
        spans.append((filename, start, start + length))
    return spans


def _check_aliases(aliases: dict[str, Any], blocks: Mapping[str, Any]) -> None:
    """Every alias chain ends at a data block: targets exist, and following the links from any
    alias never returns to a name already on the chain (three-colour walk, each name once)."""
    done: set[str] = set()
    for start in aliases:
        chain: list[str] = []
        on_chain: set[str] = set()
        name = start
        while name in aliases and name not in done:
            if name in on_chain:
                raise _layout_error("alias-cycle", name, f"alias chain {' -> '.join(chain + [name])} loops")
            chain.append(name)
            on_chain.add(name)
            target = aliases[name]
            if not isinstance(target, str) or not target:
                raise _layout_error("alias-target", name, f"alias {name!r} has target {target!r}")
            if target not in blocks or not isinstance(blocks[target], Mapping):
                raise _layout_error("alias-target", name, f"alias {name!r} points at {target!r}, which is not a block")
            name = target
        done.update(chain)


def _check_coverage(directory: Path, spans: dict[str, list[tuple[int, int, str]]]) -> None:
    """Each store file is exactly the concatenation of the ranges its blocks own."""
    for filename in QSTORE_FILES:
        path = directory / filename
        if not path.is_file():
            raise _layout_error("missing-file", filename, f"{filename} is not in {directory}")
        size = path.stat().st_size
        cursor = 0
        for start, end, name in sorted(spans[filename]):
            if end > size:
                raise _layout_error("bounds", name, f"{filename}: block {name!r} ends at byte {end}, "
                                    f"past the file's {size} bytes")
            if start != cursor:
                reason = "overlap" if start < cursor else "gap"
                raise _layout_error(reason, name, f"{filename}: block {name!r} starts at byte {start}, "
                                    f"the previous range ends at {cursor}")
            cursor = end
        if cursor != size:
            raise _layout_error("tail", filename, f"{filename}: {size - cursor} trailing byte(s) belong to no block")


def validate_int8_layout(directory: Path, manifest: Mapping[str, Any]) -> None:
    """Check that a store directory is a well-formed int8 QStore before any byte is read.

    The accept/reject rules are those of the reference's loader (engine/kernels/qstore.py:
    124-219): the manifest declares int8, carries a config and a non-empty block table with at
    least one qrow and one fp32 block; every data block's ranges match its shape; every alias
    chain ends at a data block; and each of the three files is covered by its blocks' ranges
    exactly once, with nothing left over. Raises ``QStoreLayoutError`` (a RuntimeError)."""
    directory = Path(directory)
    if manifest.get("dtype") != "int8":
        raise _layout_error("header", None, f"manifest dtype is {manifest.get('dtype')!r}, not 'int8'")
    blocks = manifest.get("blocks")
    if not isinstance(manifest.get("config"), Mapping) or not isinstance(blocks, Mapping) or not blocks:
        raise _layout_error("header", None, "manifest needs a config mapping and a non-empty block table")
    spans: dict[str, list[tuple[int, int, str]]] = {f: [] for f in QSTORE_FILES}
    aliases: dict[str, Any] = {}
    kinds_seen: set[str] = set()
    for name, block in blocks.items():
        if not isinstance(name, str) or not name or not isinstance(block, Mapping):
            raise _layout_error("header", None, f"block table entry {name!r} is not a named mapping")
        if "alias" in block:
            aliases[name] = block["alias"]
            continue
        for filename, start, end in _block_spans(name, block):
            spans[filename].append((start, end, name))
        kinds_seen.add(block["kind"])
    if kinds_seen != set(_KIND_SPANS):
        raise _layout_error("kinds", None, f"block table holds kinds {sorted(kinds_seen)}; both qrow and fp32 are needed")
    _check_aliases(aliases, blocks)
    _check_coverage(directory, spans)


def _resolve_in(blocks: Mapping[str, Any], name: str) -> Mapping[str, Any]:
    """Follow alias links (engine/kernels/qstore.py:928-942); KeyError for a missing name."""
    key = str(name)
    seen: set[str] = set()
    while True:
        if key in seen:
            raise RuntimeError(f"QStore alias cycle contains {key!r}")
        seen.add(key)
        if key not in blocks:
            raise KeyError(f"QStore has no block {key!r}")
        block = blocks[key]
        if not isinstance(block, Mapping):
            raise RuntimeError(f"QStore block {key!r} is not a mapping")
        if "alias" not in block:
            return block
        key = str(block["alias"])


def load_manifest(directory: str | Path) -> dict[str, Any]:
    directory = Path(directory)
    manifest = json.loads((directory / "manifest.json").read_text(encoding="utf-8"))
    if not isinstance(manifest, dict):
        raise RuntimeError("QStore manifest must be a JSON object")
    validate_int8_layout(directory, manifest)
    return manifest


# ------------------------------------------------------------------ prefetch ring


class _RingSlot:
    """One staging lane: pinned host buffers reused across prefetches, plus the device
    tensors of the block in flight and the event that marks its host-to-device copy."""

    __slots__ = ("pinned_q", "pinned_s", "dev_q", "dev_s", "event", "future", "name", "shape")

    def __init__(self) -> None:
        self.pinned_q: torch.Tensor | None = None
        self.pinned_s: torch.Tensor | None = None
        self.dev_q: torch.Tensor | None = None
        self.dev_s: torch.Tensor | None = None
        self.event: torch.cuda.Event | None = None  # kept across releases: the pinned
        self.future: Future | None = None           # buffers are reused only after it
        self.name: str | None = None
        self.shape: tuple[int, int] | None = None

    def release(self) -> None:
        self.dev_q = self.dev_s = None
        self.future = None
        self.name = None
        self.shape = None


class _PageRing:
    """Successor-oracle prefetch of qrow blocks (engine/kernels/qstore.py:485-660).

    ``observe(name)`` records that ``name`` followed the previous access and stages the
    ``depth`` predicted successors; ``take(name)`` hands back a staged block (waiting on its
    copy event from the caller's stream) or None. A mispredicted block is evicted when its
    slot is needed."""

    def __init__(self, store: "QStore", *, slots: int, depth: int) -> None:
        self.store = store
        self.depth = max(1, int(depth))
        self.device = store.device
        self.stream = torch.cuda.Stream(device=self.device)
        self.pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="qstore-ring")
        self.slots = [_RingSlot() for _ in range(max(2, int(slots)))]
        self.inflight: OrderedDict[str, _RingSlot] = OrderedDict()
        self.successor: dict[str, str] = {}
        self.last_access: str | None = None
        self.stats = {"hits": 0, "late_hits": 0, "misses": 0, "prefetches": 0, "staged": 0, "prefetch_bytes": 0,
                      "evicted_unused": 0, "successor_entries": 0}

    def preallocate(self, max_codes: int, max_rows: int) -> None:
        """Pinned buffers of every slot, allocated on the calling thread once."""
        for slot in self.slots:
            slot.pinned_q = torch.empty(max_codes, dtype=torch.int8, pin_memory=True)
            slot.pinned_s = torch.empty(max_rows, dtype=torch.float32, pin_memory=True)

    def close(self) -> None:
        for slot in self.inflight.values():
            if slot.future is not None:
                slot.future.result()
            slot.release()
        self.inflight.clear()
        self.pool.shutdown(wait=True)

    def take(self, name: str) -> tuple[torch.Tensor, torch.Tensor] | None:
        slot = self.inflight.pop(name, None)
        if slot is None:
            self.stats["misses"] += 1
            return None
        assert slot.future is not None
        self.stats["hits" if slot.future.done() else "late_hits"] += 1
        try:
            slot.future.result()  # staged and its copy issued (re-raises a staging error)
        except BaseException:
            slot.release()  # the slot serves the next prefetch; the error reaches the caller
            raise
        consumer = torch.cuda.current_stream(self.device)
        consumer.wait_event(slot.event)
        # allocated on the ring stream, used on the consumer's: keep the allocator from
        # handing the memory to the next prefetch while consumer kernels still read it
        slot.dev_q.record_stream(consumer)
        slot.dev_s.record_stream(consumer)
        rows, cols = slot.shape
        codes, scales = slot.dev_q.view(rows, cols), slot.dev_s
        slot.release()
        return codes, scales

    def observe(self, name: str) -> None:
        if self.last_access is not None and self.last_access != name:
            self.successor[self.last_access] = name
            self.stats["successor_entries"] = len(self.successor)
        self.last_access = name
        nxt: str | None = name
        for _ in range(self.depth):
            nxt = self.successor.get(nxt)
            if nxt is None:
                return
            self._prefetch(nxt)

    def _free_slot(self) -> _RingSlot | None:
        for slot in self.slots:
            if slot.name is None:
                return slot
        for key, slot in list(self.inflight.items()):  # oldest staged, never taken
            if slot.future is not None and slot.future.done():
                self.inflight.pop(key)
                slot.release()
                self.stats["evicted_unused"] += 1
                return slot
        return None

    def _prefetch(self, name: str) -> None:
        if name in self.inflight:
            return
        try:
            block = self.store._resolve(name)
        except KeyError:
            return
        if block.get("kind") != "qrow":
            return
        slot = self._free_slot()
        if slot is None:
            return
        rows, cols = (int(v) for v in block["shape"])
        slot.name, slot.shape = name, (rows, cols)
        slot.future = self.pool.submit(self._stage, slot, block)
        self.inflight[name] = slot
        self.stats["prefetches"] += 1
        self.stats["prefetch_bytes"] += rows * cols + rows * 4

    def _stage(self, slot: _RingSlot, block: Mapping[str, Any]) -> None:
        if slot.event is not None:
            slot.event.synchronize()  # the previous copy out of these pinned buffers is done
        rows, cols = slot.shape
        n = rows * cols
        self.store._read_block(block, slot.pinned_q, slot.pinned_s)
        with torch.cuda.stream(self.stream):
            slot.dev_q = torch.empty(n, dtype=torch.int8, device=self.device)
            slot.dev_q.copy_(slot.pinned_q[:n], non_blocking=True)
            slot.dev_s = torch.empty(rows, dtype=torch.float32, device=self.device)
            slot.dev_s.copy_(slot.pinned_s[:rows], non_blocking=True)
            slot.event = torch.cuda.Event()
            slot.event.record(self.stream)
        self.stats["staged"] += 1


# ------------------------------------------------------------------ resident page cache


class ResidentPageCache:
    """Byte-budgeted set of pages kept in HBM (engine/kernels/qstore.py:948-1006). Policy
    ``pin-fill`` (the reference's default) admits pages while they fit and never evicts: a
    decode loop touches blocks in a fixed cycle, where LRU under a budget smaller than the model
    evicts every block before its reuse while a static resident set keeps the budget's share.
    ``lru`` evicts the least recently used page. Here the cached pages are the int8 codes and
    row scales (what the kernels read), not fp32 expansions, so a budget holds 4x the weights."""

    POLICIES = ("pin-fill", "lru")

    def __init__(self, budget_bytes: int, policy: str = "pin-fill") -> None:
        if policy not in self.POLICIES:
            raise ValueError(f"unknown cache policy {policy!r}; expected one of {self.POLICIES}")
        self.budget = max(0, int(budget_bytes))
        self.policy = policy
        self.pages: OrderedDict[str, Any] = OrderedDict()
        self.bytes = 0
        self.stats = {"hits": 0, "admitted": 0, "evicted": 0, "rejected": 0}

    def get(self, name: str):
        entry = self.pages.get(name)
        if entry is None:
            return None
        self.pages.move_to_end(name)
        self.stats["hits"] += 1
        return entry[0]

    def put(self, name: str, page, nbytes: int) -> None:
        if self.budget <= 0 or name in self.pages:
            return
        if self.policy == "lru":
            if nbytes > self.budget:
                self.stats["rejected"] += 1
                return
            while self.bytes + nbytes > self.budget and self.pages:
                _, (_, old_bytes) = self.pages.popitem(last=False)
                self.bytes -= old_bytes
                self.stats["evicted"] += 1
        elif self.bytes + nbytes > self.budget:
            self.stats["rejected"] += 1
            return
        self.pages[name] = (page, nbytes)
        self.bytes += nbytes
        self.stats["admitted"] += 1


# ------------------------------------------------------------------ store


class QStore:
    """Paged int8 store on disk, served to the B200 kernels as device pages.

    Mirrors ``QStore`` (engine/kernels/qstore.py:662-1128) on its CUDA path: ``weight``
    returns the dequantised fp32 matrix exactly as the reference computes it on the device
    (``codes.float() * scales[:, None]``), while ``page`` / ``matmul`` keep the int8 codes and
    run the W8A16 kernel (``mrb_qrow_matmul``) without materialising fp32 weights."""

    def __init__(self, model_name: str, *, root: str | Path, device: str | torch.device = "cuda",
                 enable_prefetch_ring: bool = True, ring_slots: int = 3, ring_depth: int = 2,
                 read_threads: int = DEFAULT_READ_THREADS, drop_read_pages: bool = True) -> None:
        self.directory = (Path(root) / model_name).resolve()
        self.man = load_manifest(self.directory)
        self.blocks = self.man["blocks"]
        self.cfg = self.man["config"]
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("the B200 QStore serves CUDA devices only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.read_threads = int(read_threads)
        self.drop_read_pages = bool(drop_read_pages)
        self.w = StoreFile(self.directory / "weights.i8")
        self.s = StoreFile(self.directory / "scales.f32")
        self.e = StoreFile(self.directory / "extras.f32")
        self._ring: _PageRing | None = None
        self._cache: ResidentPageCache | None = None  # set_cache_budget() enables it
        self._miss_q: torch.Tensor | None = None  # pinned staging of direct (unprefetched) reads
        self._miss_s: torch.Tensor | None = None
        self._miss_event: torch.cuda.Event | None = None
        opts = store_options_from_env(ring=enable_prefetch_ring, ring_slots=ring_slots)
        if opts["ring"]:
            self.enable_ring(slots=opts["ring_slots"], depth=ring_depth)

    # ---- lifecycle

    def _max_qrow(self) -> tuple[int, int]:
        max_codes = max_rows = 1
        for block in self.blocks.values():
            if isinstance(block, Mapping) and block.get("kind") == "qrow":
                rows, cols = (int(v) for v in block["shape"])
                max_codes, max_rows = max(max_codes, rows * cols), max(max_rows, rows)
        return max_codes, max_rows

    def enable_ring(self, *, slots: int = 3, depth: int = 2) -> None:
        if self._ring is None:
            ring = _PageRing(self, slots=slots, depth=depth)
            ring.preallocate(*self._max_qrow())
            self._ring = ring

    def disable_ring(self) -> None:
        if self._ring is not None:
            self._ring.close()
            self._ring = None

    def ring_stats(self) -> dict[str, int] | None:
        return dict(self._ring.stats) if self._ring is not None else None

    def ring_allocated_bytes(self) -> int:
        """Pinned bytes the ring holds (device tensors are per prefetch)."""
        if self._ring is None:
            return 0
        return sum(t.numel() * t.element_size() for s in self._ring.slots for t in (s.pinned_q, s.pinned_s)
                   if t is not None)

    def close(self) -> None:
        self.disable_ring()
        self._cache = None
        if self._miss_event is not None:
            self._miss_event.synchronize()
        for f in (self.w, self.s, self.e):
            f.close()

    def __enter__(self) -> "QStore":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    # ---- blocks

    def _resolve(self, name: str) -> Mapping[str, Any]:
        return _resolve_in(self.blocks, name)

    def has(self, name: str) -> bool:
        return name in self.blocks

    def _read_block(self, block: Mapping[str, Any], pinned_q: torch.Tensor, pinned_s: torch.Tensor,
                    start: int = 0, end: int | None = None) -> None:
        """Rows [start, end) of a qrow block (all by default) into the pinned buffers."""
        total, cols = (int(v) for v in block["shape"])
        end = total if end is None else end
        rows = end - start
        self.w.read_into(int(block["w_off"]) + start * cols, rows * cols, pinned_q, threads=self.read_threads,
                         drop_after=self.drop_read_pages)
        self.s.read_into(int(block["s_off"]) + start * 4, rows * 4, pinned_s, drop_after=self.drop_read_pages)

    def _direct(self, block: Mapping[str, Any], start: int = 0,
                end: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Read rows [start, end) of a block (all by default) through the store's own pinned
        buffers and copy them on the current stream (the previous direct copy must have left
        those buffers first)."""
        total, cols = (int(v) for v in block["shape"])
        end = total if end is None else end
        rows = end - start
        n = rows * cols
        if self._miss_q is None or self._miss_q.numel() < n or self._miss_s.numel() < rows:
            max_codes, max_rows = self._max_qrow()
            if self._miss_event is not None:
                self._miss_event.synchronize()
            self._miss_q = torch.empty(max_codes, dtype=torch.int8, pin_memory=True)
            self._miss_s = torch.empty(max_rows, dtype=torch.float32, pin_memory=True)
        elif self._miss_event is not None:
            self._miss_event.synchronize()
        self._read_block(block, self._miss_q, self._miss_s, start, end)
        codes = torch.empty((rows, cols), dtype=torch.int8, device=self.device)
        scales = torch.empty(rows, dtype=torch.float32, device=self.device)
        codes.view(-1).copy_(self._miss_q[:n], non_blocking=True)
        scales.copy_(self._miss_s[:rows], non_blocking=True)
        self._miss_event = torch.cuda.Event()
        self._miss_event.record(torch.cuda.current_stream(self.device))
        return codes, scales

    def page(self, name: str) -> CompactQRowPage:
        """The int8 codes [out, in] and fp32 row scales of a qrow block, in HBM (through the
        ring when it predicted this block)."""
        block = self._resolve(name)
        if block.get("kind") != "qrow":
            raise ValueError(f"QStore block {name!r} is not a qrow block")
        rows, cols = (int(v) for v in block["shape"])
        cached = self._cache.get(name) if self._cache is not None else None
        if cached is not None:
            return cached
        hit = None
        if self._ring is not None:
            hit = self._ring.take(name)
            self._ring.observe(name)
        codes, scales = hit if hit is not None else self._direct(block)
        page = CompactQRowPage(name=name, start_row=0, end_row=rows, in_features=cols, codes=codes, scales=scales)
        if self._cache is not None:
            self._cache.put(name, page, rows * cols + rows * 4)
        return page

    def row_pages(self, name: str, bs: int = 8192):
        """Stream a qrow matrix in output-row chunks: yields (start, end, page of rows
        [start, end)) read straight from disk, so a head larger than the staging buffers never
        needs one whole-matrix copy. Chunks join the resident cache under ``name[start:end]``
        (engine/kernels/qstore.py:1130-1186)."""
        block = self._resolve(name)
        if block.get("kind") != "qrow":
            raise ValueError(f"QStore block {name!r} is not a qrow block")
        if bs < 1:
            raise ValueError("row block size must be positive")
        rows, cols = (int(v) for v in block["shape"])
        for start in range(0, rows, bs):
            end = min(start + bs, rows)
            key = f"{name}[{start}:{end}]"
            page = self._cache.get(key) if self._cache is not None else None
            if page is None:
                codes, scales = self._direct(block, start, end)
                page = CompactQRowPage(name=key, start_row=start, end_row=end, in_features=cols, codes=codes,
                                       scales=scales)
                if self._cache is not None:
                    self._cache.put(key, page, (end - start) * (cols + 4))
            yield start, end, page

    @torch.inference_mode()
    def row_blocks(self, name: str, bs: int = 8192):
        """``row_pages`` with each chunk dequantised to fp32 on the device (the reference's
        ``QStore.row_blocks`` contract, engine/kernels/qstore.py:1130-1186)."""
        for start, end, page in self.row_pages(name, bs):
            yield start, end, page.codes.float() * page.scales[:, None]

    def set_cache_budget(self, cache_mb: float, *, policy: str | None = None) -> None:
        """Keep up to `cache_mb` MB of pages resident in HBM (0 drops the cache); see
        ``ResidentPageCache`` for the policies (default from MRUN_QSTORE_CACHE_POLICY)."""
        budget = int(float(cache_mb) * 1e6)
        policy = store_options_from_env(cache_policy=policy)["cache_policy"]
        self._cache = ResidentPageCache(budget, policy) if budget > 0 else None

    def cache_stats(self) -> dict | None:
        return None if self._cache is None else {**self._cache.stats, "bytes": self._cache.bytes,
                                                 "budget": self._cache.budget, "policy": self._cache.policy}

    def matmul_row_stable(self, name: str, x: torch.Tensor) -> torch.Tensor:
        """``x @ weight(name).T`` with each row computed exactly as a one-row call would
        (engine/kernels/qstore.py:1094-1097): the page is loaded once and every row runs the
        M = 1 projection, so a row's bits never depend on the batch it came in."""
        page = self.page(name)
        flat = x.reshape(-1, x.shape[-1])
        rows = [qrow_linear(page.codes, page.scales, flat[i:i + 1]) for i in range(flat.shape[0])]
        out = torch.cat(rows) if rows else flat.new_empty((0, page.out_features))
        return out.reshape(*x.shape[:-1], page.out_features)

    @torch.inference_mode()
    def weight(self, name: str) -> torch.Tensor:
        """fp32 [out, in] = codes * row scale (engine/kernels/qstore.py:1026-1080, CUDA path)."""
        page = self.page(name)
        return page.codes.float() * page.scales[:, None]

    def matmul(self, name: str, x: torch.Tensor) -> torch.Tensor:
        """``x @ weight(name).T`` on the W8A16 kernel (the codes are never widened in HBM)."""
        page = self.page(name)
        return qrow_linear(page.codes, page.scales, x)

    def fp32(self, name: str) -> torch.Tensor:
        block = self._resolve(name)
        if block.get("kind") != "fp32":
            raise ValueError(f"QStore block {name!r} is not an fp32 block")
        shape = tuple(int(v) for v in block["shape"])
        host = np.empty(shape, dtype=np.float32)
        self.e.read_into(int(block["e_off"]), host.nbytes, host)
        return torch.from_numpy(host).to(self.device)

    @torch.inference_mode()
    def embed_rows(self, name: str, ids) -> torch.Tensor:
        """fp32 rows ``codes[ids] * scales[ids]`` reading only the requested rows from disk
        (engine/kernels/qstore.py:1099-1128). Out-of-range ids raise IndexError."""
        block = self._resolve(name)
        if block.get("kind") != "qrow":
            raise ValueError(f"QStore block {name!r} is not a qrow block")
        rows, cols = (int(v) for v in block["shape"])
        flat = np.asarray(ids, dtype=np.int64).reshape(-1)
        if flat.size and (flat.min() < 0 or flat.max() >= rows):
            raise IndexError("embedding id out of range")
        uniq, inverse = np.unique(flat, return_inverse=True)
        q = np.empty((uniq.size, cols), dtype=np.int8)
        sc = np.empty(uniq.size, dtype=np.float32)
        w_off, s_off = int(block["w_off"]), int(block["s_off"])
        for i, row in enumerate(uniq.tolist()):
            self.w.read_into(w_off + row * cols, cols, q[i])
            self.s.read_into(s_off + row * 4, 4, sc[i:i + 1])
        codes = torch.from_numpy(q).to(self.device)
        scales = torch.from_numpy(sc).to(self.device)
        out = codes.float() * scales[:, None]
        return out[torch.from_numpy(inverse).to(self.device)].reshape(*np.shape(ids), cols)
