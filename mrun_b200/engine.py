"""Engine entry points: ``open_engine`` and the dense QStore engine on the B200 kernels.

mrun opens its engines by backend name (engine/__init__.py:223-348, ``open_engine(model,
backend=..., fresh=False, **kwargs)``) and pools one warm instance per (model, backend,
kwargs). This module registers the B200 dense decoder under the reference's dense backend
names and keeps the same pooling rule (``fresh=True`` or ``MRUN_ENGINE_REUSE=0`` opens an
unshared instance). ``DenseQStoreCudaEngine`` keeps the generation surface of the reference's
engine of that name (engine/dense_qstore_cuda.py:1725, 2218-2478): ``prefill_ids``,
``generate_ids``, ``generate_batch``, ``generate``, ``runtime_stats``, ``close``. Weights come
from a ``DenseQStore`` (device int8 pages, never widened); prefill runs the paged flash
prefill kernel, decode the captured CUDA-graph step, greedy on the fused argmax head.
"""
from __future__ import annotations

import os
import threading
from collections.abc import Sequence
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np
import torch

DENSE_BACKENDS = ("dense-qstore-cuda", "dense_qstore_cuda", "dense-cuda")


@dataclass
class DensePrefillResult:
    """What a prefill produced: ``top1`` [batch, 1] greedy tokens after the last prompt
    position (the decoder keeps no full logits; its head fuses the argmax)."""

    top1: torch.Tensor
    token_count: int


@dataclass
class DenseSequenceCache:
    """The paged-KV sequences a prefill filled (slots of the engine's decoder)."""

    slots: list[int]
    lengths: list[int]

    @property
    def batch_size(self) -> int:
        return len(self.slots)


class DenseQStoreCudaEngine:
    """Greedy dense decoding over an on-disk int8 QStore on one B200."""

    def __init__(self, model_name: str, *, stores_dir: str | Path | None = None, store_path: str | Path | None = None,
                 device: str = "cuda", compute_dtype: str = "bf16", compact_cache_mb: float = 0.0,
                 max_seq_len: int = 128, stable_block_m: int = 16, max_batch: int = 8, max_prefill_tokens: int = 2048,
                 projection_mode: str = "w8a16") -> None:
        from .dense_engine import DenseDecoder, DenseWeights
        from .dense_store import DenseQStore

        if compute_dtype != "bf16":
            raise ValueError("the B200 dense engine computes in bf16")
        if store_path is not None:
            path = Path(store_path)
            root, name = path.parent, path.name
        elif stores_dir is not None:
            root, name = Path(stores_dir), model_name
        else:
            raise ValueError("give stores_dir or store_path")
        self.model_name = model_name
        self.store = DenseQStore(name, root=root, device=device, compute_dtype=compute_dtype,
                                 compact_cache_mb=compact_cache_mb, stable_block_m=stable_block_m)
        self.device = self.store.device
        # the decoder keeps every page it binds for its lifetime, so captured graphs never
        # see an address change (the store's LRU is not their owner)
        weights = DenseWeights.from_qstore(self.store)
        self.max_seq_len = int(max_seq_len)
        self.max_batch = int(max_batch)
        self.decoder = DenseDecoder(weights, max_batch=self.max_batch, max_seq_len=self.max_seq_len + 1,
                                    device=self.device, max_prefill_tokens=max_prefill_tokens, mode=projection_mode)
        self.cfg = weights.cfg
        self._calls = {"prefill_rows": 0, "prefill_tokens": 0, "decode_steps": 0, "generated_tokens": 0}

    # ---- prefill

    @torch.inference_mode()
    def prefill_ids(self, input_ids, *, return_logits: bool = False,
                    last_top1_only: bool = False) -> tuple[DenseSequenceCache, DensePrefillResult]:
        """Prefill each row of ``input_ids`` ([tokens] or [batch, tokens]) into its own KV
        sequence; returns the sequences and the greedy next token of each row."""
        if return_logits and last_top1_only:
            raise ValueError("last-top1 prefill cannot return logits")
        if return_logits:
            raise NotImplementedError("the B200 dense engine fuses the argmax into its head and returns no logits")
        rows = torch.as_tensor(np.asarray(input_ids), dtype=torch.long)
        if rows.ndim == 1:
            rows = rows[None, :]
        if rows.ndim != 2 or rows.shape[1] == 0:
            raise ValueError("input_ids must have shape [tokens] or [batch,tokens]")
        batch, tokens = (int(v) for v in rows.shape)
        if batch > self.max_batch:
            raise ValueError(f"batch {batch} exceeds the engine's max_batch={self.max_batch}")
        if tokens > self.max_seq_len:
            raise OverflowError("prompt exceeds max_seq_len")
        dec = self.decoder
        top1 = torch.empty(batch, 1, dtype=torch.long, device=self.device)
        for seq in range(batch):
            dec.kv.release(seq)
            top1[seq, 0] = dec.prefill(seq, rows[seq])
        self._calls["prefill_rows"] += batch
        self._calls["prefill_tokens"] += batch * tokens
        return DenseSequenceCache(list(range(batch)), [tokens] * batch), DensePrefillResult(top1, tokens)

    # ---- generation

    @torch.inference_mode()
    def generate_ids(self, input_ids, *, max_new_tokens: int = 48) -> torch.Tensor:
        """Greedy tokens [batch, max_new_tokens] (on the host) for equal-length prompts."""
        if max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be positive")
        rows = torch.as_tensor(np.asarray(input_ids), dtype=torch.long)
        if rows.ndim == 1:
            rows = rows[None, :]
        if rows.ndim != 2 or rows.shape[1] == 0:
            raise ValueError("input_ids must have shape [tokens] or [batch,tokens]")
        if int(rows.shape[1]) + max_new_tokens - 1 > self.max_seq_len:
            raise OverflowError("prompt and generated tokens exceed max_seq_len")
        cache, result = self.prefill_ids(rows, last_top1_only=True)
        batch = cache.batch_size
        out = [result.top1[:, 0].cpu()]
        if max_new_tokens > 1:
            dec = self.decoder
            for seq, length in zip(cache.slots, cache.lengths):
                dec.kv.reserve(seq, length + max_new_tokens)
            dec.row_seq[:batch].copy_(torch.tensor(cache.slots, dtype=torch.int32))
            dec.begin_decode(batch, result.top1[:, 0], cache.lengths)
            if dec.graph is None or dec.graph_rows != batch:
                dec.capture(batch)
            for _ in range(max_new_tokens - 1):
                dec.step()
                out.append(dec.next_ids[:batch].cpu())
            dec.check_errors()
            for seq, length in zip(cache.slots, cache.lengths):
                dec.kv.lengths[seq] = length + max_new_tokens - 1
            self._calls["decode_steps"] += max_new_tokens - 1
        self._calls["generated_tokens"] += batch * max_new_tokens
        return torch.stack(out, dim=1)

    def generate_batch(self, prompts: Sequence[Sequence[int] | np.ndarray], *, max_new_tokens: int = 48,
                       add_special_tokens: bool = False, eos_token_id: int | None = None,
                       return_text: bool = False) -> list[list[int]]:
        """Greedy continuations of token prompts, grouped by length (one prefill + captured
        decode per group), each cut after ``eos_token_id`` when given."""
        del add_special_tokens
        if return_text:
            raise NotImplementedError("the B200 engine takes and returns token ids (no tokenizer on this path)")
        encoded = []
        for prompt in prompts:
            if isinstance(prompt, str):
                raise TypeError("prompts must be token id sequences (no tokenizer on this path)")
            row = np.asarray(prompt, dtype=np.int64)
            if row.ndim != 1 or not row.size:
                raise ValueError("each prompt must produce a non-empty token row")
            encoded.append(row)
        outputs: list[list[int] | None] = [None] * len(encoded)
        by_length: dict[int, list[int]] = {}
        for i, row in enumerate(encoded):
            by_length.setdefault(int(row.size), []).append(i)
        for indices in by_length.values():
            for lo in range(0, len(indices), self.max_batch):
                part = indices[lo:lo + self.max_batch]
                tokens = self.generate_ids(np.stack([encoded[i] for i in part]), max_new_tokens=max_new_tokens)
                for i, row in zip(part, tokens.tolist()):
                    outputs[i] = [int(t) for t in row]
        done = []
        for row in outputs:
            assert row is not None
            if eos_token_id is not None and eos_token_id in row:
                row = row[: row.index(eos_token_id) + 1]
            done.append(row)
        return done

    def generate(self, prompt, *, max_new_tokens: int = 48, eos_token_id: int | None = None,
                 add_special_tokens: bool = False, return_text: bool = False) -> list[int]:
        return self.generate_batch([prompt], max_new_tokens=max_new_tokens, eos_token_id=eos_token_id,
                                   add_special_tokens=add_special_tokens, return_text=return_text)[0]

    def runtime_stats(self) -> dict[str, Any]:
        return {"backend": "b200-dense-qstore", "projection_mode": self.decoder.mode, **self._calls,
                "store": self.store.stats_snapshot()}

    def close(self) -> None:
        self.decoder.graph = None
        self.store.close()

    def __enter__(self) -> "DenseQStoreCudaEngine":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


_POOL: dict[tuple, Any] = {}
_POOL_LOCK = threading.Lock()


def _pool_key(model_name: str, backend: str, kwargs: dict[str, Any]) -> tuple | None:
    try:
        frozen = tuple(sorted((k, v if not isinstance(v, Path) else str(v)) for k, v in kwargs.items()))
        hash(frozen)
    except TypeError:
        return None  # unhashable options: not pooled
    return (model_name, backend, frozen)


def _open_impl(model_name: str, backend: str, kwargs: dict[str, Any]):
    name = backend.lower()
    if name in DENSE_BACKENDS:
        return DenseQStoreCudaEngine(model_name, **kwargs)
    raise ValueError(f"backend {backend!r} is not served by mrun_b200 (its dense backend names: "
                     f"{', '.join(DENSE_BACKENDS)}; MoE layers plug in through PagedInt8ExpertBackend.moe)")


def open_engine(model_name: str, *, backend: str = "dense-qstore-cuda", fresh: bool = False, **kwargs: Any):
    """Open (or reuse) an engine by backend name, as mrun's ``open_engine`` does: one warm
    instance per (model, backend, kwargs) unless ``fresh=True`` or MRUN_ENGINE_REUSE=0."""
    reuse = not fresh and os.environ.get("MRUN_ENGINE_REUSE", "1") != "0"
    key = _pool_key(model_name, backend.lower(), kwargs) if reuse else None
    if key is None:
        return _open_impl(model_name, backend, kwargs)
    with _POOL_LOCK:
        engine = _POOL.get(key)
        if engine is None:
            engine = _open_impl(model_name, backend, kwargs)
            _POOL[key] = engine
        return engine


def close_pooled_engines() -> None:
    """Close and forget every pooled engine."""
    with _POOL_LOCK:
        engines = list(_POOL.values())
        _POOL.clear()
    for engine in engines:
        engine.close()


__all__ = ["DENSE_BACKENDS", "DenseQStoreCudaEngine", "close_pooled_engines", "open_engine"]
