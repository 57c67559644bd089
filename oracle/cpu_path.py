"""The reference's CPU decode path, restated for timing on host cores (test/bench only).

mrun's CPU path (``paged_forward_kv``, engine/kernels/paged_forward.py:1015-1107) runs the
whole model in fp32: every projection dequantises its int8 block to fp32
(``_dequant_qrow``, engine/kernels/qstore.py:385-399: widen, then one in-place multiply by the
row scale) and multiplies (``QStore.matmul``, :1082-1092); the head streams 8192-row blocks
(:1130-1185). This module reproduces that arithmetic and memory traffic with torch on the
CPU. It is the CPU baseline of bench.py; it is never a product path.
"""
from __future__ import annotations

import math

import numpy as np
import torch

HEAD_BLOCK = 8192


class CpuPathDecoder:
    def __init__(self, *, num_layers, hidden, heads, kv_heads, head_dim, ffn, vocab, weights,
                 rope_theta=1e6, eps=1e-6) -> None:
        self.num_layers = num_layers
        self.hidden = hidden
        self.heads = heads
        self.kv_heads = kv_heads
        self.head_dim = head_dim
        self.ffn = ffn
        self.vocab = vocab
        self.w = weights
        self.rope_theta = rope_theta
        self.eps = eps
        self.keys: list[torch.Tensor] = []
        self.values: list[torch.Tensor] = []
        self.length = 0

    @classmethod
    def synthetic_qwen25_7b(cls, seed: int = 0) -> "CpuPathDecoder":
        """Qwen2.5-7B-shape int8 weights with plausible per-row scales. Codes tile one
        seeded 64 MiB random block (the timing does not depend on code values)."""
        h, f, v, hq, hkv, d, layers = 3584, 18944, 152064, 28, 4, 128, 28
        rng = np.random.default_rng(seed)
        block = torch.from_numpy(rng.integers(-127, 128, size=64 << 20, dtype=np.int8))

        def codes(rows, cols):
            n = rows * cols
            out = torch.empty(n, dtype=torch.int8)
            whole = n // block.numel()
            if whole:  # broadcast copy: multi-threaded in torch
                out[: whole * block.numel()].view(whole, -1).copy_(block.expand(whole, -1))
            rest = n - whole * block.numel()
            if rest:
                out[whole * block.numel():].copy_(block[:rest])
            return out.view(rows, cols).numpy()

        def scales(rows):
            return (rng.random(rows, dtype=np.float32) * 2e-4 + 6e-4).astype(np.float32)

        w: dict[str, np.ndarray] = {}
        for name, rows, cols in (("embed", v, h), ("lm_head", v, h)):
            w[name + ".codes"], w[name + ".scales"] = codes(rows, cols), scales(rows)
        w["norm.final"] = np.ones(h, np.float32)
        for i in range(layers):
            for name, rows, cols in (("q", hq * d, h), ("k", hkv * d, h), ("v", hkv * d, h), ("o", h, hq * d),
                                     ("gate", f, h), ("up", f, h), ("down", h, f)):
                w[f"L{i}.{name}.codes"], w[f"L{i}.{name}.scales"] = codes(rows, cols), scales(rows)
            for name, n in (("q", hq * d), ("k", hkv * d), ("v", hkv * d)):
                w[f"L{i}.{name}.bias"] = (rng.standard_normal(n) * 0.02).astype(np.float32)
            w[f"L{i}.ln1"] = np.ones(h, np.float32)
            w[f"L{i}.ln2"] = np.ones(h, np.float32)
        return cls(num_layers=layers, hidden=h, heads=hq, kv_heads=hkv, head_dim=d, ffn=f, vocab=v, weights=w)

    def _dequant(self, name: str, start: int | None = None, end: int | None = None) -> torch.Tensor:
        q = self.w[name + ".codes"]
        s = self.w[name + ".scales"]
        if start is not None:
            q, s = q[start:end], s[start:end]
        weight = torch.from_numpy(np.ascontiguousarray(q)).to(torch.float32)
        weight.mul_(torch.from_numpy(np.ascontiguousarray(s))[:, None])
        return weight

    def _matmul(self, name: str, x: torch.Tensor) -> torch.Tensor:
        y = x @ self._dequant(name).T
        bias = self.w.get(name + ".bias")
        if bias is not None:
            y = y + torch.from_numpy(bias)
        return y

    def _rms(self, x: torch.Tensor, name: str) -> torch.Tensor:
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * torch.from_numpy(self.w[name])

    def _rope(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        d = self.head_dim
        inv = 1.0 / (self.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        emb = torch.cat((positions.float()[:, None] * inv,) * 2, dim=-1)
        half = d // 2
        rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
        return x * emb.cos()[:, None, :] + rot * emb.sin()[:, None, :]

    # ---------------------------------------------------------------- timing units

    def head_blocks(self) -> int:
        return (self.vocab + HEAD_BLOCK - 1) // HEAD_BLOCK

    def units(self) -> int:
        """One decode token = num_layers layer units + the head's 8192-row block units."""
        return self.num_layers + self.head_blocks()

    def prepare_context(self, context: int, seed: int = 0) -> None:
        """Random committed K/V of ``context`` positions per layer (the decode step's reads)."""
        g = torch.Generator().manual_seed(seed)
        self.keys = [torch.randn(context, self.kv_heads, self.head_dim, generator=g) for _ in range(self.num_layers)]
        self.values = [torch.randn(context, self.kv_heads, self.head_dim, generator=g) for _ in range(self.num_layers)]
        self.length = context

    @torch.inference_mode()
    def run_unit(self, unit: int, x: torch.Tensor) -> torch.Tensor:
        """Execute one unit of a one-token decode step at the prepared context; returns the
        next hidden state (layer units) or the block's logits (head units). K/V are read
        but not appended so units can be repeated."""
        if unit < self.num_layers:
            i = unit
            pos = torch.tensor([self.length])
            h = self._rms(x, f"L{i}.ln1")
            q = self._rope(self._matmul(f"L{i}.q", h).view(1, self.heads, self.head_dim), pos)
            k = self._rope(self._matmul(f"L{i}.k", h).view(1, self.kv_heads, self.head_dim), pos)
            v = self._matmul(f"L{i}.v", h).view(1, self.kv_heads, self.head_dim)
            group = self.heads // self.kv_heads
            keys = torch.cat((self.keys[i], k)).repeat_interleave(group, dim=1)
            vals = torch.cat((self.values[i], v)).repeat_interleave(group, dim=1)
            probs = torch.softmax(torch.einsum("thd,shd->hts", q, keys) / math.sqrt(self.head_dim), dim=-1)
            ctx = torch.einsum("hts,shd->thd", probs, vals).reshape(1, -1)
            x = x + self._matmul(f"L{i}.o", ctx)
            h = self._rms(x, f"L{i}.ln2")
            mlp = torch.nn.functional.silu(self._matmul(f"L{i}.gate", h)) * self._matmul(f"L{i}.up", h)
            return x + self._matmul(f"L{i}.down", mlp)
        b = unit - self.num_layers
        start, end = b * HEAD_BLOCK, min((b + 1) * HEAD_BLOCK, self.vocab)
        return self._rms(x, "norm.final") @ self._dequant("lm_head", start, end).T

    @torch.inference_mode()
    def forward(self, ids) -> torch.Tensor:
        ids = np.asarray(ids, dtype=np.int64).reshape(-1)
        t = ids.size
        positions = torch.arange(self.length, self.length + t)
        q = self.w["embed.codes"][ids].astype(np.float32) * self.w["embed.scales"][ids][:, None]
        hidden = torch.from_numpy(q)
        group = self.heads // self.kv_heads
        for i in range(self.num_layers):
            x = self._rms(hidden, f"L{i}.ln1")
            q = self._rope(self._matmul(f"L{i}.q", x).view(t, self.heads, self.head_dim), positions)
            k = self._rope(self._matmul(f"L{i}.k", x).view(t, self.kv_heads, self.head_dim), positions)
            v = self._matmul(f"L{i}.v", x).view(t, self.kv_heads, self.head_dim)
            if len(self.keys) <= i:
                self.keys.append(k)
                self.values.append(v)
            else:
                self.keys[i] = torch.cat((self.keys[i], k))
                self.values[i] = torch.cat((self.values[i], v))
            keys = self.keys[i].repeat_interleave(group, dim=1)
            vals = self.values[i].repeat_interleave(group, dim=1)
            scores = torch.einsum("thd,shd->hts", q, keys) / math.sqrt(self.head_dim)
            allowed = torch.arange(keys.shape[0])[None, :] <= positions[:, None]
            probs = torch.softmax(scores.masked_fill(~allowed[None], float("-inf")), dim=-1)
            ctx = torch.einsum("hts,shd->thd", probs, vals).reshape(t, -1)
            hidden = hidden + self._matmul(f"L{i}.o", ctx)
            x = self._rms(hidden, f"L{i}.ln2")
            mlp = torch.nn.functional.silu(self._matmul(f"L{i}.gate", x)) * self._matmul(f"L{i}.up", x)
            hidden = hidden + self._matmul(f"L{i}.down", mlp)
        self.length += t
        x = self._rms(hidden[-1:], "norm.final")
        logits = torch.empty(1, self.vocab)
        for start in range(0, self.vocab, HEAD_BLOCK):
            end = min(start + HEAD_BLOCK, self.vocab)
            logits[:, start:end] = x @ self._dequant("lm_head", start, end).T
        return logits
