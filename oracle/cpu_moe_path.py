"""The routed-MoE decode step on the CPU, for timing on host cores (bench only; never a product
path, and not a parity oracle -- oracle/moe_decoder.py is that).

It runs one greedy decode token for every row of a ragged batch the way mrun's MoE runtime
does on a CPU device (``Qwen3MoeDecodeRuntime.forward_decode_rows``,
engine/qwen3_moe_cuda.py:3790-3960, with ``dtype=float32``): dense projections (q/k/v, o,
router, head) are fp32 matrices held in memory, attention is per row over its own committed
K/V with per-head q/k RMSNorm and RoPE, the router is softmax/top-k/renorm, and each expert a
row routes to is dequantised from its int8 page (``codes * scale`` in fp32, the
``_dequant_qrow`` arithmetic of engine/kernels/qstore.py:385-399) once per layer and applied
to all of that expert's rows (SwiGLU), then the k outputs are added in route-rank order
(engine/qwen3_moe_cuda.py:2654-2664). The reference has no CPU expert kernel of its own, so
this is the restatement its CPU runtime would execute with an int8 expert store.
"""
from __future__ import annotations

import math

import torch


class CpuMoePathDecoder:
    def __init__(self, *, num_layers: int, hidden: int, heads: int, kv_heads: int, head_dim: int, experts: int,
                 top_k: int, expert_ffn: int, vocab: int, rope_theta: float = 1e6, eps: float = 1e-6,
                 seed: int = 0) -> None:
        self.L, self.h, self.hq, self.hkv, self.d = num_layers, hidden, heads, kv_heads, head_dim
        self.e, self.k, self.f, self.v = experts, top_k, expert_ffn, vocab
        self.theta, self.eps = rope_theta, eps
        g = torch.Generator().manual_seed(seed)
        std = 0.02
        # dense weights: one random fp32 set shared by every layer (the timing depends only on
        # the bytes each layer reads, and a shared set keeps host memory small); expert pages
        # are distinct per (layer, expert) since they are what a decode step streams
        qkv_rows = (heads + 2 * kv_heads) * head_dim
        self.qkv = torch.randn(qkv_rows, hidden, generator=g) * std
        self.o = torch.randn(hidden, heads * head_dim, generator=g) * std
        self.router = torch.randn(experts, hidden, generator=g) * 0.05
        self.head = torch.randn(vocab, hidden, generator=g) * std
        self.embed = torch.randn(vocab, hidden, generator=g)
        block = torch.randint(-127, 128, (1 << 26,), dtype=torch.int8, generator=g)
        per = 3 * expert_ffn * hidden
        self.codes = []  # [layer][expert] -> (gate_up int8 [2F, H], down int8 [H, F]) views of one block
        for layer in range(num_layers):
            row = []
            for ex in range(experts):
                start = ((layer * experts + ex) * 7919 * 4096) % (block.numel() - per)
                flat = block[start:start + per]
                row.append((flat[: 2 * expert_ffn * hidden].view(2 * expert_ffn, hidden),
                            flat[2 * expert_ffn * hidden:].view(hidden, expert_ffn)))
            self.codes.append(row)
        self.gu_scale = torch.full((2 * expert_ffn,), std / 73.6)
        self.dn_scale = torch.full((hidden,), std / 73.6)
        self.k_cache: list[list[torch.Tensor]] = []
        self.v_cache: list[list[torch.Tensor]] = []

    @classmethod
    def qwen3_30b_a3b(cls, seed: int = 0) -> "CpuMoePathDecoder":
        return cls(num_layers=48, hidden=2048, heads=32, kv_heads=4, head_dim=128, experts=128, top_k=8,
                   expert_ffn=768, vocab=151936, seed=seed)

    def set_context(self, lengths: list[int], seed: int = 0) -> None:
        """Random committed K/V of the given lengths for each row (a stand-in for prefill). One
        set serves every layer: each layer still reads all of it (far more than the host's
        last-level cache), and 48 separate fp32 copies would not fit a host's memory."""
        g = torch.Generator().manual_seed(seed)
        keys = [torch.randn(n, self.hkv, self.d, generator=g) for n in lengths]
        vals = [torch.randn(n, self.hkv, self.d, generator=g) for n in lengths]
        self.k_cache = [keys] * self.L
        self.v_cache = [vals] * self.L
        self.lengths = list(lengths)

    def _rms(self, x: torch.Tensor) -> torch.Tensor:
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps)

    def _rope(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        d = self.d
        inv = 1.0 / (self.theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        emb = torch.cat((pos.float()[:, None] * inv,) * 2, dim=-1)[:, None, :]
        half = d // 2
        rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
        return x * emb.cos() + rot * emb.sin()

    def units(self) -> int:
        """One decode step = num_layers layer units + one head unit."""
        return self.L + 1

    def embed_rows(self, ids: torch.Tensor) -> torch.Tensor:
        return self.embed[ids]

    @torch.inference_mode()
    def run_unit(self, unit: int, x: torch.Tensor) -> torch.Tensor:
        """Layer ``unit`` for every row (K/V read, not appended, so units repeat), returning the
        next hidden states; the last unit is the head, returning greedy ids."""
        if unit == self.L:
            return torch.argmax(self._rms(x) @ self.head.T, dim=-1)
        li, rows = unit, x.shape[0]
        pos = torch.tensor(self.lengths)
        group = self.hq // self.hkv
        h = self._rms(x)
        qkv = h @ self.qkv.T
        q = qkv[:, : self.hq * self.d].view(rows, self.hq, self.d)
        k = qkv[:, self.hq * self.d: (self.hq + self.hkv) * self.d].view(rows, self.hkv, self.d)
        v = qkv[:, (self.hq + self.hkv) * self.d:].view(rows, self.hkv, self.d)
        q = self._rope(self._rms(q), pos)
        k = self._rope(self._rms(k), pos)
        ctx = torch.empty(rows, self.hq, self.d)
        for r in range(rows):
            keys = torch.cat((self.k_cache[li][r], k[r:r + 1])).repeat_interleave(group, dim=1)
            vals = torch.cat((self.v_cache[li][r], v[r:r + 1])).repeat_interleave(group, dim=1)
            sc = torch.einsum("hd,shd->hs", q[r], keys) / math.sqrt(self.d)
            ctx[r] = torch.einsum("hs,shd->hd", torch.softmax(sc, dim=-1), vals)
        x = x + ctx.reshape(rows, -1) @ self.o.T
        h = self._rms(x)
        probs = torch.softmax(h @ self.router.T, dim=-1)
        w, idx = torch.topk(probs, self.k, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        out = torch.zeros(rows, self.k, self.h)
        for ex in torch.unique(idx).tolist():
            r_idx, slot = (idx == ex).nonzero(as_tuple=True)
            gu_codes, dn_codes = self.codes[li][ex]
            w_gu = gu_codes.float() * self.gu_scale[:, None]  # dequantise the page (fp32)
            w_dn = dn_codes.float() * self.dn_scale[:, None]
            gu = h[r_idx] @ w_gu.T
            a = torch.nn.functional.silu(gu[:, : self.f]) * gu[:, self.f:]
            out[r_idx, slot] = (a @ w_dn.T) * w[r_idx, slot][:, None]
        acc = out[:, 0]
        for r in range(1, self.k):  # the k expert outputs added in route-rank order
            acc = acc + out[:, r]
        return x + acc

    @torch.inference_mode()
    def step(self, ids: torch.Tensor) -> torch.Tensor:
        """One greedy token for every row; returns the next ids."""
        x = self.embed_rows(ids)
        for unit in range(self.units()):
            x = self.run_unit(unit, x)
        return x


__all__ = ["CpuMoePathDecoder"]
