"""Dense QStore decoder oracle on the CPU (test infrastructure only).

Restates the fused-body forward of ``DenseQStoreTarget._forward_impl``
(engine/dense_qstore_cuda.py:927-1172) with the reference's CPU reference kernels:
  * embeddings: ``QStore.embed_rows`` fp32 dequant, then bf16 (:979-984)
  * projections: ``dequantized_reference_matmul`` — weights ``bf16(code * scale)``, fp32
    accumulation, bf16 output (engine/kernels/dense_qstore_cuda.py:1003-1013); bias added in
    bf16 (:1052-1056)
  * RoPE: ``_rope`` fp32 rotate-half, bf16 output (:689-704)
  * attention: causal GQA, fp32 softmax, bf16 output (:706-791)
  * residual + RMSNorm and paired SwiGLU with the reference's bf16 boundaries
  * head: the streamed exact head — fp32 hidden @ fp32 dequantised rows, first maximal
    index (:838-896)
``mode="w8a8"``: every body projection is the W8A8 store matmul of ``enable_w8a8``
(engine/kernels/w8a8.py:67-125, 145-177) — per-token int8 activations, exact int32
accumulation, ``(acc * s_x) * s_w`` in fp32, + fp32 bias, then the engine's bf16 boundary.
Torch on the CPU does the dense fp32 arithmetic, as the reference's CPU path does.
Weights come as a dict in QStore naming (``embed``, ``L{i}.q`` ... ``lm_head``), each a
``.codes`` int8 / ``.scales`` fp32 pair, plus fp32 ``L{i}.ln1``/``ln2``/``norm.final`` and
optional ``L{i}.{q,k,v}.bias``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


@dataclass
class OracleConfig:
    num_layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 1e6
    eps: float = 1e-6


class OracleDecoder:
    def __init__(self, cfg: OracleConfig, weights: dict[str, np.ndarray], *, threads: int | None = None,
                 mode: str = "w8a16") -> None:
        self.cfg = cfg
        self.w = weights
        self.mode = mode
        if threads:
            torch.set_num_threads(int(threads))
        self.k_cache: list[torch.Tensor] = []
        self.v_cache: list[torch.Tensor] = []
        self.length = 0

    # ---------------------------------------------------------------- primitives

    def _dequant(self, name: str) -> torch.Tensor:
        q = torch.from_numpy(self.w[name + ".codes"]).to(torch.float32)
        return q.mul_(torch.from_numpy(self.w[name + ".scales"])[:, None])

    def _linear(self, name: str, x: torch.Tensor) -> torch.Tensor:
        """bf16-valued x [T, in] -> bf16-valued [T, out] (the W8A16 contract, or W8A8)."""
        if self.mode == "w8a8":
            from .w8a8 import int8_gemm, quantize_activations

            qx, sx = quantize_activations(x.numpy())
            acc = int8_gemm(qx, self.w[name + ".codes"])
            y = (acc.astype(np.float32) * sx).astype(np.float32) * self.w[name + ".scales"][None, :]
            bias = self.w.get(name + ".bias")
            if bias is not None:
                y = (y + np.asarray(bias, np.float32)[None, :]).astype(np.float32)
            return _bf16(torch.from_numpy(np.ascontiguousarray(y, np.float32)))
        w = _bf16(self._dequant(name))
        y = _bf16(x @ w.T)
        bias = self.w.get(name + ".bias")
        if bias is not None:
            y = _bf16(y + _bf16(torch.from_numpy(bias))[None, :])
        return y

    def _rms(self, x: torch.Tensor, weight: str) -> torch.Tensor:
        inv = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.eps)
        return _bf16((x * inv) * torch.from_numpy(self.w[weight])[None, :])

    def _rope(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        d = self.cfg.head_dim
        inv = 1.0 / (self.cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
        freqs = positions.float()[:, None] * inv
        emb = torch.cat((freqs, freqs), dim=-1)
        cos, sin = emb.cos()[:, None, :], emb.sin()[:, None, :]
        half = d // 2
        rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
        return _bf16(x * cos + rot * sin)

    # ---------------------------------------------------------------- forward

    def reset(self) -> None:
        self.k_cache, self.v_cache, self.length = [], [], 0

    @torch.inference_mode()
    def forward(self, ids, *, all_logits: bool = False) -> torch.Tensor:
        """Append ``ids`` to the cached sequence; return fp32 logits of the last position
        (or of every new position with ``all_logits``)."""
        cfg = self.cfg
        ids = torch.as_tensor(np.asarray(ids, dtype=np.int64))
        t = int(ids.numel())
        start = self.length
        positions = torch.arange(start, start + t)
        emb = self._dequant_rows("embed", ids)
        hidden = _bf16(emb)
        normed = self._rms(hidden, "L0.ln1")
        group = cfg.heads // cfg.kv_heads
        for i in range(cfg.num_layers):
            q = self._linear(f"L{i}.q", normed).view(t, cfg.heads, cfg.head_dim)
            k = self._linear(f"L{i}.k", normed).view(t, cfg.kv_heads, cfg.head_dim)
            v = self._linear(f"L{i}.v", normed).view(t, cfg.kv_heads, cfg.head_dim)
            q = self._rope(q, positions)
            k = self._rope(k, positions)
            if len(self.k_cache) <= i:
                self.k_cache.append(k)
                self.v_cache.append(v)
            else:
                self.k_cache[i] = torch.cat((self.k_cache[i], k), 0)
                self.v_cache[i] = torch.cat((self.v_cache[i], v), 0)
            keys = self.k_cache[i].repeat_interleave(group, dim=1)  # [S, H, D]
            vals = self.v_cache[i].repeat_interleave(group, dim=1)
            scores = torch.einsum("thd,shd->hts", q, keys) * (1.0 / math.sqrt(cfg.head_dim))
            s_total = keys.shape[0]
            allowed = torch.arange(s_total)[None, :] <= positions[:, None]
            scores = scores.masked_fill(~allowed[None], float("-inf"))
            probs = torch.softmax(scores, dim=-1)
            ctx = _bf16(torch.einsum("hts,shd->thd", probs, vals)).reshape(t, cfg.heads * cfg.head_dim)
            o = self._linear(f"L{i}.o", ctx)
            hidden = _bf16(hidden + o)
            normed = self._rms(hidden, f"L{i}.ln2")
            g = self._linear(f"L{i}.gate", normed)
            u = self._linear(f"L{i}.up", normed)
            mlp = _bf16(_bf16(g * torch.sigmoid(g)) * u)
            down = self._linear(f"L{i}.down", mlp)
            hidden = _bf16(hidden + down)
            nxt = f"L{i + 1}.ln1" if i + 1 < cfg.num_layers else "norm.final"
            normed = self._rms(hidden, nxt)
        self.length += t
        head = self._dequant("lm_head")
        rows = normed if all_logits else normed[-1:]
        return rows @ head.T

    def _dequant_rows(self, name: str, ids: torch.Tensor) -> torch.Tensor:
        codes = torch.from_numpy(self.w[name + ".codes"][ids.numpy()]).to(torch.float32)
        return codes * torch.from_numpy(self.w[name + ".scales"][ids.numpy()])[:, None]

    def greedy(self, prompt, steps: int) -> list[int]:
        self.reset()
        logits = self.forward(prompt)
        out = [int(torch.argmax(logits[-1]))]
        for _ in range(steps - 1):
            logits = self.forward([out[-1]])
            out.append(int(torch.argmax(logits[-1])))
        return out

    def teacher_forced(self, prompt, tokens) -> tuple[list[int], list[float], list[float]]:
        """Score a token sequence chosen elsewhere: per step the oracle's argmax, its top-1
        minus the chosen token's logit, and the oracle's own top-1/top-2 margin."""
        self.reset()
        logits = self.forward(prompt)[-1]
        picks, gaps, margins = [], [], []
        for step, tok in enumerate(tokens):
            top2 = torch.topk(logits, 2)
            picks.append(int(top2.indices[0]))
            gaps.append(float(top2.values[0] - logits[int(tok)]))
            margins.append(float(top2.values[0] - top2.values[1]))
            if step + 1 < len(tokens):
                logits = self.forward([int(tok)])[-1]
        return picks, gaps, margins
