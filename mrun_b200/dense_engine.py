"""Dense QStore decoder on B200: the engine loop around the hot-path kernels.

Mirrors ``DenseQStoreTarget._forward_impl`` (engine/dense_qstore_cuda.py:927-1172) in its
fused-body mode — RMSNorm, W8A16 q|k|v (+ bias), RoPE, attention, o-projection, residual +
RMSNorm, paired gate/up SwiGLU, down-projection, residual + RMSNorm into the next layer's
norm — and the greedy loop of ``DenseQStoreCudaEngine.generate_ids`` (:2389-2416). The KV
cache is block-paged (16-token pages). The one-token decode step is captured once in a CUDA
graph and replays with no host work; the greedy head computes exact fp32 logits and takes
the first maximal index on the device.

Weights live in HBM as int8 codes + fp32 row scales (the QStore ``qrow`` layout); q/k/v are
stored as one concatenated page so one GEMV streams all three.

``mode="w8a8"`` runs every body projection as the W8A8 store matmul of ``enable_w8a8``
(engine/kernels/w8a8.py:145-177): per-token int8 activations, exact int32 accumulation on the
tensor cores (split over k in clusters for skinny row blocks), fp32 rescale (+ fp32 bias), one bf16
rounding; gate/up stay paired with the SwiGLU epilogue. The greedy head keeps the exact fp32
head of ``_head`` (engine/dense_qstore_cuda.py:800-896).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from .dense_qstore_cuda import (qrow_argmax, qrow_linear, qrow_swiglu, qrow_workspace_bytes, residual_rms_norm_into,
                                rms_norm_into)
from .paged_kv import PagedKVCache
from .qstore_build import embed_rows, quant_row_int8
from .w8a8 import w8a8_linear_bf16


@dataclass(frozen=True)
class DenseConfig:
    num_layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 1e6
    eps: float = 1e-6
    qkv_bias: bool = True

    @classmethod
    def qwen25_7b(cls) -> "DenseConfig":
        """Qwen2.5-7B shape: 28 layers, hidden 3584, 28/4 heads, FFN 18944, vocab 152064."""
        return cls(num_layers=28, hidden=3584, heads=28, kv_heads=4, head_dim=128, ffn=18944, vocab=152064)

    @classmethod
    def from_hf_config(cls, config: dict, *, qkv_bias: bool = True) -> "DenseConfig":
        """From the Hugging Face config a QStore manifest carries (its ``config`` entry)."""
        heads = int(config["num_attention_heads"])
        hidden = int(config["hidden_size"])
        return cls(num_layers=int(config["num_hidden_layers"]), hidden=hidden, heads=heads,
                   kv_heads=int(config.get("num_key_value_heads", heads)),
                   head_dim=int(config.get("head_dim") or hidden // heads), ffn=int(config["intermediate_size"]),
                   vocab=int(config["vocab_size"]), rope_theta=float(config.get("rope_theta", 1e6)),
                   eps=float(config.get("rms_norm_eps", 1e-6)), qkv_bias=qkv_bias)

    @property
    def qkv_rows(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    def weight_bytes(self) -> dict[str, int]:
        """int8 code + fp32 scale bytes read by one decode step (embedding rows excluded)."""
        h, f = self.hidden, self.ffn
        per_layer = self.qkv_rows * h + h * self.heads * self.head_dim + 2 * f * h + h * f
        per_layer_scales = 4 * (self.qkv_rows + h + 2 * f + h)
        head = self.vocab * h
        return {
            "body": self.num_layers * per_layer,
            "head": head,
            "scales": self.num_layers * per_layer_scales + 4 * self.vocab,
        }


@dataclass
class QRow:
    codes: torch.Tensor  # int8 [rows, cols]
    scales: torch.Tensor  # fp32 [rows]


@dataclass
class DenseLayer:
    qkv: QRow
    qkv_bias: torch.Tensor | None
    o: QRow
    gate: QRow
    up: QRow
    down: QRow
    ln1: torch.Tensor
    ln2: torch.Tensor


@dataclass
class DenseWeights:
    cfg: DenseConfig
    embed: QRow
    layers: list[DenseLayer]
    final_norm: torch.Tensor
    head: QRow
    extras: dict = field(default_factory=dict)

    @staticmethod
    @torch.inference_mode()
    def from_blocks(cfg: DenseConfig, qrow, fp32, has) -> "DenseWeights":
        """Assemble the decoder's weights from QStore blocks under the reference's canonical
        names (engine/kernels/qstore_build.py:257-276, 340-360): ``L{i}.q/k/v/o/gate/up/down``
        (qrow), ``L{i}.q.bias/k.bias/v.bias``, ``L{i}.ln1/ln2``, ``norm.final`` (fp32; ``norm`` is
        accepted too), ``embed``,
        ``lm_head`` (qrow, often an alias of ``embed``). ``qrow(name)`` returns (int8 codes,
        fp32 scales) and ``fp32(name)`` a float32 tensor, both on the target device; ``has``
        tells whether a block exists. q, k and v are stacked into one [(Hq + 2 Hkv) D, H] page."""
        layers = []
        for i in range(cfg.num_layers):
            parts = [qrow(f"L{i}.{p}") for p in ("q", "k", "v")]
            qkv = QRow(torch.cat([c for c, _ in parts]).contiguous(), torch.cat([s for _, s in parts]).contiguous())
            if qkv.codes.shape != (cfg.qkv_rows, cfg.hidden):
                raise ValueError(f"layer {i}: q/k/v blocks give {tuple(qkv.codes.shape)}, "
                                 f"expected {(cfg.qkv_rows, cfg.hidden)}")
            bias = None
            if cfg.qkv_bias and has(f"L{i}.q.bias"):
                bias = torch.cat([fp32(f"L{i}.{p}.bias").reshape(-1) for p in ("q", "k", "v")]).contiguous()
            layers.append(DenseLayer(qkv=qkv, qkv_bias=bias, o=QRow(*qrow(f"L{i}.o")), gate=QRow(*qrow(f"L{i}.gate")),
                                     up=QRow(*qrow(f"L{i}.up")), down=QRow(*qrow(f"L{i}.down")),
                                     ln1=fp32(f"L{i}.ln1").reshape(-1).contiguous(),
                                     ln2=fp32(f"L{i}.ln2").reshape(-1).contiguous()))
        embed = QRow(*qrow("embed"))
        head = QRow(*qrow("lm_head" if has("lm_head") else "embed"))
        if embed.codes.shape != (cfg.vocab, cfg.hidden) or head.codes.shape[1] != cfg.hidden:
            raise ValueError("embedding / head blocks do not match the config")
        final = "norm.final" if has("norm.final") else "norm"
        return DenseWeights(cfg=cfg, embed=embed, layers=layers, final_norm=fp32(final).reshape(-1).contiguous(),
                            head=head)

    @staticmethod
    def from_qstore(store, cfg: DenseConfig | None = None) -> "DenseWeights":
        """Load a dense decoder from an on-disk int8 QStore (``mrun_b200.qstore.QStore``): the
        int8 pages go to HBM as they are (no fp32 weight copy)."""
        cfg = cfg or DenseConfig.from_hf_config(store.cfg)

        def qrow(name):
            page = store.page(name)
            return page.codes, page.scales

        return DenseWeights.from_blocks(cfg, qrow, store.fp32, store.has)

    @staticmethod
    @torch.inference_mode()
    def synthetic(cfg: DenseConfig, device: torch.device, seed: int = 0) -> "DenseWeights":
        """Random-init N(0, 0.02) matrices quantised per output channel on the device
        (bit-identical to the reference quantiser), N(0, 0.02) biases, unit norm weights."""
        gen = torch.Generator(device=device)
        counter = [seed * 1000003]

        def mat(rows: int, cols: int) -> QRow:
            gen.manual_seed(counter[0])
            counter[0] += 1
            w = torch.randn((rows, cols), generator=gen, device=device, dtype=torch.float32).mul_(0.02)
            codes, scales = quant_row_int8(w)
            del w
            return QRow(codes, scales)

        def vec(n: int) -> torch.Tensor:
            gen.manual_seed(counter[0])
            counter[0] += 1
            return torch.randn((n,), generator=gen, device=device, dtype=torch.float32).mul_(0.02)

        h = cfg.hidden
        embed = mat(cfg.vocab, h)
        layers = []
        for _ in range(cfg.num_layers):
            layers.append(
                DenseLayer(
                    qkv=mat(cfg.qkv_rows, h),
                    qkv_bias=vec(cfg.qkv_rows) if cfg.qkv_bias else None,
                    o=mat(h, cfg.heads * cfg.head_dim),
                    gate=mat(cfg.ffn, h),
                    up=mat(cfg.ffn, h),
                    down=mat(h, cfg.ffn),
                    ln1=torch.ones(h, device=device),
                    ln2=torch.ones(h, device=device),
                )
            )
        head = mat(cfg.vocab, h)
        return DenseWeights(cfg, embed, layers, torch.ones(h, device=device), head)

    def to_host(self) -> dict[str, np.ndarray]:
        """Host copies in QStore naming (``L{i}.q|k|v|o|gate|up|down``) for the CPU oracle."""
        cfg = self.cfg
        out: dict[str, np.ndarray] = {}

        def put(name: str, q: QRow) -> None:
            out[name + ".codes"] = q.codes.cpu().numpy()
            out[name + ".scales"] = q.scales.cpu().numpy()

        put("embed", self.embed)
        put("lm_head", self.head)
        out["norm.final"] = self.final_norm.cpu().numpy()
        qd, kd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        for i, layer in enumerate(self.layers):
            codes = layer.qkv.codes.cpu().numpy()
            scales = layer.qkv.scales.cpu().numpy()
            for name, lo, hi in (("q", 0, qd), ("k", qd, qd + kd), ("v", qd + kd, qd + 2 * kd)):
                out[f"L{i}.{name}.codes"] = codes[lo:hi]
                out[f"L{i}.{name}.scales"] = scales[lo:hi]
                if layer.qkv_bias is not None:
                    out[f"L{i}.{name}.bias"] = layer.qkv_bias[lo:hi].cpu().numpy()
            put(f"L{i}.o", layer.o)
            put(f"L{i}.gate", layer.gate)
            put(f"L{i}.up", layer.up)
            put(f"L{i}.down", layer.down)
            out[f"L{i}.ln1"] = layer.ln1.cpu().numpy()
            out[f"L{i}.ln2"] = layer.ln2.cpu().numpy()
        return out


# Decode batches with at most this many (row, KV head) pairs run RoPE + KV append + attention
# as one clustered launch per layer; larger batches keep the tensor-core split-K attention.
FUSED_DECODE_MAX_GROUPS = 32


def rope_tables(head_dim: int, theta: float, length: int, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [length, head_dim/2] computed with the reference's fp32 torch recipe
    (engine/dense_qstore_cuda.py:689-704) on the host, then uploaded."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    freqs = torch.arange(length, dtype=torch.float32)[:, None] * inv
    return freqs.cos().contiguous().to(device), freqs.sin().contiguous().to(device)


class DenseDecoder:
    """Prefill + greedy decode of a dense QStore model on one GPU."""

    def __init__(
        self,
        weights: DenseWeights,
        *,
        max_batch: int,
        max_seq_len: int,
        device: torch.device,
        num_pages: int | None = None,
        max_prefill_tokens: int = 2048,
        mode: str = "w8a16",
    ) -> None:
        if mode not in ("w8a16", "w8a8"):
            raise ValueError(f"unknown projection mode {mode!r}")
        self.mode = mode
        self.w = weights
        self.cfg = cfg = weights.cfg
        self.device = device
        self.max_batch = int(max_batch)
        self.max_seq_len = int(max_seq_len)
        pages_per_seq = (self.max_seq_len + 15) // 16
        self.kv = PagedKVCache(
            num_layers=cfg.num_layers,
            num_pages=num_pages if num_pages is not None else pages_per_seq * self.max_batch,
            kv_heads=cfg.kv_heads,
            head_dim=cfg.head_dim,
            max_seqs=self.max_batch,
            max_pages_per_seq=pages_per_seq,
            device=device,
        )
        self.cos, self.sin = rope_tables(cfg.head_dim, cfg.rope_theta, self.max_seq_len, device)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.max_prefill_tokens = int(max_prefill_tokens)
        rows = max(self.max_batch, self.max_prefill_tokens)
        # the split plan depends on the row count: size for the worst row count we will run
        ws = max(self.kv.workspace_bytes(r, cfg.heads, self.max_seq_len) for r in range(1, rows + 1))
        self.workspace = torch.zeros(max(ws, 256), dtype=torch.uint8, device=device)
        # GEMV stream-K workspace shared by every projection (all ordered on one stream)
        gemv_ws = max(qrow_workspace_bytes(device, n) for n in (cfg.qkv_rows, cfg.hidden, cfg.ffn))
        self.gemv_workspace = torch.zeros(gemv_ws, dtype=torch.uint8, device=device)
        if mode == "w8a8":
            # per-token int8 activations of the projection being run (all ordered on one stream)
            self.w8_qx = torch.empty(rows, max(cfg.hidden, cfg.ffn, cfg.heads * cfg.head_dim), dtype=torch.int8,
                                     device=device)
            self.w8_scale = torch.empty(rows, dtype=torch.float32, device=device)
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=device)
        bf = torch.bfloat16
        h = cfg.hidden
        self.buf = {
            "hidden": torch.empty(rows, h, dtype=bf, device=device),
            "normed": torch.empty(rows, h, dtype=bf, device=device),
            "qkv": torch.empty(rows, cfg.qkv_rows, dtype=bf, device=device),
            "q": torch.empty(rows, cfg.heads, cfg.head_dim, dtype=bf, device=device),
            "ctx": torch.empty(rows, cfg.heads, cfg.head_dim, dtype=bf, device=device),
            "proj": torch.empty(rows, h, dtype=bf, device=device),
            "mlp": torch.empty(rows, cfg.ffn, dtype=bf, device=device),
        }
        b = self.max_batch
        self.next_ids = torch.zeros(b, dtype=torch.int64, device=device)
        self.next_val = torch.zeros(b, dtype=torch.float32, device=device)
        # decode-step state (device-resident so a captured graph can advance itself)
        self.in_ids = torch.zeros(b, dtype=torch.int64, device=device)
        self.positions = torch.zeros(b, dtype=torch.int32, device=device)
        self.row_len = torch.zeros(b, dtype=torch.int32, device=device)
        self.row_seq = torch.arange(b, dtype=torch.int32, device=device)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.graph_rows = 0
        self.launches_per_step = 0

    # ------------------------------------------------------------------ body

    def _layers(self, rows: int, positions: torch.Tensor, token_rows: torch.Tensor, row_len: torch.Tensor,
                max_total: int, *, last_only: bool, fused: bool = False,
                prefill: tuple[int, int] | None = None) -> torch.Tensor:
        """Run embeddings-to-final-norm for ``rows`` tokens already embedded in buf['hidden'].

        ``fused``: each row is the next token of a different sequence, so RoPE, the KV append
        and the attention run as one launch per layer. ``prefill`` = (sequence, first
        position): the rows are consecutive tokens of that sequence, attended causally by the
        flash prefill kernel."""
        cfg, buf, w = self.cfg, self.buf, self.w
        hidden = buf["hidden"][:rows]
        normed = buf["normed"][:rows]
        qkv = buf["qkv"][:rows]
        q = buf["q"][:rows]
        ctx = buf["ctx"][:rows]
        proj = buf["proj"][:rows]
        mlp = buf["mlp"][:rows]
        qd, kd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        gws = self.gemv_workspace
        if self.mode == "w8a8":
            def linear(page, x, out, bias=None):
                k = int(x.shape[1])
                return w8a8_linear_bf16(page.codes, page.scales, x, bias=bias, out=out,
                                        qx_ws=self.w8_qx[:rows, :k], scale_ws=self.w8_scale[:rows])

            def swiglu(gate, up, x, out):
                k = int(x.shape[1])
                return w8a8_linear_bf16(gate.codes, gate.scales, x, up=(up.codes, up.scales), out=out,
                                        qx_ws=self.w8_qx[:rows, :k], scale_ws=self.w8_scale[:rows])
        else:
            def linear(page, x, out, bias=None):
                return qrow_linear(page.codes, page.scales, x, bias=bias, out=out, workspace=gws)

            def swiglu(gate, up, x, out):
                return qrow_swiglu(gate.codes, gate.scales, up.codes, up.scales, x, out=out, workspace=gws)
        rms_norm_into(hidden, w.layers[0].ln1, cfg.eps, normed)
        for i, layer in enumerate(w.layers):
            linear(layer.qkv, normed, qkv, bias=layer.qkv_bias)
            if fused:
                # the step's bookkeeping (decode_advance) runs after every layer: the step state
                # and the cached K/V are settled when a layer's attention starts
                self.kv.append_attend(
                    i, qkv, qkv[:, qd:], qkv[:, qd + kd:], positions, token_rows, num_heads=cfg.heads,
                    max_total_tokens=max_total, in_row_stride=cfg.qkv_rows, rope=(self.cos, self.sin),
                    error_flag=self.error_flag, scale=self.scale, out=ctx, state_ready=True,
                )
            else:
                self.kv.append(
                    i, qkv[:, qd:], qkv[:, qd + kd:], positions, token_rows, q_rows=qkv, q_out=q,
                    rope=(self.cos, self.sin), in_row_stride=cfg.qkv_rows, num_heads=cfg.heads,
                    error_flag=self.error_flag,
                )
                if prefill is not None and cfg.head_dim == 128:
                    self.kv.attend_prefill(i, q, prefill[0], prefill[1], scale=self.scale, out=ctx,
                                           error_flag=self.error_flag)
                else:
                    self.kv.attend(i, q, row_len, max_total_tokens=max_total, row_seq=token_rows, out=ctx,
                                   workspace=self.workspace, scale=self.scale)
            linear(layer.o, ctx.view(rows, qd), proj)
            residual_rms_norm_into(hidden, proj, layer.ln2, cfg.eps, hidden, normed)
            swiglu(layer.gate, layer.up, normed, mlp)
            linear(layer.down, mlp, proj)
            nxt = w.layers[i + 1].ln1 if i + 1 < len(w.layers) else w.final_norm
            residual_rms_norm_into(hidden, proj, nxt, cfg.eps, hidden, normed)
        return normed

    # ------------------------------------------------------------------ prefill

    @torch.inference_mode()
    def prefill(self, seq: int, prompt_ids: torch.Tensor) -> torch.Tensor:
        """Prefill one sequence; returns the greedy next token (device int64 scalar tensor)."""
        cfg = self.cfg
        ids = prompt_ids.to(self.device, torch.int64).reshape(-1)
        n = int(ids.numel())
        if n == 0:
            raise ValueError("input block cannot be empty")
        if n > self.max_prefill_tokens:
            raise ValueError(f"prompt of {n} tokens exceeds max_prefill_tokens={self.max_prefill_tokens}")
        start = self.kv.lengths[seq]
        if start + n > self.max_seq_len:
            raise OverflowError("input block exceeds KV cache capacity")
        self.kv.reserve(seq, start + n)
        positions = torch.arange(start, start + n, dtype=torch.int32, device=self.device)
        token_rows = torch.full((n,), seq, dtype=torch.int32, device=self.device)
        row_len = positions + 1
        embed_rows(self.w.embed.codes, self.w.embed.scales, ids, out=self.buf["hidden"][:n])
        normed = self._layers(n, positions, token_rows, row_len, start + n, last_only=True, prefill=(seq, start))
        self.kv.lengths[seq] = start + n
        idx, _, _ = qrow_argmax(self.w.head.codes, self.w.head.scales, normed[n - 1 : n],
                                out_index=self.next_ids[seq : seq + 1], out_value=self.next_val[seq : seq + 1],
                                store_logits=False)
        return idx[0]

    # ------------------------------------------------------------------ decode

    def _decode_body(self, rows: int) -> None:
        """One greedy step for rows [0, rows) using the device-resident step state."""
        cfg = self.cfg
        embed_rows(self.w.embed.codes, self.w.embed.scales, self.in_ids[:rows], out=self.buf["hidden"][:rows])
        normed = self._layers(rows, self.positions[:rows], self.row_seq[:rows], self.row_len[:rows],
                              self.max_seq_len, last_only=False,
                              fused=rows * self.cfg.kv_heads <= FUSED_DECODE_MAX_GROUPS)
        qrow_argmax(self.w.head.codes, self.w.head.scales, normed, out_index=self.next_ids[:rows],
                    out_value=self.next_val[:rows], store_logits=False)
        _lib.call("mrb_decode_advance", self.next_ids.data_ptr(), self.in_ids.data_ptr(),
                  self.positions.data_ptr(), self.row_len.data_ptr(), rows, _lib.stream_handle(self.device))
        del cfg

    def begin_decode(self, rows: int, first_ids: torch.Tensor, lengths: list[int]) -> None:
        """Load the step state: row i continues sequence i at position lengths[i]."""
        self.in_ids[:rows].copy_(first_ids.to(self.device, torch.int64).reshape(rows))
        pos = torch.tensor(lengths, dtype=torch.int32)
        self.positions[:rows].copy_(pos)
        self.row_len[:rows].copy_(pos + 1)

    @torch.inference_mode()
    def capture(self, rows: int) -> None:
        """Capture the decode step for ``rows`` rows (warm-up run first, outside the graph).
        The captured step advances in_ids/positions/row_len itself; call begin_decode again
        before replaying on new inputs."""
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        saved = (self.in_ids.clone(), self.positions.clone(), self.row_len.clone())
        with torch.cuda.stream(stream):
            self._decode_body(rows)  # warm-up (lazy attribute setup happens here)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        self.in_ids.copy_(saved[0])
        self.positions.copy_(saved[1])
        self.row_len.copy_(saved[2])
        graph = torch.cuda.CUDAGraph(keep_graph=True)  # kept so tools can list its kernel nodes
        with torch.cuda.graph(graph, stream=stream):
            self._decode_body(rows)
        graph.instantiate()
        self.graph = graph
        self.graph_rows = rows
        # kernels: embed, final norm, 8 per layer (7 with the fused RoPE/append/attention; W8A8:
        # + 4 activation quantisers), head GEMV + argmax unpack, advance (the argmax key reset
        # is a memset node, not a kernel)
        fused = rows * self.cfg.kv_heads <= FUSED_DECODE_MAX_GROUPS
        per_layer = (7 if fused else 8) + (4 if self.mode == "w8a8" else 0)
        self.launches_per_step = 2 + per_layer * self.cfg.num_layers + 2 + 1

    def step(self) -> None:
        """Advance every captured row by one greedy token (graph replay, no host sync)."""
        if self.graph is None:
            raise RuntimeError("capture() the decode step first")
        self.graph.replay()

    @torch.inference_mode()
    def generate(self, prompt_ids: torch.Tensor, max_new_tokens: int, *, seq: int = 0) -> list[int]:
        """Greedy generation for one sequence through the public path: host ids in, host ids
        out, one device->host read per token (the reference's `token.cpu()` boundary)."""
        first = self.prefill(seq, prompt_ids)
        tokens = [int(first.item())]
        if max_new_tokens <= 1:
            return tokens[:max_new_tokens]
        length = self.kv.lengths[seq]
        self.kv.reserve(seq, length + max_new_tokens)
        self.row_seq[0] = seq
        self.begin_decode(1, first.reshape(1), [length])
        if self.graph is None or self.graph_rows != 1:
            self.capture(1)
        for _ in range(max_new_tokens - 1):
            self.step()
            tokens.append(int(self.next_ids[0].item()))
        self.kv.lengths[seq] = length + max_new_tokens - 1
        return tokens

    def check_errors(self) -> None:
        if int(self.error_flag.item()):
            raise RuntimeError("KV append saw a position outside the mapped pages")
