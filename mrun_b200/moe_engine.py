"""Routed-MoE decoder (Qwen3-MoE family) on the B200 kernels: ragged continuous-batch decode.

Mirrors ``Qwen3MoeDecodeRuntime.forward_decode_rows`` (engine/qwen3_moe_cuda.py:3790-3960):
per layer, input RMSNorm -> fused qkv projection -> per-head q/k RMSNorm -> RoPE -> K/V
append at each row's own position -> GQA decode attention over that row's pages -> o
projection -> residual -> post RMSNorm -> router softmax / top-k / renorm (bf16 weights) ->
the ``.moe`` backend (route compiler, grouped int8 expert SwiGLU MLP, fixed-order combine) ->
residual; then the final norm and a greedy head. Every dense projection (qkv, o, router,
head, embedding) is an int8 qrow matrix; expert weights are int8 qrow pages.

The whole step is captured in a CUDA graph (no host synchronisation inside) when the expert
pages are resident in HBM. With the pages in a pinned host tier (``MoeWeights.synthetic(...,
host_experts=True)``, the Mixtral-shape config 5) they stream through an HBM slot cache whose
copies are planned on the host from each layer's routes, so that step runs eagerly. With a process
group of N ranks the experts are sharded (rank r owns experts [r*E/N, (r+1)*E/N)) and each
layer's MoE runs through ``P2PExpertParallelMoE`` (real rows stored straight into the owners'
peer-mapped mailboxes over NVLink, epoch flags with bounded waits) or, with
``exchange="nccl"``, ``FixedCapacityExpertParallelMoE`` (fixed-size NCCL all-to-all); both are
captured with the rest of the step. Every rank decodes its own rows
(data-parallel attention), so per-GPU work stays fixed as N grows.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .dense_engine import QRow, rope_tables
from .dense_qstore_cuda import qrow_argmax, qrow_linear, qrow_workspace_bytes, residual_rms_norm_into, rms_norm_into
from .expert_parallel import ExpertShard, FixedCapacityExpertParallelMoE, P2PExpertParallelMoE
from .moe import ExpertPageLayout, PagedInt8ExpertBackend, ResidentInt8ExpertPages, router_qrow_topk
from .paged_kv import PagedKVCache
from .qstore_build import embed_rows
from .streaming import ExpertPageCache, HostPageTier


@dataclass(frozen=True)
class MoeConfig:
    num_layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    experts: int
    top_k: int
    expert_ffn: int
    vocab: int
    rope_theta: float = 1e6
    eps: float = 1e-6
    norm_topk: bool = True
    qk_norm: bool = True  # per-head q/k RMSNorm (Qwen3); Mixtral has none

    @classmethod
    def qwen3_30b_a3b(cls) -> "MoeConfig":
        """Qwen3-30B-A3B shape: 48 layers, hidden 2048, 32/4 heads, 128 experts top-8, expert FFN 768."""
        return cls(num_layers=48, hidden=2048, heads=32, kv_heads=4, head_dim=128, experts=128, top_k=8,
                   expert_ffn=768, vocab=151936)

    @classmethod
    def mixtral_8x7b(cls) -> "MoeConfig":
        """Mixtral-8x7B shape: 32 layers, hidden 4096, 32/8 heads, 8 experts top-2 (softmax over
        the two picks), expert FFN 14336 (176 MB int8 pages), vocab 32000, no q/k norm."""
        return cls(num_layers=32, hidden=4096, heads=32, kv_heads=8, head_dim=128, experts=8, top_k=2,
                   expert_ffn=14336, vocab=32000, eps=1e-5, qk_norm=False)

    @property
    def qkv_rows(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim


@dataclass
class MoeLayer:
    qkv: QRow
    o: QRow
    router: QRow
    q_norm: torch.Tensor | None   # bf16 [head_dim]; None without q/k norm
    k_norm: torch.Tensor | None
    ln1: torch.Tensor      # input norm, fp32 [hidden] holding bf16 values
    ln2: torch.Tensor      # post-attention norm
    pages: torch.Tensor | None    # uint8 [local experts, page_stride]; None when the pages live in a host tier


def _random_qrow(rows: int, cols: int, gen: torch.Generator, device: torch.device, std: float = 0.02) -> QRow:
    """Random int8 codes with per-row scales giving weights of about `std` (synthetic model)."""
    codes = torch.randint(-127, 128, (rows, cols), dtype=torch.int8, device=device, generator=gen)
    base = std / 73.6  # std of uniform codes in [-127, 127]
    scales = (torch.rand(rows, device=device, generator=gen) + 0.5) * base
    return QRow(codes, scales.float())


def _random_norm(n: int, gen: torch.Generator, device: torch.device) -> torch.Tensor:
    return (1.0 + 0.1 * torch.randn(n, device=device, generator=gen)).to(torch.bfloat16)


@dataclass
class MoeWeights:
    cfg: MoeConfig
    layout: ExpertPageLayout
    embed: QRow
    layers: list[MoeLayer]
    final_norm: torch.Tensor
    head: QRow
    expert_first: int
    experts_local: int
    host: HostPageTier | None = None  # expert pages in pinned host memory (streamed decode)

    @classmethod
    def synthetic(cls, cfg: MoeConfig, device: torch.device, seed: int = 0, *,
                  shard: ExpertShard | None = None, host_experts: bool = False) -> "MoeWeights":
        """Random-init int8 weights of the given shape (no checkpoint). With ``shard`` only the
        rank's experts are materialised; dense weights are identical on every rank. With
        ``host_experts`` every expert page goes to a pinned host tier (layer by layer, so HBM
        never holds more than one layer's pages) and the layers carry no device pages."""
        gen = torch.Generator(device=device).manual_seed(seed)
        layout = ExpertPageLayout.create(cfg.hidden, cfg.expert_ffn)
        first, local = (shard.first, shard.per_rank) if shard is not None else (0, cfg.experts)
        host = HostPageTier(layout, cfg.num_layers, local) if host_experts else None
        embed = _random_qrow(cfg.vocab, cfg.hidden, gen, device, std=1.0)
        layers = []
        for i in range(cfg.num_layers):
            layer = cls._draw_layer(cfg, layout, gen, device, first, local)
            if host is not None:
                host.pages[i].copy_(layer.pages)
                layer.pages = None
            layers.append(layer)
        final_norm = _random_norm(cfg.hidden, gen, device).float()
        head = _random_qrow(cfg.vocab, cfg.hidden, gen, device)
        return cls(cfg, layout, embed, layers, final_norm, head, first, local, host)

    @classmethod
    def _draw_layer(cls, cfg: MoeConfig, layout: ExpertPageLayout, gen: torch.Generator, device: torch.device,
                    first: int, local: int) -> MoeLayer:
        """One layer's random weights, drawn in a fixed order from ``gen``."""
        h, d = cfg.hidden, cfg.head_dim
        qkv = _random_qrow(cfg.qkv_rows, h, gen, device)
        o = _random_qrow(h, cfg.heads * d, gen, device)
        router = _random_qrow(cfg.experts, h, gen, device, std=0.05)
        q_norm, k_norm = _random_norm(d, gen, device), _random_norm(d, gen, device)
        if not cfg.qk_norm:  # drawn all the same, so the later draws do not depend on the flag
            q_norm = k_norm = None
        ln1, ln2 = _random_norm(h, gen, device).float(), _random_norm(h, gen, device).float()
        pages = cls._expert_pages(cfg, layout, gen, device, first, local)
        return MoeLayer(qkv, o, router, q_norm, k_norm, ln1, ln2, pages)

    @classmethod
    def synthetic_full_layer_pages(cls, cfg: MoeConfig, device: torch.device, layer: int,
                                   seed: int = 0) -> torch.Tensor:
        """Every expert page ([experts, page_stride]) of one layer of ``synthetic(cfg, device,
        seed)``, whatever shard a rank holds: the generator replays the draws up to that layer
        (used to check an expert-parallel layer against one GPU holding all experts)."""
        gen = torch.Generator(device=device).manual_seed(seed)
        layout = ExpertPageLayout.create(cfg.hidden, cfg.expert_ffn)
        _random_qrow(cfg.vocab, cfg.hidden, gen, device, std=1.0)
        for _ in range(layer):
            cls._draw_layer(cfg, layout, gen, device, 0, 0)
        return cls._draw_layer(cfg, layout, gen, device, 0, cfg.experts).pages

    @staticmethod
    def _expert_pages(cfg: MoeConfig, layout: ExpertPageLayout, gen: torch.Generator, device: torch.device,
                      first: int, local: int) -> torch.Tensor:
        """[local, page_stride] pages of experts [first, first + local): the layer's pages are
        drawn for all experts from the layer's generator state and sliced, so a sharded model
        holds exactly the same experts as the unsharded one."""
        ly = layout
        e, f, h = cfg.experts, ly.intermediate_size, ly.hidden_size
        codes = torch.randint(-127, 128, (e, ly.page_stride), dtype=torch.int8, device=device, generator=gen)
        pages = codes[first:first + local].view(torch.uint8).clone()
        del codes
        gus = ((torch.rand(e, 2 * f, device=device, generator=gen) + 0.5) * (0.02 / 73.6))[first:first + local]
        dns = ((torch.rand(e, h, device=device, generator=gen) + 0.5) * (0.02 / 73.6))[first:first + local]
        pages[:, ly.gate_up_scales_offset: ly.gate_up_scales_offset + ly.gate_up_scales_bytes].copy_(
            gus.contiguous().view(torch.uint8))
        pages[:, ly.down_scales_offset: ly.down_scales_offset + ly.down_scales_bytes].copy_(
            dns.contiguous().view(torch.uint8))
        return pages

    def to_host(self) -> dict:
        """numpy copy for the CPU oracle (small configurations only)."""
        def q(x: QRow):
            return x.codes.cpu().numpy(), x.scales.cpu().numpy()

        def b(x):
            return x.float().cpu().numpy()

        return {
            "embed": q(self.embed), "final_norm": b(self.final_norm), "head": q(self.head),
            "layout": self.layout.as_dict(),
            "layers": [{"qkv": q(L.qkv), "o": q(L.o), "router": q(L.router),
                        "q_norm": None if L.q_norm is None else b(L.q_norm),
                        "k_norm": None if L.k_norm is None else b(L.k_norm), "ln1": b(L.ln1), "ln2": b(L.ln2),
                        "pages": (self.host.pages[i] if L.pages is None else L.pages).cpu().numpy()}
                       for i, L in enumerate(self.layers)],
        }

    def expert_bytes(self) -> int:
        return self.cfg.num_layers * self.experts_local * self.layout.page_stride


class MoeDecoder:
    """Ragged continuous-batch greedy decode over a paged KV cache (one token per row per step)."""

    def __init__(self, weights: MoeWeights, *, max_rows: int, max_seq_len: int, device: torch.device,
                 group=None, world: int = 1, exchange: str = "p2p", expert_cache_bytes: int | None = None,
                 route_prefetch: bool = True, cache_policy: str | None = None) -> None:
        cfg = weights.cfg
        self.w = weights
        self.cfg = cfg
        self.device = device
        self.max_rows = int(max_rows)
        self.max_seq_len = int(max_seq_len)
        pages_per_seq = (self.max_seq_len + 15) // 16
        self.kv = PagedKVCache(num_layers=cfg.num_layers, num_pages=self.max_rows * pages_per_seq,
                               kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, max_seqs=self.max_rows,
                               max_pages_per_seq=pages_per_seq, device=device)
        self.cos, self.sin = rope_tables(cfg.head_dim, cfg.rope_theta, self.max_seq_len, device)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        r, bf = self.max_rows, torch.bfloat16
        ws = max(self.kv.workspace_bytes(n, cfg.heads, self.max_seq_len) for n in range(1, r + 1))
        self.attn_ws = torch.zeros(max(ws, 256), dtype=torch.uint8, device=device)
        gemv_ws = max(qrow_workspace_bytes(device, n) for n in (cfg.qkv_rows, cfg.hidden, cfg.experts))
        self.gemv_ws = torch.zeros(gemv_ws, dtype=torch.uint8, device=device)
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=device)
        self.buf = {
            "hidden": torch.empty(r, cfg.hidden, dtype=bf, device=device),
            "normed": torch.empty(r, cfg.hidden, dtype=bf, device=device),
            "qkv": torch.empty(r, cfg.qkv_rows, dtype=bf, device=device),
            "q": torch.empty(r, cfg.heads, cfg.head_dim, dtype=bf, device=device),
            "ctx": torch.empty(r, cfg.heads, cfg.head_dim, dtype=bf, device=device),
            "proj": torch.empty(r, cfg.hidden, dtype=bf, device=device),
        }
        # router outputs: expert ids, bf16 weights and their fp32 images (route coefficients)
        self.route_buf = (torch.empty(r, cfg.top_k, dtype=torch.int64, device=device),
                          torch.empty(r, cfg.top_k, dtype=bf, device=device),
                          torch.empty(r, cfg.top_k, dtype=torch.float32, device=device))
        self.router_logits = torch.empty(r, cfg.experts, dtype=bf, device=device)
        self.in_ids = torch.zeros(r, dtype=torch.int64, device=device)
        self.positions = torch.zeros(r, dtype=torch.int32, device=device)
        self.row_len = torch.zeros(r, dtype=torch.int32, device=device)
        self.row_seq = torch.arange(r, dtype=torch.int32, device=device)
        self.next_ids = torch.zeros(r, dtype=torch.int64, device=device)
        self.next_val = torch.zeros(r, dtype=torch.float32, device=device)
        self.world = int(world)
        self.group = group
        self.streamed = weights.host is not None
        if self.streamed and self.world > 1 and exchange != "p2p":
            raise ValueError("host-tier experts stream only under the peer-memory exchange")
        self.expert_cache = None
        if self.world > 1:
            shard = ExpertShard(self.world, torch.distributed.get_rank(group), cfg.experts)
            if exchange not in ("p2p", "nccl"):
                raise ValueError(f"unknown expert exchange {exchange!r}")
            if exchange == "p2p":
                self.ep = [P2PExpertParallelMoE(shard, L.pages, weights.layout, tokens=self.max_rows, k=cfg.top_k,
                                                hidden=cfg.hidden, group=group, layer=i, device=device)
                           for i, L in enumerate(weights.layers)]
                if self.streamed:  # each rank streams its own experts under its own budget
                    self.backend = None
                    self.set_expert_cache(budget_bytes=expert_cache_bytes, cache_policy=cache_policy,
                                          route_prefetch=route_prefetch)
            else:
                self.ep = [FixedCapacityExpertParallelMoE(shard, L.pages, weights.layout, group=group)
                           for L in weights.layers]
            self.backend = None
        elif self.streamed:
            self.ep = None
            self.backend = None
            self.set_expert_cache(budget_bytes=expert_cache_bytes, cache_policy=cache_policy,
                                  route_prefetch=route_prefetch)
        else:
            self.ep = None
            self.backend = PagedInt8ExpertBackend(
                ResidentInt8ExpertPages(weights.layout, [L.pages for L in weights.layers]), num_experts=cfg.experts)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.graph_rows = 0
        self.max_context = 0
        self.routes: list[torch.Tensor] | None = None  # filled when record_routes is set
        # set to {"layer": i} before an eager step to keep that layer's MoE input, routes and
        # output (clones) in the dict
        self.probe: dict | None = None

    def set_expert_cache(self, *, budget_bytes: int | None = None, cache_policy: str | None = None,
                         route_prefetch: bool = True) -> None:
        """(Re)build the HBM slot cache the host-tier experts stream through: ``budget_bytes``
        (25 % of the expert bytes this GPU owns when None) under ``cache_policy``. Each layer's routes are
        read on the host to plan its copies, as the reference's ExpertPageCache does, so a
        streamed step runs eagerly. The previous cache's slots are freed first."""
        if not self.streamed:
            raise RuntimeError("the decoder's experts are resident in HBM")
        torch.cuda.synchronize(self.device)
        host = self.w.host
        budget = int(budget_bytes if budget_bytes is not None else host.nbytes // 4)
        for ep in self.ep or []:
            ep.page_cache = None
        self.backend = self.expert_cache = None
        self.expert_cache = ExpertPageCache(host, budget_bytes=budget, device=self.device,
                                            route_prefetch=route_prefetch, cache_policy=cache_policy)
        if self.ep is not None:  # expert parallel: the cache holds this rank's experts only
            for ep in self.ep:
                ep.page_cache = self.expert_cache
        else:
            self.backend = PagedInt8ExpertBackend(self.expert_cache, num_experts=self.cfg.experts)

    # ------------------------------------------------------------------ context

    def load_synthetic_context(self, lengths: list[int], first_ids: torch.Tensor, *, steps: int, seed: int = 0) -> None:
        """Give row i a committed context of lengths[i] tokens whose K/V pages hold random bf16
        values (a stand-in for prefill; decode cost depends only on the lengths), reserve room
        for `steps` more tokens and load the step state."""
        rows = len(lengths)
        if rows > self.max_rows:
            raise ValueError("more rows than the decoder was sized for")
        gen = torch.Generator(device=self.device).manual_seed(seed)
        for i, n in enumerate(lengths):
            if n + steps > self.max_seq_len:
                raise ValueError("context plus decode steps exceed max_seq_len")
            self.kv.release(i)
            self.kv.reserve(i, n + steps)
            self.kv.lengths[i] = n
        for layer in range(self.cfg.num_layers):
            for cache in (self.kv.k[layer], self.kv.v[layer]):
                cache.normal_(0.0, 1.0, generator=gen)
        self.in_ids[:rows].copy_(first_ids.to(self.device, torch.int64).reshape(rows))
        pos = torch.tensor(lengths, dtype=torch.int32)
        self.positions[:rows].copy_(pos)
        self.row_len[:rows].copy_(pos + 1)
        self.max_context = max(lengths) + steps + 1

    # ------------------------------------------------------------------ step

    def _decode_body(self, rows: int) -> None:
        cfg, buf, w = self.cfg, self.buf, self.w
        hidden, normed = buf["hidden"][:rows], buf["normed"][:rows]
        qkv, q, ctx = buf["qkv"][:rows], buf["q"][:rows], buf["ctx"][:rows]
        proj = buf["proj"][:rows]
        qd, kd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        ws = self.gemv_ws
        embed_rows(w.embed.codes, w.embed.scales, self.in_ids[:rows], dtype=torch.bfloat16, out=hidden)
        rms_norm_into(hidden, w.layers[0].ln1, cfg.eps, normed)
        positions, row_len, row_seq = self.positions[:rows], self.row_len[:rows], self.row_seq[:rows]
        for i, layer in enumerate(w.layers):
            qrow_linear(layer.qkv.codes, layer.qkv.scales, normed, out=qkv, workspace=ws)
            self.kv.append(i, qkv[:, qd:], qkv[:, qd + kd:], positions, row_seq, q_rows=qkv, q_out=q,
                           rope=(self.cos, self.sin), in_row_stride=cfg.qkv_rows, num_heads=cfg.heads,
                           error_flag=self.error_flag,
                           qk_norm=None if layer.q_norm is None else (layer.q_norm, layer.k_norm), norm_eps=cfg.eps)
            self.kv.attend(i, q, row_len, max_total_tokens=self.max_seq_len, row_seq=row_seq, out=ctx,
                           workspace=self.attn_ws, scale=self.scale)
            qrow_linear(layer.o.codes, layer.o.scales, ctx.view(rows, qd), out=proj, workspace=ws)
            residual_rms_norm_into(hidden, proj, layer.ln2, cfg.eps, hidden, normed)
            # router linear, then softmax / top-k waiting on it; the backends take the fp32
            # images of the bf16 weights (the values the reference's .float() would give)
            top_idx, _, top_w = router_qrow_topk(normed, layer.router.codes, layer.router.scales, cfg.top_k,
                                                 renorm=cfg.norm_topk, logits=self.router_logits,
                                                 out=self.route_buf)
            if self.routes is not None:
                self.routes.append(top_idx.clone())  # the router buffers are reused per layer
            if self.ep is not None:
                moe_out = self.ep[i].forward(normed, top_idx, top_w)
            else:
                moe_out = self.backend.moe(i, normed, top_idx, top_w)
            if self.probe is not None and self.probe.get("layer") == i:
                self.probe.update(source=normed.clone(), top_indices=top_idx.clone(), top_weights=top_w.clone(),
                                  output=moe_out.clone())
            nxt = w.layers[i + 1].ln1 if i + 1 < len(w.layers) else w.final_norm
            residual_rms_norm_into(hidden, moe_out, nxt, cfg.eps, hidden, normed)
        qrow_argmax(w.head.codes, w.head.scales, normed, out_index=self.next_ids[:rows],
                    out_value=self.next_val[:rows], store_logits=False)
        _lib.call("mrb_decode_advance", self.next_ids.data_ptr(), self.in_ids.data_ptr(), self.positions.data_ptr(),
                  self.row_len.data_ptr(), rows, _lib.stream_handle(self.device))

    @torch.inference_mode()
    def capture(self, rows: int) -> None:
        """Capture one decode step for `rows` rows in a CUDA graph (with expert parallelism the
        NCCL exchanges are captured too; every rank must capture). Streamed experts cannot be
        captured: their copies are planned on the host from each layer's routes."""
        if self.streamed:
            raise RuntimeError("a decoder with host-tier experts steps eagerly (routes are read on the host)")
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        saved = (self.in_ids.clone(), self.positions.clone(), self.row_len.clone())
        with torch.cuda.stream(stream):
            self._decode_body(rows)  # warm-up outside the graph
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

    @torch.inference_mode()
    def step_eager(self, rows: int) -> None:
        """One greedy token without the captured graph (same kernels, launched one by one;
        with expert parallelism every rank must call it too)."""
        self._decode_body(rows)

    @torch.inference_mode()
    def step(self, rows: int) -> None:
        """One greedy token for rows [0, rows): graph replay when captured, else eager."""
        if self.graph is not None and self.graph_rows == rows:
            self.graph.replay()
        else:
            self._decode_body(rows)

    def check_errors(self) -> None:
        if int(self.error_flag.item()):
            raise RuntimeError("KV append saw a position outside the mapped pages")
        for ep in self.ep or []:
            if hasattr(ep, "check"):
                ep.check()
        if self.backend is not None:
            self.backend.check()

    def close(self) -> None:
        """Release the captured graph and the peer mailboxes of the expert exchange (call on
        every rank before the process group is destroyed)."""
        self.graph = None
        for ep in self.ep or []:
            if hasattr(ep, "close"):
                torch.cuda.synchronize(self.device)
                ep.close()

    def gather_kv(self, layer: int, row: int, length: int) -> tuple[np.ndarray, np.ndarray]:
        """Committed K/V of one row as float arrays [length, Hkv, D] (test support)."""
        pages = self.kv.block_table[row, : (length + 15) // 16].long()
        k = self.kv.k[layer][pages].permute(0, 2, 1, 3).reshape(-1, self.cfg.kv_heads, self.cfg.head_dim)[:length]
        v = self.kv.v[layer][pages].permute(0, 2, 1, 3).reshape(-1, self.cfg.kv_heads, self.cfg.head_dim)[:length]
        return k.float().cpu().numpy(), v.float().cpu().numpy()


__all__ = ["MoeConfig", "MoeDecoder", "MoeLayer", "MoeWeights"]
