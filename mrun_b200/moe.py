"""Routed-MoE chain on B200: router top-k, route compiler, grouped int8 expert MLP, stable
combine, and the ``.moe`` backend protocol of mrun's Qwen3-MoE engine.

Reference interfaces mirrored here (same names and argument meaning):
  * ``grouped_route_tensors`` / ``grouped_route_tensors_with_inverse`` (engine/olmoe_cuda.py:1092-1135)
  * ``stable_route_reduce`` (engine/qwen3_moe_cuda.py:2561-2664)
  * ``ExpertPageLayout`` (engine/qwen3_moe_cuda.py:187-231)
  * backend ``.moe(layer, source, top_indices, top_weights, *, prefill)`` / ``.report()`` /
    ``.reset_stats(clear_pages=)`` (engine/qwen3_moe_cuda.py:2698-2822)
Expert weights use the int8 qrow codec (per-output-channel scales) instead of the
reference's FP8/int4 pages; every computation runs in libmrun_b200.so.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any

import torch

from . import _lib

PAGE_ALIGNMENT = 4096


def align_up(value: int, alignment: int = PAGE_ALIGNMENT) -> int:
    return (value + alignment - 1) // alignment * alignment


@dataclass(frozen=True)
class ExpertPageLayout:
    """One expert's page: gate_up codes [2F, H] | gate_up scales [2F] fp32 | down codes
    [H, F] | down scales [H] fp32, padded to 4 KiB (the reference's page layout with the
    int8 qrow codec)."""

    hidden_size: int
    intermediate_size: int
    gate_up_codes_offset: int
    gate_up_codes_bytes: int
    gate_up_scales_offset: int
    gate_up_scales_bytes: int
    down_codes_offset: int
    down_codes_bytes: int
    down_scales_offset: int
    down_scales_bytes: int
    page_stride: int

    @classmethod
    def create(cls, hidden_size: int, intermediate_size: int) -> "ExpertPageLayout":
        gate_up_rows = 2 * intermediate_size
        gu_codes = gate_up_rows * hidden_size
        gu_scales_off = align_up(gu_codes, 16)
        gu_scales = gate_up_rows * 4
        down_off = align_up(gu_scales_off + gu_scales, 16)
        down_codes = hidden_size * intermediate_size
        down_scales_off = align_up(down_off + down_codes, 16)
        down_scales = hidden_size * 4
        return cls(
            hidden_size=hidden_size,
            intermediate_size=intermediate_size,
            gate_up_codes_offset=0,
            gate_up_codes_bytes=gu_codes,
            gate_up_scales_offset=gu_scales_off,
            gate_up_scales_bytes=gu_scales,
            down_codes_offset=down_off,
            down_codes_bytes=down_codes,
            down_scales_offset=down_scales_off,
            down_scales_bytes=down_scales,
            page_stride=align_up(down_scales_off + down_scales),
        )

    @classmethod
    def from_dict(cls, payload: dict[str, Any]) -> "ExpertPageLayout":
        """A layout recorded in a store manifest. The B200 kernels read every part with
        16-byte vector loads, so each offset must be 16-byte aligned (``create`` always is,
        and so is the reference's layout whenever H and F are multiples of 4)."""
        layout = cls(**{name: int(payload[name]) for name in cls.__dataclass_fields__})
        offsets = (layout.gate_up_scales_offset, layout.down_codes_offset, layout.down_scales_offset,
                   layout.page_stride)
        if layout.gate_up_codes_offset % 16 or any(o % 16 for o in offsets):
            raise ValueError("expert page parts must start on 16-byte boundaries")
        return layout

    def as_dict(self) -> dict[str, int]:
        return {name: int(getattr(self, name)) for name in self.__dataclass_fields__}


def pack_expert_page(layout: ExpertPageLayout, gate_up_codes, gate_up_scales, down_codes, down_scales,
                     out: torch.Tensor) -> None:
    """Write one expert's tensors into a uint8 page (device or pinned host)."""
    ly = layout

    def put(offset: int, tensor: torch.Tensor) -> None:
        raw = tensor.contiguous().view(torch.uint8).reshape(-1)
        out[offset : offset + raw.numel()].copy_(raw)

    put(ly.gate_up_codes_offset, gate_up_codes)
    put(ly.gate_up_scales_offset, gate_up_scales)
    put(ly.down_codes_offset, down_codes)
    put(ly.down_scales_offset, down_scales)


@dataclass(frozen=True)
class DeviceExpertLayer:
    """Typed views of a block of expert pages (engine/qwen3_moe_cuda.py:765-769): for ``G``
    pages, gate_up int8 [G, 2F, H], gate_up_scales fp32 [G, 2F], down int8 [G, H, F],
    down_scales fp32 [G, H]. The codes are int8 here (the reference's fp8 codec stores
    float8_e4m3fn at the same offsets)."""

    gate_up: torch.Tensor
    gate_up_scales: torch.Tensor
    down: torch.Tensor
    down_scales: torch.Tensor


def expert_page_views(raw: torch.Tensor, layout: ExpertPageLayout) -> DeviceExpertLayer:
    """Views (no copies) of every part of the pages in ``raw`` (uint8 ``[groups,
    page_stride]``; one page ``[page_stride]`` counts as one group), with the reference's
    argument order and result type (engine/qwen3_moe_cuda.py:1819-1853)."""
    ly = layout
    block = raw.unsqueeze(0) if raw.dim() == 1 else raw
    if block.dim() != 2 or int(block.shape[1]) < ly.page_stride or block.dtype != torch.uint8:
        raise ValueError("expert pages must be uint8 [groups, page_stride]")
    groups, f, h = int(block.shape[0]), ly.intermediate_size, ly.hidden_size

    def part(offset: int, nbytes: int, dtype: torch.dtype, *shape: int) -> torch.Tensor:
        return block[:, offset: offset + nbytes].view(dtype).reshape(groups, *shape)

    return DeviceExpertLayer(
        gate_up=part(ly.gate_up_codes_offset, ly.gate_up_codes_bytes, torch.int8, 2 * f, h),
        gate_up_scales=part(ly.gate_up_scales_offset, ly.gate_up_scales_bytes, torch.float32, 2 * f),
        down=part(ly.down_codes_offset, ly.down_codes_bytes, torch.int8, h, f),
        down_scales=part(ly.down_scales_offset, ly.down_scales_bytes, torch.float32, h),
    )


# ------------------------------------------------------------------ router


def router_topk(logits: torch.Tensor, k: int, *, renorm: bool = True) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """softmax(fp32) -> top-k (ties -> lower expert) -> optional renorm -> bf16 weights.

    Returns (indices int64 [T, k], weights bf16 [T, k], weights fp32 [T, k])."""
    device = _lib.require_cuda(logits, what="router top-k")
    lg = logits.reshape(-1, logits.shape[-1])
    if lg.dtype not in (torch.float32, torch.bfloat16):
        lg = lg.float()
    lg = lg.contiguous()
    t, e = (int(v) for v in lg.shape)
    idx = torch.empty((t, k), dtype=torch.int64, device=device)
    w32 = torch.empty((t, k), dtype=torch.float32, device=device)
    w16 = torch.empty((t, k), dtype=torch.bfloat16, device=device)
    _lib.ops().router_topk(lg, int(k), bool(renorm), idx, w32, w16)
    return idx, w16, w32


def router_qrow_topk(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, k: int, *, renorm: bool = True,
                     logits: torch.Tensor | None = None, out: tuple | None = None):
    """The router linear and selection of one MoE layer in one launch (qwen3_moe_cuda.py:
    3700-3707): bf16 logits of x [T, H] against int8 router codes [E, H] (W8A16 boundary),
    softmax / top-k (ties -> lower expert) / optional renorm. Returns (indices int64 [T, k],
    weights bf16 [T, k], coefficients fp32 [T, k] = the bf16 weights as fp32).

    Two launches: the logits (expert-major), then the selection waiting on them. ``logits``
    (bf16, at least [T, E], row stride E) receives the logits; ``out`` reuses (indices,
    weights, coefficients) buffers. A captured step passes both so their addresses stay
    fixed."""
    device = _lib.require_cuda(x, codes, scales, what="router")
    xr = x.reshape(-1, x.shape[-1])
    if xr.dtype != torch.bfloat16:
        raise ValueError("the router takes bf16 activations")
    if not xr.is_contiguous() or xr.data_ptr() % 16:
        xr = xr.contiguous().clone() if xr.data_ptr() % 16 else xr.contiguous()
    t, h = (int(v) for v in xr.shape)
    e = int(codes.shape[0])
    if int(codes.shape[1]) != h:
        raise ValueError("router codes do not match the activation width")
    if logits is None:
        logits = torch.empty((t, e), dtype=torch.bfloat16, device=device)
    elif (logits.dtype != torch.bfloat16 or not logits.is_contiguous() or logits.dim() != 2
          or int(logits.shape[1]) != e or int(logits.shape[0]) < t):
        raise ValueError("router logits must be contiguous bf16 [>= tokens, experts]")
    if out is None:
        out = (torch.empty((t, k), dtype=torch.int64, device=device),
               torch.empty((t, k), dtype=torch.bfloat16, device=device),
               torch.empty((t, k), dtype=torch.float32, device=device))
    idx, w16, coef = (o[:t] for o in out)
    _lib.call("mrb_router_qrow_topk", xr.data_ptr(), t, h, codes.data_ptr(), scales.data_ptr(), e, int(k),
              int(bool(renorm)), logits.data_ptr(), idx.data_ptr(), None, w16.data_ptr(), coef.data_ptr(),
              _lib.stream_handle(device))
    return idx, w16, coef


# ------------------------------------------------------------------ route compiler


def _grouped_route_tensors_impl(top_indices, top_weights, *, num_experts, include_inverse):
    started = time.perf_counter()
    device = _lib.require_cuda(top_indices, top_weights, what="route compiler")
    idx = top_indices.to(torch.int64).contiguous()
    rows, top_k = (int(v) for v in idx.shape)
    w = top_weights.to(torch.float32).reshape(-1).contiguous()
    a = rows * top_k
    counts = torch.empty(num_experts, dtype=torch.int32, device=device)
    starts = torch.empty(num_experts, dtype=torch.int32, device=device)
    token_ids = torch.empty(a, dtype=torch.int64, device=device)
    coefficients = torch.empty(a, dtype=torch.float32, device=device)
    inverse = torch.empty(a, dtype=torch.int64, device=device)
    _lib.ops().route_compile(idx, w, int(num_experts), counts, starts, token_ids, coefficients, inverse)
    if top_weights.dtype != torch.float32:
        coefficients = coefficients.to(top_weights.dtype)
    return token_ids, coefficients, starts, counts, (inverse if include_inverse else None), time.perf_counter() - started


def grouped_route_tensors(top_indices, top_weights, *, num_experts):
    """Expert-major route plan without a host sync (reference: engine/olmoe_cuda.py:1092)."""
    token_ids, coefficients, starts, counts, _, metadata_s = _grouped_route_tensors_impl(
        top_indices, top_weights, num_experts=num_experts, include_inverse=False)
    return token_ids, coefficients, starts, counts, metadata_s


def grouped_route_tensors_with_inverse(top_indices, top_weights, *, num_experts):
    """Route plan plus the original-rank -> expert-major-row bijection (engine/olmoe_cuda.py:1108)."""
    return _grouped_route_tensors_impl(top_indices, top_weights, num_experts=num_experts, include_inverse=True)


# ------------------------------------------------------------------ combine


def stable_route_reduce(
    expert_output: torch.Tensor,
    coefficients: torch.Tensor,
    token_ids: torch.Tensor,
    counts: torch.Tensor,
    top_indices: torch.Tensor,
    selected_experts: torch.Tensor,
    *,
    inverse_assignments: torch.Tensor | None = None,
    out_bf16: torch.Tensor | None = None,
) -> torch.Tensor:
    """fp32 [rows, hidden] combine in original route-rank order (engine/qwen3_moe_cuda.py:2561)."""
    if top_indices.ndim != 2:
        raise ValueError("stable route reduction requires [rows, top_k] indices")
    rows, top_k = map(int, top_indices.shape)
    assignments = rows * top_k
    if expert_output.ndim != 2 or int(expert_output.shape[0]) != assignments:
        raise ValueError("expert output rows must equal rows * top_k")
    if token_ids.ndim != 1 or int(token_ids.numel()) != assignments:
        raise ValueError("stable route token IDs must cover every assignment")
    if coefficients.ndim != 1 or int(coefficients.numel()) != assignments:
        raise ValueError("stable route coefficients must cover every assignment")
    if counts.ndim != 1 or int(counts.numel()) != int(selected_experts.numel()):
        raise ValueError("stable route counts must match selected experts")
    device = _lib.require_cuda(expert_output, coefficients, token_ids, counts, top_indices, what="stable route reduce")
    inverse = inverse_assignments
    if inverse is None:
        compact = torch.searchsorted(selected_experts.to(device), top_indices)
        _, _, _, _, inverse, _ = _grouped_route_tensors_impl(
            compact, torch.zeros(top_indices.shape, dtype=torch.float32, device=device),
            num_experts=int(selected_experts.numel()), include_inverse=True)
    elif inverse.ndim != 1 or int(inverse.numel()) != assignments:
        raise ValueError("stable route inverse must cover every assignment")
    eo = expert_output if expert_output.dtype == torch.bfloat16 else expert_output.to(torch.bfloat16)
    eo = eo.contiguous()
    hidden = int(eo.shape[1])
    out = torch.empty((rows, hidden), dtype=torch.float32, device=device)
    _lib.ops().stable_route_reduce(eo, coefficients.float().contiguous(), inverse.to(torch.int64).contiguous(), rows,
                                   top_k, out, out_bf16)
    return out


# ------------------------------------------------------------------ grouped expert MLP


def grouped_expert_mlp(
    source: torch.Tensor,
    token_ids: torch.Tensor,
    starts: torch.Tensor,
    counts: torch.Tensor,
    pages: torch.Tensor,
    layout: ExpertPageLayout,
    *,
    slot_of: torch.Tensor | None = None,
    act_out: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    sync: torch.Tensor | None = None,
) -> torch.Tensor:
    """Expert-major rows -> bf16 expert outputs [A, H]: gate/up (SwiGLU fused) then down.

    ``pages`` is a uint8 buffer of expert pages ``[slots, page_stride]``; expert ``e`` uses
    slot ``slot_of[e]`` (identity when None). The down launch starts on each expert as soon
    as its gate/up work is stored, through per-expert counters in ``sync`` (int32 ``[2E + 1]``,
    zeroed, left zeroed by every call; the last word is set when a wait gave up). Calls that
    may run at the same time need their own ``sync``."""
    device = _lib.require_cuda(source, token_ids, starts, counts, pages, what="grouped expert MLP")
    ly = layout
    f, h = ly.intermediate_size, ly.hidden_size
    a = int(token_ids.numel())
    e = int(counts.numel())
    base = pages.data_ptr()
    stride = ly.page_stride
    act = act_out if act_out is not None else torch.empty((a, f), dtype=torch.bfloat16, device=device)
    y = out if out is not None else torch.empty((a, h), dtype=torch.bfloat16, device=device)
    if a == 0:
        return y
    stream = _lib.stream_handle(device)
    src = source.contiguous()
    if sync is None:
        sync = expert_mlp_sync(e, device)
    elif sync.dtype != torch.int32 or sync.numel() < 2 * e + 1:
        raise ValueError(f"the expert MLP sync buffer is int32 [2 * experts + 1] = [{2 * e + 1}]")
    _lib.ops().grouped_expert_mlp(src, token_ids, starts, counts, pages, stride, ly.gate_up_codes_offset,
                                  ly.gate_up_scales_offset, ly.down_codes_offset, ly.down_scales_offset, slot_of, act,
                                  y, sync)
    return y


#: Routed rows from which an expert's MLP runs on the tensor-core GEMMs instead of the grouped
#: kernel, whose 16-row passes re-stream the expert's page once per pass.
LARGE_EXPERT_ROWS = 64


def expert_page_matrices(pages: torch.Tensor, layout: ExpertPageLayout, slot: int):
    """(gate codes, gate scales, up codes, up scales, down codes, down scales) views of the
    expert page in slot ``slot`` of ``pages`` (uint8 ``[slots, page_stride]``)."""
    ly = layout
    f, h = ly.intermediate_size, ly.hidden_size
    page = pages[int(slot)]
    gu = page[ly.gate_up_codes_offset: ly.gate_up_codes_offset + ly.gate_up_codes_bytes].view(torch.int8).view(2 * f, h)
    gus = page[ly.gate_up_scales_offset: ly.gate_up_scales_offset + ly.gate_up_scales_bytes].view(torch.float32)
    dn = page[ly.down_codes_offset: ly.down_codes_offset + ly.down_codes_bytes].view(torch.int8).view(h, f)
    dns = page[ly.down_scales_offset: ly.down_scales_offset + ly.down_scales_bytes].view(torch.float32)
    return gu[:f], gus[:f], gu[f:], gus[f:], dn, dns


def expert_mlp_large_counts(
    source: torch.Tensor,
    token_ids: torch.Tensor,
    starts: torch.Tensor,
    counts: torch.Tensor,
    pages: torch.Tensor,
    layout: ExpertPageLayout,
    *,
    slot_of: torch.Tensor | None = None,
    sync: torch.Tensor | None = None,
    min_rows: int = LARGE_EXPERT_ROWS,
) -> torch.Tensor:
    """``grouped_expert_mlp`` with every expert that received ``min_rows`` rows or more moved
    to the tcgen05 W8A16 GEMMs: its rows are gathered, the paired gate/up GEMM applies the
    SwiGLU boundaries (``qrow_swiglu``) and the down GEMM (``qrow_linear``) writes straight
    into the expert's rows of the route-ordered output; the other experts run on the grouped
    kernel. Prefill-sized groups (hundreds of rows per expert) thus read each page once
    instead of once per 16 rows. Reads the counts on the host (one synchronisation), so it
    serves eager calls -- prefill and host-planned streamed decode -- not captured steps.
    Each output row agrees with the grouped kernel's within the bf16 tolerance (the two sum
    the same exact products in a different order)."""
    from .dense_qstore_cuda import qrow_linear, qrow_swiglu

    device = _lib.require_cuda(source, token_ids, starts, counts, pages, what="expert MLP")
    counts_h = counts.cpu().tolist()
    big = [e for e, c in enumerate(counts_h) if c >= min_rows]
    small = counts
    if big:
        small = counts.clone()
        small[torch.tensor(big, dtype=torch.int64, device=device)] = 0
    y = grouped_expert_mlp(source, token_ids, starts, small, pages, layout, slot_of=slot_of, sync=sync)
    if big:
        starts_h = starts.cpu().tolist()
        slots_h = slot_of.cpu().tolist() if slot_of is not None else None
        src = source.reshape(-1, layout.hidden_size)
        for e in big:
            s, c = starts_h[e], counts_h[e]
            gate, gate_s, up, up_s, down, down_s = expert_page_matrices(
                pages, layout, slots_h[e] if slots_h is not None else e)
            rows = src.index_select(0, token_ids[s:s + c])
            act = qrow_swiglu(gate, gate_s, up, up_s, rows)
            qrow_linear(down, down_s, act, out=y[s:s + c])
    return y


def expert_mlp_sync(experts: int, device: torch.device) -> torch.Tensor:
    """A zeroed sync buffer for ``grouped_expert_mlp`` over ``experts`` experts."""
    return torch.zeros(2 * int(experts) + 1, dtype=torch.int32, device=device)


# ------------------------------------------------------------------ backends


@dataclass
class ExpertBackendStats:
    grouped_kernel_calls: int = 0
    route_compiler_calls: int = 0
    expert_assignments: int = 0
    addressed_source_bytes: int = 0

    def as_dict(self) -> dict[str, int]:
        return dict(self.__dict__)


class ResidentInt8ExpertPages:
    """All experts of every layer resident in HBM: pages[layer] is [experts, page_stride]."""

    def __init__(self, layout: ExpertPageLayout, pages: list[torch.Tensor]) -> None:
        self.layout = layout
        self.pages = pages

    def layer_pages(self, layer: int, top_indices: torch.Tensor, *, prefill: bool):
        return self.pages[layer], None

    def reset(self, *, clear_pages: bool) -> None:
        del clear_pages

    def report(self) -> dict[str, Any]:
        return {"kind": "resident", "layers": len(self.pages)}


@dataclass
class PagedInt8ExpertBackend:
    """The reference's `.moe` protocol over int8 expert pages (engine/qwen3_moe_cuda.py:2698)."""

    cache: Any
    dtype: torch.dtype = torch.bfloat16
    num_experts: int = 0
    stats: ExpertBackendStats = field(default_factory=ExpertBackendStats)
    # experts with this many routed rows or more run on the tensor-core GEMMs in prefill calls
    # and under a cache that plans its copies on the host (None: always the grouped kernel)
    large_expert_rows: int | None = LARGE_EXPERT_ROWS
    _sync: dict = field(default_factory=dict, repr=False)

    def _sync_for(self, experts: int, device: torch.device) -> torch.Tensor:
        key = (device.index, experts)
        if key not in self._sync:
            self._sync[key] = expert_mlp_sync(experts, device)
        return self._sync[key]

    def check(self) -> None:
        """Raise if a down launch gave up waiting for its gate/up work (its output is then not
        to be trusted)."""
        for buf in self._sync.values():
            if int(buf[-1].item()):
                raise RuntimeError("expert MLP: the down projection timed out waiting for the gate/up projection")

    def reset_stats(self, *, clear_pages: bool) -> None:
        self.stats = ExpertBackendStats()
        self.cache.reset(clear_pages=clear_pages)

    def moe(self, layer: int, source: torch.Tensor, top_indices: torch.Tensor, top_weights: torch.Tensor, *,
            prefill: bool = False) -> torch.Tensor:
        pages, slot_of = self.cache.layer_pages(layer, top_indices, prefill=prefill)
        token_ids, coefficients, starts, counts, inverse, _ = grouped_route_tensors_with_inverse(
            top_indices, top_weights.float(), num_experts=self.num_experts)
        sync = self._sync_for(self.num_experts, source.device)
        if self.large_expert_rows is not None and (prefill or getattr(self.cache, "plans_on_host", False)):
            expert_output = expert_mlp_large_counts(source, token_ids, starts, counts, pages, self.cache.layout,
                                                    slot_of=slot_of, sync=sync, min_rows=self.large_expert_rows)
        else:
            expert_output = grouped_expert_mlp(source, token_ids, starts, counts, pages, self.cache.layout,
                                               slot_of=slot_of, sync=sync)
        out = torch.empty((source.shape[0], source.shape[1]), dtype=torch.bfloat16, device=source.device)
        _lib.ops().stable_route_reduce(expert_output, coefficients, inverse, int(top_indices.shape[0]),
                                       int(top_indices.shape[1]), None, out)
        release = getattr(self.cache, "release_layer", None)
        if release is not None:  # streamed pages: slots may be reused after these kernels
            release()
        self.stats.grouped_kernel_calls += 2
        self.stats.route_compiler_calls += 1
        self.stats.expert_assignments += int(top_indices.numel())
        return out if self.dtype == torch.bfloat16 else out.to(self.dtype)

    def report(self) -> dict[str, Any]:
        return {"kind": "paged-int8-qstore", "kernel": "b200-grouped-int8-qrow", "backend": self.stats.as_dict(),
                "page_cache": self.cache.report(), "page_stride": self.cache.layout.page_stride}


__all__ = [
    "DeviceExpertLayer",
    "ExpertPageLayout",
    "PagedInt8ExpertBackend",
    "ResidentInt8ExpertPages",
    "expert_page_views",
    "expert_mlp_large_counts",
    "expert_mlp_sync",
    "expert_page_matrices",
    "grouped_expert_mlp",
    "grouped_route_tensors",
    "grouped_route_tensors_with_inverse",
    "pack_expert_page",
    "router_qrow_topk",
    "router_topk",
    "stable_route_reduce",
]
