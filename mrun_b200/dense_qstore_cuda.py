"""B200 drop-in for mrun's dense QStore CUDA kernels (engine/kernels/dense_qstore_cuda.py).

Same function names, argument meaning, return tuples and validation errors as the
reference; every computation runs in ``libmrun_b200.so`` (hand-written sm_100a kernels) on
torch's current CUDA stream. There is no CPU or Triton path: CPU tensors raise.
The ``require_triton`` keyword is accepted for call-site compatibility; the native kernel is
always required.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib

IMPL_W8A16 = "b200-w8a16-qrow-v1"
IMPL_SWIGLU = "b200-paired-w8a16-swiglu-bf16-v1"
IMPL_RESIDUAL_RMS = "b200-residual-bf16-rms-v1"
IMPL_RMS = "b200-row-stable-rms-v1"
IMPL_ARGMAX = "b200-w8a16-qrow-exact-argmax-v1"


def _tensor_bytes(tensor: torch.Tensor) -> int:
    return int(tensor.numel() * tensor.element_size())


def _rows(activations: torch.Tensor, in_features: int) -> torch.Tensor:
    """Contiguous, 16-byte aligned [rows, in_features] view (copied only when needed)."""
    flat = activations.reshape(-1, in_features)
    if not flat.is_contiguous() or flat.data_ptr() % 16:
        flat = flat.contiguous() if not flat.is_contiguous() else flat.clone()
    return flat


@dataclass(frozen=True)
class CompactQRowPage:
    """Device-resident int8 codes [rows, in] + fp32 row scales [rows].

    Mirrors ``CompactQRowPage`` (engine/kernels/dense_qstore_cuda.py:78-101)."""

    name: str
    start_row: int
    end_row: int
    in_features: int
    codes: torch.Tensor
    scales: torch.Tensor

    @property
    def out_features(self) -> int:
        return self.end_row - self.start_row

    @property
    def compact_bytes(self) -> int:
        return _tensor_bytes(self.codes) + _tensor_bytes(self.scales)

    @property
    def expanded_fp32_bytes(self) -> int:
        return self.out_features * self.in_features * 4

    def expanded_compute_bytes(self, dtype: torch.dtype) -> int:
        return self.out_features * self.in_features * torch.empty((), dtype=dtype).element_size()


def _check_block_m(block_m: int) -> None:
    if block_m not in {16, 32, 64}:
        raise ValueError("block_m must be one of 16, 32, or 64")


def _check_page(page: CompactQRowPage) -> None:
    if page.codes.dtype != torch.int8 or page.scales.dtype != torch.float32:
        raise ValueError("compact qrow pages hold int8 codes and fp32 scales")
    if not page.codes.is_contiguous() or not page.scales.is_contiguous():
        raise ValueError("compact qrow page tensors must be contiguous")
    if tuple(page.codes.shape) != (page.out_features, page.in_features):
        raise ValueError("compact qrow page codes do not match its row range")


_GEMV_SCRATCH = _lib.StreamScratch()
_GEMV_WS_BYTES: dict[tuple[int, int], int] = {}


def qrow_workspace_bytes(device: torch.device, out_features: int) -> int:
    """Bytes of the optional GEMV workspace (stream-K tile splitting) for ``out_features``."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, int(out_features))
    nbytes = _GEMV_WS_BYTES.get(key)
    if nbytes is None:
        with torch.cuda.device(index):
            nbytes = int(_lib.load().mrb_qrow_workspace(int(out_features)))
        _GEMV_WS_BYTES[key] = nbytes
    return nbytes


def _gemv_workspace(device: torch.device, out_features: int, workspace: torch.Tensor | None):
    """(pointer, bytes) of the workspace for one GEMV call: the caller's, else this stream's."""
    if workspace is None:
        workspace = _GEMV_SCRATCH.get(device, qrow_workspace_bytes(device, out_features))
        if workspace is None:
            return None, 0
    elif workspace.device != device or workspace.dtype != torch.uint8 or not workspace.is_contiguous():
        raise ValueError("workspace must be a contiguous uint8 tensor on the activations' device")
    return workspace.data_ptr(), workspace.numel()


def _gemv_workspace_tensor(device: torch.device, out_features: int, workspace: torch.Tensor | None):
    """The workspace tensor for one GEMV call: the caller's (checked), else this stream's."""
    if workspace is None:
        return _GEMV_SCRATCH.get(device, qrow_workspace_bytes(device, out_features))
    if workspace.device != device or workspace.dtype != torch.uint8 or not workspace.is_contiguous():
        raise ValueError("workspace must be a contiguous uint8 tensor on the activations' device")
    return workspace


def qrow_linear(
    codes: torch.Tensor,
    scales: torch.Tensor,
    activations: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """``activations @ (codes * scales[:, None]).T (+ bias)`` in the activation dtype.

    ``workspace`` (zeroed uint8, ``qrow_workspace_bytes`` long) lets decode-size calls
    split uneven tiles over all SMs; by default a per-stream workspace is used."""
    out_features, in_features = (int(v) for v in codes.shape)
    if activations.shape[-1] != in_features:
        raise ValueError("activation width does not match compact qrow page")
    device = _lib.require_cuda(codes, scales, activations, bias, what="qrow matmul")
    flat = _rows(activations, in_features)
    rows = int(flat.shape[0])
    if out is None:
        out = torch.empty((rows, out_features), device=device, dtype=flat.dtype)
    elif out.shape != (rows, out_features) or out.dtype != flat.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous [rows, out_features] tensor in the activation dtype")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != out_features):
        raise ValueError("bias must be fp32 [out_features]")
    _lib.dtype_code(flat.dtype)  # ValueError for an unsupported activation dtype
    ws = _gemv_workspace_tensor(device, out_features, workspace) if rows <= 32 else None
    _lib.ops().qrow_linear(flat, codes, scales, bias, out, ws)
    return out.reshape(*activations.shape[:-1], out_features)


@torch.inference_mode()
def dequantized_reference_matmul(page: CompactQRowPage, activations: torch.Tensor) -> torch.Tensor:
    """Device execution of the reference's materialised contract (no fp32 weight copy).

    The reference rounds the dequantised weight to the activation dtype before the dot
    (engine/kernels/dense_qstore_cuda.py:1003-1013); the B200 kernel keeps the exact int8
    code, accumulates exact products in fp32 and applies the row scale once, which stays
    within the bf16 tolerance of that contract."""
    return qrow_linear(page.codes, page.scales, activations)


@torch.inference_mode()
def fused_qrow_matmul(
    page: CompactQRowPage,
    activations: torch.Tensor,
    *,
    require_triton: bool = False,
    block_m: int = 16,
) -> tuple[torch.Tensor, str]:
    """W8A16 projection (reference: engine/kernels/dense_qstore_cuda.py:1105-1152)."""
    del require_triton
    if activations.shape[-1] != page.in_features:
        raise ValueError("activation width does not match compact qrow page")
    if page.codes.device != activations.device or page.scales.device != activations.device:
        raise ValueError("compact qrow page and activations must use one device")
    _check_block_m(block_m)
    _check_page(page)
    return qrow_linear(page.codes, page.scales, activations), IMPL_W8A16


def _validate_paired_qrow_pages(
    gate_page: CompactQRowPage,
    up_page: CompactQRowPage,
    activations: torch.Tensor,
) -> None:
    if activations.ndim < 2 or activations.dtype is not torch.bfloat16:
        raise ValueError("paired SwiGLU requires BF16 activation rows")
    if gate_page.in_features != activations.shape[-1]:
        raise ValueError("activation width does not match paired compact qrow pages")
    if (
        gate_page.in_features != up_page.in_features
        or gate_page.out_features != up_page.out_features
        or gate_page.start_row != up_page.start_row
        or gate_page.end_row != up_page.end_row
    ):
        raise ValueError("gate/up compact qrow pages must have identical geometry")
    tensors = (gate_page.codes, gate_page.scales, up_page.codes, up_page.scales)
    if any(tensor.device != activations.device for tensor in tensors):
        raise ValueError("paired compact qrow pages and activations must use one device")


def qrow_swiglu(
    gate_codes: torch.Tensor,
    gate_scales: torch.Tensor,
    up_codes: torch.Tensor,
    up_scales: torch.Tensor,
    activations: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    out_features, in_features = (int(v) for v in gate_codes.shape)
    device = _lib.require_cuda(gate_codes, up_codes, activations, what="paired SwiGLU")
    flat = _rows(activations, in_features)
    rows = int(flat.shape[0])
    if out is None:
        out = torch.empty((rows, out_features), device=device, dtype=torch.bfloat16)
    ws = _gemv_workspace_tensor(device, out_features, workspace) if rows <= 32 else None
    _lib.ops().qrow_swiglu(flat, gate_codes, gate_scales, up_codes, up_scales, out, ws)
    return out.reshape(*activations.shape[:-1], out_features)


@torch.inference_mode()
def fused_qrow_swiglu(
    gate_page: CompactQRowPage,
    up_page: CompactQRowPage,
    activations: torch.Tensor,
    *,
    require_triton: bool = False,
    block_m: int = 16,
) -> tuple[torch.Tensor, str]:
    """Paired gate/up W8A16 + BF16 SwiGLU (reference: dense_qstore_cuda.py:1052-1102)."""
    del require_triton
    _validate_paired_qrow_pages(gate_page, up_page, activations)
    _check_block_m(block_m)
    _check_page(gate_page)
    _check_page(up_page)
    return (
        qrow_swiglu(gate_page.codes, gate_page.scales, up_page.codes, up_page.scales, activations),
        IMPL_SWIGLU,
    )


def _validate_residual_rms_norm(residual: torch.Tensor, update: torch.Tensor, weight: torch.Tensor) -> int:
    if residual.ndim < 2 or update.shape != residual.shape:
        raise ValueError("residual and update must have identical row-major shapes")
    if residual.dtype is not torch.bfloat16 or update.dtype is not torch.bfloat16:
        raise ValueError("fused residual RMSNorm requires a BF16 residual boundary")
    width = int(residual.shape[-1])
    if weight.ndim != 1 or weight.numel() != width:
        raise ValueError("RMSNorm weight width does not match the residual")
    if residual.device != update.device or residual.device != weight.device:
        raise ValueError("residual, update, and RMSNorm weight must use one device")
    return width


def residual_rms_norm_into(
    residual: torch.Tensor,
    update: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    residual_out: torch.Tensor,
    normed_out: torch.Tensor,
) -> None:
    width = int(residual.shape[-1])
    rows = residual.numel() // width
    device = _lib.require_cuda(residual, update, weight, what="fused residual RMSNorm")
    _lib.call(
        "mrb_residual_rms_norm",
        residual.data_ptr(),
        update.data_ptr(),
        rows,
        width,
        weight.data_ptr(),
        float(eps),
        residual_out.data_ptr(),
        normed_out.data_ptr(),
        _lib.stream_handle(device),
    )


@torch.inference_mode()
def fused_residual_rms_norm(
    residual: torch.Tensor,
    update: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    *,
    require_triton: bool = False,
) -> tuple[torch.Tensor, torch.Tensor, str]:
    """Residual add (fp32), BF16 round, RMSNorm (reference: dense_qstore_cuda.py:1411-1459)."""
    del require_triton
    _validate_residual_rms_norm(residual, update, weight)
    if weight.dtype != torch.float32:
        weight = weight.float()
    residual_rows = residual.contiguous()
    update_rows = update.contiguous()
    rounded = torch.empty_like(residual_rows)
    normalized = torch.empty_like(residual_rows)
    residual_rms_norm_into(residual_rows, update_rows, weight.contiguous(), eps, rounded, normalized)
    return rounded, normalized, IMPL_RESIDUAL_RMS


def rms_norm_into(activations: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor) -> None:
    width = int(activations.shape[-1])
    rows = activations.numel() // width
    device = _lib.require_cuda(activations, weight, what="stable RMSNorm")
    _lib.call(
        "mrb_rms_norm",
        activations.data_ptr(),
        _lib.dtype_code(activations.dtype),
        rows,
        width,
        weight.data_ptr(),
        float(eps),
        out.data_ptr(),
        _lib.stream_handle(device),
    )


@torch.inference_mode()
def stable_rms_norm(
    activations: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    *,
    require_triton: bool = False,
) -> tuple[torch.Tensor, str]:
    """Row RMSNorm (reference: engine/kernels/dense_qstore_cuda.py:1473-1511)."""
    del require_triton
    if activations.ndim < 2 or weight.ndim != 1:
        raise ValueError("activations need rows and weight must be a vector")
    width = int(activations.shape[-1])
    if weight.numel() != width or activations.device != weight.device:
        raise ValueError("RMSNorm weight width/device does not match activations")
    flat = activations.contiguous()
    out = torch.empty_like(flat)
    rms_norm_into(flat, weight.float().contiguous(), eps, out)
    return out, IMPL_RMS


def qrow_argmax(
    codes: torch.Tensor,
    scales: torch.Tensor,
    activations: torch.Tensor,
    *,
    semantic_rows: int | None = None,
    logits: torch.Tensor | None = None,
    out_index: torch.Tensor | None = None,
    out_value: torch.Tensor | None = None,
    store_logits: bool = True,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """Exact fp32 head logits and their first maximal index (lowest index on ties).

    The argmax is fused into the head GEMV (no logits pass); ``store_logits=False`` also
    skips writing the logits."""
    vocab, in_features = (int(v) for v in codes.shape)
    device = _lib.require_cuda(codes, scales, activations, what="qrow argmax head")
    flat = _rows(activations, in_features)
    rows = int(flat.shape[0])
    semantic = vocab if semantic_rows is None else int(semantic_rows)
    if logits is None and store_logits:
        logits = torch.empty((rows, vocab), device=device, dtype=torch.float32)
    if out_index is None:
        out_index = torch.empty((rows,), device=device, dtype=torch.int64)
    if out_value is None:
        out_value = torch.empty((rows,), device=device, dtype=torch.float32)
    _lib.call(
        "mrb_qrow_argmax",
        flat.data_ptr(),
        _lib.dtype_code(flat.dtype),
        rows,
        in_features,
        codes.data_ptr(),
        scales.data_ptr(),
        vocab,
        semantic,
        _lib.ptr(logits if store_logits else None),
        out_index.data_ptr(),
        out_value.data_ptr(),
        _lib.stream_handle(device),
    )
    return out_index, out_value, logits if store_logits else None


@torch.inference_mode()
def fused_qrow_exact_argmax(
    page: CompactQRowPage,
    activations: torch.Tensor,
    *,
    semantic_row_count: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor, str]:
    """Greedy head: exact fp32 logits + first maximal index, the semantics of the
    streamed exact head (engine/dense_qstore_cuda.py:838-896)."""
    row_count = page.out_features if semantic_row_count is None else int(semantic_row_count)
    if row_count < 1 or row_count > page.out_features:
        raise ValueError("semantic_row_count must select rows inside the compact page")
    index, value, _ = qrow_argmax(page.codes, page.scales, activations, semantic_rows=row_count)
    shape = activations.shape[:-1]
    return (index + page.start_row).reshape(shape), value.reshape(shape), IMPL_ARGMAX


def __getattr__(name: str):
    """``DenseQStore`` and ``load_compact_qrow_page`` live in ``mrun_b200.dense_store`` (they
    build on ``qstore.QStore``, which imports this module) and are served from here too, where
    the reference keeps them (engine/kernels/dense_qstore_cuda.py:963, 1857)."""
    if name in ("DenseQStore", "DenseQStoreStats", "load_compact_qrow_page"):
        from . import dense_store

        return getattr(dense_store, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


__all__ = [
    "CompactQRowPage",
    "DenseQStore",
    "DenseQStoreStats",
    "dequantized_reference_matmul",
    "fused_qrow_exact_argmax",
    "fused_qrow_matmul",
    "fused_qrow_swiglu",
    "fused_residual_rms_norm",
    "load_compact_qrow_page",
    "qrow_argmax",
    "qrow_linear",
    "qrow_swiglu",
    "qrow_workspace_bytes",
    "residual_rms_norm_into",
    "rms_norm_into",
    "stable_rms_norm",
]
