"""Device-side QStore build helpers (reference: engine/kernels/qstore_build.py:496-501,
engine/kernels/qstore.py:1099-1128)."""
from __future__ import annotations

import torch

from . import _lib


@torch.inference_mode()
def quant_row_int8(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel symmetric int8 of an fp32 CUDA matrix -> (codes int8, scales fp32).

    Bit-identical to the reference quantiser: scale = max|w|/127 (1 for a zero row),
    code = round-half-even(w / scale) clipped to [-127, 127]."""
    if weight.ndim != 2:
        raise ValueError("weight must be a [rows, cols] matrix")
    if weight.dtype != torch.float32:
        raise ValueError("weight must be fp32")
    device = _lib.require_cuda(weight, what="quant_row_int8")
    w = weight.contiguous()
    rows, cols = (int(v) for v in w.shape)
    codes = torch.empty((rows, cols), device=device, dtype=torch.int8)
    scales = torch.empty((rows,), device=device, dtype=torch.float32)
    _lib.call("mrb_quant_row_int8", w.data_ptr(), rows, cols, codes.data_ptr(), scales.data_ptr(),
              _lib.stream_handle(device))
    return codes, scales


@torch.inference_mode()
def embed_rows(
    codes: torch.Tensor,
    scales: torch.Tensor,
    ids: torch.Tensor,
    *,
    dtype: torch.dtype = torch.float32,
    out: torch.Tensor | None = None,
    bad_ids: torch.Tensor | None = None,
) -> torch.Tensor:
    """Dequantised rows ``codes[ids] * scales[ids]`` (fp32 product) in ``dtype``.

    Out-of-range ids yield zero rows and set ``bad_ids`` (int32 device flag) when given."""
    rows, cols = (int(v) for v in codes.shape)
    device = _lib.require_cuda(codes, scales, ids, what="embed_rows")
    flat = ids.reshape(-1)
    if flat.dtype != torch.int64:
        flat = flat.to(torch.int64)
    flat = flat.contiguous()
    if out is None:
        out = torch.empty((flat.numel(), cols), device=device, dtype=dtype)
    _lib.call("mrb_qrow_embed_rows", codes.data_ptr(), scales.data_ptr(), rows, cols, flat.data_ptr(),
              flat.numel(), out.data_ptr(), _lib.dtype_code(out.dtype), _lib.ptr(bad_ids),
              _lib.stream_handle(device))
    return out.reshape(*ids.shape, cols)
