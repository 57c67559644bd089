"""W8A8 QStore linear on B200 (drop-in for engine/kernels/w8a8.py).

``w8a8_matmul`` keeps the reference signature and numerics: per-token dynamic int8
activations, exact int32 accumulation (integer tensor pipe), ``acc * act_scale * w_scale`` in
fp32, and an exact fp32 side path for protected outlier columns. With no protected columns
the result is bit-identical to the reference. ``enable_w8a8`` / ``disable_w8a8`` rebind a
store's ``matmul`` exactly as the reference does.
"""
from __future__ import annotations

import types
from typing import Any

import numpy as np
import torch

from . import _lib


def _int8_gemm(q_x: torch.Tensor, q_w: torch.Tensor, use_int_mm: bool = True) -> torch.Tensor:
    """[T, in] int8 @ [out, in] int8 -> [T, out] int32, exact (reference: w8a8.py:33-64).

    ``use_int_mm`` is accepted for call compatibility; the native kernel is always used."""
    del use_int_mm
    if q_x.dtype != torch.int8 or q_w.dtype != torch.int8:
        raise ValueError("int8 GEMM operands must be int8")
    device = _lib.require_cuda(q_x, q_w, what="int8 GEMM")
    qx = q_x.contiguous()
    qw = q_w.contiguous()
    m, k = (int(v) for v in qx.shape)
    n = int(qw.shape[0])
    if int(qw.shape[1]) != k:
        raise ValueError("int8 GEMM inner dimensions differ")
    acc = torch.empty((m, n), dtype=torch.int32, device=device)
    _lib.call("mrb_int8_gemm", qx.data_ptr(), qw.data_ptr(), m, n, k, acc.data_ptr(), _lib.stream_handle(device))
    return acc


def quantize_activations(x: torch.Tensor, keep: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token int8 codes and scales (reference: w8a8.py:117-121)."""
    device = _lib.require_cuda(x, what="W8A8 activation quantiser")
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    m, k = (int(v) for v in x2.shape)
    qx = torch.empty((m, k), dtype=torch.int8, device=device)
    scale = torch.empty((m, 1), dtype=torch.float32, device=device)
    _lib.call("mrb_w8a8_quantize", x2.data_ptr(), _lib.dtype_code(x2.dtype), m, k, _lib.ptr(keep), qx.data_ptr(),
              scale.data_ptr(), _lib.stream_handle(device))
    return qx, scale


def w8a8_matmul(
    q_w: torch.Tensor,
    sc_w: torch.Tensor,
    x: torch.Tensor,
    *,
    protect_idx: torch.Tensor | None = None,
    protect_k: int = 0,
    use_int_mm: bool = True,
    acc_out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``x @ (q_w * sc_w[:,None]).T`` through int8 x int8 -> int32 (reference: w8a8.py:67-125).

    Returns fp32 ``[..., out]``. ``acc_out`` (int32 [T, out]) optionally receives the exact
    accumulator."""
    del use_int_mm
    device = _lib.require_cuda(q_w, sc_w, x, what="W8A8 matmul")
    out_features, in_features = (int(v) for v in q_w.shape)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        x2 = x2.float()
    x2 = x2.contiguous()
    t = int(x2.shape[0])
    if int(x2.shape[1]) != in_features:
        raise ValueError("activation width does not match the int8 weight")
    qw = q_w.contiguous()
    sw = sc_w.to(device=device, dtype=torch.float32).contiguous()
    stream = _lib.stream_handle(device)
    keep = None
    idx = None
    if protect_idx is None and protect_k > 0:
        k = min(int(protect_k), in_features)
        idx = torch.empty(k, dtype=torch.int64, device=device)
        keep = torch.empty(in_features, dtype=torch.float32, device=device)
        _lib.call("mrb_w8a8_protect_topk", x2.data_ptr(), _lib.dtype_code(x2.dtype), t, in_features, k,
                  idx.data_ptr(), keep.data_ptr(), stream)
    elif protect_idx is not None:
        idx = torch.as_tensor(protect_idx, dtype=torch.int64, device=device).reshape(-1).contiguous()
        if idx.numel() == 0:
            idx = None
        else:
            keep = torch.ones(in_features, dtype=torch.float32, device=device)
            keep[idx] = 0.0
    nprotect = 0 if idx is None else int(idx.numel())
    y = torch.empty((t, out_features), dtype=torch.float32, device=device)
    qx_ws = torch.empty((t, in_features), dtype=torch.int8, device=device)
    scale_ws = torch.empty((t,), dtype=torch.float32, device=device)
    side_ws = torch.empty((t, out_features), dtype=torch.float32, device=device) if nprotect else None
    _lib.call("mrb_w8a8_matmul", x2.data_ptr(), _lib.dtype_code(x2.dtype), t, in_features, qw.data_ptr(),
              sw.data_ptr(), out_features, _lib.ptr(idx), nprotect, _lib.ptr(keep), y.data_ptr(), _lib.ptr(acc_out),
              _lib.ptr(qx_ws), scale_ws.data_ptr(), _lib.ptr(side_ws), stream)
    return y.reshape(*x.shape[:-1], out_features)


def w8a8_linear_bf16(
    codes: torch.Tensor,
    scales: torch.Tensor,
    x: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    up: tuple[torch.Tensor, torch.Tensor] | None = None,
    out: torch.Tensor | None = None,
    qx_ws: torch.Tensor | None = None,
    scale_ws: torch.Tensor | None = None,
) -> torch.Tensor:
    """W8A8 projection for a bf16 decoder: ``bf16((acc * s_x) * s_w + bias)`` with per-token
    int8 activations and exact int32 accumulation (the ``enable_w8a8`` store matmul,
    engine/kernels/w8a8.py:145-177, at the dense engine's bf16 boundary). ``up=(codes, scales)``
    gives the paired gate/up SwiGLU instead. ``qx_ws`` / ``scale_ws``: optional int8 [m, k]
    and fp32 [m] buffers for the quantised activations."""
    device = _lib.require_cuda(codes, scales, x, what="W8A8 linear")
    if x.dtype != torch.bfloat16:
        raise ValueError("W8A8 linear takes bf16 activations")
    x2 = x.reshape(-1, x.shape[-1])
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    m, k = (int(v) for v in x2.shape)
    n = int(codes.shape[0])
    if int(codes.shape[1]) != k:
        raise ValueError("activation width does not match the int8 weight")
    if up is not None and (tuple(up[0].shape) != tuple(codes.shape)):
        raise ValueError("gate and up pages differ in shape")
    y = out if out is not None else torch.empty((m, n), dtype=torch.bfloat16, device=device)
    qx = qx_ws if qx_ws is not None else torch.empty((m, k), dtype=torch.int8, device=device)
    sx = scale_ws if scale_ws is not None else torch.empty((m,), dtype=torch.float32, device=device)
    _lib.call("mrb_w8a8_linear_bf16", x2.data_ptr(), m, k, codes.data_ptr(), scales.data_ptr(),
              _lib.ptr(up[0] if up is not None else None), _lib.ptr(up[1] if up is not None else None),
              _lib.ptr(bias), n, y.data_ptr(), qx.data_ptr(), sx.data_ptr(), _lib.stream_handle(device))
    return y


# ---- opt-in store hook (reference: w8a8.py:145-187) -----------------------------------------

_ORIG_MATMUL: dict[int, Any] = {}


def _raw_qrow(store: Any, name: str) -> tuple[torch.Tensor, torch.Tensor]:
    """(int8 codes [out, in], fp32 row scales [out]) of a qrow block, never dequantised
    (engine/kernels/w8a8.py:130-143). Reads through what the store offers: the device page of
    a B200 ``QStore`` / ``DenseQStore`` (``page``), a ``compact_page`` of another dense store,
    or the reference QStore's memory-mapped ``w`` / ``s`` files (then moved to the store's
    device)."""
    reader = getattr(store, "page", None) or getattr(store, "compact_page", None)
    if callable(reader):
        page = reader(name)
        return page.codes, page.scales
    block = store._resolve(name)
    rows, cols = (int(v) for v in block["shape"])
    w0, s0 = int(block["w_off"]), int(block["s_off"]) // 4
    codes = torch.from_numpy(np.array(store.w[w0:w0 + rows * cols], dtype=np.int8).reshape(rows, cols))
    scales = torch.from_numpy(np.array(store.s[s0:s0 + rows], dtype=np.float32))
    device = getattr(store, "device", "cpu")
    if str(device) != "cpu":
        codes, scales = codes.to(device), scales.to(device)
    return codes, scales


def _w8a8_matmul_method(self: Any, name: str, x: torch.Tensor) -> torch.Tensor:
    b = self._resolve(name)
    if b.get("kind") != "qrow":
        return _ORIG_MATMUL[id(self)](name, x)
    cfg = self._w8a8
    codes, scales = _raw_qrow(self, name)
    if codes.device != x.device:  # a host-resident store feeding device activations
        codes, scales = codes.to(x.device), scales.to(x.device)
    return w8a8_matmul(codes, scales, x, protect_idx=cfg["lists"].get(name), protect_k=cfg["k"],
                       use_int_mm=cfg["use_int_mm"])


def enable_w8a8(
    store: Any,
    *,
    protect_k: int = 8,
    protect_lists: dict[str, Any] | None = None,
    use_int_mm: bool = True,
) -> Any:
    """Flip one store into W8A8 mode by rebinding ``matmul`` (reversible via disable_w8a8)."""
    _ORIG_MATMUL[id(store)] = store.matmul
    store._w8a8 = {"k": int(protect_k), "lists": protect_lists or {}, "use_int_mm": bool(use_int_mm)}
    store.matmul = types.MethodType(_w8a8_matmul_method, store)
    return store


def disable_w8a8(store: Any) -> Any:
    orig = _ORIG_MATMUL.pop(id(store), None)
    if orig is not None:
        store.matmul = orig
    if hasattr(store, "_w8a8"):
        del store._w8a8
    return store


__all__ = ["_int8_gemm", "disable_w8a8", "enable_w8a8", "quantize_activations", "w8a8_linear_bf16", "w8a8_matmul"]
