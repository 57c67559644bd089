"""ctypes binding of the in-tree CUDA library ``libmrun_b200.so`` (the C ABI boundary), and the
loader of its PyTorch operator library ``libmrun_b200_torch.so`` (``torch.ops.mrun_b200``).

Loading is strict: if a library is missing or lacks a declared symbol, importing any
operator raises instead of falling back to another implementation. Status codes follow
``include/mrun_b200.h``: argument errors raise ``ValueError`` (the reference's validation
errors), CUDA and unsupported-shape errors raise ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import c_int32, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "libmrun_b200.so"
OPS_LIBRARY_PATH = Path(__file__).resolve().parent / "libmrun_b200_torch.so"
OPS = ("qrow_linear", "qrow_swiglu", "quant_row_int8", "router_topk", "route_compile", "stable_route_reduce",
       "grouped_expert_mlp")

MRB_OK = 0
MRB_ERR_ARG = 1
MRB_ERR_CUDA = 2
MRB_ERR_UNSUPPORTED = 3
MRB_ERR_IO = 4

MRB_F32 = 0
MRB_BF16 = 1
MRB_F16 = 2

_P = c_void_p
_I64 = c_int64

# name -> argtypes (all functions return int unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "mrb_abi_version": [],
    "mrb_last_error": [],
    "mrb_quant_row_int8": [_P, _I64, _I64, _P, _P, _P],
    "mrb_qrow_embed_rows": [_P, _P, _I64, _I64, _P, _I64, _P, c_int, _P, _P],
    "mrb_qrow_matmul": [_P, c_int, _I64, _I64, _P, _P, _I64, _P, _P, c_int, _P, c_size_t, _P],
    "mrb_qrow_workspace": [_I64],
    "mrb_qrow_swiglu": [_P, _I64, _I64, _P, _P, _P, _P, _I64, _P, _P, c_size_t, _P],
    "mrb_qrow_argmax": [_P, c_int, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _P, _P],
    "mrb_rms_norm": [_P, c_int, _I64, _I64, _P, c_float, _P, _P],
    "mrb_residual_rms_norm": [_P, _P, _I64, _I64, _P, c_float, _P, _P, _P],
    "mrb_w8a8_quantize": [_P, c_int, _I64, _I64, _P, _P, _P, _P],
    "mrb_int8_gemm": [_P, _P, _I64, _I64, _I64, _P, _P],
    "mrb_tc_status": [_P],
    "mrb_w8a8_protect_topk": [_P, c_int, _I64, _I64, c_int, _P, _P, _P],
    "mrb_w8a8_matmul": [_P, c_int, _I64, _I64, _P, _P, _I64, _P, c_int, _P, _P, _P, _P, _P, _P, _P],
    "mrb_router_topk": [_P, c_int, _I64, _I64, _I64, c_int, _P, _P, _P, _P],
    "mrb_router_qrow_topk": [_P, _I64, _I64, _P, _P, _I64, _I64, c_int, _P, _P, _P, _P, _P, _P],
    "mrb_route_compile": [_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P],
    "mrb_grouped_qrow": [_P, _P, _P, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, c_int, _I64, _P, _P],
    "mrb_grouped_expert_mlp": [_P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64, _I64, _P, _P,
                               _P, _P],
    "mrb_stable_route_reduce": [_P, _P, _P, _I64, _I64, _I64, _P, _P, _P],
    "mrb_ep_pack": [_P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P],
    "mrb_ep_gather_rows": [_P, _I64, _P, _I64, _P, _P],
    "mrb_rope_kv_append": [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _P, _P, _P,
                           _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _P, c_float, _P],
    "mrb_rope_append_attention": [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _P, _P, c_float,
                                  _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, c_float, _I64, c_int, _P,
                                  _P],
    "mrb_rope_append_attention_cluster": [_I64, _I64, _I64, _I64, _I64],
    "mrb_paged_prefill_attention": [_P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P,
                                    c_float, _P, _P],
    "mrb_store_file_open": [ctypes.c_char_p, ctypes.POINTER(c_void_p), ctypes.POINTER(ctypes.c_uint64)],
    "mrb_store_file_close": [_P],
    "mrb_store_file_read": [_P, ctypes.c_uint64, ctypes.c_uint64, _P, c_int, c_int],
    "mrb_store_file_advise": [_P, ctypes.c_uint64, ctypes.c_uint64, c_int],
    "mrb_paged_attention_workspace": [_I64, _I64, _I64, _I64, _I64],
    "mrb_paged_attention_timeouts": [],
    "mrb_paged_attention": [_P, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _P,
                            _P, _P, c_float, _I64, _P, _P, c_size_t, _P],
    "mrb_paged_attention_static_capacity": [],
    "mrb_paged_attention_static": [_P, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _P,
                                   _P, _P, c_float, _I64, _P, _P],
    "mrb_decode_advance": [_P, _P, _P, _P, _I64, _P],
    "mrb_copy_pages": [_P, _I64, _P, _I64, _P, _P, _I64, _I64, _P, _P],
    "mrb_w8a8_linear_bf16": [_P, _I64, _I64, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _P],
    "mrb_ep_mailbox_bytes": [_I64, _I64, _I64],
    "mrb_ep_mailbox_offsets": [_I64, _I64, _I64, _P],
    "mrb_ep_mailbox_create": [c_size_t, _P, _P],
    "mrb_ep_mailbox_open": [_P, _P],
    "mrb_ep_mailbox_close": [_P, c_int],
    "mrb_ep_p2p_dispatch": [_P, _I64, _P, _P, _I64, _I64, _I64, _P, _P, _P],
    "mrb_ep_p2p_wait_dispatch": [_P, _I64, _I64, _I64, c_int32, _P, _P, _P],
    "mrb_ep_p2p_return": [_P, _P, _I64, _I64, _I64, _I64, _P, _P, _P],
    "mrb_ep_p2p_wait_return": [_P, _I64, _I64, _I64, _P, _P],
    "mrb_ep_p2p_wait_route": [_P, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    "mrb_ep_p2p_combine": [_P, _I64, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _P],
    "mrb_ep_set_wait_limit": [_I64],
    "mrb_ep_wait_limit": [],
}
_RESTYPES = {"mrb_last_error": ctypes.c_char_p, "mrb_abi_version": c_int, "mrb_paged_attention_workspace": c_size_t,
             "mrb_paged_attention_static_capacity": c_size_t, "mrb_qrow_workspace": c_size_t,
             "mrb_ep_mailbox_bytes": c_size_t, "mrb_ep_wait_limit": ctypes.c_int64,
             "mrb_paged_attention_timeouts": ctypes.c_int64}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class MrbError(RuntimeError):
    """A CUDA or unsupported-shape failure reported by the native library."""


def load() -> ctypes.CDLL:
    """Load the native library once; raise if it is absent (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIBRARY_PATH.exists():
            raise ImportError(
                f"mrun_b200 native library not built: {LIBRARY_PATH} is missing "
                "(run `python -c 'import __graft_entry__ as g; g.build()'`)"
            )
        lib = ctypes.CDLL(str(LIBRARY_PATH))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)  # AttributeError if a declared symbol is missing
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, c_int)
        _lib = lib
        return lib


_ops = None


def ops():
    """``torch.ops.mrun_b200``: the operator library over the C ABI (csrc/torch_ops.cpp), loaded
    once after the C library; raises if it is absent or lacks an operator."""
    global _ops
    if _ops is not None:
        return _ops
    load()
    with _lock:
        if _ops is None:
            if not OPS_LIBRARY_PATH.exists():
                raise ImportError(f"mrun_b200 operator library not built: {OPS_LIBRARY_PATH} is missing")
            torch.ops.load_library(str(OPS_LIBRARY_PATH))
            namespace = torch.ops.mrun_b200
            for name in OPS:
                getattr(namespace, name)  # AttributeError if an operator is not registered
            _ops = namespace
    return _ops


def check(status: int, what: str) -> None:
    if status == MRB_OK:
        return
    message = load().mrb_last_error().decode("utf-8", "replace")
    text = f"{what}: {message}" if message else f"{what}: status {status}"
    if status == MRB_ERR_ARG:
        raise ValueError(text)
    if status == MRB_ERR_IO:
        raise OSError(text)
    raise MrbError(text)


def call(name: str, *args) -> None:
    """Invoke a C-ABI entry point and raise on a non-zero status."""
    check(getattr(load(), name)(*args), name)


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    """Raw cudaStream_t of torch's current stream on ``device``."""
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    if dtype is torch.float32:
        return MRB_F32
    if dtype is torch.bfloat16:
        return MRB_BF16
    if dtype is torch.float16:
        return MRB_F16
    raise ValueError(f"unsupported activation dtype {dtype}")


def require_cuda(*tensors: torch.Tensor, what: str) -> torch.device:
    """Every hot-path operator runs on CUDA only; CPU tensors are a caller error."""
    device = None
    for tensor in tensors:
        if tensor is None:
            continue
        if tensor.device.type != "cuda":
            raise RuntimeError(f"{what} requires CUDA tensors (got {tensor.device}); there is no CPU path")
        if device is None:
            device = tensor.device
        elif tensor.device != device:
            raise ValueError(f"{what}: tensors must share one device")
    if device is None:
        raise ValueError(f"{what}: no tensor given")
    return device


class DeviceScratch:
    """Grow-only, zero-initialised scratch buffer per device for kernels that keep
    self-resetting counters in their workspace. Calls that share it must be stream-ordered."""

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._buffers: dict[int, torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor | None:
        if nbytes <= 0:
            return None
        index = device.index if device.index is not None else torch.cuda.current_device()
        with self._lock:
            buf = self._buffers.get(index)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(int(nbytes), 1 << 20), dtype=torch.uint8, device=device)
                self._buffers[index] = buf
            return buf


class StreamScratch:
    """Zero-initialised workspace per (device, CUDA stream) for kernels whose workspace
    holds self-resetting counters: calls ordered on one stream may share it, calls on
    different streams never do. While the current stream is being captured only an
    existing buffer is handed out (None otherwise), so a CUDA graph never owns one."""

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._buffers: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor | None:
        if nbytes <= 0:
            return None
        index = device.index if device.index is not None else torch.cuda.current_device()
        key = (index, torch.cuda.current_stream(device).cuda_stream)
        with self._lock:
            buf = self._buffers.get(key)
            if buf is not None and buf.numel() >= nbytes:
                return buf
            if torch.cuda.is_current_stream_capturing():
                return None
            buf = torch.zeros(max(int(nbytes), 1 << 20), dtype=torch.uint8, device=device)
            self._buffers[key] = buf
            return buf


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


__all__ = [
    "LIBRARY_PATH",
    "MRB_BF16",
    "MRB_F16",
    "MRB_F32",
    "MrbError",
    "c_size_t",
    "call",
    "check",
    "dtype_code",
    "exported_symbols",
    "load",
    "ptr",
    "require_cuda",
    "stream_handle",
]
