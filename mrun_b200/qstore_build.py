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
    _lib.ops().quant_row_int8(w, codes, scales)
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


def write_qstore(
    directory,
    *,
    qrows: dict,
    fp32: dict,
    aliases: dict | None = None,
    config: dict | None = None,
    arch: str = "qwen2",
    model_name: str | None = None,
) -> dict:
    """Write a paged int8 store in the reference's on-disk layout (the block table of
    engine/kernels/qstore_build.py:615-690): ``weights.i8`` and ``scales.f32`` hold the qrow
    blocks back to back in the order given, ``extras.f32`` the fp32 blocks, and
    ``manifest.json`` maps names to offsets.

    qrows: name -> (int8 codes [out, in], fp32 scales [out]) as numpy arrays (from
    ``quant_row_int8`` or the reference quantiser); fp32: name -> fp32 array; aliases:
    name -> target name. Provenance digests are not written. Returns the manifest."""
    import json
    from pathlib import Path

    import numpy as np

    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    blocks: dict[str, dict] = {}
    w_off = s_off = e_off = 0
    with (directory / "weights.i8").open("wb") as wf, (directory / "scales.f32").open("wb") as sf:
        for name, (codes, scales) in qrows.items():
            codes = np.ascontiguousarray(codes, dtype=np.int8)
            scales = np.ascontiguousarray(scales, dtype=np.float32)
            if codes.ndim != 2 or scales.shape != (codes.shape[0],):
                raise ValueError(f"{name}: codes [out, in] and scales [out] required")
            wf.write(codes.tobytes())
            sf.write(scales.tobytes())
            blocks[name] = {"kind": "qrow", "shape": list(codes.shape), "w_off": w_off, "w_len": codes.nbytes,
                            "s_off": s_off, "s_len": scales.nbytes}
            w_off += codes.nbytes
            s_off += scales.nbytes
    with (directory / "extras.f32").open("wb") as ef:
        for name, array in fp32.items():
            array = np.ascontiguousarray(array, dtype=np.float32)
            ef.write(array.tobytes())
            blocks[name] = {"kind": "fp32", "shape": list(array.shape), "e_off": e_off, "e_len": array.nbytes}
            e_off += array.nbytes
    for name, target in (aliases or {}).items():
        blocks[name] = {"alias": target}
    manifest = {"schema_version": "mrun-qstore-int8-v3", "model_name": model_name or directory.name, "arch": arch,
                "dtype": "int8", "config": dict(config or {}), "blocks": blocks}
    (directory / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    return manifest
