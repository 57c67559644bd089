"""The C ABI library loads without a GPU and exports every symbol the header declares."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _declared() -> list[str]:
    names = []
    for header in sorted((REPO / "include").glob("*.h")):
        text = header.read_text()
        names += re.findall(r"^\s*(?:const\s+)?(?:int64_t|int|void|size_t|char)\s*\*?\s*(mrb_\w+)\s*\(", text, re.M)
    return names


def test_header_declares_entry_points():
    names = _declared()
    assert "mrb_qrow_matmul" in names and "mrb_last_error" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    from mrun_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIBRARY_PATH))
    missing = [name for name in _declared() if not hasattr(lib, name)]
    assert not missing, missing


def test_python_binding_covers_header():
    from mrun_b200 import _lib

    assert sorted(_lib.SIGNATURES) == sorted(_declared())


def test_abi_version_and_error_text_without_gpu():
    from mrun_b200 import _lib

    lib = _lib.load()
    assert lib.mrb_abi_version() >= 1
    # argument validation runs on the host and needs no device
    status = lib.mrb_qrow_matmul(None, 1, 1, 64, None, None, 8, None, None, 1, None, 0, None)
    assert status == _lib.MRB_ERR_ARG
    assert b"null" in lib.mrb_last_error()
    with pytest.raises(ValueError):
        _lib.check(status, "probe")


def test_operators_refuse_cpu_tensors():
    import torch

    from mrun_b200.dense_qstore_cuda import qrow_linear

    codes = torch.zeros(8, 64, dtype=torch.int8)
    scales = torch.ones(8)
    with pytest.raises(RuntimeError, match="CUDA"):
        qrow_linear(codes, scales, torch.zeros(1, 64, dtype=torch.bfloat16))


def test_new_attention_entry_points_validate_on_the_host():
    """The fused decode step and the prefill attention reject bad shapes, unsupported head
    sizes and null pointers before touching a device."""
    from mrun_b200 import _lib

    lib = _lib.load()
    P = 256  # a non-null, 16-byte aligned stand-in address (never dereferenced: validation fails first)
    # prefill: head_dim 64 is unsupported, pages must hold a multiple of 16 tokens
    rc = lib.mrb_paged_prefill_attention(P, 4, 8, 2, 64, 0, P, P, 4096, 1024, 128, 16, P, 4, None, 0.1, P, None)
    assert rc == _lib.MRB_ERR_UNSUPPORTED and b"head_dim 128" in lib.mrb_last_error()
    rc = lib.mrb_paged_prefill_attention(P, 4, 8, 2, 128, 0, P, P, 4096, 1024, 128, 8, P, 4, None, 0.1, P, None)
    assert rc == _lib.MRB_ERR_UNSUPPORTED
    rc = lib.mrb_paged_prefill_attention(P, 4, 34, 2, 128, 0, P, P, 4096, 1024, 128, 16, P, 4, None, 0.1, P, None)
    assert rc == _lib.MRB_ERR_UNSUPPORTED and b"group" in lib.mrb_last_error()
    rc = lib.mrb_paged_prefill_attention(None, 4, 8, 2, 128, 0, P, P, 4096, 1024, 128, 16, P, 4, None, 0.1, P, None)
    assert rc == _lib.MRB_ERR_ARG and b"null" in lib.mrb_last_error()
    rc = lib.mrb_paged_prefill_attention(P + 2, 4, 8, 2, 128, 0, P, P, 4096, 1024, 128, 16, P, 4, None, 0.1, P, None)
    assert rc == _lib.MRB_ERR_ARG and b"aligned" in lib.mrb_last_error()
    assert lib.mrb_paged_prefill_attention(P, 0, 8, 2, 128, 0, P, P, 4096, 1024, 128, 16, P, 4, None, 0.1, P,
                                           None) == _lib.MRB_OK  # no tokens: nothing to do
    # fused decode step
    args = dict(q=P, k=P, v=P, stride=1024, rows=2, hq=8, hkv=2, d=128)

    def fused(**kw):
        a = {**args, **kw}
        return lib.mrb_rope_append_attention(a["q"], a["k"], a["v"], a["stride"], a["rows"], a["hq"], a["hkv"],
                                             a["d"], P, None, None, None, 0, None, None, 1e-6, P, P, 4096, 1024,
                                             128, 16, P, 8, 4, None, 0.1, 64, 0, P, None)

    assert fused(d=96) == _lib.MRB_ERR_UNSUPPORTED
    assert fused(hq=40, hkv=2) == _lib.MRB_ERR_UNSUPPORTED
    assert fused(hq=7) == _lib.MRB_ERR_ARG
    assert fused(q=None) == _lib.MRB_ERR_ARG
    assert fused(k=P + 2) == _lib.MRB_ERR_ARG
    assert fused(rows=0) == _lib.MRB_OK


def test_torch_operator_library_registers_every_op():
    """libmrun_b200_torch.so loads without a GPU and registers torch.ops.mrun_b200.* with
    caller-allocated outputs (mutable `Tensor(a!)` arguments, no return values)."""
    import torch

    from mrun_b200 import _lib

    ops = _lib.ops()
    for name in _lib.OPS:
        schema = getattr(ops, name).default._schema
        assert schema.name == f"mrun_b200::{name}"
        assert len(schema.returns) == 0
        assert any(a.alias_info is not None and a.alias_info.is_write for a in schema.arguments), name
    # the built library carries the schemas the Python mirror calls with
    args = {name: [a.name for a in getattr(ops, name).default._schema.arguments] for name in _lib.OPS}
    assert args["stable_route_reduce"] == ["expert_out", "coef", "inverse", "tokens", "k", "out_f32", "out_bf16"]
    assert args["qrow_linear"] == ["x", "codes", "scales", "bias", "out", "workspace"]
    assert args["grouped_expert_mlp"][-4:] == ["slot_of", "act", "y", "sync"]
    # every operator has a CUDA kernel registered and nothing else (no CPU path)
    for name in _lib.OPS:
        assert torch._C._dispatch_has_kernel_for_dispatch_key(f"mrun_b200::{name}", "CUDA"), name
        assert not torch._C._dispatch_has_kernel_for_dispatch_key(f"mrun_b200::{name}", "CPU"), name
