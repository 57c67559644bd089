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
        names += re.findall(r"^\s*(?:const\s+)?(?:int|void|size_t|char)\s*\*?\s*(mrb_\w+)\s*\(", text, re.M)
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
