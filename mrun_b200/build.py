"""Build the in-tree CUDA library ``libmrun_b200.so`` for sm_100a with nvcc, and the PyTorch
operator library ``libmrun_b200_torch.so`` over it.

Each ``csrc/*.cu`` compiles to its own object (in parallel) and the objects link into one
shared library next to this file. The library exports only the C ABI declared in
``include/mrun_b200.h``; Python reaches it through ctypes (``mrun_b200._lib``) and through
``torch.ops.mrun_b200`` (``csrc/torch_ops.cpp``, compiled with g++ against torch's headers and
linked to the CUDA library by its soname, found next to it at load time).
"""
from __future__ import annotations

import concurrent.futures as _cf
import os
import shutil
import subprocess
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC_DIR = PACKAGE_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
BUILD_DIR = PACKAGE_DIR / "_build"
LIBRARY_PATH = PACKAGE_DIR / "libmrun_b200.so"
OPS_LIBRARY_PATH = PACKAGE_DIR / "libmrun_b200_torch.so"
OPS_SOURCE = CSRC_DIR / "torch_ops.cpp"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-I",
    str(INCLUDE_DIR),
]


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path("/usr/local/cuda/bin/nvcc")
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build mrun_b200")


def _sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in deps)


def build(*, force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile every CUDA source that changed and relink the library when needed."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    flags = NVCC_FLAGS + list(extra_flags or [])
    jobs = []
    objects = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers, Path(__file__)]):
            jobs.append([nvcc, *flags, "-c", str(src), "-o", str(obj)])

    def run(cmd: list[str]) -> None:
        if verbose:
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed for {cmd[-3]}:\n{proc.stdout}\n{proc.stderr}")
        if verbose and proc.stderr.strip():
            print(proc.stderr, flush=True)

    if jobs:
        workers = max(1, min(len(jobs), os.cpu_count() or 1))
        with _cf.ThreadPoolExecutor(max_workers=workers) as pool:
            for future in [pool.submit(run, job) for job in jobs]:
                future.result()
    if force or jobs or _stale(LIBRARY_PATH, objects):
        tmp = LIBRARY_PATH.with_suffix(".so.tmp")
        run([nvcc, *ARCH_FLAGS, "-shared", "-Xlinker", "-soname=libmrun_b200.so", "-o", str(tmp),
             *map(str, objects)])
        os.replace(tmp, LIBRARY_PATH)
    build_ops(force=force, verbose=verbose)
    return LIBRARY_PATH


def build_ops(*, force: bool = False, verbose: bool = False) -> Path:
    """Compile the torch.ops.mrun_b200 operator library (g++, torch's C++ ABI) when stale."""
    if not (force or _stale(OPS_LIBRARY_PATH, [OPS_SOURCE, LIBRARY_PATH, *_headers(), Path(__file__)])):
        return OPS_LIBRARY_PATH
    import torch
    from torch.utils import cpp_extension

    cuda_home = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    cmd = [shutil.which("g++") or "g++", "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch.compiled_with_cxx11_abi())}",
           *[f"-I{p}" for p in cpp_extension.include_paths()], f"-I{cuda_home / 'include'}", f"-I{INCLUDE_DIR}",
           str(OPS_SOURCE), "-o", str(OPS_LIBRARY_PATH.with_suffix(".so.tmp")),
           *[f"-L{p}" for p in cpp_extension.library_paths()], "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           "-lc10_cuda", f"-L{PACKAGE_DIR}", "-lmrun_b200", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"g++ failed for {OPS_SOURCE}:\n{proc.stdout}\n{proc.stderr}")
    os.replace(OPS_LIBRARY_PATH.with_suffix(".so.tmp"), OPS_LIBRARY_PATH)
    return OPS_LIBRARY_PATH


if __name__ == "__main__":  # pragma: no cover - manual rebuild entry point
    import sys

    print(build(force="--force" in sys.argv, verbose=True))
