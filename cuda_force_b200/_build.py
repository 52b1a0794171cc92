"""Builds the in-tree native libraries.

* ``libcudaforge_b200.so`` — the C-ABI library (``include/cudaforge_b200.h``),
  compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``),
  no fast-math: the quantiser relies on IEEE division and round-half-even.
* ``_C.so`` — the thin PyTorch dispatcher shim that registers the reference's
  ``torch.ops.cudaforge`` schemas over the C ABI. Plain g++ against torch's
  headers; it links ``libcudaforge_b200.so`` through ``$ORIGIN``.

Both land next to this file so they travel with the source tree. Rebuilds only
when a source is newer than its output.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libcudaforge_b200.so"
SHIM = PKG / "_C.so"

CUDA_SOURCES = ["abi.cu", "quant.cu", "lora_gemm.cu", "norm.cu"]
HEADERS = ["quant_math.cuh", "cf_common.cuh", "ptx.cuh"]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _cuda_home() -> Path:
    env = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if env:
        return Path(env)
    return Path("/usr/local/cuda")


def _stale(output: Path, inputs: list[Path]) -> bool:
    if not output.exists():
        return True
    built = output.stat().st_mtime
    return any(p.exists() and p.stat().st_mtime > built for p in inputs)


def _run(cmd: list[str]) -> None:
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(result.stdout + result.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")


def build_library(force: bool = False, verbose: bool = False) -> Path:
    nvcc = str(_cuda_home() / "bin" / "nvcc")
    sources = [CSRC / s for s in CUDA_SOURCES]
    deps = sources + [CSRC / h for h in HEADERS] + [INCLUDE / "cudaforge_b200.h", Path(__file__)]
    if not force and not _stale(LIB, deps):
        return LIB
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    objects = []
    for src in sources:
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
        objects.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    _run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objects, "-o", str(tmp)])
    os.replace(tmp, LIB)
    return LIB


def build_shim(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "torch_shim.cpp"
    deps = [src, INCLUDE / "cudaforge_b200.h", LIB, Path(__file__)]
    if not force and not _stale(SHIM, deps):
        return SHIM
    import sysconfig

    include_dirs = cpp_extension.include_paths() + [
        str(_cuda_home() / "include"), str(INCLUDE), sysconfig.get_paths()["include"]]
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = SHIM.with_suffix(".so.tmp")
    cmd = [
        "g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        *[f"-I{d}" for d in include_dirs], str(src), "-o", str(tmp),
        f"-L{torch_lib}", "-lc10", "-ltorch_cpu", "-ltorch", "-lc10_cuda",
        f"-L{PKG}", "-l:libcudaforge_b200.so",
        "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}",
    ]
    _run(cmd)
    os.replace(tmp, SHIM)
    return SHIM


def build_all(force: bool = False) -> None:
    build_library(force=force)
    build_shim(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(LIB)
    print(SHIM)
