"""Compiles the reference's own native CPU operators into ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY: the product never loads this library. Tests, the
``cpu_baseline`` leg of ``bench.py`` and ``bench.py --impl reference`` use it as
the reference implementation of the path on the host cores.

Recipe: the single translation unit ``cpp/src/bindings.cpp`` of the reference
(CudaForge) is compiled unmodified with g++ against PyTorch's headers, without
``CUDAFORGE_WITH_CUDA``, so only its CPU implementations are built
(bindings.cpp:255-329, registered at :379-390). ``-Dcudaforge=cudaforge_ref``
renames its C++ and operator namespace, so its ops appear as
``torch.ops.cudaforge_ref.*`` and can be loaded in the same process as this
package's ``torch.ops.cudaforge.*``. The reference's build system (CMake,
setup.py) is not used. Sources are read where they lie; nothing is copied.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
OUT = OUT_DIR / "cudaforge_ref_cpu.so"


def reference_root() -> Path | None:
    """The reference checkout: ``$CUDAFORGE_REFERENCE``, else BASELINE.json's
    ``reference_path``; None when neither names one."""
    env = os.environ.get("CUDAFORGE_REFERENCE")
    if env:
        return Path(env)
    baseline = HERE.parent / "BASELINE.json"
    if baseline.exists():
        import json

        path = json.loads(baseline.read_text()).get("reference_path")
        if path:
            return Path(path)
    return None


def build(force: bool = False) -> Path | None:
    """Builds the library if the reference tree is present; returns its path or None."""
    root = reference_root()
    src = root / "cpp" / "src" / "bindings.cpp" if root is not None else None
    if src is None or not src.exists():
        return OUT if OUT.exists() else None
    if OUT.exists() and not force and OUT.stat().st_mtime > src.stat().st_mtime:
        return OUT
    import torch
    from torch.utils import cpp_extension

    OUT_DIR.mkdir(exist_ok=True)
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    includes = cpp_extension.include_paths() + [
        sysconfig.get_paths()["include"],
        str(root / "cpp" / "include"),
        str(root / "cuda" / "include"),
    ]
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [
        "g++", "-O3", "-std=c++20", "-shared", "-fPIC",
        f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
        "-Dcudaforge=cudaforge_ref", "-DTORCH_EXTENSION_NAME=cudaforge_ref_cpu",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        *[f"-I{d}" for d in includes], str(src), "-o", str(tmp),
        f"-L{torch_lib}", "-lc10", "-ltorch_cpu", "-ltorch", "-ltorch_python",
        f"-Wl,-rpath,{torch_lib}",
    ]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(result.stderr[-4000:])
        raise RuntimeError("building the reference CPU operators failed")
    os.replace(tmp, OUT)
    return OUT


def load() -> bool:
    """Registers torch.ops.cudaforge_ref.* in this process. False if not built."""
    import torch

    if not OUT.exists():
        return False
    if not hasattr(torch.ops, "cudaforge_ref") or not hasattr(torch.ops.cudaforge_ref, "quantize_int8"):
        torch.ops.load_library(str(OUT))
    return True


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
