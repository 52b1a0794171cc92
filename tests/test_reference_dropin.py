"""The reference's own operator tests, run with this build as its extension.

CPU only, and only where the reference tree is available (the build
container); skipped elsewhere. A package stub under ``oracle/_ref/dropin``
makes ``cudaforge`` resolve to the reference's Python package, with this
build's ``_C.so`` in place of the reference's ``cudaforge._C``
(python/cudaforge/ops.py:44-58 imports it and asks
``cuda_kernels_available()``). The reference's tests for the operators, their
autograd guard, the block-size constant and the LoRA module then run
unmodified through the dispatcher schemas this build registers: host tensors
reach the host kernels, as they reach the reference's.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

from oracle import build_ref

ROOT = Path(__file__).resolve().parents[1]
_REF_ROOT = build_ref.reference_root() or ROOT / "missing-reference"
REF_PKG = _REF_ROOT / "python" / "cudaforge"
REF_TESTS = _REF_ROOT / "tests" / "python"
DROPIN = ROOT / "oracle" / "_ref" / "dropin"

STUB = '''"""The reference package with another build's extension module first on its path."""
import os
_REF = {ref!r}
__path__ = [os.path.dirname(os.path.abspath(__file__)), _REF]
__file__ = os.path.join(_REF, "__init__.py")
exec(compile(open(__file__).read(), __file__, "exec"))
'''


def make_stub(dropin: Path, ref_pkg: Path) -> Path:
    """A ``cudaforge`` package under ``dropin`` that runs the reference package at
    ``ref_pkg`` with this build's extension modules first on its path."""
    pkg = dropin / "cudaforge"
    pkg.mkdir(parents=True, exist_ok=True)
    (pkg / "__init__.py").write_text(STUB.format(ref=str(ref_pkg)))
    for name in ("_C.so", "libcudaforge_b200.so"):
        link = pkg / name
        if link.is_symlink() or link.exists():
            link.unlink()
        link.symlink_to(ROOT / "cuda_force_b200" / name)
    return dropin


@pytest.mark.skipif(not (REF_PKG / "ops.py").exists(), reason="reference tree not available")
def test_reference_operator_tests_pass_with_this_extension():
    root = make_stub(DROPIN, REF_PKG)
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=os.pathsep.join([str(root), str(_REF_ROOT)]))
    files = [str(REF_TESTS / f) for f in ("test_ops.py", "test_autograd.py",
                                           "test_constant_parity.py", "test_lora.py")]
    probe = ("from cudaforge import ops; r = ops.backend_report(); "
             "assert r.extension_loaded and r.cuda_compiled, r")
    subprocess.run([sys.executable, "-c", probe], env=env, cwd=root, check=True, timeout=300)
    result = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", *files],
        env=env, cwd=root, capture_output=True, text=True, timeout=600)
    tail = "\n".join(result.stdout.splitlines()[-15:])
    assert result.returncode == 0, tail
    assert " passed" in tail and "failed" not in tail, tail
