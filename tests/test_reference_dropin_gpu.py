"""The reference's Python package driving this build's kernels on the GPU.

``cudaforge`` resolves to the reference's own package (the copy installed
into ``baseline/_ref`` from the reference checkout, which travels with the
repository; or the checkout itself where it is mounted) with this build's
``_C.so`` as ``cudaforge._C``. The reference's wrapper then routes CUDA
tensors to ``torch.ops.cudaforge.*`` exactly as it would route them to its
own extension, and ``tests/dropin_gpu_checks.py`` runs the reference's
on-GPU parity checks (examples/kernel_parity.py:57-133) and operator-test
tolerances through it.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

from oracle import build_ref
from tests.test_reference_dropin import make_stub

ROOT = Path(__file__).resolve().parents[1]

pytestmark = pytest.mark.gpu


def reference_package() -> Path | None:
    installed = ROOT / "baseline" / "_ref" / "cudaforge"
    if (installed / "ops.py").exists():
        return installed
    root = build_ref.reference_root()
    if root is not None and (root / "python" / "cudaforge" / "ops.py").exists():
        return root / "python" / "cudaforge"
    return None


def test_reference_wrapper_runs_this_build_on_the_gpu(tmp_path, cuda_device):
    pkg = reference_package()
    if pkg is None:
        pytest.skip("the reference's Python package is not installed (baseline/_ref)")
    root = make_stub(tmp_path / "dropin", pkg)
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=os.pathsep.join([str(root), str(pkg.parent)]))
    result = subprocess.run([sys.executable, str(ROOT / "tests" / "dropin_gpu_checks.py")],
                            env=env, cwd=root, capture_output=True, text=True, timeout=600)
    assert result.stdout.strip(), result.stderr[-3000:]
    out = json.loads(result.stdout.strip().splitlines()[-1])
    assert Path(out["extension"]).resolve() == (ROOT / "cuda_force_b200" / "_C.so").resolve()
    failed = [c for c in out["checks"] if not c["ok"]]
    assert not failed and result.returncode == 0, failed
    assert len(out["checks"]) >= 35
