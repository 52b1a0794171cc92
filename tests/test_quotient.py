"""CPU proof obligation of the quantiser's division-free code path.

The kernels form fl32(x / s) as q0 = x*r, e = fma(-q0, s, x), q = fma(e, r, q0)
with r = fl32(1/s) and round q half-to-even. tests/native/verify_quotient.c
compares that code against rint(fl32(x / s)) for every (x, absmax) pair of bf16
and fp16 (about 1.9e9 pairs) and a seeded fp32 sample steered onto
half-integer quotients. Any mismatch fails.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent


def test_division_free_codes_match_ieee_division(tmp_path):
    exe = tmp_path / "verify_quotient"
    subprocess.run(["gcc", "-O2", "-std=c11", "-fno-fast-math", "-ffp-contract=off",
                    str(HERE / "native" / "verify_quotient.c"), "-o", str(exe), "-lm"], check=True)
    out = subprocess.run([str(exe), "4000000"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "bf16 pairs 878165502 mismatches 0" in out.stdout
    assert "f16 pairs 1007713278 mismatches 0" in out.stdout
    assert "mismatches 0" in out.stdout.splitlines()[-1]
