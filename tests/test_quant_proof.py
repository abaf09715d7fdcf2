"""CPU: the exhaustive proof behind the quantizer's branch-free rounding.

tests/native/quant_exhaustive.c checks, for every fp16 absmax and every fp16
|x| <= absmax (503,856,639 pairs), that the division-free quotient of
quant_math.cuh (Markstein's correction step on fl(|x| * fl(1/s))) equals the
correctly rounded |x| / s and that the integer equals the reference's
trunc(fl(q + 0.5)) clamped to 127. It runs in seconds with gcc.
"""
import shutil
import subprocess
from pathlib import Path

import pytest

SRC = Path(__file__).resolve().parent / "native" / "quant_exhaustive.c"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_branch_free_rounding_is_exact_on_every_fp16_pair(tmp_path):
    exe = tmp_path / "quant_exhaustive"
    subprocess.run(["gcc", "-std=c11", "-O2", "-mfma", "-ffp-contract=off", "-fopenmp", str(SRC), "-o", str(exe),
                    "-lm"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "checked 503856639 pairs: quotient mismatches 0, integer mismatches 0" in out.stdout, out.stdout
