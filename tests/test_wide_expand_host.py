"""The wide product's Q4_K / Q5_K weight expansion, the kernel's own
per-thread source (inferq_b200/csrc/wide_expand.cuh) compiled for the host
and run on the CPU (tests/native/wide_expand_check.cu): every operand value
sc*q (Q4_K) or sc*(q-16) (Q5_K) and every min / centring tile entry equals an
independent decode of random GGUF blocks put into the device layout."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _nvcc():
    for cand in ("/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    return None


def test_expansion_matches_an_independent_decode(tmp_path):
    nvcc = _nvcc()
    if nvcc is None:
        pytest.skip("nvcc not found")
    exe = tmp_path / "wide_expand_check"
    build = subprocess.run([nvcc, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a",
                            "-I" + str(ROOT / "inferq_b200" / "csrc"), "-I" + str(ROOT / "include"),
                            str(ROOT / "tests" / "native" / "wide_expand_check.cu"), "-o", str(exe)],
                           capture_output=True, text=True, timeout=600)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    print(run.stdout)
    assert run.returncode == 0, run.stdout
    assert "Q5_K expansion: 131 rows x 3 blocks, 0 mismatches" in run.stdout
