"""The decode kernel's stream-K partitions, checked on the CPU: tests/streamk_check.cu (host code only, the same
header the kernel's host side uses) is compiled with nvcc and run; it verifies full, non-overlapping coverage of every
part by stages, cuts at stage starts, one finalizer and at most 16 contributors per tile, for several shapes and
grid sizes, and that the 20b shape's gate/up split is the equal-unit split."""
import os
import shutil
import subprocess
import tempfile
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


def _nvcc():
    for c in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    return None


def test_streamk_partitions():
    nvcc = _nvcc()
    if nvcc is None:
        pytest.skip("nvcc not found")
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "streamk_check")
        r = subprocess.run([nvcc, "-std=c++17", "-O1", "-Wno-deprecated-gpu-targets", "-o", exe,
                            str(HERE / "streamk_check.cu")], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stdout + r.stderr
        out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
        assert out.returncode == 0 and out.stdout.strip().endswith("OK"), out.stdout + out.stderr
