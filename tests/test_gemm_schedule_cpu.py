"""The GEMM kernels' work distribution, checked on the CPU from the package's own header.

tests/cpu_helpers/worklist_check.cu includes csrc/gemm_sm100.cuh and runs reax::WorkList -- the same host/device code
every GEMM CTA uses to pick its tiles and k-blocks -- for work-unit counts of 148 and 132 SMs, their pairs (74 and 66
clusters of two for the CTA-pair kernels) and small counts.  It uses k-blocks per tile from 1 to 128 and every tile
count up to four waves past the unit count, unsplit and with the split last waves.  It checks that every k-block of
every tile is run exactly once, that a tile is cut at most once, that a head piece (unit c) and the tail piece
(unit c + 1) agree on the tile and the cut, that every share holds a whole tile, and that with two or more waves split
a whole tile separates a unit's head from its tail.  The kernels' hand-over of partial accumulators, and their freedom
from waits on one another in a chain, rest on these properties.  nvcc compiles the program for the host; no GPU is
used.
"""
import os
import shutil
import subprocess
import tempfile

import pytest

from reax_engine_kernels_b200 import build as B

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists(B.NVCC), reason="needs nvcc")
def test_gemm_work_distribution():
    nvcc = shutil.which("nvcc") or B.NVCC
    with tempfile.TemporaryDirectory() as td:
        exe = os.path.join(td, "worklist_check")
        cmd = [nvcc] + B.ARCH + ["-O2", "-std=c++17", "-I", B.CSRC,
                                 os.path.join(HERE, "cpu_helpers", "worklist_check.cu"), "-o", exe]
        subprocess.run(cmd, check=True, capture_output=True)
        r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok "), r.stdout
    assert int(r.stdout.split()[1]) > 10000
