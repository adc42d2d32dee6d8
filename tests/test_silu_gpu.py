"""The gate of the fused gated RMSNorm (reax_howu_norm): silu_gate computes z / (1 + exp(-z)) by Markstein's quotient
(approximate reciprocal, one Newton step, one remainder correction) instead of the IEEE division with its out-of-range
branch.  It must give exactly the IEEE quotient's bits: checked here for all 65536 bf16 gates (the gate z is a bf16
input), NaN matching NaN."""
import ctypes
import os
import shutil
import subprocess
import tempfile

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "reax_engine_kernels_b200", "csrc")


@pytest.mark.gpu
def test_silu_gate_is_bitwise_the_ieee_quotient_for_every_bf16_gate():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    with tempfile.TemporaryDirectory() as td:
        so = os.path.join(td, "libsilu_check.so")
        subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-shared",
                        "-Xcompiler", "-fPIC", "-I", CSRC, os.path.join(HERE, "gpu_helpers", "silu_check.cu"), "-o", so],
                       check=True, capture_output=True)
        lib = ctypes.CDLL(so)
        out = (ctypes.c_uint * 2)()
        assert lib.run_silu_check(out) == 0
        assert out[0] == 0, f"{out[0]} bf16 gates differ, first pattern {out[1]:#06x}"
