"""Failure detection without a GPU fault: the bounded mbarrier wait every kernel of the package uses gives up, records
a status code and lets the kernel return when the awaited event never happens.

A helper (tests/gpu_helpers/bounded_wait.cu, built here with nvcc for sm_100a from the package's own header, with
the wait limit shortened to ~2 M cycles, about 1 ms) waits on an mbarrier that nothing arrives on.  The test checks
that every thread's wait returned failure, that the CTA's abort flag and the device status word were set, and that
an ordinary kernel still runs in the same context afterwards.
"""
import ctypes
import os
import shutil
import subprocess
import tempfile

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "reax_engine_kernels_b200", "csrc")
ST_TIMEOUT_ATTN = 0x201


@pytest.mark.gpu
def test_bounded_wait_gives_up_and_reports():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    with tempfile.TemporaryDirectory() as td:
        so = os.path.join(td, "libbounded_wait.so")
        subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-shared",
                        "-Xcompiler", "-fPIC", "-DREAX_WAIT_LIMIT=(1ll<<21)", "-I", CSRC,
                        os.path.join(HERE, "gpu_helpers", "bounded_wait.cu"), "-o", so],
                       check=True, capture_output=True)
        lib = ctypes.CDLL(so)
        lib.reax_b200_status.restype = ctypes.c_int
        lib.reax_b200_status.argtypes = [ctypes.c_void_p]
        res = (ctypes.c_int * 2)()
        assert lib.run_stuck_wait(res) == 0            # the kernel returned: no hang, no fault
        assert res[0] == 64, res[0]                    # every thread's wait reported failure
        assert res[1] == 1                             # the CTA-wide abort flag was raised
        assert lib.reax_b200_status(None) == ST_TIMEOUT_ATTN  # the device status word names the timed-out wait
        assert lib.reax_b200_status(None) == 0         # reading it clears it
        val = ctypes.c_int(0)
        assert lib.run_after(ctypes.byref(val)) == 0   # the context is still usable
        assert val.value == 1
