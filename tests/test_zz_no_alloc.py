"""reax_gv_noalloc: the gate-up entry point for callers that cannot allocate device memory.

An engine that reserves all of the GPU's memory for its own arena, or a serving loop that cannot let a library call
cudaMalloc in the middle of a step, calls reax_gv_noalloc instead of reax_gv: it takes the split-last-waves scratch
from a static array in the library rather than allocating it.  Called through the C ABI twice in a row on each
shape, its output must equal reax_gv's bit for bit (the two run the same kernels; equality is the tolerance the
gate-up tests use between kernel variants), and the device status word must stay clear.  The shapes take the split
kernel, which uses the scratch (BASELINE config 2's 4- and 8-way column shards, a ragged one, 128-wide tiles), and
one takes the unsplit kernel.  This file sorts last, so a run that stops at the first failure has run every other
test before it; it also passes alone in a fresh process (the first call does the per-device set-up)."""
import ctypes

import pytest
import torch

from reax_engine_kernels_b200 import abi
from reax_engine_kernels_b200 import synth

pytestmark = pytest.mark.gpu

CASES = [
    (2048, 1792, 4096, 0),   # 8-way shard of config 2: 1.51 waves, split
    (2048, 3584, 4096, 0),   # 4-way shard: 3.03 waves, split
    (2000, 1800, 4000, 0),   # ragged M, N2, K
    (2048, 1792, 4096, 1),   # 128-wide tiles: 3.03 waves, split
    (256, 512, 1024, 0),     # 8 tiles: unsplit
]


def _call(fn, x, w, out, M, N2, K, cfg):
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return fn(cfg, x.data_ptr(), w.data_ptr(), out.data_ptr(), M, N2, K, s)


@pytest.mark.parametrize("M,N2,K,cfg", CASES)
def test_noalloc_equals_reax_gv_twice_in_a_row(M, N2, K, cfg):
    lib = abi.load("libreax_gv")
    x = synth.device_normal_bf16((M, K), 1.0, 71)
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 72)
    ref = torch.empty(M, N2, dtype=torch.bfloat16, device="cuda")
    assert _call(lib.reax_gv, x, w, ref, M, N2, K, cfg) == 0
    for _ in range(2):
        out = torch.full((M, N2), float("nan"), dtype=torch.bfloat16, device="cuda")
        assert _call(lib.reax_gv_noalloc, x, w, out, M, N2, K, cfg) == 0
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    assert lib.reax_b200_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0


def test_noalloc_rejects_bad_arguments_without_launching():
    lib = abi.load("libreax_gv")
    x = synth.device_normal_bf16((128, 64), 1.0, 73)
    w = synth.device_normal_bf16((256, 64), 0.02, 74)
    out = torch.empty(128, 128, dtype=torch.bfloat16, device="cuda")
    assert _call(lib.reax_gv_noalloc, x, w, out, 128, 128, 60, 0) == 1   # K % 8
    assert _call(lib.reax_gv_noalloc, x, w, out, 128, 126, 64, 0) == 1   # N2 % 4
    assert _call(lib.reax_gv_noalloc, x, w, out, 128, 128, 64, 20) == 9  # unknown cfg
