"""Failure detection in the product kernels: the gate-up GEMM's and the attention kernels' own pipelines give up
mid-launch, unwind and report.

libreax_gv is rebuilt here from its own sources with the wait limit cut to ~20 K cycles (about 10 us) and the
suspension between checks to 0.5 us.  A 128 x 256 tile of BASELINE config 2 takes ~25 us, so the epilogue's first wait
for an accumulator runs out while the TMA producer and the MMA issuer are mid-pipeline.  The roles must then unwind as
built: the abort flag stops the others at their next wait, the producer waits for every copy it armed, the MMA issuer
for every MMA it issued, TMEM is released and the CTAs exit.  Checked: the launch returns, the library's status word
holds a pipeline timeout code (and reading clears it), and the same context then computes a layer correctly with the
normal build -- for the one-SM and the CTA-pair kernels, each unsplit and with the split last waves (whose epilogue
warps also wait on partial-accumulator flags published by other CTAs).  The pair kernels also exchange their
producers' fill counts at teardown, so that neither CTA of a pair leaves while a copy it issued, counted on the other
CTA's barrier, may still be in flight.  No fault and no hang is involved: only bounded waits run out.
"""
import ctypes
import os
import shutil
import subprocess
import tempfile

import pytest
import torch

from reax_engine_kernels_b200 import build as B
from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import synth

pytestmark = pytest.mark.gpu

TIMEOUT_CODES = {0x101, 0x102, 0x103, 0x104, 0x106}  # producer, MMA (stage / accumulator), epilogue, split flag


@pytest.fixture(scope="module")
def short_limit_gv():
    nvcc = shutil.which("nvcc") or B.NVCC
    with tempfile.TemporaryDirectory() as td:
        so = os.path.join(td, "libreax_gv_shortwait.so")
        cmd = ([nvcc] + B.ARCH + B.NVCC_FLAGS + ["-DREAX_WAIT_LIMIT=(20000ll)", "-DREAX_WAIT_SLEEP_NS=500",
                                                  os.path.join(B.CSRC, "gv.cu"), "-o", so])
        subprocess.run(cmd, check=True, capture_output=True)
        lib = ctypes.CDLL(so)
        lib.reax_gv.restype = ctypes.c_int
        lib.reax_gv.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
        lib.reax_b200_status.restype = ctypes.c_int
        lib.reax_b200_status.argtypes = [ctypes.c_void_p]
        yield lib


@pytest.mark.parametrize("N2,pair,split", [(14336, "0", "0"), (1792, "0", "1"), (14336, "1", "0"), (1792, "1", "1")])
def test_gemm_pipeline_gives_up_and_context_survives(short_limit_gv, N2, pair, split):
    M, K = 2048, 4096
    x = synth.device_normal_bf16((M, K), 1.0, 81)
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 82)
    out = torch.zeros(M, N2, dtype=torch.bfloat16, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    env = {"REAX_GEMM_SPLIT": split, "REAX_GEMM_PAIR": pair}
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        assert short_limit_gv.reax_gv(0, x.data_ptr(), w.data_ptr(), out.data_ptr(), M, N2, K, s) == 0
        torch.cuda.synchronize()  # the launch ends: no hang
        code = short_limit_gv.reax_b200_status(s)
        assert code in TIMEOUT_CODES, hex(code)
        assert short_limit_gv.reax_b200_status(s) == 0  # read and cleared
        # the context is intact: the normal build computes the layer, identical to a fresh computation
        a = rk.gv(x, w)
        b = rk.gv(x, w)
        torch.cuda.synchronize()
        assert rk.status("libreax_gv") == 0
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        assert bool(torch.isfinite(a.float()).all())
    finally:
        for k, v in old.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v


@pytest.fixture(scope="module")
def zero_limit_fmha():
    """libreax_fmha_post rebuilt with no patience at all: the first wait that is not already satisfied gives up (every
    attention wait lasts a few us, so a finite short limit would not reliably run out).  The producer has issued its
    first Q / K / V copies by then, so the drain of copies in flight is exercised."""
    from reax_engine_kernels_b200 import abi

    nvcc = shutil.which("nvcc") or B.NVCC
    with tempfile.TemporaryDirectory() as td:
        so = os.path.join(td, "libreax_fmha_post_nowait.so")
        cmd = ([nvcc] + B.ARCH + B.NVCC_FLAGS + ["-DREAX_WAIT_LIMIT=(0ll)", "-DREAX_WAIT_SLEEP_NS=50",
                                                  os.path.join(B.CSRC, "fmha_post_lib.cu"), "-o", so])
        subprocess.run(cmd, check=True, capture_output=True)
        lib = ctypes.CDLL(so)
        for name in ("reax_fmha_q_hd", "reax_b200_status"):
            res, args = abi.PROTOTYPES["libreax_fmha_post"][name]
            getattr(lib, name).restype, getattr(lib, name).argtypes = res, args
        yield lib


@pytest.mark.parametrize("B_,H", [(1, 2), (4, 8)])  # 64 CTAs of one query tile; 1024 two-tile CTAs (fmha2_kernel)
def test_attention_pipeline_gives_up_and_context_survives(zero_limit_fmha, B_, H):
    import math

    G, S, D = 4, 2048, 128
    M = S * G
    q = synth.device_normal_bf16((B_, H, M, D), 1.0, 83)
    k = synth.device_normal_bf16((B_, H, S, D), 1.0, 84)
    v = synth.device_normal_bf16((B_, H, S, D), 1.0, 85)
    qpos = torch.arange(S, dtype=torch.int32, device="cuda").repeat(B_, 1).contiguous()
    out = torch.zeros(B_, H, M, D, dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    st = lambda t: (t.stride(0), t.stride(1), t.stride(2))
    rc = zero_limit_fmha.reax_fmha_q_hd(q.data_ptr(), k.data_ptr(), v.data_ptr(), qpos.data_ptr(), G, S,
                                        out.data_ptr(), 1 / math.sqrt(D), B_, H, M, S, *st(q), *st(k), *st(v), *st(out),
                                        D, s)
    assert rc == 0
    torch.cuda.synchronize()  # the launch ends: no hang
    assert zero_limit_fmha.reax_b200_status(s) == 0x201  # attention pipeline wait
    assert zero_limit_fmha.reax_b200_status(s) == 0
    a = rk.fmha(q, k, v, 1 / math.sqrt(D), qpos=qpos, G=G)
    b = rk.fmha(q, k, v, 1 / math.sqrt(D), qpos=qpos, G=G)
    torch.cuda.synchronize()
    assert rk.status("libreax_fmha_post") == 0
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert bool(torch.isfinite(a.float()).all())
