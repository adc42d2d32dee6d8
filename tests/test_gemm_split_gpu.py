"""Split last waves of the tcgen05 GEMM (gv, plain GEMM, sliced GEMM) against the unsplit kernel, bit for bit.

When a GEMM's tiles leave a partly full last wave, the launcher hands the last one to three waves of tiles out by
k-blocks; a tile cut between two CTAs carries its fp32 accumulator from one to the other, so every output keeps the
unsplit kernel's k order and the two kernels must agree exactly.  REAX_GEMM_SPLIT=0 / 1 forces each kernel; these
tests run the one-SM kernels (REAX_GEMM_PAIR=0: the CTA-pair kernels are checked in tests/test_gemm_pair_gpu.py).  The
shapes cover 1, 3, 63 and 64 k-blocks per tile, ragged M / N / K tails, the 256-, 128- and 64-wide tiles, and the
BASELINE config-2 layer and its 8-way column shard.  The unsplit kernel itself is pinned to the fp64 oracle in
tests/test_gemm_gpu.py."""
import contextlib
import os

import pytest
import torch

from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import synth

pytestmark = pytest.mark.gpu


@contextlib.contextmanager
def _split(mode):
    env = {"REAX_GEMM_SPLIT": mode, "REAX_GEMM_PAIR": "0"}
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        yield
    finally:
        for k, v in old.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v


def _both(fn):
    with _split("0"):
        a = fn()
    with _split("1"):
        b = fn()
    torch.cuda.synchronize()
    return a, b


def _takes_split(tiles):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    return tiles > sms and tiles % sms != 0


def _cdiv(a, b):
    return (a + b - 1) // b


def _same_bits(a, b):
    ia = a.view(torch.int16) if a.dtype == torch.bfloat16 else a.view(torch.int32)
    ib = b.view(torch.int16) if b.dtype == torch.bfloat16 else b.view(torch.int32)
    return torch.equal(ia, ib)


GV_CASES = [
    (2048, 14336, 4096),  # config 2
    (2048, 1792, 4096),   # its 8-way column shard
    (2000, 1800, 4000),   # ragged M, N2 and K (63 k-blocks, the last zero-filled)
    (1536, 2500, 136),    # 3 k-blocks
    (2304, 2400, 64),     # 1 k-block: tiles are never cut, only re-dealt
]


@pytest.mark.parametrize("M,N2,K", GV_CASES)
@pytest.mark.parametrize("cfg,bn", [(0, 256), (1, 128)])
def test_gv_split_equals_unsplit(M, N2, K, cfg, bn):
    assert _takes_split(_cdiv(M, 128) * _cdiv(2 * N2, bn))
    x = synth.device_normal_bf16((M, K), 1.0, 51)
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 52)
    a, b = _both(lambda: rk.gv(x, w, cfg=cfg))
    assert rk.status("libreax_gv") == 0
    assert _same_bits(a, b)


@pytest.mark.parametrize("cfg,bn", [(0, 256), (1, 128), (12, 64)])
def test_gemm_split_equals_unsplit_strided_out(cfg, bn):
    M, N, K = 2048, 6000, 4096
    assert _takes_split(_cdiv(M, 128) * _cdiv(N, bn))
    x = synth.device_normal_bf16((M, K), 1.0, 53)
    w = synth.device_normal_bf16((N, K), 0.02, 54)
    wide = torch.zeros(M, N + 40, dtype=torch.bfloat16, device="cuda")

    def run():
        wide.zero_()
        rk.gemm(x, w, cfg=cfg, out=wide[:, 8:8 + N])
        return wide.clone()

    a, b = _both(run)
    assert rk.status("libreax_plain") == 0
    assert _same_bits(a, b)
    assert not wide[:, :8].any() and not wide[:, 8 + N:].any()  # nothing written outside the output view


@pytest.mark.parametrize("cfg,bn", [(0, 256), (1, 128), (8, 64)])
@pytest.mark.parametrize("part_fp32", [True, False])
def test_slices_split_equals_unsplit(cfg, bn, part_fp32):
    M, N, S, kps = 4096, 4096, 4, 1024  # config 4
    assert _takes_split(S * _cdiv(M, 128) * _cdiv(N, bn))
    x = synth.device_normal_bf16((M, S * kps), 1.0, 55)
    w = synth.device_normal_bf16((N, S * kps), 0.02, 56)
    a, b = _both(lambda: rk.slices(x, w, S, kps, part_fp32=part_fp32, cfg=cfg))
    assert rk.status("libreax_slices") == 0
    assert _same_bits(a, b)


def test_gv_split_on_concurrent_streams():
    """Split launches on two streams take different scratch blocks of the pool and may run at the same time: each
    gives the output it gives alone."""
    M, N2, K = 2048, 1792, 4096
    xs = [synth.device_normal_bf16((M, K), 1.0, 60 + i) for i in range(2)]
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 62)
    with _split("1"):
        alone = [rk.gv(x, w) for x in xs]
        torch.cuda.synchronize()
        streams = [torch.cuda.Stream() for _ in range(2)]
        outs = [None, None]
        for _ in range(3):
            for i, s in enumerate(streams):
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    outs[i] = rk.gv(xs[i], w)
            torch.cuda.synchronize()
            for i in range(2):
                assert _same_bits(outs[i], alone[i])
    assert rk.status("libreax_gv") == 0


def test_split_scratch_stays_bounded_across_many_streams():
    """The split kernel's scratch comes from a pool of at most four blocks per device, whichever streams launch it:
    split launches on twelve fresh streams give the single-stream result bit for bit and leave device memory within
    four scratch blocks (18.9 MB each on a 148-SM GPU) of where it was."""
    M, N2, K = 2048, 1792, 4096
    x = synth.device_normal_bf16((M, K), 1.0, 63)
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 64)
    with _split("1"):
        ref = rk.gv(x, w)
        outs = [torch.empty_like(ref) for _ in range(12)]
        streams = [torch.cuda.Stream() for _ in range(12)]
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for s, o in zip(streams, outs):
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                rk.gv(x, w, out=o)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
    assert rk.status("libreax_gv") == 0
    for o in outs:
        assert _same_bits(o, ref)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    block = sms * 128 * 256 * 4 + 8 * sms * 4 + 256
    assert free0 - free1 <= 4 * block + (2 << 20), (free0 - free1) / 1e6
