"""CTA-pair tiles of the tcgen05 GEMM (gv, plain GEMM, sliced GEMM) against the one-SM kernel, bit for bit.

With REAX_GEMM_PAIR=1 a row-major GEMM runs on clusters of two CTAs: each tile is 256 rows, each CTA loads its own
128 rows of A and half of the tile's B rows, and the leader issues cta_group::2 MMAs that read both CTAs' halves and
accumulate into both CTAs' tensor memory.  Each output element still takes the same K = 16 MMA steps in the same k
order, so the outputs must equal the one-SM kernel's exactly -- with the pair kernel's split of the last waves too
(REAX_GEMM_SPLIT=1, the default: k-blocks of the last waves shared out over the clusters, partial accumulators of
both CTAs of a pair handed to the same CTAs of the next cluster).  The shapes cover 1, 3, 63 and 64 k-blocks per tile,
a pair whose second CTA holds no valid rows (M = 100), ragged N whose last tile's second B half lies past N, the
256- and 128-wide tiles, a strided output and the sliced GEMM's batches.  Every case also checks, through the CUDA
profiler's kernel list, that the pair kernel (split or not, as asked) is the one that ran."""
import contextlib
import os

import pytest
import torch
from torch.profiler import ProfilerActivity, profile

from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import synth

pytestmark = pytest.mark.gpu


@contextlib.contextmanager
def _env(**kv):
    old = {k: os.environ.get(k) for k in kv}
    os.environ.update(kv)
    try:
        yield
    finally:
        for k, v in old.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v


def _gemm_kernels(fn):
    """fn's result and the (SPLIT, PAIR) template flags of the gemm_kernel launches it made"""
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        out = fn()
        torch.cuda.synchronize()
    flags = set()
    for e in prof.events():
        if "gemm_kernel<" in e.name:
            args = [a.strip() for a in e.name.split("gemm_kernel<", 1)[1].split(">", 1)[0].split(",")]
            flags.add((args[-2] == "true", args[-1] == "true"))
    return out, flags


def _pair_tiles_split(tiles):
    clusters = torch.cuda.get_device_properties(0).multi_processor_count // 2
    return tiles > clusters and tiles % clusters != 0


def _both(fn, split="0", expect_split=False):
    """(one-SM unsplit result, pair result) of fn; asserts that the pair run used the pair kernel, split as expected"""
    with _env(REAX_GEMM_PAIR="0", REAX_GEMM_SPLIT="0"):
        a = fn()
        torch.cuda.synchronize()
    with _env(REAX_GEMM_PAIR="1", REAX_GEMM_SPLIT=split):
        b, flags = _gemm_kernels(fn)
    assert flags == {(expect_split, True)}, flags
    return a, b


def _same_bits(a, b):
    ia = a.view(torch.int16) if a.dtype == torch.bfloat16 else a.view(torch.int32)
    ib = b.view(torch.int16) if b.dtype == torch.bfloat16 else b.view(torch.int32)
    return torch.equal(ia, ib)


GV_CASES = [
    (2048, 14336, 4096),  # config 2
    (2048, 1792, 4096),   # its 8-way column shard
    (2000, 1800, 4000),   # ragged M, N2 and K (63 k-blocks, the last zero-filled)
    (1536, 2500, 136),    # 3 k-blocks
    (2304, 2400, 64),     # 1 k-block
    (100, 700, 304),      # one pair of rows, its second CTA entirely past M
]


@pytest.mark.parametrize("M,N2,K", GV_CASES)
@pytest.mark.parametrize("cfg,bn", [(0, 256), (1, 128)])
@pytest.mark.parametrize("split", ["0", "1"])
def test_gv_pair_equals_one_sm(M, N2, K, cfg, bn, split):
    x = synth.device_normal_bf16((M, K), 1.0, 71)
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 72)
    tiles = -(-M // 256) * -(-(2 * N2) // bn)
    a, b = _both(lambda: rk.gv(x, w, cfg=cfg), split, split == "1" and _pair_tiles_split(tiles))
    assert rk.status("libreax_gv") == 0
    assert _same_bits(a, b)


@pytest.mark.parametrize("cfg,bn", [(0, 256), (1, 128), (12, 64)])
@pytest.mark.parametrize("split", ["0", "1"])
def test_gemm_pair_equals_one_sm_strided_out(cfg, bn, split):
    M, N, K = 2048, 6000, 4096
    x = synth.device_normal_bf16((M, K), 1.0, 73)
    w = synth.device_normal_bf16((N, K), 0.02, 74)
    wide = torch.zeros(M, N + 40, dtype=torch.bfloat16, device="cuda")

    def run():
        wide.zero_()
        rk.gemm(x, w, cfg=cfg, out=wide[:, 8:8 + N])
        return wide.clone()

    a, b = _both(run, split, split == "1" and _pair_tiles_split((M // 256) * -(-N // bn)))
    assert rk.status("libreax_plain") == 0
    assert _same_bits(a, b)
    assert not b[:, :8].any() and not b[:, 8 + N:].any()  # nothing written outside the output view


@pytest.mark.parametrize("M", [256, 4096])
@pytest.mark.parametrize("part_fp32", [True, False])
@pytest.mark.parametrize("cfg,bn", [(0, 256), (1, 128), (8, 64)])
@pytest.mark.parametrize("split", ["0", "1"])
def test_slices_pair_equals_one_sm(M, part_fp32, cfg, bn, split):
    S, kps, N = 4, 1024, 4096  # config 4
    x = synth.device_normal_bf16((M, S * kps), 1.0, 75)
    w = synth.device_normal_bf16((N, S * kps), 0.02, 76)
    tiles = S * (M // 256) * (N // bn)
    a, b = _both(lambda: rk.slices(x, w, S, kps, part_fp32=part_fp32, cfg=cfg), split,
                 split == "1" and _pair_tiles_split(tiles))
    assert rk.status("libreax_slices") == 0
    assert _same_bits(a, b)


def test_pair_split_on_concurrent_streams_and_bounded_scratch():
    """Pair-split launches on several streams take blocks of the same bounded scratch pool as the one-SM split kernel:
    each gives the single-stream result bit for bit, and device memory stays within four scratch blocks of where it
    was."""
    M, N2, K = 2048, 1792, 4096
    xs = [synth.device_normal_bf16((M, K), 1.0, 77 + i) for i in range(2)]
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 79)
    with _env(REAX_GEMM_PAIR="1", REAX_GEMM_SPLIT="1"):
        alone = [rk.gv(x, w) for x in xs]
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        streams = [torch.cuda.Stream() for _ in range(6)]
        outs = [torch.empty_like(alone[0]) for _ in streams]
        for _ in range(3):
            for i, st in enumerate(streams):
                st.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(st):
                    rk.gv(xs[i % 2], w, out=outs[i])
            torch.cuda.synchronize()
            for i in range(len(streams)):
                assert _same_bits(outs[i], alone[i % 2])
        free1 = torch.cuda.mem_get_info()[0]
    assert rk.status("libreax_gv") == 0
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    block = sms * 128 * 256 * 4 + 8 * sms * 4 + 256
    assert free0 - free1 <= 4 * block + (2 << 20), (free0 - free1) / 1e6
