"""GEMM family (libreax_gv / libreax_plain / libreax_slices) on the GPU against the fp64 oracle.

Small and medium shapes are checked in full; BASELINE-sized shapes are checked on a sample of rows (every row
of a GEMM output is independent, so a row sample is an unbiased parity check of the whole kernel)."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import synth
from tests.tolerance import assert_close, assert_close_interval

pytestmark = pytest.mark.gpu
bf = synth.bf16_bits_to_f32


def _inputs(M, N, K, seed, xstd=1.0, wstd=0.02):
    x = synth.bf16_normal(seed, (M, K), xstd)
    w = synth.bf16_normal(seed + 1, (N, K), wstd)
    return x, w, synth.to_torch_bf16(x), synth.to_torch_bf16(w)


@pytest.mark.parametrize("M,N2,K", [(128, 128, 64), (256, 512, 256), (200, 300, 136), (1, 64, 4096), (130, 1024, 4096)])
@pytest.mark.parametrize("cfg", [0, 2])
def test_gv_vs_oracle(M, N2, K, cfg):
    x, w, xt, wt = _inputs(M, 2 * N2, K, 100 + M)
    out = synth.from_torch_bf16(rk.gv(xt, wt, cfg=cfg))
    assert rk.status("libreax_gv") == 0
    ref, lo, hi = orc.gv(x, w)
    assert_close_interval(bf(out), bf(ref), bf(lo), bf(hi))


def test_gv_baseline_shape_row_sample():
    # M=2048, K=4096, N2=14336 (W ~ N(0, 0.02) gate/up halves packed into groups of 4)
    M, N2, K = 2048, 14336, 4096
    x = synth.bf16_normal(synth.SEED_BASE + 2, (M, K))
    wg = synth.bf16_normal(synth.SEED_BASE + 2 + 100, (N2, K), 0.02)
    wu = synth.bf16_normal(synth.SEED_BASE + 2 + 200, (N2, K), 0.02)
    w = synth.gv_pack_g4(wg, wu)
    out = synth.from_torch_bf16(rk.gv(synth.to_torch_bf16(x), synth.to_torch_bf16(w), cfg=0))
    rows = [(0, 3), (127, 130), (1021, 1024), (2045, 2048)]  # tile edges and the last tile
    for r0, r1 in rows:
        ref, lo, hi = orc.gv(x[r0:r1], w)
        assert_close_interval(bf(out[r0:r1]), bf(ref), bf(lo), bf(hi))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gv_column_shards_reproduce_full_layer_bitwise(world):
    """Strong-scaling split of BASELINE config 2 on one GPU: each rank's w_g4 row shard (whole groups of 4 gate/up
    features) run alone gives exactly the full layer's columns -- bit for bit, although the shard and the full layer
    leave different partial last waves (different 16-column pieces and MMA widths)."""
    from reax_engine_kernels_b200 import dist as rd

    M, N2, K = 2048, 14336, 4096
    x = synth.device_normal_bf16((M, K), 1.0, 31)
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 32)
    full = rk.gv(x, w, cfg=0)
    for r in range(world):
        c, rows = rd.gate_up_columns(N2, world, r), rd.gate_up_weight_rows(N2, world, r)
        part = rk.gv(x, w[rows.start:rows.stop], cfg=0)
        assert torch.equal(part.view(torch.int16), full[:, c.start:c.stop].view(torch.int16)), (world, r)
    assert rk.status("libreax_gv") == 0


def test_gv_all_cfgs_bitwise_identical():
    x, w, xt, wt = _inputs(300, 2 * 640, 512, 7)
    outs = [synth.from_torch_bf16(rk.gv(xt, wt, cfg=c)) for c in range(20)]
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


def test_gv_write_mask_and_errors():
    M, N2, K = 100, 60, 64
    x, w, xt, wt = _inputs(M, 2 * N2, K, 11)
    buf = torch.full((M + 3, N2), float("nan"), dtype=torch.bfloat16, device="cuda")
    rk.gv(xt, wt, cfg=1, out=buf[:M])
    torch.cuda.synchronize()
    assert torch.isnan(buf[M:].float()).all() and not torch.isnan(buf[:M].float()).any()
    lib = rk.abi.load("libreax_gv")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.reax_gv(20, xt.data_ptr(), wt.data_ptr(), buf.data_ptr(), M, N2, K, s) == 9
    assert lib.reax_gv(-1, xt.data_ptr(), wt.data_ptr(), buf.data_ptr(), M, N2, K, s) == 9
    assert lib.reax_gv(0, xt.data_ptr(), wt.data_ptr(), buf.data_ptr(), M, N2, 60, s) == 1  # K % 8
    assert lib.reax_gv(0, xt.data_ptr(), wt.data_ptr(), buf.data_ptr(), M, 58, K, s) == 1  # N2 % 4


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 200, 1000), (16, 4096, 4096), (1, 72, 8)])
@pytest.mark.parametrize("cfg", [0, 2, 12])
def test_gemm_vs_oracle(M, N, K, cfg):
    x, w, xt, wt = _inputs(M, N, K, 200 + N)
    out = synth.from_torch_bf16(rk.gemm(xt, wt, cfg=cfg))
    assert_close(bf(out), bf(orc.gemm(x, w)))


@pytest.mark.parametrize("M,N,K", [(33, 200, 136), (64, 4096, 512), (7, 130, 72)])
def test_gemm_small_m_swapped_vs_oracle_and_write_mask(M, N, K):
    # M <= 64 runs the swapped problem (rows of W on the MMA's 128-row side) with a transposed epilogue: values, the
    # output's leading dimension and the write mask (nothing beyond N columns or M rows) must hold as for large M
    x, w, xt, wt = _inputs(M, N, K, 400 + M)
    ldd = (N + 8 + 7) // 8 * 8
    buf = torch.full((M + 2, ldd), float("nan"), dtype=torch.bfloat16, device="cuda")
    rk.gemm(xt, wt, cfg=3, out=buf[:M, :N])
    torch.cuda.synchronize()
    assert torch.isnan(buf[:, N:].float()).all() and torch.isnan(buf[M:].float()).all()
    assert_close(bf(synth.from_torch_bf16(buf[:M, :N])), bf(orc.gemm(x, w)))


@pytest.mark.parametrize("part_fp32", [True, False])
def test_slices_small_m_swapped_ragged(part_fp32):
    # swapped path (M <= 64) with ragged slices: every cfg identical, values against the oracle
    M, N, K, S, kps = 40, 96, 400, 3, 120
    x, w, xt, wt = _inputs(M, N, K, 11)
    outs = [rk.slices(xt, wt, S, kps, part_fp32=part_fp32, cfg=c) for c in range(16)]
    torch.cuda.synchronize()
    iv = torch.int32 if part_fp32 else torch.int16
    for o in outs[1:]:
        assert torch.equal(o.view(iv), outs[0].view(iv))
    got = outs[0].cpu()
    got = got.numpy() if part_fp32 else bf(got.view(torch.int16).numpy().view(np.uint16))
    ref = orc.slices(x, w, S, kps, part_fp32)
    assert_close(got, ref if part_fp32 else bf(ref))


def test_gemm_ldd_writes_only_its_columns():
    M, N, K, ldd = 70, 40, 128, 64
    x, w, xt, wt = _inputs(M, N, K, 5)
    buf = torch.full((M, ldd), float("nan"), dtype=torch.bfloat16, device="cuda")
    rk.gemm(xt, wt, cfg=1, out=buf[:, :N])
    torch.cuda.synchronize()
    assert torch.isnan(buf[:, N:].float()).all()
    assert_close(bf(synth.from_torch_bf16(buf[:, :N])), bf(orc.gemm(x, w)))


def test_gemm_qkv_projection_row_sample():
    # the linear-attention qkv projection shape: T=32768, K=2048, N=6144, W ~ N(0, 0.02)
    M, N, K = 32768, 6144, 2048
    x = synth.bf16_normal(31, (M, K))
    w = synth.bf16_normal(32, (N, K), 0.02)
    out = synth.from_torch_bf16(rk.gemm(synth.to_torch_bf16(x), synth.to_torch_bf16(w), cfg=0))
    for r0 in (0, 16383, 32765):
        assert_close(bf(out[r0:r0 + 3]), bf(orc.gemm(x[r0:r0 + 3], w)))


@pytest.mark.parametrize("M", [16, 256, 4096])
@pytest.mark.parametrize("part_fp32", [True, False])
def test_slices_all_cfgs_identical_and_vs_oracle(M, part_fp32):
    N = K = 4096
    S, kps = 4, 1024
    x, w, xt, wt = _inputs(M, N, K, 300 + M)
    outs = [rk.slices(xt, wt, S, kps, part_fp32=part_fp32, cfg=c) for c in range(16)]
    torch.cuda.synchronize()
    iv = torch.int32 if part_fp32 else torch.int16
    for o in outs[1:]:
        assert torch.equal(o.view(iv), outs[0].view(iv))
    rows = slice(0, M) if M <= 256 else slice(M - 5, M)
    got = outs[0][:, rows].cpu()
    got = got.numpy() if part_fp32 else bf(got.view(torch.int16).numpy().view(np.uint16))
    ref = orc.slices(np.ascontiguousarray(x[rows]), w, S, kps, part_fp32)
    assert_close(got, ref if part_fp32 else bf(ref))


def test_slices_ragged_kps_and_errors():
    # kps not a multiple of the 64-wide K tile: the tail of each slice must not read the next slice
    M, N, K, S, kps = 100, 96, 400, 3, 120
    x, w, xt, wt = _inputs(M, N, K, 9)
    out = rk.slices(xt, wt, S, kps, part_fp32=True, cfg=4)
    assert_close(out.cpu().numpy(), orc.slices(x, w, S, kps, True))
    lib = rk.abi.load("libreax_slices")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.reax_slices(16, 1, xt.data_ptr(), wt.data_ptr(), out.data_ptr(), M, N, kps, S, K, s) == 9
    assert lib.reax_slices(0, 1, xt.data_ptr(), wt.data_ptr(), out.data_ptr(), M, N, 121, S, K, s) == 1
    assert lib.reax_slices(0, 1, xt.data_ptr(), wt.data_ptr(), out.data_ptr(), M, N, kps, 4, K, s) == 1
