"""Attention forward (libreax_fmha_post / libreax_howu exports) on the GPU against the fp64 oracle."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import synth
from tests.tolerance import assert_close, assert_close_interval

pytestmark = pytest.mark.gpu
bf = synth.bf16_bits_to_f32


def qkv(B, H, M, N, D, seed):
    q = synth.bf16_normal(seed, (B, H, M, D))
    k = synth.bf16_normal(seed + 1, (B, H, N, D))
    v = synth.bf16_normal(seed + 2, (B, H, N, D))
    return q, k, v


def dev(*a):
    return [synth.to_torch_bf16(x) for x in a]


@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("B,H,M,N,G", [(1, 2, 300, 300, 1), (2, 1, 128, 128, 1), (1, 2, 4 * 70, 70, 4), (1, 1, 5, 200, 1)])
def test_qpos_causal_vs_oracle(D, B, H, M, N, G):
    q, k, v = qkv(B, H, M, N, D, 10 + M + D)
    Lq = M // G
    # queries are the last Lq tokens of an N-token sequence (history = N - Lq)
    qpos = np.stack([np.arange(N - Lq, N, dtype=np.int32)] * B)
    qt, kt, vt = dev(q, k, v)
    scale = 1.0 / math.sqrt(D)
    out = synth.from_torch_bf16(rk.fmha(qt, kt, vt, scale, qpos=torch.from_numpy(qpos).cuda(), G=G))
    ref, lo, hi = orc.fmha(q, k, v, scale, qpos=qpos, G=G, qpBs=Lq, intervals=True)
    assert_close_interval(bf(out), bf(ref), bf(lo), bf(hi))


@pytest.mark.parametrize("D", [128, 256])
def test_bias_mode_vs_oracle(D):
    B, H, M, N = 2, 2, 200, 333
    q, k, v = qkv(B, H, M, N, D, 77)
    bias = synth.bf16_normal(80, (B, H, M, N), 2.0)
    mask = synth.uniform(81, B * H * M * N).reshape(B, H, M, N) < 0.3
    bias[mask] = 0xFF80  # -inf
    bias[:, :, 7, :] = 0xFF80  # a fully masked row -> 0
    qt, kt, vt, bt = dev(q, k, v, bias)
    out = synth.from_torch_bf16(rk.fmha(qt, kt, vt, 0.07, bias=bt))
    ref, lo, hi = orc.fmha(q, k, v, 0.07, bias=bias, intervals=True)
    assert np.all(bf(out)[:, :, 7] == 0)
    assert_close_interval(bf(out), bf(ref), bf(lo), bf(hi))


def test_fully_masked_rows_and_write_mask():
    B, H, M, N, D = 1, 1, 200, 256, 128
    q, k, v = qkv(B, H, M, N, D, 90)
    qpos = np.full((1, M), -1, np.int32)
    qpos[0, 100:] = np.arange(100)  # rows 0..99 see nothing
    qt, kt, vt = dev(q, k, v)
    buf = torch.full((B, H, M + 5, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    rk.fmha(qt, kt, vt, 0.1, qpos=torch.from_numpy(qpos).cuda(), out=buf[:, :, :M])
    torch.cuda.synchronize()
    o = buf.float().cpu().numpy()
    assert np.isnan(o[:, :, M:]).all(), "rows >= M must not be written"
    assert np.all(o[0, 0, :100] == 0)
    ref, lo, hi = orc.fmha(q, k, v, 0.1, qpos=qpos, qpBs=M, intervals=True)
    assert_close_interval(o[:, :, :M], bf(ref), bf(lo), bf(hi))


def test_strided_layouts_match_contiguous():
    # Q as [B, M, H, D] (token-major) and K/V as [B, N, H, D]: strides, not copies
    B, H, M, N, D = 2, 3, 150, 150, 128
    q, k, v = qkv(B, H, M, N, D, 5)
    qt, kt, vt = dev(q, k, v)
    qs = qt.transpose(1, 2).contiguous().transpose(1, 2)
    ks = kt.transpose(1, 2).contiguous().transpose(1, 2)
    vs = vt.transpose(1, 2).contiguous().transpose(1, 2)
    qpos = torch.arange(M, dtype=torch.int32, device="cuda").repeat(B, 1)
    a = rk.fmha(qt, kt, vt, 0.09, qpos=qpos)
    o2 = torch.empty(B, M, H, D, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
    b = rk.fmha(qs, ks, vs, 0.09, qpos=qpos, out=o2)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.contiguous().view(torch.int16))


def test_libraries_export_identical_attention():
    B, H, M, N, D = 1, 2, 256, 256, 256
    q, k, v = qkv(B, H, M, N, D, 44)
    qt, kt, vt = dev(q, k, v)
    qpos = torch.arange(M, dtype=torch.int32, device="cuda").view(1, M)
    a = rk.fmha(qt, kt, vt, 0.0625, qpos=qpos, library="libreax_fmha_post")
    b = rk.fmha(qt, kt, vt, 0.0625, qpos=qpos, library="libreax_howu")
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_post_epilogue_vs_oracle():
    B, Hkv, G, Lq, D = 2, 2, 2, 96, 256
    M = Lq * G
    N = Lq
    q, k, v = qkv(B, Hkv, M, N, D, 55)
    qpos = np.stack([np.arange(Lq, dtype=np.int32)] * B)
    rows = B * Lq + 3
    perm = synth.uniform(56, B * Lq).argsort()
    inv = perm.astype(np.int32).reshape(B, Lq)
    inv[0, 5] = -1
    inv[1, 17] = -1
    Hq = Hkv * G
    qg = synth.bf16_normal(57, (rows, Hq * 2 * D), 3.0)
    outp0 = np.full((rows, Hq * D), 0x7FC0, np.uint16)  # NaN canaries: skipped rows keep them
    qt, kt, vt, qgt, outt = dev(q, k, v, qg, outp0)
    rk.fmha_qp(qt, kt, vt, 0.0625, torch.from_numpy(qpos).cuda(), G, torch.from_numpy(inv).cuda(), qgt, outt)
    got = synth.from_torch_bf16(outt)
    ref = outp0.copy()
    _, lo, hi = orc.fmha(q, k, v, 0.0625, qpos=qpos, G=G, qpBs=Lq, intervals=True,
                         post=dict(inv=inv, Lq=Lq, qg=qg, qg_rs=Hq * 2 * D, outp=ref, out_rs=Hq * D))
    written = ref != 0x7FC0
    assert np.array_equal(got == 0x7FC0, ref == 0x7FC0), "write mask differs"
    assert_close_interval(bf(got[written]), bf(ref[written]), bf(lo[written]), bf(hi[written]))


def test_config1_causal_mha_full():
    # B=1, S=1024, Hq=Hkv=8, D=128, scale 1/sqrt(128), qpos[t] = t
    B, H, S, D = 1, 8, 1024, 128
    q, k, v = qkv(B, H, S, S, D, synth.SEED_BASE + 1)
    qpos = np.arange(S, dtype=np.int32).reshape(1, S)
    qt, kt, vt = dev(q, k, v)
    out = synth.from_torch_bf16(rk.fmha(qt, kt, vt, 1 / math.sqrt(D), qpos=torch.from_numpy(qpos).cuda()))
    ref, lo, hi = orc.fmha(q, k, v, 1 / math.sqrt(D), qpos=qpos, qpBs=S, intervals=True)
    assert_close_interval(bf(out), bf(ref), bf(lo), bf(hi))


def test_config3_gqa_prefill_sampled_rows():
    # B=4, S=8192, Hq=32, Hkv=8 (G=4 row fold: M = 4*8192 rows per kv head), D=128
    B, Hkv, G, S, D = 4, 8, 4, 8192, 128
    M = S * G
    qt = synth.device_normal_bf16((B, Hkv, M, D), 1.0, synth.SEED_BASE + 3)
    kt = synth.device_normal_bf16((B, Hkv, S, D), 1.0, synth.SEED_BASE + 4)
    vt = synth.device_normal_bf16((B, Hkv, S, D), 1.0, synth.SEED_BASE + 5)
    qpos = torch.arange(S, dtype=torch.int32, device="cuda").repeat(B, 1).contiguous()
    out = rk.fmha(qt, kt, vt, 1 / math.sqrt(D), qpos=qpos, G=G)
    torch.cuda.synchronize()
    o = synth.from_torch_bf16(out)
    qh, kh, vh = (synth.from_torch_bf16(t) for t in (qt, kt, vt))
    for r0 in (0, 12345, M - 130):
        r1 = r0 + 2
        ref, lo, hi = orc.fmha(qh, kh, vh, 1 / math.sqrt(D), qpos=qpos.cpu().numpy(), G=G, qpBs=S, rows=(r0, r1),
                               intervals=True)
        sl = (slice(None), slice(None), slice(r0, r1))
        assert_close_interval(bf(o[sl]), bf(ref[sl]), bf(lo[sl]), bf(hi[sl]))


@pytest.mark.parametrize("mode", ["qpos", "bias"])
def test_two_tile_kernel_full_output_vs_torch(mode):
    # a shape large enough to select the two-query-tile kernel (head dim 128), every element checked against a torch
    # fp32 softmax reference: races between the tensor-core stages would show up as O(1) errors here
    B, H, G, S, D = 4, 8, 4, 1024, 128
    M = S * G
    q = synth.device_normal_bf16((B, H, M, D), 1.0, 31)
    k = synth.device_normal_bf16((B, H, S, D), 1.0, 32)
    v = synth.device_normal_bf16((B, H, S, D), 1.0, 33)
    scale = 1 / math.sqrt(D)
    if mode == "qpos":
        qpos = torch.arange(S, dtype=torch.int32, device="cuda").repeat(B, 1).contiguous()
        out = rk.fmha(q, k, v, scale, qpos=qpos, G=G)
        vis = (torch.arange(S, device="cuda")[None, :] <= (torch.arange(M, device="cuda") // G)[:, None])
        bias = torch.where(vis, 0.0, float("-inf"))
    else:
        bt = synth.device_normal_bf16((B, H, M, S), 1.0, 34)
        out = rk.fmha(q, k, v, scale, bias=bt)
        bias = bt.float()
    for b in range(B):  # per batch to bound the fp32 temporaries
        s = (q[b].float() @ k[b].float().transpose(-1, -2)) * scale + (bias if mode == "qpos" else bias[b])
        ref = torch.softmax(s, -1) @ v[b].float()
        err = (out[b].float() - ref).abs()
        assert float(err.max()) < 0.03, f"batch {b}: max abs err {float(err.max()):.4g}"
        assert float(err.mean()) < 2e-3
