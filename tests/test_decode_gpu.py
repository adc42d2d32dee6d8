"""Decode-step shapes (one new token per sequence) on the GPU against the fp64 oracle.

* GEMMs with M = 1..16 rows (the swapped small-M path of reax_gv / reax_gemm / reax_slices);
* attention for one new token per sequence over a long cached history, GQA row fold G = 4, histories of different
  lengths per batch entry through qpos (keys beyond a sequence's own position are invisible);
* conv for one token per sequence whose three earlier taps all come from the per-sequence conv cache (meta y = pos),
  including sequences with fewer than three earlier positions;
* reax_conv_v on a second stream while reax_conv_l2 (skip_v = 1) computes q and k on the first, as an engine that
  overlaps the value path does.
"""
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
T_ = synth.to_torch_bf16
H_ = synth.from_torch_bf16
NAN = 0x7FC0


def t64(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("M", [1, 2, 3, 4, 8, 16])
def test_decode_gemms(M):
    K, N = 2048, 1024
    x = synth.bf16_normal(1000 + M, (M, K))
    w = synth.bf16_normal(1100 + M, (N, K), 0.02)
    xt, wt = T_(x), T_(w)
    out = H_(rk.gemm(xt, wt))
    assert_close(bf(out), bf(orc.gemm(x, w)))
    g = H_(rk.gv(xt, wt))  # w read as the g4-interleaved gate/up pack of N/2 outputs
    ref, lo, hi = orc.gv(x, w)
    assert_close_interval(bf(g), bf(ref), bf(lo), bf(hi))
    for part_fp32 in (True, False):
        p = rk.slices(xt, wt, 4, K // 4, part_fp32=part_fp32)
        r = orc.slices(x, w, 4, K // 4, part_fp32=part_fp32)
        got = p.cpu().numpy() if part_fp32 else bf(H_(p))
        assert_close(got, r if part_fp32 else bf(r))


@pytest.mark.parametrize("D", [128, 256])
def test_decode_attention_over_cached_history(D):
    # B = 3 sequences, 2 kv heads, G = 4 query heads per kv head, one new token each; the key cache holds N = 2049
    # positions, sequence b has history hist[b] (its new token is at position hist[b], later keys are invisible)
    B, H, G, N = 3, 2, 4, 2049
    hist = np.array([2048, 700, 5], np.int32)
    q = synth.bf16_normal(1200 + D, (B, H, G, D))
    k = synth.bf16_normal(1201 + D, (B, H, N, D))
    v = synth.bf16_normal(1202 + D, (B, H, N, D))
    qpos = hist.reshape(B, 1).copy()
    scale = 1 / math.sqrt(D)
    out = H_(rk.fmha(T_(q), T_(k), T_(v), scale, qpos=t64(qpos), G=G))
    ref, lo, hi = orc.fmha(q, k, v, scale, qpos=qpos, G=G, qpBs=1, intervals=True)
    assert_close_interval(bf(out), bf(ref), bf(lo), bf(hi))
    # the keys past a sequence's position do not leak: poison them and expect the same bits
    k2, v2 = k.copy(), v.copy()
    for b in range(B):
        k2[b, :, hist[b] + 1:] = 0x4780  # 65536.0: a visible poisoned key would dominate its row's softmax
        v2[b, :, hist[b] + 1:] = 0x4780  # (finite: a masked key's probability is 0, and 0 * inf would be NaN)
    out2 = H_(rk.fmha(T_(q), T_(k2), T_(v2), scale, qpos=t64(qpos), G=G))
    assert np.array_equal(out, out2)


def test_decode_conv_taps_from_cache():
    # 6 sequences, one token each; the cache keeps each sequence's last 3 rows (rows 3s .. 3s+2 for positions
    # pos-3 .. pos-1); positions 0, 1 and 2 have fewer earlier taps (the rest are skipped)
    KD, VD = 256, 384
    Ctot = 2 * KD + VD
    pos = np.array([57, 0, 1, 2, 3, 1000], np.int32)
    S = len(pos)
    SX = Ctot + 64
    qkv = synth.bf16_normal(1300, (S, SX))
    cache = synth.bf16_normal(1301, (3 * S, Ctot))
    w = synth.bf16_normal(1302, (Ctot, 4), 0.5)
    meta = np.array([(p, p, s - p, 3 * s + 3 - p) for s, p in enumerate(pos)], np.int32)
    for rep in (1, 2):
        q0 = np.full((S, rep * KD), NAN, np.uint16)
        v0 = np.full((S, VD), NAN, np.uint16)
        qt, kt, vt = T_(q0), T_(q0), T_(v0)
        rk.conv_l2(T_(qkv), t64(meta), T_(w), KD, VD, 1e-6, rep, cache=T_(cache), q=qt, k=kt, v=vt)
        rq, rk_, rv = orc.conv(qkv, SX, cache, Ctot, meta, w, S, 1e-6, KD, VD, rep, 0)
        for got, ref in ((qt, rq), (kt, rk_), (vt, rv)):
            assert_close(bf(H_(got)), bf(ref))


def test_conv_v_on_a_side_stream():
    KD, VD = 256, 512
    lengths = [130, 1, 77]
    T = sum(lengths)
    Ctot = 2 * KD + VD
    SX = Ctot
    qkv = synth.bf16_normal(1400, (T, SX))
    w = synth.bf16_normal(1401, (Ctot, 4), 0.5)
    cu = np.concatenate([[0], np.cumsum(lengths)])
    meta = np.array([(t - cu[s], 0, cu[s], 0) for s in range(len(lengths)) for t in range(cu[s], cu[s + 1])], np.int32)
    qkvt, wt, mt = T_(qkv), T_(w), t64(meta)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    q, k, _ = rk.conv_l2(qkvt, mt, wt, KD, VD, 1e-6, skip_v=True)
    with torch.cuda.stream(side):
        v = rk.conv_v(qkvt, mt, wt, KD, VD)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    rq, rk_, rv = orc.conv(qkv, SX, None, 0, meta, w, T, 1e-6, KD, VD, 1, 0)
    assert_close(bf(H_(q)), bf(rq))
    assert_close(bf(H_(k)), bf(rk_))
    assert_close(bf(H_(v)), bf(rv))
