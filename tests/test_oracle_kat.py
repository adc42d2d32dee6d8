"""Known-answer checks of the fp64 oracle (CPU only).  Each property is computed independently in numpy."""
import math

import numpy as np

from oracle import oracle as orc
from reax_engine_kernels_b200 import synth

bf = synth.bf16_bits_to_f32
b16 = synth.f32_to_bf16_bits


def test_gv_scalar_formula():
    M, N2, K = 3, 8, 16
    x = synth.bf16_normal(1, (M, K))
    w = synth.bf16_normal(2, (2 * N2, K), 0.3)
    out, lo, hi = orc.gv(x, w)
    X, W = bf(x).astype(np.float64), bf(w).astype(np.float64)
    for m in range(M):
        for j in range(N2 // 4):
            for i in range(4):
                G = X[m] @ W[8 * j + i]
                U = X[m] @ W[8 * j + 4 + i]
                g = float(bf(b16(np.array([G], np.float32)))[0])
                u = float(bf(b16(np.array([U], np.float32)))[0])
                s = float(bf(b16(np.array([g / (1 + math.exp(-g))], np.float32)))[0])
                want = float(bf(b16(np.array([s * u], np.float32)))[0])
                assert abs(float(bf(out[m:m + 1, 4 * j + i])[0]) - want) <= abs(s * u) * 2 ** -7
    assert np.all(bf(lo) <= bf(out)) and np.all(bf(out) <= bf(hi))


def test_gemm_and_slices_consistent():
    M, N, K, S, kps = 5, 7, 64, 4, 16
    x = synth.bf16_normal(3, (M, K))
    w = synth.bf16_normal(4, (N, K))
    p = orc.slices(x, w, S, kps, True)
    full = bf(x).astype(np.float64) @ bf(w).astype(np.float64).T
    assert np.allclose(p.sum(0), full, rtol=1e-6, atol=1e-5)
    d = orc.gemm(x, w, ldd=9)
    assert np.array_equal(d[:, :N], b16(full.astype(np.float32)))


def test_fmha_identical_keys_average_visible_values():
    B, H, M, N, D = 1, 1, 6, 6, 128
    q = synth.bf16_normal(5, (B, H, M, D))
    k = np.repeat(synth.bf16_normal(6, (1, 1, 1, D)), N, axis=2)
    v = synth.bf16_normal(7, (B, H, N, D))
    qpos = np.arange(M, dtype=np.int32).reshape(1, M)
    o = orc.fmha(q, k, v, 0.1, qpos=qpos, qpBs=M)
    V = bf(v)[0, 0].astype(np.float64)
    for r in range(M):
        assert np.allclose(bf(o[0, 0, r]), V[:r + 1].mean(0), rtol=1e-2, atol=1e-2)
    assert np.array_equal(o[0, 0, 0], v[0, 0, 0])  # a single visible key returns V[0] exactly


def test_fmha_fully_masked_row_is_zero_and_bias_matches_qpos():
    B, H, M, N, D = 1, 1, 4, 4, 128
    q, k, v = (synth.bf16_normal(8 + i, (B, H, M if i == 0 else N, D)) for i in range(3))
    qpos = np.array([[-1, 0, 1, 3]], np.int32)
    o = orc.fmha(q, k, v, 0.2, qpos=qpos, qpBs=M)
    assert np.all(o[0, 0, 0] == 0)
    bias = np.zeros((B, H, M, N), np.uint16)
    for r in range(M):
        bias[0, 0, r, qpos[0, r] + 1:] = 0xFF80
    ob = orc.fmha(q, k, v, 0.2, bias=bias)
    assert np.array_equal(ob, o)


def test_rarn_zero_partials_is_rmsnorm():
    n, D = 3, 256
    part = np.zeros((2, n, D), np.uint16)
    res = synth.bf16_normal(11, (n, D))
    w = synth.bf16_normal(12, (D,), 0.1)
    h, out = orc.rarn(part, 2, 1, n * D, res, w, n, D, 1e-6, 1.0 / D)
    assert np.array_equal(h, res)
    R, Wv = bf(res).astype(np.float64), bf(w).astype(np.float64)
    ref = R / np.sqrt((R * R).mean(1, keepdims=True) + 1e-6) * (1 + Wv)
    assert np.allclose(bf(out), ref, rtol=8e-3, atol=1e-3)


def test_conv_one_hot_tap_is_shift():
    KD, VD, T = 128, 128, 10
    SX = 2 * KD + VD
    qkv = synth.bf16_normal(13, (T, SX))
    w = np.zeros((SX, 4), np.uint16)
    w[:, 1] = b16(np.ones(SX, np.float32))  # tap 1 reads position t - 2
    meta = np.array([(t, 0, 0, 0) for t in range(T)], np.int32)
    _, _, v = orc.conv(qkv, SX, None, 0, meta, w, T, 1e-6, KD, VD, 1, 0)
    X = bf(qkv).astype(np.float64)
    for t in range(T):
        y = X[t - 2, 2 * KD:] if t >= 2 else np.zeros(VD)
        s = bf(b16((y / (1 + np.exp(-y))).astype(np.float32)))
        assert np.array_equal(bf(v[t]), s)


def test_kkt_is_inverse():
    d = synth.delta_rule_inputs([90], 1, 2, 14)
    A = orc.kkt(d["k"], d["g"], d["beta"], d["cu"], d["cidx"], 1, 2)
    K = bf(d["k"]).astype(np.float64)[:, 0]
    for c0 in (0, 64):
        n = min(64, 90 - c0)
        for hv in range(2):
            g = d["g"][c0:c0 + n, hv].astype(np.float64)
            b = bf(d["beta"][c0:c0 + n, hv]).astype(np.float64)
            L = np.tril(b[:, None] * (K[c0:c0 + n] @ K[c0:c0 + n].T) * np.exp2(g[:, None] - g[None, :]), -1)
            Ainv = np.linalg.inv(np.eye(n) + L)
            got = bf(A[c0:c0 + n, hv, :n]).astype(np.float64)
            mask = np.tril(np.ones((n, n)), 0)
            # written set: blocks on/below the diagonal; entries in the strict upper part of written blocks are 0
            blk = (np.arange(n)[:, None] // 16) >= (np.arange(n)[None, :] // 16)
            assert np.allclose(got[blk], (Ainv * mask)[blk], rtol=1e-2, atol=1e-3)


def test_howu_single_chunk_matches_direct_recurrence():
    # one chunk, first chunk: o = scale * (Aq vn) with vn = A vb exactly (h = 0)
    d = synth.delta_rule_inputs([40], 1, 2, 15)
    A = orc.kkt(d["k"], d["g"], d["beta"], d["cu"], d["cidx"], 1, 2)
    o = orc.howu(d["q"], d["k"], d["v"], d["beta"], A, d["g"], d["cu"], 0.5, 1, 2)
    q, k, v = (bf(d[n])[:, 0].astype(np.float64) for n in "qkv")
    b = bf(d["beta"])[:, 0].astype(np.float64)
    g = d["g"][:, 0].astype(np.float64)
    Aa = bf(A[:, 0, :40]).astype(np.float64)
    vb = bf(b16((b[:, None] * v).astype(np.float32))).astype(np.float64)
    u = bf(b16((Aa @ vb).astype(np.float32))).astype(np.float64)
    aq = np.tril(q @ k.T * np.exp2(g[:, None] - g[None, :]))
    ref = 0.5 * (aq @ u)
    assert np.allclose(bf(o[:, 0]), ref, rtol=3e-2, atol=3e-3)
