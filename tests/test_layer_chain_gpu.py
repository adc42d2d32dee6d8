"""Per-layer chains of the libraries, in the engine's data layouts, each stage checked against the fp64 oracle.

Three chains, each as one layer of the engine calls them:
* linear attention: reax_gemm (qkv projection into a wider row buffer, ldd > N) -> reax_conv_l2 (reading that buffer
  with SX = ldd) -> reax_kkt -> reax_howu_norm (rows scattered through f2s, gated RMSNorm);
* reduce + norm: reax_slices (two bf16 K-slice partials) -> reax_rarn (partial stride = M*N, the slices' batch stride);
* gated attention: reax_gemm (q|gate and k|v projections) -> reax_fmha_qp reading q, k and v in place inside the
  projection buffers through strides, with the sigmoid-gate scatter epilogue.

Each stage is checked against the oracle run on the GPU's own inputs to that stage, with that kernel's usual
criterion (the contract per entry point).  The layer output is also checked against the all-oracle chain.  There a
one-ulp rounding flip of an early stage's bf16 output (about 1 element in 10^4 of a GEMM differs from the fp64
oracle's rounding) travels on as an absolute error of one intermediate ulp, which the element-relative measure
inflates wherever the output cancels to near zero (a residual add): run on the CPU with partials rounded from fp32
instead of fp64, the oracle chains moved single elements by up to 10 % of their value but by at most 1.6 % (rarn)
and 2.3 % (gated attention, whose rows differ in scale by 15x) of the output's rms, and the attention's legitimate
rounding interval is itself 1.1 % of the rms wide.  So the layer check is normwise, |y - r| / rms(r) with
mean <= 1e-3 and max <= 0.1: loose enough for propagated rounding, far below what a layout or plumbing error gives.
"""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import synth
from tests.tolerance import assert_close, assert_close_chain, assert_close_interval

pytestmark = pytest.mark.gpu
bf = synth.bf16_bits_to_f32
T_ = synth.to_torch_bf16
H_ = synth.from_torch_bf16
NAN = 0x7FC0


def t64(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def assert_close_layer(y, r):
    y, r = np.asarray(y, np.float64), np.asarray(r, np.float64)
    assert np.all(np.isfinite(y)), "non-finite values"
    rms = float(np.sqrt(np.mean(r * r)))
    e = np.abs(y - r) / rms
    assert e.mean() <= 1e-3, f"layer output: mean |y - r| / rms {e.mean():.3g} > 1e-3"
    assert e.max() <= 0.1, f"layer output: max |y - r| / rms {e.max():.3g} > 0.1"


def test_linear_attention_layer_chain():
    lengths = [100, 70]
    H, HV = 2, 4
    KD, VD = 128 * H, 128 * HV
    hidden = 256
    NQKV = 2 * KD + VD
    LDD = NQKV + 64  # the projection writes into a wider row buffer; conv reads it with SX = LDD
    T = sum(lengths)
    seed = 900
    x = synth.bf16_normal(seed, (T, hidden))
    W = synth.bf16_normal(seed + 1, (NQKV, hidden), 1.0 / math.sqrt(hidden))
    cw = synth.bf16_normal(seed + 2, (NQKV, 4), 0.5)
    d = synth.delta_rule_inputs(lengths, H, HV, seed + 3)  # beta, g, cu, cidx of the layer
    meta = np.array([(p, 0, int(d["cu"][s]), 0) for s, L in enumerate(lengths) for p in range(L)], np.int32)
    rows = T + 3
    f2s = synth.uniform(seed + 4, T).argsort().astype(np.int32) + 3
    f2s[5] = -1
    f2s[131] = -1
    ZS = HV * 128 + 32
    z = synth.bf16_normal(seed + 5, (rows, ZS), 2.0)
    nw = synth.bf16_normal(seed + 6, (128,), 0.1, 1.0)
    scale = 1 / math.sqrt(128)
    norm = dict(f2s=f2s, z=z, ZS=ZS, nw=nw, eps=1e-6, factor=1 / 128, rows=rows)

    # the GPU layer
    buf = torch.full((T, LDD), float("nan"), dtype=torch.bfloat16, device="cuda")
    rk.gemm(T_(x), T_(W), out=buf[:, :NQKV])
    q, k, v = rk.conv_l2(buf, t64(meta), T_(cw), KD, VD, 1e-6)
    gt, bt, cut, cit = t64(d["g"]), T_(d["beta"]), t64(d["cu"]), t64(d["cidx"])
    A = rk.kkt(k.view(T, H, 128), gt, bt, cut, cit, HV)
    out0 = np.full((rows, HV, 128), NAN, np.uint16)
    out = T_(out0)
    rk.howu_norm(q.view(T, H, 128), k.view(T, H, 128), v.view(T, HV, 128), bt, A, gt, cut, scale, t64(f2s), T_(z),
                 T_(nw), 1e-6, 1 / 128, out)
    torch.cuda.synchronize()
    g_buf, g_q, g_k, g_v, g_A, g_out = (H_(t) for t in (buf, q, k, v, A, out))

    # stage by stage, each on the GPU's own inputs
    r_qkv = orc.gemm(x, W, ldd=LDD)
    assert np.all(g_buf[:, NQKV:] == NAN), "the projection wrote outside its ldd columns"
    assert_close(bf(g_buf[:, :NQKV]), bf(r_qkv[:, :NQKV]))
    r_q, r_k, r_v = orc.conv(g_buf, LDD, None, 0, meta, cw, T, 1e-6, KD, VD, 1, 0)
    for g, r in ((g_q, r_q), (g_k, r_k), (g_v, r_v)):
        assert_close(bf(g), bf(r))
    r_A = orc.kkt(g_k.reshape(T, H, 128), d["g"], d["beta"], d["cu"], d["cidx"], H, HV)
    assert_close(bf(g_A), bf(r_A))
    r_out = orc.howu(g_q.reshape(T, H, 128), g_k.reshape(T, H, 128), g_v.reshape(T, HV, 128), d["beta"], g_A, d["g"],
                     d["cu"], scale, H, HV, norm=norm, out=out0.copy())
    assert np.array_equal(g_out == NAN, r_out == NAN), "write set of the normed output differs"
    m = r_out != NAN
    assert_close_chain(bf(g_out[m]), bf(r_out[m]))

    # the whole layer against the all-oracle chain
    o_q, o_k, o_v = orc.conv(r_qkv, LDD, None, 0, meta, cw, T, 1e-6, KD, VD, 1, 0)
    o_A = orc.kkt(o_k.reshape(T, H, 128), d["g"], d["beta"], d["cu"], d["cidx"], H, HV)
    o_out = orc.howu(o_q.reshape(T, H, 128), o_k.reshape(T, H, 128), o_v.reshape(T, HV, 128), d["beta"], o_A, d["g"],
                     d["cu"], scale, H, HV, norm=norm, out=out0.copy())
    assert np.array_equal(g_out == NAN, o_out == NAN)
    assert_close_layer(bf(g_out[m]), bf(o_out[m]))


def test_slices_into_rarn_chain():
    M, N, K, S = 200, 2048, 1024, 2
    kps = K // S
    x = synth.bf16_normal(910, (M, K))
    W = synth.bf16_normal(911, (N, K), 0.02)
    res = synth.bf16_normal(912, (M, N))
    w = synth.bf16_normal(913, (N,), 0.1, 1.0)
    eps, factor = 1e-6, 1.0 / N

    part = rk.slices(T_(x), T_(W), S, kps, part_fp32=False)
    h, out = rk.rarn(part, T_(res), T_(w), eps, factor, serial=True)
    torch.cuda.synchronize()
    g_part, g_h, g_out = H_(part), H_(h), H_(out)

    r_part = orc.slices(x, W, S, kps, part_fp32=False)
    assert_close(bf(g_part), bf(r_part))
    r_h, r_out = orc.rarn(g_part, S, 1, M * N, res, w, M, N, eps, factor)
    assert np.array_equal(g_h, r_h), "h_out must be bit-exact on the same partials"
    assert_close(bf(g_out), bf(r_out))

    o_h, o_out = orc.rarn(r_part, S, 1, M * N, res, w, M, N, eps, factor)
    assert_close_layer(bf(g_h), bf(o_h))
    assert_close_layer(bf(g_out), bf(o_out))


def test_gated_attention_layer_chain():
    # one kv head shared by G = 2 query heads (the row fold maps row r to token r / G, head r % G, so q is read in
    # place from the projection buffer with a row stride of one head), head dim 256, two sequences of Lq tokens
    B, Lq, G, D, hidden = 2, 96, 2, 256, 256
    Hq = G
    T = B * Lq
    x = synth.bf16_normal(920, (T, hidden))
    Wqg = synth.bf16_normal(921, (Hq * 2 * D, hidden), 1.0 / math.sqrt(hidden))
    Wkv = synth.bf16_normal(922, (2 * D, hidden), 1.0 / math.sqrt(hidden))
    qpos = np.stack([np.arange(Lq, dtype=np.int32)] * B)
    inv = np.arange(T, dtype=np.int32).reshape(B, Lq)
    inv[0, 7] = -1
    inv[1, 50] = -1
    scale = 1 / 16.0

    qg = rk.gemm(T_(x), T_(Wqg))  # [T, Hq * 512]: per query head 256 q columns then 256 gate columns
    kv = rk.gemm(T_(x), T_(Wkv))  # [T, 512]: k then v
    qv = torch.as_strided(qg, (B, 1, Lq * G, D), (Lq * Hq * 2 * D, 0, 2 * D, 1))
    kvv = torch.as_strided(kv, (B, 1, Lq, D), (Lq * 2 * D, 0, 2 * D, 1))
    vv = torch.as_strided(kv, (B, 1, Lq, D), (Lq * 2 * D, 0, 2 * D, 1), storage_offset=D)
    outp0 = np.full((T, Hq * D), NAN, np.uint16)
    outp = T_(outp0)
    rk.fmha_qp(qv, kvv, vv, scale, t64(qpos), G, t64(inv), qg, outp)
    torch.cuda.synchronize()
    g_qg, g_kv, g_out = H_(qg), H_(kv), H_(outp)

    r_qg = orc.gemm(x, Wqg)
    r_kv = orc.gemm(x, Wkv)
    assert_close(bf(g_qg), bf(r_qg))
    assert_close(bf(g_kv), bf(r_kv))

    def attention(qg_, kv_):
        q = np.ascontiguousarray(qg_.reshape(B, Lq, Hq, 2 * D)[:, :, :, :D].reshape(B, 1, Lq * G, D))
        k = np.ascontiguousarray(kv_.reshape(B, 1, Lq, 2 * D)[..., :D])
        v = np.ascontiguousarray(kv_.reshape(B, 1, Lq, 2 * D)[..., D:])
        ref = outp0.copy()
        _, lo, hi = orc.fmha(q, k, v, scale, qpos=qpos, G=G, qpBs=Lq, intervals=True,
                             post=dict(inv=inv, Lq=Lq, qg=qg_, qg_rs=Hq * 2 * D, outp=ref, out_rs=Hq * D))
        return ref, lo, hi

    ref, lo, hi = attention(g_qg, g_kv)
    written = ref != NAN
    assert np.array_equal(g_out == NAN, ref == NAN), "write mask of the gated scatter differs"
    assert_close_interval(bf(g_out[written]), bf(ref[written]), bf(lo[written]), bf(hi[written]))

    o_ref, _, _ = attention(r_qg, r_kv)
    assert np.array_equal(g_out == NAN, o_ref == NAN)
    assert_close_layer(bf(g_out[written]), bf(o_ref[written]))
