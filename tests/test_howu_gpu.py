"""Linear-attention layer kernels (libreax_howu) on the GPU against the fp64 oracle: rarn, conv_l2 / conv_v, kkt,
howu (skip / dense) and howu_norm, with write masks checked through NaN canaries."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import synth
from tests.tolerance import assert_close, assert_close_chain

pytestmark = pytest.mark.gpu
bf = synth.bf16_bits_to_f32
T_ = synth.to_torch_bf16
NAN = 0x7FC0


def t64(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _reference_howu(entry, args, norm=None):
    """The reference's own kernel (oracle/_ref) on the same device inputs, or None when that build is absent.
    args = (q, k, v, beta, A, g, cu) device tensors, scale, N, H, HV; norm = (out, f2s, z, ZS, nw, eps, factor)."""
    import ctypes as C
    import os

    from oracle.build import ref_path

    if not os.path.exists(ref_path("libreax_howu")):
        return None
    ref = C.CDLL(ref_path("libreax_howu"))
    (q, k, v, beta, A, g, cu), scale, N, H, HV = args
    P = lambda t: C.c_void_p(t.data_ptr())
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if norm is None:
        o = torch.empty_like(v)
        rc = getattr(ref, entry)(P(q), P(k), P(v), P(beta), P(A), P(g), P(o), P(cu), C.c_float(scale), C.c_int(N),
                                 C.c_int(H), C.c_int(HV), s)
    else:
        o, f2s, z, ZS, nw, eps, factor = norm
        rc = ref.reax_howu_norm(P(q), P(k), P(v), P(beta), P(A), P(g), P(o), P(cu), C.c_float(scale), C.c_int(N),
                                C.c_int(H), C.c_int(HV), s, P(f2s), P(z), C.c_longlong(ZS), P(nw), C.c_float(eps),
                                C.c_float(factor))
    assert rc == 0
    torch.cuda.synchronize()
    return synth.from_torch_bf16(o)


def check_chain(got, ref, theirs):
    """The delta rule's criterion: pinned to the reference's own kernel when its build is present (every element above
    the 1e-2 bound must be the reference kernel's own bits, oracle/tolerance.py reference_matched_stats), else the
    looser chain criterion."""
    from oracle.tolerance import assert_reference_matched

    if theirs is None:
        assert_close_chain(bf(got), bf(ref))
    else:
        assert_reference_matched(bf(got), bf(ref), bf(theirs))


# ------------------------------------------------------------------------------------------------ rarn
@pytest.mark.parametrize("D", [128, 2048, 2560])
@pytest.mark.parametrize("S,serial", [(2, 0), (2, 1), (3, 1), (8, 0)])
def test_rarn_vs_oracle(D, S, serial):
    n = 257
    part = synth.bf16_normal(1 + S, (S, n, D), 0.5)
    res = synth.bf16_normal(2, (n, D))
    w = synth.bf16_normal(3, (D,), 0.1, 1.0)
    h, o = rk.rarn(T_(part), T_(res), T_(w), 1e-6, 1.0 / D, bool(serial))
    rh, ro = orc.rarn(part, S, serial, n * D, res, w, n, D, 1e-6, 1.0 / D)
    assert np.array_equal(synth.from_torch_bf16(h), rh), "h_out must be bit-exact (sums of bf16 pairs)"
    assert_close(bf(synth.from_torch_bf16(o)), bf(ro))


def test_rarn_config5_and_codes():
    n, D, S = 32768, 2048, 2
    part = synth.device_normal_bf16((S, n, D), 0.5, 11)
    res = synth.device_normal_bf16((n, D), 1.0, 12)
    w = synth.device_normal_bf16((D,), 0.1, 13, mean=1.0)
    h, o = rk.rarn(part, res, w, 1e-6, 1.0 / D)
    ph, rh, wh = (synth.from_torch_bf16(t) for t in (part, res, w))
    rows = slice(n - 300, n)
    oh, oo = orc.rarn(np.ascontiguousarray(ph[:, rows]), S, 0, 300 * D, np.ascontiguousarray(rh[rows]), wh, 300, D, 1e-6,
                      1.0 / D)
    assert np.array_equal(synth.from_torch_bf16(h)[rows], oh)
    assert_close(bf(synth.from_torch_bf16(o)[rows]), bf(oo))
    lib = rk.abi.load("libreax_howu")
    s = torch.cuda.current_stream().cuda_stream
    p = part.data_ptr()
    assert lib.reax_rarn(p, 2, 0, n * D, p, p, p, p, 0, D, 1e-6, 1.0, s) == 0
    assert lib.reax_rarn(p, 2, 0, n * D, p, p, p, p, 4, 100, 1e-6, 1.0, s) == -1
    assert lib.reax_rarn(p, 1, 0, n * D, p, p, p, p, 4, D, 1e-6, 1.0, s) == -2
    assert lib.reax_rarn(p, 9, 0, n * D, p, p, p, p, 4, D, 1e-6, 1.0, s) == -2


# ------------------------------------------------------------------------------------------------ conv
def conv_case(lengths, KD, VD, cache_rows=0, seed=0):
    T = sum(lengths)
    SX = 2 * KD + VD + 64  # padded row stride
    qkv = synth.bf16_normal(seed, (T, SX))
    w = synth.bf16_normal(seed + 1, (2 * KD + VD, 4), 0.5)
    meta = []
    bos = 0
    for L in lengths:
        for p in range(L):
            meta.append((p + cache_rows, cache_rows, bos - cache_rows, 0))  # positions continue after cached rows
        bos += L
    meta = np.array(meta, np.int32)
    cache = synth.bf16_normal(seed + 2, (max(cache_rows, 1), 2 * KD + VD)) if cache_rows else None
    return qkv, w, meta, cache, SX


@pytest.mark.parametrize("rep,skip_v", [(1, 0), (2, 0), (1, 1)])
@pytest.mark.parametrize("cache_rows", [0, 3])
def test_conv_vs_oracle(rep, skip_v, cache_rows):
    KD, VD = 256, 384
    qkv, w, meta, cache, SX = conv_case([70, 131], KD, VD, cache_rows, seed=20 + rep)
    T = meta.shape[0]
    q0 = np.full((T, rep * KD), NAN, np.uint16)
    v0 = np.full((T, VD), NAN, np.uint16)
    qt, kt, vt = T_(q0), T_(q0), T_(v0)
    C = cache.shape[1] if cache is not None else 0
    rk.conv_l2(T_(qkv), t64(meta), T_(w), KD, VD, 1e-6, rep, bool(skip_v), cache=T_(cache) if cache is not None else None,
               q=qt, k=kt, v=vt)
    rq, rk_, rv = orc.conv(qkv, SX, cache, C, meta, w, T, 1e-6, KD, VD, rep, skip_v, q=q0.copy(), k=q0.copy(), v=v0.copy())
    for got, ref in ((qt, rq), (kt, rk_), (vt, rv)):
        g = synth.from_torch_bf16(got)
        assert np.array_equal(g == NAN, ref == NAN), "write set differs"
        m = ref != NAN
        assert_close(bf(g[m]), bf(ref[m]))


def test_conv_v_only_values():
    KD, VD = 256, 256
    qkv, w, meta, cache, SX = conv_case([90], KD, VD, 0, seed=33)
    T = meta.shape[0]
    v = rk.conv_v(T_(qkv), t64(meta), T_(w), KD, VD)
    _, _, rv = orc.conv(qkv, SX, None, 0, meta, w, T, 1e-6, KD, VD, 1, 0, units=(2 * KD // 128, 2 * KD // 128 + VD // 128))
    assert_close(bf(synth.from_torch_bf16(v)), bf(rv))


def test_conv_config5_sampled():
    # 2 sequences x 16384 tokens, KD = VD = 2048 (16 heads x 128), SX = 6144, conv w ~ N(0, 0.5), qkv ~ N(0, 1)
    L, KD, VD = 16384, 2048, 2048
    T, SX = 2 * L, 6144
    qkv = synth.device_normal_bf16((T, SX), 1.0, 41)
    w = synth.device_normal_bf16((SX, 4), 0.5, 42)
    meta = np.array([(p, 0, s * L, 0) for s in range(2) for p in range(L)], np.int32)
    q, k, v = rk.conv_l2(qkv, t64(meta), w, KD, VD)
    torch.cuda.synchronize()
    qh, wh = synth.from_torch_bf16(qkv), synth.from_torch_bf16(w)
    for t0 in (0, L - 2, L, T - 3):
        sub = meta[t0:t0 + 2].copy()
        rq, rk_, rv = orc.conv(qh, SX, None, 0, sub, wh, 2, 1e-6, KD, VD, 1, 0)
        assert_close(bf(synth.from_torch_bf16(q[t0:t0 + 2])), bf(rq))
        assert_close(bf(synth.from_torch_bf16(k[t0:t0 + 2])), bf(rk_))
        assert_close(bf(synth.from_torch_bf16(v[t0:t0 + 2])), bf(rv))


# ------------------------------------------------------------------------------------------------ kkt
@pytest.mark.parametrize("lengths", [[100, 150], [64], [1, 17, 200]])
def test_kkt_vs_oracle_and_write_mask(lengths):
    d = synth.delta_rule_inputs(lengths, 2, 4, seed=50 + len(lengths))
    T = d["T"]
    A0 = np.full((T, 4, 64), NAN, np.uint16)
    At = T_(A0)
    rk.kkt(T_(d["k"]), t64(d["g"]), T_(d["beta"]), t64(d["cu"]), t64(d["cidx"]), 4, A=At)
    got = synth.from_torch_bf16(At)
    ref = orc.kkt(d["k"], d["g"], d["beta"], d["cu"], d["cidx"], 2, 4, A=A0.copy())
    assert np.array_equal(got == NAN, ref == NAN), "write set differs"
    m = ref != NAN
    assert_close(bf(got[m]), bf(ref[m]))
    # unit diagonal and zero strict-upper part inside the diagonal blocks, exactly
    for t in range(T):
        r = t - d["cu"][np.searchsorted(d["cu"], t, side="right") - 1]
        rr = r % 64
        assert np.all(bf(got[t, :, rr]) == 1.0)
        blk = rr // 16
        assert np.all(bf(got[t, :, rr + 1:16 * (blk + 1)]) == 0.0)


def test_kkt_codes():
    lib = rk.abi.load("libreax_howu")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.reax_kkt(0, 0, 0, 0, 0, 0, 4, 2, 3, s) == -1  # HV != 2H
    assert lib.reax_kkt_smem() > 0


def test_kkt_config5_sampled_chunks():
    d = synth.delta_rule_inputs([16384, 16384], 16, 32, seed=61)
    At = rk.kkt(T_(d["k"]), t64(d["g"]), T_(d["beta"]), t64(d["cu"]), t64(d["cidx"]), 32)
    got = synth.from_torch_bf16(At)
    for ci in (0, 255, 256, 511):
        cidx = d["cidx"][ci:ci + 1]
        ref = orc.kkt(d["k"], d["g"], d["beta"], d["cu"], cidx, 16, 32)
        n, c = cidx[0]
        rows = slice(int(d["cu"][n] + 64 * c), int(d["cu"][n] + 64 * c + 64))
        assert_close(bf(got[rows]), bf(ref[rows]))


# ------------------------------------------------------------------------------------------------ howu
def howu_case(lengths, H, HV, seed):
    d = synth.delta_rule_inputs(lengths, H, HV, seed)
    A = orc.kkt(d["k"], d["g"], d["beta"], d["cu"], d["cidx"], H, HV)
    return d, A


@pytest.mark.parametrize("entry", ["reax_howu", "howu3_skip", "howu3_dense"])
def test_howu_vs_oracle(entry):
    d, A = howu_case([100, 150, 64], 2, 4, 70)
    scale = 1 / math.sqrt(128)
    dev = (T_(d["q"]), T_(d["k"]), T_(d["v"]), T_(d["beta"]), T_(A), t64(d["g"]), t64(d["cu"]))
    o = rk.howu(*dev, scale, entry)
    ref = orc.howu(d["q"], d["k"], d["v"], d["beta"], A, d["g"], d["cu"], scale, 2, 4, dense=entry == "howu3_dense")
    check_chain(synth.from_torch_bf16(o), ref, _reference_howu(entry, (dev, scale, 3, 2, 4)))


def test_howu_skip_ignores_upper_blocks_and_edge_lengths():
    # sequences of 1, 63, 64, 65 and 200 tokens; the strictly-upper 16x16 blocks of A (which the KKT never writes) hold
    # NaN: the skip entry points must not read them, and with zeros there the dense entry gives the same bits
    lengths = [1, 63, 64, 65, 200]
    d, A = howu_case(lengths, 2, 4, 76)
    scale = 1 / math.sqrt(128)
    Ap = A.copy()
    cu = d["cu"]
    for t in range(d["T"]):
        r = t - cu[np.searchsorted(cu, t, side="right") - 1]
        Ap[t, :, 16 * ((r % 64) // 16 + 1):] = NAN
    args = (T_(d["q"]), T_(d["k"]), T_(d["v"]), T_(d["beta"]))
    tail = (t64(d["g"]), t64(d["cu"]), scale)
    o_skip = synth.from_torch_bf16(rk.howu(*args, T_(Ap), *tail, "reax_howu"))
    o_skip3 = synth.from_torch_bf16(rk.howu(*args, T_(Ap), *tail, "howu3_skip"))
    o_dense = synth.from_torch_bf16(rk.howu(*args, T_(A), *tail, "howu3_dense"))
    ref = orc.howu(d["q"], d["k"], d["v"], d["beta"], A, d["g"], cu, scale, 2, 4)
    assert np.array_equal(o_skip, o_skip3)
    assert np.array_equal(o_skip, o_dense)
    assert_close_chain(bf(o_skip), bf(ref))


def test_howu_long_sequence():
    # 16 chunks of recurrence: the bf16 state re-publication error must stay within tolerance
    d, A = howu_case([1000], 1, 2, 71)
    scale = 1 / math.sqrt(128)
    dev = (T_(d["q"]), T_(d["k"]), T_(d["v"]), T_(d["beta"]), T_(A), t64(d["g"]), t64(d["cu"]))
    o = rk.howu(*dev, scale)
    ref = orc.howu(d["q"], d["k"], d["v"], d["beta"], A, d["g"], d["cu"], scale, 1, 2)
    check_chain(synth.from_torch_bf16(o), ref, _reference_howu("reax_howu", (dev, scale, 1, 1, 2)))


def test_howu_column_split_is_bitwise_whole_rows():
    # 5 sequences x 16 value heads: 2 * 80 CTAs exceed the SM count, so the launcher keeps whole rows (128 value
    # columns per CTA); one sequence alone (16 pairs) is split into two 64-column slices.  The recurrence is
    # independent per value column, so both launches must give the same bits for that sequence.
    lengths = [130, 70, 200, 64, 95]
    d, A = howu_case(lengths, 8, 16, 75)
    scale = 1 / math.sqrt(128)
    o = rk.howu(T_(d["q"]), T_(d["k"]), T_(d["v"]), T_(d["beta"]), T_(A), t64(d["g"]), t64(d["cu"]), scale)
    ref = orc.howu(d["q"], d["k"], d["v"], d["beta"], A, d["g"], d["cu"], scale, 8, 16)
    got = synth.from_torch_bf16(o)
    assert_close_chain(bf(got), bf(ref))
    b0, b1 = int(d["cu"][2]), int(d["cu"][3])  # the third sequence on its own
    cu1 = np.array([0, b1 - b0], np.int64)
    o1 = rk.howu(T_(d["q"][b0:b1]), T_(d["k"][b0:b1]), T_(d["v"][b0:b1]), T_(d["beta"][b0:b1]), T_(A[b0:b1]),
                 t64(d["g"][b0:b1]), t64(cu1), scale)
    assert np.array_equal(synth.from_torch_bf16(o1), got[b0:b1])


def test_howu_norm_vs_oracle():
    d, A = howu_case([100, 80], 2, 4, 72)
    T, HV = d["T"], 4
    rows = T + 5
    f2s = (np.arange(T, dtype=np.int32) + 2)
    f2s[7] = -1
    f2s[150] = -1
    ZS = HV * 128 + 32
    z = synth.bf16_normal(73, (rows, ZS), 2.0)
    nw = synth.bf16_normal(74, (128,), 0.1, 1.0)
    out0 = np.full((rows, HV, 128), NAN, np.uint16)
    outt = T_(out0)
    scale = 1 / math.sqrt(128)
    dev = (T_(d["q"]), T_(d["k"]), T_(d["v"]), T_(d["beta"]), T_(A), t64(d["g"]), t64(d["cu"]))
    f2s_t, z_t, nw_t = t64(f2s), T_(z), T_(nw)
    rk.howu_norm(*dev, scale, f2s_t, z_t, nw_t, 1e-6, 1.0 / 128, outt)
    got = synth.from_torch_bf16(outt)
    ref = orc.howu(d["q"], d["k"], d["v"], d["beta"], A, d["g"], d["cu"], scale, 2, 4,
                   norm=dict(f2s=f2s, z=z, ZS=ZS, nw=nw, eps=1e-6, factor=1.0 / 128, rows=rows), out=out0.copy())
    assert np.array_equal(got == NAN, ref == NAN), "write set differs"
    theirs = _reference_howu("reax_howu_norm", (dev, scale, 2, 2, 4),
                             norm=(T_(out0), f2s_t, z_t, ZS, nw_t, 1e-6, 1.0 / 128))
    m = ref != NAN
    check_chain(got[m], ref[m], None if theirs is None else theirs[m])
