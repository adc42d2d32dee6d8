"""The fp64 oracle against outputs of the reference itself: tests/golden/*.npz were produced by the reference's
own kernels (its unmodified sources compiled for sm_100a, run on a B200 by tests/golden/make_golden.py).
Bit-exact where the function is exact (write sets, residual sums); the project tolerance elsewhere."""
import glob
import math
import os

import numpy as np
import pytest

from oracle import oracle as orc
from reax_engine_kernels_b200 import synth
from tests.tolerance import assert_close, assert_close_interval

bf = synth.bf16_bits_to_f32
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NAN = 0x7FC0


def load(name):
    p = os.path.join(GOLD, name + ".npz")
    if not os.path.exists(p):
        pytest.fail(f"golden fixture {name} missing (run tests/golden/make_golden.py on a GPU box)")
    return np.load(p)


def test_fixture_set_complete():
    names = {os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLD, "*.npz"))}
    want = {"gv", "gemm", "slices", "fmha_q_g1", "fmha_q_g2", "fmha_b", "fmha_qp", "rarn_s2_serial0", "rarn_s2_serial1",
            "rarn_s3_serial1", "conv_rep1", "conv_rep2", "kkt", "howu"}
    assert want <= names, want - names


def test_gv_golden():
    z = load("gv")
    out, lo, hi = orc.gv(z["x"], z["w"])
    assert_close_interval(bf(z["out"]), bf(out), bf(lo), bf(hi))


def test_gemm_golden():
    z = load("gemm")
    M, N, K, ldd = z["dims"]
    d = orc.gemm(z["x"], z["w"])
    assert np.all(z["d"][:, N:] == NAN), "reference wrote past N"
    assert_close(bf(z["d"][:, :N]), bf(d))


def test_slices_golden():
    z = load("slices")
    M, N, K, S, kps = z["dims"]
    assert_close(z["p_fp32"], orc.slices(z["x"], z["w"], S, kps, True))
    assert_close(bf(z["p_bf16"]), bf(orc.slices(z["x"], z["w"], S, kps, False)))


@pytest.mark.parametrize("G", [1, 2])
def test_fmha_q_golden(G):
    z = load(f"fmha_q_g{G}")
    B, H, M, N, D, G_, Lq = z["dims"]
    o = orc.fmha(z["q"], z["k"], z["v"], float(z["scale"][0]), qpos=z["qpos"], G=int(G_), qpBs=int(Lq))
    assert_close(bf(z["o"]), bf(o))


def test_fmha_b_golden():
    z = load("fmha_b")
    o = orc.fmha(z["q"], z["k"], z["v"], float(z["scale"][0]), bias=z["bias"])
    assert_close(bf(z["o"]), bf(o))


def test_fmha_qp_golden():
    z = load("fmha_qp")
    B, H, G, Lq, D = z["dims"]
    ref = np.full_like(z["outp"], NAN)
    orc.fmha(z["q"], z["k"], z["v"], float(z["scale"][0]), qpos=z["qpos"], G=int(G), qpBs=int(Lq),
             post=dict(inv=z["inv"], Lq=int(Lq), qg=z["qg"], qg_rs=int(H * G * 2 * D), outp=ref, out_rs=int(H * G * D)))
    assert np.array_equal(ref == NAN, z["outp"] == NAN), "write set"
    m = ref != NAN
    assert_close(bf(z["outp"][m]), bf(ref[m]))


@pytest.mark.parametrize("name", ["rarn_s2_serial0", "rarn_s2_serial1", "rarn_s3_serial1"])
def test_rarn_golden(name):
    z = load(name)
    S, serial, n, D = z["dims"]
    h, o = orc.rarn(z["part"], S, serial, n * D, z["res"], z["w"], n, D, 1e-6, 1.0 / D)
    assert np.array_equal(h, z["h_out"]), "h_out is exact"
    assert_close(bf(z["out"]), bf(o))


@pytest.mark.parametrize("rep", [1, 2])
def test_conv_golden(rep):
    z = load(f"conv_rep{rep}")
    T, SX, Ct, KD, VD, rep_ = z["dims"]
    q0 = np.full((T, rep * KD), NAN, np.uint16)
    q, k, v = orc.conv(z["qkv"], SX, z["cache"], Ct, z["meta"], z["w"], T, 1e-6, KD, VD, rep, 0, q=q0.copy(), k=q0.copy(),
                       v=np.full((T, VD), NAN, np.uint16))
    for a, b in ((q, z["q"]), (k, z["k"]), (v, z["v"])):
        assert np.array_equal(a == NAN, b == NAN)
        assert_close(bf(b[a != NAN]), bf(a[a != NAN]))


def test_kkt_golden():
    z = load("kkt")
    A0 = np.full(z["A"].shape, NAN, np.uint16)
    A = orc.kkt(z["k"], z["g"], z["beta"], z["cu"], z["cidx"], 2, 4, A=A0)
    assert np.array_equal(A == NAN, z["A"] == NAN), "write set (upper 16x16 blocks never written)"
    m = A != NAN
    assert_close(bf(z["A"][m]), bf(A[m]))


def test_howu_golden():
    z = load("howu")
    sc = float(z["scale"][0])
    for key, dense in (("o_skip", False), ("o_dense", True)):
        o = orc.howu(z["q"], z["k"], z["v"], z["beta"], z["A"], z["g"], z["cu"], sc, 2, 4, dense=dense)
        assert_close(bf(z[key]), bf(o))
    rows = z["out_norm"].shape[0]
    ref = np.full_like(z["out_norm"], NAN)
    orc.howu(z["q"], z["k"], z["v"], z["beta"], z["A"], z["g"], z["cu"], sc, 2, 4,
             norm=dict(f2s=z["f2s"], z=z["z"], ZS=z["z"].shape[1], nw=z["nw"], eps=1e-6, factor=1.0 / 128, rows=rows), out=ref)
    assert np.array_equal(ref == NAN, z["out_norm"] == NAN)
    m = ref != NAN
    assert_close(bf(z["out_norm"][m]), bf(ref[m]))
