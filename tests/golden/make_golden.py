"""Generate the golden fixtures that pin the fp64 oracle to the reference implementation.

Runs on a B200: loads the reference's own libraries (the unmodified reference sources compiled for sm_100a by
oracle/build.py into oracle/_ref/), calls their C entry points exactly as the engine does on small seeded inputs,
and stores inputs + outputs as tests/golden/<case>.npz (bf16 as uint16 bits).  The CPU test suite
(tests/test_oracle_golden.py) then checks the oracle against these outputs.

    python tests/golden/make_golden.py            # on a GPU box, from the repository root
"""
import ctypes as C
import math
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from oracle.build import ref_path  # noqa: E402
from reax_engine_kernels_b200 import synth  # noqa: E402

OUT = os.environ.get("GOLDEN_OUT", os.path.dirname(os.path.abspath(__file__)))
c_int, c_float, c_ll, c_vp = C.c_int, C.c_float, C.c_longlong, C.c_void_p
NAN = 0x7FC0


def lib(name):
    return C.CDLL(ref_path(name))


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if a.dtype == np.uint16:
        t = t.view(torch.int16)
    return t.cuda()


def host(t, dtype=np.uint16):
    torch.cuda.synchronize()
    a = t.cpu().numpy()
    return a.view(dtype) if dtype == np.uint16 else a


def P(t):
    return c_vp(t.data_ptr())


def S():
    return c_vp(torch.cuda.current_stream().cuda_stream)


def save(name, **arrays):
    np.savez_compressed(os.path.join(OUT, name + ".npz"), **arrays)
    print("wrote", name, {k: v.shape for k, v in arrays.items()})


def case_gv():
    M, N2, K = 96, 128, 256
    x = synth.bf16_normal(1001, (M, K))
    w = synth.bf16_normal(1002, (2 * N2, K), 0.05)
    xt, wt = dev(x), dev(w)
    out = torch.zeros(M, N2, dtype=torch.int16, device="cuda")
    rc = lib("libreax_gv").reax_gv(c_int(0), P(xt), P(wt), P(out), c_int(M), c_int(N2), c_int(K), S())
    assert rc == 0, rc
    save("gv", x=x, w=w, out=host(out), dims=np.array([M, N2, K]))


def case_gemm():
    M, N, K, ldd = 80, 96, 192, 104
    x = synth.bf16_normal(1011, (M, K))
    w = synth.bf16_normal(1012, (N, K), 0.05)
    xt, wt = dev(x), dev(w)
    d = dev(np.full((M, ldd), NAN, np.uint16))
    rc = lib("libreax_plain").reax_gemm(c_int(2), P(xt), P(wt), P(d), c_int(M), c_int(N), c_int(K), c_int(ldd), S())
    assert rc == 0, rc
    save("gemm", x=x, w=w, d=host(d), dims=np.array([M, N, K, ldd]))


def case_slices():
    M, N, K, S_, kps = 40, 64, 256, 2, 128
    x = synth.bf16_normal(1021, (M, K))
    w = synth.bf16_normal(1022, (N, K), 0.05)
    xt, wt = dev(x), dev(w)
    outs = {}
    for fp32 in (0, 1):
        p = torch.zeros(S_ * M * N * (2 if fp32 else 1), dtype=torch.int16, device="cuda")
        rc = lib("libreax_slices").reax_slices(c_int(4), c_int(fp32), P(xt), P(wt), P(p), c_int(M), c_int(N), c_int(kps),
                                               c_int(S_), c_int(K), S())
        assert rc == 0, rc
        torch.cuda.synchronize()
        a = p.cpu().numpy()
        outs["p_fp32" if fp32 else "p_bf16"] = a.view(np.float32).reshape(S_, M, N) if fp32 else a.view(np.uint16).reshape(S_, M, N)
    save("slices", x=x, w=w, dims=np.array([M, N, K, S_, kps]), **outs)


def fmha_strides(B, H, R, D):
    return [c_ll(H * R * D), c_ll(R * D), c_ll(D)]


def case_fmha_q():
    for G in (1, 2):
        B, H, Lq, D = 1, 1, 100 // G * 1, 256
        M = Lq * G
        N = Lq + 7  # 7 tokens of history
        q = synth.bf16_normal(1031 + G, (B, H, M, D))
        k = synth.bf16_normal(1033 + G, (B, H, N, D))
        v = synth.bf16_normal(1035 + G, (B, H, N, D))
        qpos = (np.arange(Lq, dtype=np.int32) + 7).reshape(1, Lq)
        qt, kt, vt, qp = dev(q), dev(k), dev(v), dev(qpos)
        o = dev(np.full((B, H, M, D), NAN, np.uint16))
        scale = 1 / math.sqrt(D)
        f = lib("libreax_fmha_post").reax_fmha_q
        rc = f(P(qt), P(kt), P(vt), P(qp), c_int(G), c_ll(Lq), P(o), c_float(scale), c_int(B), c_int(H), c_int(M), c_int(N),
               *fmha_strides(B, H, M, D), *fmha_strides(B, H, N, D), *fmha_strides(B, H, N, D), *fmha_strides(B, H, M, D), S())
        assert rc == 0, rc
        save(f"fmha_q_g{G}", q=q, k=k, v=v, qpos=qpos, o=host(o), dims=np.array([B, H, M, N, D, G, Lq]),
             scale=np.array([scale], np.float32))


def case_fmha_b():
    B, H, M, N, D = 1, 1, 70, 140, 256
    q = synth.bf16_normal(1041, (B, H, M, D))
    k = synth.bf16_normal(1042, (B, H, N, D))
    v = synth.bf16_normal(1043, (B, H, N, D))
    bias = synth.bf16_normal(1044, (B, H, M, N), 2.0)
    bias[synth.uniform(1045, B * H * M * N).reshape(B, H, M, N) < 0.25] = 0xFF80
    qt, kt, vt, bt = dev(q), dev(k), dev(v), dev(bias)
    o = dev(np.full((B, H, M, D), NAN, np.uint16))
    f = lib("libreax_fmha_post").reax_fmha_b
    rc = f(P(qt), P(kt), P(vt), P(bt), P(o), c_float(0.07), c_int(B), c_int(H), c_int(M), c_int(N),
           *fmha_strides(B, H, M, D), *fmha_strides(B, H, N, D), *fmha_strides(B, H, N, D), *fmha_strides(B, H, M, N),
           *fmha_strides(B, H, M, D), S())
    assert rc == 0, rc
    save("fmha_b", q=q, k=k, v=v, bias=bias, o=host(o), dims=np.array([B, H, M, N, D]), scale=np.array([0.07], np.float32))


def case_fmha_qp():
    B, H, G, Lq, D = 1, 1, 2, 40, 256
    M, N = Lq * G, Lq
    q = synth.bf16_normal(1051, (B, H, M, D))
    k = synth.bf16_normal(1052, (B, H, N, D))
    v = synth.bf16_normal(1053, (B, H, N, D))
    qpos = np.arange(Lq, dtype=np.int32).reshape(1, Lq)
    rows = Lq + 2
    inv = synth.uniform(1054, Lq).argsort().astype(np.int32).reshape(1, Lq)
    inv[0, 3] = -1
    Hq = H * G
    qg = synth.bf16_normal(1055, (rows, Hq * 2 * D), 3.0)
    outp0 = np.full((rows, Hq * D), NAN, np.uint16)
    qt, kt, vt, qp, it, gt, ot = dev(q), dev(k), dev(v), dev(qpos), dev(inv), dev(qg), dev(outp0)
    f = lib("libreax_fmha_post").reax_fmha_qp
    rc = f(P(qt), P(kt), P(vt), P(qp), c_int(G), c_ll(Lq), c_float(0.0625), c_int(B), c_int(H), c_int(M), c_int(N),
           *fmha_strides(B, H, M, D), *fmha_strides(B, H, N, D), *fmha_strides(B, H, N, D), P(it), c_int(Lq), P(gt),
           c_ll(Hq * 2 * D), P(ot), c_ll(Hq * D), S())
    assert rc == 0, rc
    save("fmha_qp", q=q, k=k, v=v, qpos=qpos, inv=inv, qg=qg, outp=host(ot), dims=np.array([B, H, G, Lq, D]),
         scale=np.array([0.0625], np.float32))


def case_rarn():
    n, D = 20, 2560
    for S_, serial in ((2, 0), (2, 1), (3, 1)):
        part = synth.bf16_normal(1061 + S_, (S_, n, D), 0.5)
        res = synth.bf16_normal(1064, (n, D))
        w = synth.bf16_normal(1065, (D,), 0.1, 1.0)
        pt, rt, wt = dev(part), dev(res), dev(w)
        h = torch.zeros(n, D, dtype=torch.int16, device="cuda")
        o = torch.zeros(n, D, dtype=torch.int16, device="cuda")
        rc = lib("libreax_howu").reax_rarn(P(pt), c_int(S_), c_int(serial), c_ll(n * D), P(rt), P(wt), P(h), P(o), c_int(n),
                                            c_int(D), c_float(1e-6), c_float(1.0 / D), S())
        assert rc == 0, rc
        save(f"rarn_s{S_}_serial{serial}", part=part, res=res, w=w, h_out=host(h), out=host(o), dims=np.array([S_, serial, n, D]))


def case_conv():
    KD, VD, cache_rows = 256, 256, 3
    lengths = [30, 50]
    T = sum(lengths)
    SX = 2 * KD + VD + 64
    Ct = 2 * KD + VD
    qkv = synth.bf16_normal(1071, (T, SX))
    w = synth.bf16_normal(1072, (Ct, 4), 0.5)
    cache = synth.bf16_normal(1073, (cache_rows, Ct))
    meta, bos = [], 0
    for L in lengths:
        for p in range(L):
            meta.append((p + cache_rows, cache_rows, bos - cache_rows, 0))
        bos += L
    meta = np.array(meta, np.int32)
    # every device tensor stays referenced until the kernel has finished (a temporary freed while the argument
    # list is built would be handed to the next argument by the caching allocator)
    qkv_d, cache_d, meta_d, w_d = dev(qkv), dev(cache), dev(meta), dev(w)
    for rep in (1, 2):
        qt, kt, vt = (dev(np.full(s, NAN, np.uint16)) for s in ((T, rep * KD), (T, rep * KD), (T, VD)))
        rc = lib("libreax_howu").reax_conv_l2(P(qkv_d), c_ll(SX), P(cache_d), c_int(Ct), P(meta_d), P(w_d), P(qt),
                                               P(kt), P(vt), c_int(T), c_float(1e-6), c_int(KD), c_int(VD), c_int(rep), c_int(0),
                                               c_int(16), S())
        assert rc == 0, rc
        save(f"conv_rep{rep}", qkv=qkv, w=w, cache=cache, meta=meta, q=host(qt), k=host(kt), v=host(vt),
             dims=np.array([T, SX, Ct, KD, VD, rep]))


def delta_inputs(seed):
    return synth.delta_rule_inputs([100, 40], 2, 4, seed)


def case_kkt():
    d = delta_inputs(1081)
    T = d["T"]
    At = dev(np.full((T, 4, 64), NAN, np.uint16))
    dd = {n: dev(d[n]) for n in ("k", "g", "beta", "cu", "cidx")}
    rc = lib("libreax_howu").reax_kkt(P(dd["k"]), P(dd["g"]), P(dd["beta"]), P(At), P(dd["cu"]), P(dd["cidx"]),
                                       c_int(d["cidx"].shape[0]), c_int(2), c_int(4), S())
    assert rc == 0, rc
    save("kkt", k=d["k"], g=d["g"], beta=d["beta"], cu=d["cu"], cidx=d["cidx"], A=host(At))


def case_howu():
    d = delta_inputs(1091)
    T = d["T"]
    L = lib("libreax_howu")
    # A from the reference's own KKT, upper blocks zero-filled (what howu3_dense requires)
    At = dev(np.zeros((T, 4, 64), np.uint16))
    dd = {n: dev(d[n]) for n in ("q", "k", "v", "g", "beta", "cu", "cidx")}
    rc = L.reax_kkt(P(dd["k"]), P(dd["g"]), P(dd["beta"]), P(At), P(dd["cu"]), P(dd["cidx"]), c_int(d["cidx"].shape[0]),
                    c_int(2), c_int(4), S())
    assert rc == 0, rc
    A = host(At)
    scale = 1 / math.sqrt(128)
    outs = {}
    for entry in ("reax_howu", "howu3_dense"):
        o = dev(np.full((T, 4, 128), NAN, np.uint16))
        rc = getattr(L, entry)(P(dd["q"]), P(dd["k"]), P(dd["v"]), P(dd["beta"]), P(At), P(dd["g"]), P(o), P(dd["cu"]),
                               c_float(scale), c_int(2), c_int(2), c_int(4), S())
        assert rc == 0, rc
        outs[entry] = host(o)
    rows = T + 3
    f2s = np.arange(T, dtype=np.int32) + 1
    f2s[5] = -1
    ZS = 4 * 128 + 32
    z = synth.bf16_normal(1092, (rows, ZS), 2.0)
    nw = synth.bf16_normal(1093, (128,), 0.1, 1.0)
    on = dev(np.full((rows, 4, 128), NAN, np.uint16))
    f2s_d, z_d, nw_d = dev(f2s), dev(z), dev(nw)
    rc = L.reax_howu_norm(P(dd["q"]), P(dd["k"]), P(dd["v"]), P(dd["beta"]), P(At), P(dd["g"]), P(on), P(dd["cu"]),
                          c_float(scale), c_int(2), c_int(2), c_int(4), S(), P(f2s_d), P(z_d), c_ll(ZS), P(nw_d),
                          c_float(1e-6), c_float(1.0 / 128))
    assert rc == 0, rc
    save("howu", q=d["q"], k=d["k"], v=d["v"], beta=d["beta"], g=d["g"], cu=d["cu"], A=A, o_skip=outs["reax_howu"],
         o_dense=outs["howu3_dense"], f2s=f2s, z=z, nw=nw, out_norm=host(on), scale=np.array([scale], np.float32))


if __name__ == "__main__":
    os.makedirs(OUT, exist_ok=True)
    torch.cuda.set_device(0)
    cases = {f.__name__[5:]: f for f in (case_gv, case_gemm, case_slices, case_fmha_q, case_fmha_b, case_fmha_qp, case_rarn,
                                         case_conv, case_kkt, case_howu)}
    for name in (sys.argv[1:] or cases):
        cases[name]()
