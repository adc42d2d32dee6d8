"""The reference's own kernels, compiled unmodified for sm_100a into oracle/_ref, timed on the GPU at the BASELINE
shapes (TEST INFRASTRUCTURE: a second reference point for the benchmark's reference arm and for tests; never a product
path).  Every time is the mean of CUDA-event-timed launches on one stream with the L2 flushed (a 256 MiB write)
between them; for the libraries with configuration tables every index is timed and the best is reported.

Shapes where the reference cannot run BASELINE's own shape use the nearest shape it can run, stated in the result:
attention at head dim 256 (its only head dim, libreax_fmha_post/reax_fmha_v11.cu:25) and the RMSNorm at D = 2560
(libreax_howu/reax_rarn_final.cu:7).  The benchmark's own arm times this package's kernels at the same shapes.
"""
from __future__ import annotations

import ctypes as C
import math
import os

from .build import ref_path

REF_SHAPES = {
    "gv": "config 2: M=2048, K=4096, N2=14336",
    "gemm": "config-5 qkv projection: M=32768, K=2048, N=6144",
    "slices": "config 4: K=N=4096, S=4 x 1024, bf16 partials, M in {16, 256, 4096}",
    "rarn": "config-5 tokens at the reference's D: n=32768, D=2560, S=2",
    "conv_l2": "config 5: T=32768, KD=VD=2048, SX=6144",
    "kkt": "config 5: 2 x 16384 tokens, H=16, HV=32",
    "howu": "config 5: 2 x 16384 tokens, H=16, HV=32",
    "howu_norm": "config 5: 2 x 16384 tokens, H=16, HV=32, every row written",
    "fmha_q": "config 3 at the reference's head dim: B=4, S=8192, Hq=32, Hkv=8, D=256",
}


def _timer(torch, flush, steps):
    def time_fn(fn):
        fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            tot += a.elapsed_time(b)
        return tot / steps

    return time_fn


def time_all(steps: int = 5) -> dict:
    import numpy as np
    import torch

    from reax_engine_kernels_b200 import synth

    for n in ("libreax_gv", "libreax_plain", "libreax_slices", "libreax_howu", "libreax_fmha_post"):
        if not os.path.exists(ref_path(n)):
            raise FileNotFoundError(ref_path(n))
    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA device")
    torch.cuda.set_device(0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    tm = _timer(torch, flush, steps)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())
    out = {}

    def cfg_sweep(ncfg, call):
        best = None
        for cfg in range(ncfg):
            if call(cfg) != 0:
                continue
            ms = tm(lambda: call(cfg))
            if best is None or ms < best[1]:
                best = (cfg, ms)
        return best

    # ---- gate-up GEMM
    gv = C.CDLL(ref_path("libreax_gv"))
    Mg, Kg, N2 = 2048, 4096, 14336
    x = synth.device_normal_bf16((Mg, Kg), 1.0, 1)
    w = synth.device_normal_bf16((2 * N2, Kg), 0.02, 2)
    o = torch.empty(Mg, N2, dtype=torch.bfloat16, device="cuda")
    call = lambda cfg: gv.reax_gv(C.c_int(cfg), P(x), P(w), P(o), C.c_int(Mg), C.c_int(N2), C.c_int(Kg), s)
    cfg, ms = cfg_sweep(20, call)
    out["gv"] = {"ms": round(ms, 4), "best_cfg": cfg, "tflops": round(2.0 * Mg * 2 * N2 * Kg / ms / 1e9, 1)}
    del x, w, o
    # ---- plain GEMM (qkv projection of the linear-attention chain)
    pl = C.CDLL(ref_path("libreax_plain"))
    Mp, Kp, Np = 32768, 2048, 6144
    x = synth.device_normal_bf16((Mp, Kp), 1.0, 3)
    w = synth.device_normal_bf16((Np, Kp), 0.02, 4)
    d = torch.empty(Mp, Np, dtype=torch.bfloat16, device="cuda")
    call = lambda cfg: pl.reax_gemm(C.c_int(cfg), P(x), P(w), P(d), C.c_int(Mp), C.c_int(Np), C.c_int(Kp), C.c_int(Np), s)
    cfg, ms = cfg_sweep(15, call)
    out["gemm"] = {"ms": round(ms, 4), "best_cfg": cfg, "tflops": round(2.0 * Mp * Np * Kp / ms / 1e9, 1)}
    del x, w, d
    # ---- sliced GEMM sweep
    sl = C.CDLL(ref_path("libreax_slices"))
    Ks = Ns = 4096
    S = 4
    w = synth.device_normal_bf16((Ns, Ks), 0.02, 5)
    per_m = {}
    for Mi in (16, 256, 4096):
        x = synth.device_normal_bf16((Mi, Ks), 1.0, 6 + Mi)
        p = torch.empty(S, Mi, Ns, dtype=torch.bfloat16, device="cuda")
        call = lambda cfg: sl.reax_slices(C.c_int(cfg), C.c_int(0), P(x), P(w), P(p), C.c_int(Mi), C.c_int(Ns),
                                          C.c_int(Ks // S), C.c_int(S), C.c_int(Ks), s)
        cfg, ms = cfg_sweep(16, call)
        per_m[f"M={Mi}"] = {"ms": round(ms, 5), "best_cfg": cfg, "tflops": round(2.0 * Mi * Ns * Ks / ms / 1e9, 1)}
    out["slices"] = per_m
    del x, w, p
    # ---- linear-attention kernels
    hw = C.CDLL(ref_path("libreax_howu"))
    n, D = 32768, 2560
    part = synth.device_normal_bf16((2, n, D), 0.5, 7)
    res = synth.device_normal_bf16((n, D), 1.0, 8)
    wn = synth.device_normal_bf16((D,), 0.1, 9, mean=1.0)
    h_out, o = torch.empty(n, D, dtype=torch.bfloat16, device="cuda"), torch.empty(n, D, dtype=torch.bfloat16, device="cuda")
    ms = tm(lambda: hw.reax_rarn(P(part), C.c_int(2), C.c_int(0), C.c_longlong(n * D), P(res), P(wn), P(h_out), P(o),
                                 C.c_int(n), C.c_int(D), C.c_float(1e-6), C.c_float(1.0 / D), s))
    out["rarn"] = {"ms": round(ms, 4), "gbs": round(5 * n * D * 2 / ms / 1e6, 1)}
    del part, res, h_out, o
    T, KD = 32768, 2048
    SX = 3 * KD
    qkv = synth.device_normal_bf16((T, SX), 1.0, 10)
    cw = synth.device_normal_bf16((SX, 4), 0.5, 11)
    meta = torch.from_numpy(np.array([(p_, 0, s_ * 16384, 0) for s_ in range(2) for p_ in range(16384)], np.int32)).cuda()
    q = torch.empty(T, KD, dtype=torch.bfloat16, device="cuda")
    k, v = torch.empty_like(q), torch.empty_like(q)
    ms = tm(lambda: hw.reax_conv_l2(P(qkv), C.c_longlong(SX), C.c_void_p(0), C.c_int(0), P(meta), P(cw), P(q), P(k), P(v),
                                    C.c_int(T), C.c_float(1e-6), C.c_int(KD), C.c_int(KD), C.c_int(1), C.c_int(0),
                                    C.c_int(16), s))
    out["conv_l2"] = {"ms": round(ms, 4), "gbs": round(T * SX * 2 * 2 / ms / 1e6, 1)}
    del qkv, q, k, v
    H, HV = 16, 32
    dd = synth.delta_rule_inputs([16384, 16384], H, HV, 12)
    t16 = synth.to_torch_bf16
    t64 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    qq, kk, vv, beta = t16(dd["q"]), t16(dd["k"]), t16(dd["v"]), t16(dd["beta"])
    g, cu, cidx = t64(dd["g"]), t64(dd["cu"]), t64(dd["cidx"])
    A = torch.zeros(T, HV, 64, dtype=torch.bfloat16, device="cuda")
    ms = tm(lambda: hw.reax_kkt(P(kk), P(g), P(beta), P(A), P(cu), P(cidx), C.c_int(cidx.shape[0]), C.c_int(H),
                                C.c_int(HV), s))
    out["kkt"] = {"ms": round(ms, 4), "gbs": round((T * H * 256 + T * HV * 6 + T * HV * 80) / ms / 1e6, 1)}
    oo = torch.empty(T, HV, 128, dtype=torch.bfloat16, device="cuda")
    sc = C.c_float(1 / math.sqrt(128))
    ms = tm(lambda: hw.reax_howu(P(qq), P(kk), P(vv), P(beta), P(A), P(g), P(oo), P(cu), sc, C.c_int(2), C.c_int(H),
                                 C.c_int(HV), s))
    hb = T * (2 * H * 256 + 2 * HV * 256 + HV * 128)
    out["howu"] = {"ms": round(ms, 4), "gbs": round(hb / ms / 1e6, 1)}
    f2s = torch.arange(T, dtype=torch.int32, device="cuda")
    z = synth.device_normal_bf16((T, HV * 128), 1.0, 13)
    nw = synth.device_normal_bf16((128,), 0.1, 14, mean=1.0)
    ms = tm(lambda: hw.reax_howu_norm(P(qq), P(kk), P(vv), P(beta), P(A), P(g), P(oo), P(cu), sc, C.c_int(2), C.c_int(H),
                                      C.c_int(HV), s, P(f2s), P(z), C.c_longlong(HV * 128), P(nw), C.c_float(1e-6),
                                      C.c_float(1.0 / 128)))
    out["howu_norm"] = {"ms": round(ms, 4), "gbs": round((hb + T * HV * 256 + T * 4) / ms / 1e6, 1)}
    del qq, kk, vv, beta, g, cu, cidx, A, oo, z
    # ---- attention (head dim 256)
    fm = C.CDLL(ref_path("libreax_fmha_post"))
    B, Hk, G, Sa, Da = 4, 8, 4, 8192, 256
    Mr = Sa * G
    q = synth.device_normal_bf16((B, Hk, Mr, Da), 1.0, 15)
    k = synth.device_normal_bf16((B, Hk, Sa, Da), 1.0, 16)
    v = synth.device_normal_bf16((B, Hk, Sa, Da), 1.0, 17)
    o = torch.empty_like(q)
    qpos = torch.arange(Sa, dtype=torch.int32, device="cuda").repeat(B, 1).contiguous()
    st = lambda t: [C.c_longlong(x_) for x_ in (t.stride(0), t.stride(1), t.stride(2))]
    ms = tm(lambda: fm.reax_fmha_q(P(q), P(k), P(v), P(qpos), C.c_int(G), C.c_longlong(Sa), P(o),
                                   C.c_float(1 / math.sqrt(Da)), C.c_int(B), C.c_int(Hk), C.c_int(Mr), C.c_int(Sa),
                                   *st(q), *st(k), *st(v), *st(o), s))
    fl = 4.0 * Da * B * Hk * G * Sa * (Sa + 1) / 2
    out["fmha_q"] = {"ms": round(ms, 3), "tflops": round(fl / ms / 1e9, 1)}
    torch.cuda.synchronize()
    return {"what": "the reference's own kernels (unmodified sources compiled for sm_100a) timed on this GPU",
            "steps": steps, "l2": "flushed between launches (256 MiB write)", "shapes": REF_SHAPES, "kernels": out}
