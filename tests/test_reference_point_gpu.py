"""Second reference point: the reference's own gate-up kernel (its unmodified source compiled for sm_100a into
oracle/_ref) timed on this B200 on the BASELINE config-2 shape beside ours, same inputs, and checked for agreement.
Run with -s to see the numbers."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

from oracle.build import ref_path
from reax_engine_kernels_b200 import abi, synth

pytestmark = pytest.mark.gpu


def _time(fn, n=20):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    torch.cuda._sleep(50_000_000)
    e0.record()
    for _ in range(n):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n


@pytest.mark.skipif(not os.path.exists(ref_path("libreax_gv")), reason="reference build absent")
def test_gate_up_vs_reference_kernel_on_b200():
    M, N2, K = 2048, 14336, 4096
    x = synth.device_normal_bf16((M, K), 1.0, 1)
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 2)
    ours = torch.empty(M, N2, dtype=torch.bfloat16, device="cuda")
    theirs = torch.empty_like(ours)
    ref = C.CDLL(ref_path("libreax_gv"))
    lib = abi.load("libreax_gv")
    s = torch.cuda.current_stream().cuda_stream
    flops = 2.0 * M * 2 * N2 * K
    best = None
    for cfg in range(20):
        rc = ref.reax_gv(C.c_int(cfg), C.c_void_p(x.data_ptr()), C.c_void_p(w.data_ptr()), C.c_void_p(theirs.data_ptr()),
                         C.c_int(M), C.c_int(N2), C.c_int(K), C.c_void_p(s))
        if rc:
            continue
        ms = _time(lambda: ref.reax_gv(C.c_int(cfg), C.c_void_p(x.data_ptr()), C.c_void_p(w.data_ptr()),
                                       C.c_void_p(theirs.data_ptr()), C.c_int(M), C.c_int(N2), C.c_int(K), C.c_void_p(s)))
        if best is None or ms < best[1]:
            best = (cfg, ms)
    ms_ours = _time(lambda: lib.reax_gv(0, x.data_ptr(), w.data_ptr(), ours.data_ptr(), M, N2, K, s))
    ref.reax_gv(C.c_int(best[0]), C.c_void_p(x.data_ptr()), C.c_void_p(w.data_ptr()), C.c_void_p(theirs.data_ptr()),
                C.c_int(M), C.c_int(N2), C.c_int(K), C.c_void_p(s))
    torch.cuda.synchronize()
    print(f"\nreference reax_gv best cfg {best[0]}: {best[1]*1e3:.1f} us = {flops/best[1]/1e9:.1f} TFLOP/s;"
          f" ours: {ms_ours*1e3:.1f} us = {flops/ms_ours/1e9:.1f} TFLOP/s; speed-up {best[1]/ms_ours:.2f}x")
    d = (ours.float() - theirs.float()).abs()
    frac_exact = float((ours.view(torch.int16) == theirs.view(torch.int16)).float().mean())
    print(f"bitwise-equal fraction vs reference kernel: {frac_exact:.6f}; max abs diff {float(d.max()):.4g}")
    assert frac_exact > 0.999
    assert ms_ours < best[1]


@pytest.mark.skipif(not os.path.exists(ref_path("libreax_fmha_post")), reason="reference build absent")
def test_attention_d256_vs_reference_kernel_on_b200():
    # GQA causal prefill at the reference's head dim (256): B=1, Hkv=4, G=4, S=2048 (M = 8192 rows per kv head)
    import math

    from reax_engine_kernels_b200 import kernels as rk
    B, H, G, S, D = 1, 4, 4, 2048, 256
    M = S * G
    q = synth.device_normal_bf16((B, H, M, D), 1.0, 21)
    k = synth.device_normal_bf16((B, H, S, D), 1.0, 22)
    v = synth.device_normal_bf16((B, H, S, D), 1.0, 23)
    qpos = torch.arange(S, dtype=torch.int32, device="cuda").view(1, S)
    scale = 1 / math.sqrt(D)
    ours = torch.empty(B, H, M, D, dtype=torch.bfloat16, device="cuda")
    theirs = torch.empty_like(ours)
    ref = C.CDLL(ref_path("libreax_fmha_post"))
    s = torch.cuda.current_stream().cuda_stream
    st = lambda t: [C.c_longlong(x) for x in (t.stride(0), t.stride(1), t.stride(2))]

    def run_ref():
        rc = ref.reax_fmha_q(C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()),
                             C.c_void_p(qpos.data_ptr()), C.c_int(G), C.c_longlong(S), C.c_void_p(theirs.data_ptr()),
                             C.c_float(scale), C.c_int(B), C.c_int(H), C.c_int(M), C.c_int(S), *st(q), *st(k), *st(v),
                             *st(theirs), C.c_void_p(s))
        assert rc == 0

    def run_ours():
        rk.fmha(q, k, v, scale, qpos=qpos, G=G, out=ours)

    ms_ref = _time(run_ref, 5)
    ms_ours = _time(run_ours, 5)
    torch.cuda.synchronize()
    # causal FLOPs: 4 * D * (visible (row, key) pairs)
    pairs = B * H * sum((t + 1) * G for t in range(S))
    flops = 4.0 * D * pairs
    frac = float((ours.view(torch.int16) == theirs.view(torch.int16)).float().mean())
    print(f"\nreference reax_fmha_q (D=256): {ms_ref*1e3:.1f} us = {flops/ms_ref/1e9:.1f} TFLOP/s; ours: {ms_ours*1e3:.1f} us = "
          f"{flops/ms_ours/1e9:.1f} TFLOP/s; speed-up {ms_ref/ms_ours:.2f}x; bitwise-equal fraction {frac:.4f}")
    # both kernels against the oracle's rounding interval on sampled rows (the two differ only where a probability
    # sits on a bf16 rounding midpoint and their fp32 score accumulations round it differently)
    from oracle import oracle as orc
    from tests.tolerance import assert_close_interval

    bf = synth.bf16_bits_to_f32
    qh, kh, vh = (synth.from_torch_bf16(t) for t in (q, k, v))
    oh, th = synth.from_torch_bf16(ours), synth.from_torch_bf16(theirs)
    for r0 in (0, 4097, M - 3):
        ref, lo, hi = orc.fmha(qh, kh, vh, scale, qpos=qpos.cpu().numpy(), G=G, qpBs=S, rows=(r0, r0 + 3), intervals=True)
        sl = (slice(None), slice(None), slice(r0, r0 + 3))
        assert_close_interval(bf(oh[sl]), bf(ref[sl]), bf(lo[sl]), bf(hi[sl]))
        assert_close_interval(bf(th[sl]), bf(ref[sl]), bf(lo[sl]), bf(hi[sl]))
    assert ms_ours < ms_ref


@pytest.mark.skipif(not os.path.exists(ref_path("libreax_howu")), reason="reference build absent")
@pytest.mark.parametrize("entry", ["reax_howu", "reax_kkt", "reax_conv_l2", "reax_rarn"])
def test_linear_attention_vs_reference_kernels(entry):
    """Our linear-attention kernels against the reference's own kernels on identical inputs: report the bitwise-equal
    fraction and both implementations' error statistics against the oracle; ours must be at least as close to the
    oracle as the reference is (max and mean of the project's relative error)."""
    import math

    from oracle import oracle as orc
    from reax_engine_kernels_b200 import kernels as rk
    from tests.tolerance import rel_errors

    bf = synth.bf16_bits_to_f32
    ref = C.CDLL(ref_path("libreax_howu"))
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())
    T_ = synth.to_torch_bf16
    t64 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    if entry in ("reax_howu", "reax_kkt"):
        d = synth.delta_rule_inputs([300, 200, 64], 2, 4, 90)
        dd = {n: (T_(d[n]) if d[n].dtype == np.uint16 else t64(d[n])) for n in ("q", "k", "v", "beta", "g", "cu", "cidx")}
        A_ref = torch.zeros(d["T"], 4, 64, dtype=torch.bfloat16, device="cuda")
        assert ref.reax_kkt(P(dd["k"]), P(dd["g"]), P(dd["beta"]), P(A_ref), P(dd["cu"]), P(dd["cidx"]),
                            C.c_int(d["cidx"].shape[0]), C.c_int(2), C.c_int(4), s) == 0
        if entry == "reax_kkt":
            ours = rk.kkt(dd["k"], dd["g"], dd["beta"], dd["cu"], dd["cidx"], 4)
            theirs = A_ref
            oracle = orc.kkt(d["k"], d["g"], d["beta"], d["cu"], d["cidx"], 2, 4)
        else:
            sc = 1 / math.sqrt(128)
            ours = rk.howu(dd["q"], dd["k"], dd["v"], dd["beta"], A_ref, dd["g"], dd["cu"], sc)
            theirs = torch.empty_like(ours)
            assert ref.reax_howu(P(dd["q"]), P(dd["k"]), P(dd["v"]), P(dd["beta"]), P(A_ref), P(dd["g"]), P(theirs),
                                 P(dd["cu"]), C.c_float(sc), C.c_int(3), C.c_int(2), C.c_int(4), s) == 0
            oracle = orc.howu(d["q"], d["k"], d["v"], d["beta"], synth.from_torch_bf16(A_ref), d["g"], d["cu"], sc, 2, 4)
    elif entry == "reax_conv_l2":
        T, KD, VD = 2048, 256, 256
        SX = 2 * KD + VD
        qkv = synth.device_normal_bf16((T, SX), 1.0, 91)
        w = synth.device_normal_bf16((SX, 4), 0.5, 92)
        meta = t64(np.array([(t, 0, 0, 0) for t in range(T)], np.int32))
        q, k, v = rk.conv_l2(qkv, meta, w, KD, VD)
        q2, k2, v2 = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        assert ref.reax_conv_l2(P(qkv), C.c_longlong(SX), C.c_void_p(0), C.c_int(0), P(meta), P(w), P(q2), P(k2), P(v2),
                                C.c_int(T), C.c_float(1e-6), C.c_int(KD), C.c_int(VD), C.c_int(1), C.c_int(0), C.c_int(16), s) == 0
        ours, theirs = torch.cat([q, k, v], 1), torch.cat([q2, k2, v2], 1)
        rq, rk_, rv = orc.conv(synth.from_torch_bf16(qkv), SX, None, 0, meta.cpu().numpy(), synth.from_torch_bf16(w), T,
                               1e-6, KD, VD, 1, 0)
        oracle = np.concatenate([rq, rk_, rv], 1)
    else:
        n, D, S_ = 4096, 2560, 2
        part = synth.device_normal_bf16((S_, n, D), 0.5, 93)
        res = synth.device_normal_bf16((n, D), 1.0, 94)
        w = synth.device_normal_bf16((D,), 0.1, 95, mean=1.0)
        _, ours = rk.rarn(part, res, w, 1e-6, 1.0 / D)
        h2, theirs = torch.empty_like(ours), torch.empty_like(ours)
        assert ref.reax_rarn(P(part), C.c_int(S_), C.c_int(0), C.c_longlong(n * D), P(res), P(w), P(h2), P(theirs), C.c_int(n),
                             C.c_int(D), C.c_float(1e-6), C.c_float(1.0 / D), s) == 0
        _, oracle = orc.rarn(synth.from_torch_bf16(part), S_, 0, n * D, synth.from_torch_bf16(res), synth.from_torch_bf16(w),
                             n, D, 1e-6, 1.0 / D)
    torch.cuda.synchronize()
    o, t = synth.from_torch_bf16(ours), synth.from_torch_bf16(theirs)
    frac = float(np.mean(o == t))
    eo, et = rel_errors(bf(o), bf(oracle)), rel_errors(bf(t), bf(oracle))
    print(f"\n{entry}: bitwise-equal fraction vs reference {frac:.6f}; vs oracle -- ours max {eo.max():.3g} mean {eo.mean():.3g}"
          f" (>1e-2: {int((eo > 1e-2).sum())}); reference max {et.max():.3g} mean {et.mean():.3g} (>1e-2: {int((et > 1e-2).sum())})")
    assert eo.mean() <= max(1e-3, 1.1 * et.mean())
    assert eo.max() <= max(1e-2, 1.5 * et.max())
