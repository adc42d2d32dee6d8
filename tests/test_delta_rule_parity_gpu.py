"""Parity of the chunked gated delta rule (reax_howu, reax_howu_norm) at BASELINE config-5 head counts, pinned to the
reference's own kernel: ours and the reference's unmodified sources built for sm_100a (oracle/_ref) run on identical
inputs, and both are checked against the fp64 oracle on a prefix of one sequence.

Criterion (oracle/tolerance.py reference_matched_stats): mean relative error <= 1e-3; every element above the 1e-2
element bound equals the reference kernel's output bit for bit (the chain of ~10 bf16 roundings per chunk over a
128x128 recurrent state makes a few intermediates land on the other side of a bf16 midpoint than the fp64 oracle's,
and the reference's kernel shows the same outliers); wherever ours differs from the reference kernel, it is within 1e-2
of the oracle.  The measured statistics are printed (-s) and asserted against the reference kernel's own."""
import ctypes as C
import math
import os

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from oracle.build import ref_path
from oracle.tolerance import reference_matched_stats
from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import synth

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(ref_path("libreax_howu")), reason="reference build absent")]
bf = synth.bf16_bits_to_f32
T_ = synth.to_torch_bf16
P = lambda t: C.c_void_p(t.data_ptr())
H, HV, L = 16, 32, 4096           # config-5 head counts; 2 sequences of 4096 tokens
TP, H1, HV1 = 2048, 2, 4          # oracle prefix: sequence 0, tokens < 2048, key heads 0-1 (value heads 0-3)


@pytest.fixture(scope="module")
def case():
    d = synth.delta_rule_inputs([L, L], H, HV, 0x5EED0000 + 55)
    t64 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dd = {n: (T_(d[n]) if d[n].dtype == np.uint16 else t64(d[n])) for n in ("q", "k", "v", "beta", "g", "cu", "cidx")}
    A = rk.kkt(dd["k"], dd["g"], dd["beta"], dd["cu"], dd["cidx"], HV)
    return d, dd, A


def _prefix(a, nh):
    return np.ascontiguousarray(a[:TP, :nh])


def test_delta_rule_outliers_are_the_reference_kernels(case):
    d, dd, A = case
    sc = 1 / math.sqrt(128)
    ours = rk.howu(dd["q"], dd["k"], dd["v"], dd["beta"], A, dd["g"], dd["cu"], sc)
    theirs = torch.empty_like(ours)
    ref = C.CDLL(ref_path("libreax_howu"))
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert ref.reax_howu(P(dd["q"]), P(dd["k"]), P(dd["v"]), P(dd["beta"]), P(A), P(dd["g"]), P(theirs), P(dd["cu"]),
                         C.c_float(sc), C.c_int(2), C.c_int(H), C.c_int(HV), s) == 0
    torch.cuda.synchronize()
    o, t = synth.from_torch_bf16(ours), synth.from_torch_bf16(theirs)
    frac = float(np.mean(o == t))
    Ah = synth.from_torch_bf16(A)
    oracle = orc.howu(_prefix(d["q"], H1), _prefix(d["k"], H1), _prefix(d["v"], HV1), _prefix(d["beta"], HV1),
                      _prefix(Ah, HV1), _prefix(d["g"], HV1), np.array([0, TP], np.int64), sc, H1, HV1)
    st = reference_matched_stats(bf(o[:TP, :HV1]), bf(oracle), bf(t[:TP, :HV1]))
    print(f"\nreax_howu, {2 * L} tokens x {HV} value heads: bitwise equal to the reference kernel on {frac:.6f} of "
          f"{o.size} outputs; vs oracle ({st['elements']} outputs): {st}")
    assert frac > 0.999
    assert st["within_tolerance"], st
    assert st["mean_rel"] <= max(1e-3, 1.01 * st["reference_kernel_mean_rel"])


def test_delta_rule_norm_outliers_are_the_reference_kernels(case):
    d, dd, A = case
    sc = 1 / math.sqrt(128)
    T = 2 * L
    f2s = torch.arange(T, dtype=torch.int32, device="cuda")
    z = synth.device_normal_bf16((T, HV * 128), 1.0, 0x5EED0000 + 56)
    nw = synth.device_normal_bf16((128,), 0.1, 0x5EED0000 + 57, mean=1.0)
    ours = torch.empty(T, HV, 128, dtype=torch.bfloat16, device="cuda")
    theirs = torch.empty_like(ours)
    rk.howu_norm(dd["q"], dd["k"], dd["v"], dd["beta"], A, dd["g"], dd["cu"], sc, f2s, z, nw, 1e-6, 1.0 / 128, ours)
    ref = C.CDLL(ref_path("libreax_howu"))
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert ref.reax_howu_norm(P(dd["q"]), P(dd["k"]), P(dd["v"]), P(dd["beta"]), P(A), P(dd["g"]), P(theirs), P(dd["cu"]),
                              C.c_float(sc), C.c_int(2), C.c_int(H), C.c_int(HV), s, P(f2s), P(z),
                              C.c_longlong(HV * 128), P(nw), C.c_float(1e-6), C.c_float(1.0 / 128)) == 0
    torch.cuda.synchronize()
    o, t = synth.from_torch_bf16(ours), synth.from_torch_bf16(theirs)
    frac = float(np.mean(o == t))
    Ah = synth.from_torch_bf16(A)
    zs = np.ascontiguousarray(synth.from_torch_bf16(z[:TP]).reshape(TP, HV, 128)[:, :HV1].reshape(TP, -1))
    oracle = orc.howu(_prefix(d["q"], H1), _prefix(d["k"], H1), _prefix(d["v"], HV1), _prefix(d["beta"], HV1),
                      _prefix(Ah, HV1), _prefix(d["g"], HV1), np.array([0, TP], np.int64), sc, H1, HV1,
                      norm=dict(f2s=np.arange(TP, dtype=np.int32), z=zs, ZS=zs.shape[1], nw=synth.from_torch_bf16(nw),
                                eps=1e-6, factor=1.0 / 128, rows=TP))
    st = reference_matched_stats(bf(o[:TP, :HV1]), bf(oracle), bf(t[:TP, :HV1]))
    print(f"\nreax_howu_norm, {T} tokens x {HV} value heads: bitwise equal to the reference kernel on {frac:.6f} of "
          f"{o.size} outputs; vs oracle ({st['elements']} outputs): {st}")
    assert frac > 0.999
    assert st["within_tolerance"], st
