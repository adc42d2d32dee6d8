"""One small, seeded invocation of a kernel of this package, for profilers (ncu) and quick timing.

    python profile_cases.py CASE [--launches N]      (CASE: see CASES at the end)

Each case builds its inputs on the device, launches the kernel N times (default 3) through the package's C-ABI front
end and synchronises.  The shapes are sized for a profiler: inputs larger than the 126 MB L2 where the kernel streams
memory, a few GB on the device at most, and kernels of well under a second.
"""
from __future__ import annotations

import argparse
import math
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import numpy as np
import torch

from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import synth


def case_gv(n):
    # BASELINE config 2 at a quarter of the output width: X [2048, 4096], w_g4 [2 * 3584, 4096]
    M, K, N2 = 2048, 4096, 3584
    x = synth.device_normal_bf16((M, K), 1.0, 1)
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 2)
    out = torch.empty(M, N2, dtype=torch.bfloat16, device="cuda")
    for _ in range(n):
        rk.gv(x, w, cfg=0, out=out)


def _gv_case(n, N2):
    M, K = 2048, 4096
    x = synth.device_normal_bf16((M, K), 1.0, 1)
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 2)
    out = torch.empty(M, N2, dtype=torch.bfloat16, device="cuda")
    for _ in range(n):
        rk.gv(x, w, cfg=0, out=out)


def case_gv_config2(n):
    # BASELINE config 2 itself: X [2048, 4096], w_g4 [2 * 14336, 4096] (0.3 GB on the device)
    _gv_case(n, 14336)


def case_gv_shard8(n):
    # one rank's shard of config 2 split over 8 GPUs: N2 = 1792, 224 tiles = 1.51 waves -> the split-last-waves kernel
    _gv_case(n, 1792)


def case_slices_m16(n):
    # BASELINE config 4 at its smallest M: X [16, 4096], W [4096, 4096], 4 slices of 1024, fp32 partials
    M, K, N, S = 16, 4096, 4096, 4
    x = synth.device_normal_bf16((M, K), 1.0, 1)
    w = synth.device_normal_bf16((N, K), 0.02, 2)
    out = torch.empty(S, M, N, dtype=torch.float32, device="cuda")
    for _ in range(n):
        rk.slices(x, w, S, K // S, True, cfg=1, out=out)


def case_attention(n):
    # causal GQA prefill, one batch: 8 kv heads x 4 query rows per position, 4096 positions, head dim 128
    B, H, G, S, D = 1, 8, 4, 4096, 128
    M = S * G
    q = synth.device_normal_bf16((B, H, M, D), 1.0, 1)
    k = synth.device_normal_bf16((B, H, S, D), 1.0, 2)
    v = synth.device_normal_bf16((B, H, S, D), 1.0, 3)
    qpos = torch.arange(S, dtype=torch.int32, device="cuda").view(1, S)
    o = torch.empty_like(q)
    for _ in range(n):
        rk.fmha(q, k, v, 1 / math.sqrt(D), qpos=qpos, G=G, out=o)


def case_conv(n):
    # the config-5 channel layout (q/k/v 3 x 2048 channels) over one 8192-token sequence
    T, KD, VD, SX = 8192, 2048, 2048, 6144
    qkv = synth.device_normal_bf16((T, SX), 1.0, 4)
    cw = synth.device_normal_bf16((SX, 4), 0.5, 5)
    meta = torch.from_numpy(np.array([(p, 0, 0, 0) for p in range(T)], np.int32)).cuda()
    q = torch.empty(T, KD, dtype=torch.bfloat16, device="cuda")
    k = torch.empty_like(q)
    v = torch.empty(T, VD, dtype=torch.bfloat16, device="cuda")
    for _ in range(n):
        rk.conv_l2(qkv, meta, cw, KD, VD, q=q, k=k, v=v)


def _delta_inputs():
    d = synth.delta_rule_inputs([8192, 8192], 16, 32, 7)
    t = {n: synth.to_torch_bf16(d[n]) for n in ("q", "k", "beta")}
    t.update({n: torch.from_numpy(d[n]).cuda() for n in ("g", "cu", "cidx")})
    return d, t


def case_kkt(n):
    # config-5 heads (16 key / 32 value heads) over 2 x 8192 tokens
    d, t = _delta_inputs()
    A = torch.zeros(d["T"], 32, 64, dtype=torch.bfloat16, device="cuda")
    for _ in range(n):
        rk.kkt(t["k"], t["g"], t["beta"], t["cu"], t["cidx"], 32, A=A)


def case_delta_rule(n):
    d, t = _delta_inputs()
    A = torch.zeros(d["T"], 32, 64, dtype=torch.bfloat16, device="cuda")
    rk.kkt(t["k"], t["g"], t["beta"], t["cu"], t["cidx"], 32, A=A)
    v = synth.device_normal_bf16((d["T"], 32, 128), 1.0, 8)
    o = torch.empty_like(v)
    for _ in range(n):
        rk.howu(t["q"], t["k"], v, t["beta"], A, t["g"], t["cu"], 1 / math.sqrt(128), o=o)


def case_rarn(n):
    # residual add of two partial sums + RMSNorm over hidden 2048, 32768 rows
    rows, D, S = 32768, 2048, 2
    part = synth.device_normal_bf16((S, rows, D), 0.5, 1)
    res = synth.device_normal_bf16((rows, D), 1.0, 2)
    w = synth.device_normal_bf16((D,), 0.1, 3, mean=1.0)
    h = torch.empty(rows, D, dtype=torch.bfloat16, device="cuda")
    o = torch.empty_like(h)
    for _ in range(n):
        rk.rarn(part, res, w, 1e-6, 1.0 / D, h_out=h, out=o)


def case_gemm_qkv(n):
    # the linear-attention layer's qkv projection (plain GEMM) at a quarter of config 5's tokens: X [8192, 2048],
    # W [6144, 2048]
    M, K, N = 8192, 2048, 6144
    x = synth.device_normal_bf16((M, K), 1.0, 1)
    w = synth.device_normal_bf16((N, K), 0.02, 2)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    for _ in range(n):
        rk.gemm(x, w, cfg=0, out=out)


def case_slices_m16_bf16(n):
    # BASELINE config 4's smallest M with its bf16 partials (the swapped small-M kernel, transposed bf16 epilogue)
    M, K, N, S = 16, 4096, 4096, 4
    x = synth.device_normal_bf16((M, K), 1.0, 1)
    w = synth.device_normal_bf16((N, K), 0.02, 2)
    out = torch.empty(S, M, N, dtype=torch.bfloat16, device="cuda")
    for _ in range(n):
        rk.slices(x, w, S, K // S, False, cfg=0, out=out)


def case_slices_m4096(n):
    # BASELINE config 4's largest M with bf16 partials: X [4096, 4096], W [4096, 4096], 4 slices of 1024 (cfg 0,
    # 256-wide tiles: 2048 tiles of 16 k-blocks each)
    M, K, N, S = 4096, 4096, 4096, 4
    x = synth.device_normal_bf16((M, K), 1.0, 1)
    w = synth.device_normal_bf16((N, K), 0.02, 2)
    out = torch.empty(S, M, N, dtype=torch.bfloat16, device="cuda")
    for _ in range(n):
        rk.slices(x, w, S, K // S, False, cfg=0, out=out)


def case_attention_d256(n):
    # the reference's head dim (256): causal GQA, one batch, 4 kv heads x 4 query rows, 2048 positions
    B, H, G, S, D = 1, 4, 4, 2048, 256
    M = S * G
    q = synth.device_normal_bf16((B, H, M, D), 1.0, 1)
    k = synth.device_normal_bf16((B, H, S, D), 1.0, 2)
    v = synth.device_normal_bf16((B, H, S, D), 1.0, 3)
    qpos = torch.arange(S, dtype=torch.int32, device="cuda").view(1, S)
    o = torch.empty_like(q)
    for _ in range(n):
        rk.fmha(q, k, v, 1 / math.sqrt(D), qpos=qpos, G=G, out=o)


def case_attention_post(n):
    # reax_fmha_qp: the same head-dim-256 attention with the sigmoid-gate scatter epilogue (every row written)
    B, H, G, S, D = 1, 4, 4, 2048, 256
    M = S * G
    q = synth.device_normal_bf16((B, H, M, D), 1.0, 1)
    k = synth.device_normal_bf16((B, H, S, D), 1.0, 2)
    v = synth.device_normal_bf16((B, H, S, D), 1.0, 3)
    qpos = torch.arange(S, dtype=torch.int32, device="cuda").view(1, S)
    inv = torch.arange(S, dtype=torch.int32, device="cuda").view(1, S)
    qg = synth.device_normal_bf16((S, H * G * 2 * D), 1.0, 4)
    outp = torch.empty(S, H * G * D, dtype=torch.bfloat16, device="cuda")
    for _ in range(n):
        rk.fmha_qp(q, k, v, 1 / math.sqrt(D), qpos, G, inv, qg, outp)


def case_attention_config1(n):
    # causal MHA, B=1, S=1024, 8 heads, D=128 (the one-tile kernel: 64 CTAs)
    B, H, S, D = 1, 8, 1024, 128
    q = synth.device_normal_bf16((B, H, S, D), 1.0, 1)
    k = synth.device_normal_bf16((B, H, S, D), 1.0, 2)
    v = synth.device_normal_bf16((B, H, S, D), 1.0, 3)
    qpos = torch.arange(S, dtype=torch.int32, device="cuda").view(1, S)
    o = torch.empty_like(q)
    for _ in range(n):
        rk.fmha(q, k, v, 1 / math.sqrt(D), qpos=qpos, G=1, out=o)


def case_conv_v(n):
    # reax_conv_v: the v channels only (conv + SiLU, no norm), config-5 channel layout over 8192 tokens
    T, KD, VD, SX = 8192, 2048, 2048, 6144
    qkv = synth.device_normal_bf16((T, SX), 1.0, 4)
    cw = synth.device_normal_bf16((SX, 4), 0.5, 5)
    meta = torch.from_numpy(np.array([(p, 0, 0, 0) for p in range(T)], np.int32)).cuda()
    v = torch.empty(T, VD, dtype=torch.bfloat16, device="cuda")
    for _ in range(n):
        rk.conv_v(qkv, meta, cw, KD, VD, v=v)


def case_delta_rule_norm(n):
    # reax_howu_norm (the delta rule, then the in-place gated RMSNorm pass howu_gnorm_kernel), 2 x 8192 tokens
    d, t = _delta_inputs()
    T = d["T"]
    A = torch.zeros(T, 32, 64, dtype=torch.bfloat16, device="cuda")
    rk.kkt(t["k"], t["g"], t["beta"], t["cu"], t["cidx"], 32, A=A)
    v = synth.device_normal_bf16((T, 32, 128), 1.0, 8)
    f2s = torch.arange(T, dtype=torch.int32, device="cuda")
    z = synth.device_normal_bf16((T, 32 * 128), 1.0, 9)
    nw = synth.device_normal_bf16((128,), 0.1, 10, mean=1.0)
    out = torch.empty(T, 32, 128, dtype=torch.bfloat16, device="cuda")
    for _ in range(n):
        rk.howu_norm(t["q"], t["k"], v, t["beta"], A, t["g"], t["cu"], 1 / math.sqrt(128), f2s, z, nw, 1e-6, 1.0 / 128,
                     out)


CASES = {"gv": case_gv, "gv_config2": case_gv_config2, "gv_shard8": case_gv_shard8, "slices_m16": case_slices_m16, "slices_m16_bf16": case_slices_m16_bf16, "slices_m4096": case_slices_m4096,
         "gemm_qkv": case_gemm_qkv, "attention": case_attention, "attention_d256": case_attention_d256,
         "attention_post": case_attention_post, "attention_config1": case_attention_config1, "conv": case_conv,
         "conv_v": case_conv_v, "kkt": case_kkt, "rarn": case_rarn, "delta_rule": case_delta_rule,
         "delta_rule_norm": case_delta_rule_norm}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--launches", type=int, default=3)
    a = ap.parse_args()
    CASES[a.case](a.launches)
    torch.cuda.synchronize()
    print("ok", a.case)


if __name__ == "__main__":
    main()
