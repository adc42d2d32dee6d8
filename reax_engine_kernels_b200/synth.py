"""Seeded synthetic inputs shared by the tests, the benchmark and the oracle checks.

Element i of a stream with seed s is a function of (s, i) only:
    z_j  = splitmix64 output for counter j (state s + j * 0x9E3779B97F4A7C15)
    u1   = ((z_{2i} >> 11) + 1) * 2^-53,  u2 = (z_{2i+1} >> 11) * 2^-53
    n_i  = sqrt(-2 ln u1) * cos(2 pi u2)          (Box-Muller, one normal per pair)
and bf16 values are n_i * std + mean rounded to nearest even.  Any slice of a tensor can be regenerated
without the rest (the benchmark's CPU sample uses that).  Seeds follow 0x5EED0000 + config number.
"""
from __future__ import annotations

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)
SEED_BASE = 0x5EED0000


def _splitmix(seed: int, idx: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (idx.astype(np.uint64) + np.uint64(1)) * GOLDEN
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
        return z ^ (z >> np.uint64(31))


def normal(seed: int, n: int, start: int = 0, chunk: int = 1 << 22) -> np.ndarray:
    out = np.empty(n, np.float32)
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        i = np.arange(start + c0, start + c1, dtype=np.uint64)
        z1 = _splitmix(seed, 2 * i)
        z2 = _splitmix(seed, 2 * i + 1)
        u1 = ((z1 >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53
        u2 = (z2 >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
        out[c0:c1] = (np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)).astype(np.float32)
    return out


def uniform(seed: int, n: int, start: int = 0) -> np.ndarray:
    i = np.arange(start, start + n, dtype=np.uint64)
    return ((_splitmix(seed, i) >> np.uint64(11)).astype(np.float64) * 2.0 ** -53).astype(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def bf16_normal(seed: int, shape, std: float = 1.0, mean: float = 0.0, start: int = 0) -> np.ndarray:
    n = int(np.prod(shape))
    return f32_to_bf16_bits(normal(seed, n, start) * np.float32(std) + np.float32(mean)).reshape(shape)


def to_torch_bf16(bits: np.ndarray, device="cuda"):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
    return t.to(device) if device else t


def from_torch_bf16(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def gv_pack_g4(w_gate: np.ndarray, w_up: np.ndarray) -> np.ndarray:
    """[N2, K] gate and up weights (row n = output feature n) -> [2*N2, K] rows interleaved in groups of 4:
    rows 8j..8j+3 = gate 4j..4j+3, rows 8j+4..8j+7 = up 4j..4j+3 (the layout reax_gv consumes)."""
    N2, K = w_gate.shape
    assert N2 % 4 == 0 and w_up.shape == w_gate.shape
    out = np.empty((N2 // 4, 2, 4, K), w_gate.dtype)
    out[:, 0] = w_gate.reshape(N2 // 4, 4, K)
    out[:, 1] = w_up.reshape(N2 // 4, 4, K)
    return out.reshape(2 * N2, K)


def device_normal_bf16(shape, std: float = 1.0, seed: int = 0, device="cuda", mean: float = 0.0):
    """Large seeded inputs generated on the device (torch's Philox generator): used where the host generator
    above would dominate the run time (the benchmark's 224 MiB weights).  Host copies for the oracle are taken
    from the device tensor, so both sides still see identical bits."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    t = torch.randn(tuple(shape), generator=g, device=device, dtype=torch.float32)
    return (t * std + mean).to(torch.bfloat16)


def delta_rule_inputs(lengths, H, HV, seed, dk=128):
    """Seeded inputs of the linear-attention (gated delta rule) path for sequences of the given lengths:
    q, k [T, H, 128] bf16 (k unit-norm per head, as the conv + L2 stage produces), v [T, HV, 128] bf16,
    beta = sigmoid(N(0,1)) bf16 [T, HV], g [T, HV] fp32 = log2(e) * chunk-local cumsum over 64-token chunks of
    -softplus(N(0,1)) (the log2-domain decay the kernels consume), cu [N+1] int64, cidx [NT, 2] int64."""
    lengths = list(lengths)
    T = int(sum(lengths))
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    q = normal(seed, T * H * dk).reshape(T, H, dk)
    k = normal(seed + 1, T * H * dk).reshape(T, H, dk)
    k = k / np.sqrt((k.astype(np.float64) ** 2).sum(-1, keepdims=True)).astype(np.float32)
    q = q / np.sqrt((q.astype(np.float64) ** 2).sum(-1, keepdims=True)).astype(np.float32)
    v = normal(seed + 2, T * HV * dk).reshape(T, HV, dk)
    beta = 1.0 / (1.0 + np.exp(-normal(seed + 3, T * HV).reshape(T, HV).astype(np.float64)))
    x = normal(seed + 4, T * HV).reshape(T, HV).astype(np.float64)
    ls = -np.log1p(np.exp(x))  # -softplus
    g = np.zeros((T, HV), np.float64)
    cidx = []
    for n, L in enumerate(lengths):
        b = cu[n]
        for c0 in range(0, L, 64):
            c1 = min(L, c0 + 64)
            g[b + c0:b + c1] = np.cumsum(ls[b + c0:b + c1], axis=0)
            cidx.append((n, c0 // 64))
    g *= np.log2(np.e)
    return dict(q=f32_to_bf16_bits(q), k=f32_to_bf16_bits(k), v=f32_to_bf16_bits(v),
                beta=f32_to_bf16_bits(beta.astype(np.float32)), g=g.astype(np.float32), cu=cu,
                cidx=np.array(cidx, np.int64).reshape(-1, 2), T=T, H=H, HV=HV)
