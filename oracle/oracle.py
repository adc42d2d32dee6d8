"""ctypes wrapper of the fp64 CPU oracle (TEST INFRASTRUCTURE: used only by tests/, __graft_entry__.smoke() and
the CPU-baseline leg of bench.py, always as the checker).  Arrays are numpy; bf16 is carried as uint16 bits."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .build import build_oracle, oracle_path

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = oracle_path()
        if not os.path.exists(path):
            build_oracle()
        _lib = C.CDLL(path)
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def set_threads(n: int):
    lib().oracle_set_threads(C.c_int(n))


def threads() -> int:
    return lib().oracle_threads()


def _u16(a):
    a = np.ascontiguousarray(a)
    assert a.dtype == np.uint16, a.dtype
    return a


def gv(x, w, band=2.0 ** -19, rows=None, intervals=True):
    """-> (out, lo, hi) uint16 [M, N2]; rows=(m0, m1) restricts the computation (other rows stay 0);
    intervals=False skips the rounding-interval outputs (lo, hi returned as None)."""
    x, w = _u16(x), _u16(w)
    M, K = x.shape
    N2 = w.shape[0] // 2
    m0, m1 = rows if rows else (0, M)
    out = np.zeros((M, N2), np.uint16)
    lo = np.zeros_like(out)
    hi = np.zeros_like(out)
    f = lib().oracle_gv_rows
    f.argtypes = [C.c_void_p] * 5 + [C.c_int] * 5 + [C.c_double]
    if not intervals:
        lo = hi = None
    f(_p(x), _p(w), _p(out), _p(lo), _p(hi), M, N2, K, m0, m1, band)
    return out, lo, hi


def gemm(x, w, ldd=None):
    x, w = _u16(x), _u16(w)
    M, K = x.shape
    N = w.shape[0]
    ldd = ldd or N
    d = np.zeros((M, ldd), np.uint16)
    f = lib().oracle_gemm
    f.argtypes = [C.c_void_p] * 3 + [C.c_int] * 4
    f(_p(x), _p(w), _p(d), M, N, K, ldd)
    return d


def slices(x, w, S, kps, part_fp32=True):
    x, w = _u16(x), _u16(w)
    M, K = x.shape
    N = w.shape[0]
    p = np.zeros((S, M, N), np.float32 if part_fp32 else np.uint16)
    f = lib().oracle_slices
    f.argtypes = [C.c_int] + [C.c_void_p] * 3 + [C.c_int] * 5
    f(int(part_fp32), _p(x), _p(w), _p(p), M, N, kps, S, K)
    return p


def fmha(q, k, v, scale, *, qpos=None, G=1, qpBs=0, bias=None, post=None, rows=None, intervals=False, band=2.0 ** -19):
    """q [B, H, M, D], k/v [B, H, N, D], bias [B, H, M, N] (uint16 bf16 bits, contiguous).
    qpos mode when qpos is given (int32 [B, qpBs-strided]); post = dict(inv, Lq, qg, qg_rs, outp, out_rs) fuses
    the sigmoid-gate scatter and writes into post['outp'] (uint16, modified in place).  Returns O [B, H, M, D], or
    (O, lo, hi) with intervals=True (for post, lo/hi have outp's layout and untouched entries equal outp's)."""
    q, k, v = _u16(q), _u16(k), _u16(v)
    B, H, M, D = q.shape
    N = k.shape[2]
    o = np.zeros((B, H, M, D), np.uint16)
    mode = 1 if qpos is not None else 0
    if bias is not None:
        bias = _u16(bias)
    if qpos is not None:
        qpos = np.ascontiguousarray(qpos, np.int32)
    r0, r1 = rows if rows else (0, M)
    f = lib().oracle_fmha
    f.argtypes = ([C.c_int, C.c_int] + [C.c_void_p] * 5 + [C.c_int, C.c_longlong, C.c_void_p, C.c_float] +
                  [C.c_int] * 4 + [C.c_longlong] * 15 + [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_longlong,
                                                          C.c_void_p, C.c_longlong, C.c_int, C.c_int, C.c_void_p,
                                                          C.c_void_p, C.c_double])
    qs = (H * M * D, M * D, D)
    ks = (H * N * D, N * D, D)
    bs = (H * M * N, M * N, N) if bias is not None else (0, 0, 0)
    if post is None:
        lo = np.zeros_like(o) if intervals else None
        hi = np.zeros_like(o) if intervals else None
        f(mode, D, _p(q), _p(k), _p(v), _p(bias), _p(qpos), G, qpBs, _p(o), scale, B, H, M, N, *qs, *ks, *ks, *bs,
          *qs, 0, None, 0, None, 0, None, 0, r0, r1, _p(lo), _p(hi), band)
    else:
        outp = post["outp"]
        lo = outp.copy() if intervals else None
        hi = outp.copy() if intervals else None
        inv = np.ascontiguousarray(post["inv"], np.int32)
        f(mode, D, _p(q), _p(k), _p(v), _p(bias), _p(qpos), G, qpBs, _p(o), scale, B, H, M, N, *qs, *ks, *ks, *bs,
          *qs, 1, _p(inv), post["Lq"], _p(_u16(post["qg"])), post["qg_rs"], _p(outp), post["out_rs"], r0, r1, _p(lo),
          _p(hi), band)
    return (o, lo, hi) if intervals else o


def rarn(part, S, serial, pstride, res, w, n, D, eps, factor):
    part, res, w = _u16(part), _u16(res), _u16(w)
    h_out = np.zeros((n, D), np.uint16)
    out = np.zeros((n, D), np.uint16)
    f = lib().oracle_rarn
    f.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_longlong] + [C.c_void_p] * 4 + [C.c_int, C.c_int, C.c_float, C.c_float]
    f(_p(part), S, serial, pstride, _p(res), _p(w), _p(h_out), _p(out), n, D, eps, factor)
    return h_out, out


def conv(qkv, SX, cache, C_, meta, w, Tf, eps, KD, VD, rep, skip_v, units=None, q=None, k=None, v=None):
    """Returns (q, k, v) uint16 arrays (given arrays are written in place; unwritten elements keep their value)."""
    qkv, w = _u16(qkv), _u16(w)
    meta = np.ascontiguousarray(meta, np.int32)
    q = np.zeros((Tf, rep * KD), np.uint16) if q is None else q
    k = np.zeros((Tf, rep * KD), np.uint16) if k is None else k
    v = np.zeros((Tf, VD), np.uint16) if v is None else v
    lo, hi = units if units else (0, 2 * KD // 128 + VD // 128)
    f = lib().oracle_conv
    f.argtypes = [C.c_void_p, C.c_longlong, C.c_void_p, C.c_int] + [C.c_void_p] * 5 + [C.c_int, C.c_float] + [C.c_int] * 6
    f(_p(qkv), SX, _p(cache), C_, _p(meta), _p(w), _p(q), _p(k), _p(v), Tf, eps, KD, VD, rep, skip_v, lo, hi)
    return q, k, v


def kkt(k, g, beta, cu, cidx, H, HV, A=None):
    k, beta = _u16(k), _u16(beta)
    g = np.ascontiguousarray(g, np.float32)
    cu = np.ascontiguousarray(cu, np.int64)
    cidx = np.ascontiguousarray(cidx, np.int64)
    T = k.shape[0]
    A = np.zeros((T, HV, 64), np.uint16) if A is None else A
    f = lib().oracle_kkt
    f.argtypes = [C.c_void_p] * 6 + [C.c_int] * 3
    f(_p(k), _p(g), _p(beta), _p(A), _p(cu), _p(cidx), cidx.shape[0], H, HV)
    return A


def howu(q, k, v, beta, A, g, cu, scale, H, HV, dense=False, norm=None, out=None):
    """norm = dict(f2s, z, ZS, nw, eps, factor, rows) for the gated-RMSNorm variant (out [rows, HV, 128])."""
    q, k, v, beta, A = _u16(q), _u16(k), _u16(v), _u16(beta), _u16(A)
    g = np.ascontiguousarray(g, np.float32)
    cu = np.ascontiguousarray(cu, np.int64)
    N = cu.shape[0] - 1
    T = q.shape[0]
    f = lib().oracle_howu
    f.argtypes = ([C.c_void_p] * 6 + [C.c_void_p, C.c_void_p, C.c_float, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p, C.c_float, C.c_float])
    if norm is None:
        o = np.zeros((T, HV, 128), np.uint16) if out is None else out
        f(_p(q), _p(k), _p(v), _p(beta), _p(A), _p(g), _p(o), _p(cu), scale, N, H, HV, int(dense), 0, None, None, 0,
          None, 0.0, 0.0)
        return o
    f2s = np.ascontiguousarray(norm["f2s"], np.int32)
    z, nw = _u16(norm["z"]), _u16(norm["nw"])
    o = np.zeros((norm["rows"], HV, 128), np.uint16) if out is None else out
    f(_p(q), _p(k), _p(v), _p(beta), _p(A), _p(g), _p(o), _p(cu), scale, N, H, HV, int(dense), 1, _p(f2s), _p(z),
      norm["ZS"], _p(nw), norm["eps"], norm["factor"])
    return o
