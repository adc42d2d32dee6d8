"""Torch-tensor front end over the C ABI (the call a Python user of the libraries makes).

Each function validates shapes on the host, takes raw device pointers from the tensors, passes torch's
current CUDA stream, calls the library entry point by name and raises ``ReaxCallError`` on a nonzero
return code.  Nothing here computes on the CPU: without the built libraries every call raises.
"""
from __future__ import annotations

import torch

from . import abi


class ReaxCallError(RuntimeError):
    pass


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(dev=None):
    return torch.cuda.current_stream(dev).cuda_stream


def _check(rc, fn):
    if rc != 0:
        raise ReaxCallError(f"{fn} returned {rc}")


def _dev(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("all tensors must be CUDA tensors")


# ------------------------------------------------------------------ GEMM family
def gv(x: torch.Tensor, w_g4: torch.Tensor, cfg: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """Gate/up GEMM + SiLU*mul.  x [M, K] bf16, w_g4 [2*N2, K] bf16 (groups of 4 gate rows then 4 up rows)."""
    _dev(x, w_g4)
    M, K = x.shape
    N2 = w_g4.shape[0] // 2
    if out is None:
        out = torch.empty(M, N2, dtype=torch.bfloat16, device=x.device)
    lib = abi.load("libreax_gv")
    _check(lib.reax_gv(cfg, _ptr(x), _ptr(w_g4), _ptr(out), M, N2, K, _stream(x.device)), "reax_gv")
    return out


def gemm(x: torch.Tensor, w: torch.Tensor, cfg: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """D = X W^T, bf16 out.  ``out`` may be a column slice of a wider row-major buffer (ldd = out.stride(0))."""
    _dev(x, w)
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    ldd = out.stride(0)
    lib = abi.load("libreax_plain")
    _check(lib.reax_gemm(cfg, _ptr(x), _ptr(w), _ptr(out), M, N, K, ldd, _stream(x.device)), "reax_gemm")
    return out


def slices(x: torch.Tensor, w: torch.Tensor, S: int, kps: int, part_fp32: bool = True, cfg: int = 0,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """P[s] = X[:, s*kps:(s+1)*kps] W[:, s*kps:(s+1)*kps]^T -> [S, M, N] fp32 or bf16."""
    _dev(x, w)
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(S, M, N, dtype=torch.float32 if part_fp32 else torch.bfloat16, device=x.device)
    lib = abi.load("libreax_slices")
    _check(lib.reax_slices(cfg, int(part_fp32), _ptr(x), _ptr(w), _ptr(out), M, N, kps, S, K, _stream(x.device)),
           "reax_slices")
    return out


def cfg_names(library: str) -> list[str]:
    lib = abi.load(library)
    stem = {"libreax_gv": "reax_gv", "libreax_plain": "reax_gemm", "libreax_slices": "reax_slices"}[library]
    n = getattr(lib, stem + "_ncfg")()
    return [getattr(lib, stem + "_cfgname")(i).decode() for i in range(n)]


def status(library: str) -> int:
    """Read and clear the library's device status word (nonzero = a bounded wait ran out)."""
    return abi.load(library).reax_b200_status(_stream())


# ------------------------------------------------------------------ attention
def _s3(t):
    return t.stride(0), t.stride(1), t.stride(2)


def _last_dim_contiguous(**ts):
    """The attention entry points take strides for the first three dims only: every operand's last dim must be dense."""
    for name, t in ts.items():
        if t is not None and t.dim() > 0 and t.shape[-1] > 1 and t.stride(-1) != 1:
            raise ValueError(f"{name}: the last dimension must be contiguous (stride {t.stride(-1)})")


def _check_qpos(qpos, device):
    if qpos is None:
        raise ValueError("qpos mode needs a qpos tensor")
    if qpos.dtype != torch.int32:
        raise ValueError(f"qpos must be int32, got {qpos.dtype}")
    if qpos.device != device:
        raise ValueError(f"qpos is on {qpos.device}, the operands on {device}")


def fmha(q, k, v, scale: float, *, qpos=None, G: int = 1, qpBs: int | None = None, bias=None, out=None,
         library: str = "libreax_fmha_post"):
    """q [B, H, M, D], k/v [B, H, N, D] (bf16, last dim contiguous, any other strides), D in {128, 256}.
    qpos mode (qpos int32 [B, *], row r of batch b sees keys <= qpos[b*qpBs + r/G]) or bias mode (bias [B, H, M, N])."""
    _dev(q, k, v, qpos, bias)
    B, H, M, D = q.shape
    N = k.shape[2]
    if out is None:
        out = torch.empty(B, H, M, D, dtype=torch.bfloat16, device=q.device)
    _last_dim_contiguous(q=q, k=k, v=v, out=out, bias=bias)
    if bias is None:
        _check_qpos(qpos, q.device)
    lib = abi.load(library)
    st = _stream(q.device)
    if qpos is not None:
        qpBs = qpos.stride(0) if qpBs is None else qpBs
        rc = lib.reax_fmha_q_hd(_ptr(q), _ptr(k), _ptr(v), _ptr(qpos), G, qpBs, _ptr(out), scale, B, H, M, N, *_s3(q),
                                *_s3(k), *_s3(v), *_s3(out), D, st)
        _check(rc, "reax_fmha_q_hd")
    else:
        rc = lib.reax_fmha_b_hd(_ptr(q), _ptr(k), _ptr(v), _ptr(bias), _ptr(out), scale, B, H, M, N, *_s3(q), *_s3(k),
                                *_s3(v), *_s3(bias), *_s3(out), D, st)
        _check(rc, "reax_fmha_b_hd")
    return out


def fmha_qp(q, k, v, scale: float, qpos, G: int, inv, qg, outp, qpBs: int | None = None):
    """qpos-mode attention (head dim 256) with the fused attn_post epilogue: for row r of (b, h), R = inv[b*Lq + r/G];
    outp[R, (h*G + r%G)*256 : +256] = bf16(bf16(O) * bf16(sigmoid(qg[R, (h*G + r%G)*512 + 256 : +256]))), R < 0 skipped.
    inv int32 [B, Lq]; qg [rows, Hq*512]; outp [rows, Hq*256]."""
    _dev(q, k, v, qpos, inv, qg, outp)
    B, H, M, D = q.shape
    assert D == 256, "reax_fmha_qp has head dim 256"
    _last_dim_contiguous(q=q, k=k, v=v, qg=qg, outp=outp)
    _check_qpos(qpos, q.device)
    if inv.dtype != torch.int32 or inv.device != q.device:
        raise ValueError("inv must be an int32 tensor on the operands' device")
    N = k.shape[2]
    qpBs = qpos.stride(0) if qpBs is None else qpBs
    lib = abi.load("libreax_fmha_post")
    rc = lib.reax_fmha_qp(_ptr(q), _ptr(k), _ptr(v), _ptr(qpos), G, qpBs, scale, B, H, M, N, *_s3(q), *_s3(k), *_s3(v),
                          _ptr(inv), inv.shape[1], _ptr(qg), qg.stride(0), _ptr(outp), outp.stride(0), _stream(q.device))
    _check(rc, "reax_fmha_qp")
    return outp


# ------------------------------------------------------------------ linear-attention layer (libreax_howu)
def rarn(part, res, w, eps: float, factor: float, serial: bool = False, h_out=None, out=None):
    """part [S, n, D] bf16 (partial stride = part.stride(0)), res [n, D], w [D] -> (h_out, out)."""
    _dev(part, res, w)
    S, n, D = part.shape
    h_out = torch.empty(n, D, dtype=torch.bfloat16, device=res.device) if h_out is None else h_out
    out = torch.empty(n, D, dtype=torch.bfloat16, device=res.device) if out is None else out
    rc = abi.load("libreax_howu").reax_rarn(_ptr(part), S, int(serial), part.stride(0), _ptr(res), _ptr(w), _ptr(h_out),
                                            _ptr(out), n, D, eps, factor, _stream(res.device))
    _check(rc, "reax_rarn")
    return h_out, out


def conv_l2(qkv, meta, w, KD: int, VD: int, eps: float = 1e-6, rep: int = 1, skip_v: bool = False, cache=None,
            RT: int = 16, q=None, k=None, v=None):
    """qkv [T, SX] bf16, meta [T, 4] int32 (pos, y, z, w), w [channels, 4] bf16 -> (q, k, v)."""
    _dev(qkv, meta, w, cache)
    T = meta.shape[0]
    dev = qkv.device
    q = torch.empty(T, rep * KD, dtype=torch.bfloat16, device=dev) if q is None else q
    k = torch.empty(T, rep * KD, dtype=torch.bfloat16, device=dev) if k is None else k
    v = torch.empty(T, VD, dtype=torch.bfloat16, device=dev) if v is None else v
    C = cache.stride(0) if cache is not None else 0
    rc = abi.load("libreax_howu").reax_conv_l2(_ptr(qkv), qkv.stride(0), _ptr(cache), C, _ptr(meta), _ptr(w), _ptr(q),
                                               _ptr(k), _ptr(v), T, eps, KD, VD, rep, int(skip_v), RT, _stream(dev))
    _check(rc, "reax_conv_l2")
    return q, k, v


def conv_v(qkv, meta, w, KD: int, VD: int, cache=None, v=None):
    _dev(qkv, meta, w, cache)
    T = meta.shape[0]
    v = torch.empty(T, VD, dtype=torch.bfloat16, device=qkv.device) if v is None else v
    C = cache.stride(0) if cache is not None else 0
    rc = abi.load("libreax_howu").reax_conv_v(_ptr(qkv), qkv.stride(0), _ptr(cache), C, _ptr(meta), _ptr(w), _ptr(v), T,
                                              KD, VD, _stream(qkv.device))
    _check(rc, "reax_conv_v")
    return v


def kkt(k, g, beta, cu, cidx, HV: int, A=None):
    """k [T, H, 128] bf16, g [T, HV] fp32, beta [T, HV] bf16, cu [N+1] int64, cidx [NT, 2] int64 -> A [T, HV, 64]
    (only rows < chunk length and 16x16 blocks on/below the diagonal are written; a new A starts zeroed)."""
    _dev(k, g, beta, cu, cidx)
    T, H, _ = k.shape
    A = torch.zeros(T, HV, 64, dtype=torch.bfloat16, device=k.device) if A is None else A
    rc = abi.load("libreax_howu").reax_kkt(_ptr(k), _ptr(g), _ptr(beta), _ptr(A), _ptr(cu), _ptr(cidx), cidx.shape[0], H,
                                           HV, _stream(k.device))
    _check(rc, "reax_kkt")
    return A


def howu(q, k, v, beta, A, g, cu, scale: float, entry: str = "reax_howu", o=None):
    """Chunked gated delta rule output o [T, HV, 128]; entry in {reax_howu, howu3_skip, howu3_dense}."""
    _dev(q, k, v, beta, A, g, cu)
    T, H, _ = q.shape
    HV = v.shape[1]
    o = torch.empty(T, HV, 128, dtype=torch.bfloat16, device=q.device) if o is None else o
    fn = getattr(abi.load("libreax_howu"), entry)
    rc = fn(_ptr(q), _ptr(k), _ptr(v), _ptr(beta), _ptr(A), _ptr(g), _ptr(o), _ptr(cu), scale, cu.shape[0] - 1, H, HV,
            _stream(q.device))
    _check(rc, entry)
    return o


def howu_norm(q, k, v, beta, A, g, cu, scale: float, f2s, z, nw, eps: float, factor: float, out):
    """reax_howu + gated RMSNorm: out[f2s[t], hv] (rows with f2s < 0 untouched); z [rows, ZS] with ZS = z.stride(0)."""
    _dev(q, k, v, beta, A, g, cu, f2s, z, nw, out)
    T, H, _ = q.shape
    HV = v.shape[1]
    rc = abi.load("libreax_howu").reax_howu_norm(_ptr(q), _ptr(k), _ptr(v), _ptr(beta), _ptr(A), _ptr(g), _ptr(out),
                                                 _ptr(cu), scale, cu.shape[0] - 1, H, HV, _stream(q.device), _ptr(f2s),
                                                 _ptr(z), z.stride(0), _ptr(nw), eps, factor)
    _check(rc, "reax_howu_norm")
    return out
