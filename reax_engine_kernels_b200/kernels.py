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
