"""ctypes binding of the five sm_100a libraries -- the same binding the REAX engine makes to the reference
libraries (``dlopen`` + symbol lookup by name, raw device pointers and ``cudaStream_t`` passed as integers).

Every prototype mirrors ``include/reax_abi.h`` (which cites the reference definition of each entry point).
Loading is strict: a missing or unloadable library raises ``ReaxLibraryError``; there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from .build import LIBRARIES, lib_path

c_int, c_float, c_ll, c_vp, c_char_p = C.c_int, C.c_float, C.c_longlong, C.c_void_p, C.c_char_p


class ReaxLibraryError(RuntimeError):
    pass


_FMHA_B = [c_vp, c_vp, c_vp, c_vp, c_vp, c_float, c_int, c_int, c_int, c_int] + [c_ll] * 15 + [c_vp]
_FMHA_Q = [c_vp, c_vp, c_vp, c_vp, c_int, c_ll, c_vp, c_float, c_int, c_int, c_int, c_int] + [c_ll] * 12 + [c_vp]
_FMHA_QP = ([c_vp, c_vp, c_vp, c_vp, c_int, c_ll, c_float, c_int, c_int, c_int, c_int] + [c_ll] * 9 +
            [c_vp, c_int, c_vp, c_ll, c_vp, c_ll, c_vp])
_HOWU = [c_vp] * 8 + [c_float, c_int, c_int, c_int, c_vp]

# name -> (restype, argtypes); per library
PROTOTYPES = {
    "libreax_gv": {
        "reax_gv_ncfg": (c_int, []),
        "reax_gv_cfgname": (c_char_p, [c_int]),
        "reax_gv": (c_int, [c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp]),
        "reax_gv_noalloc": (c_int, [c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp]),
        "reax_b200_status": (c_int, [c_vp]),
    },
    "libreax_plain": {
        "reax_gemm_ncfg": (c_int, []),
        "reax_gemm_cfgname": (c_char_p, [c_int]),
        "reax_gemm": (c_int, [c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp]),
        "reax_b200_status": (c_int, [c_vp]),
    },
    "libreax_slices": {
        "reax_slices_ncfg": (c_int, []),
        "reax_slices_cfgname": (c_char_p, [c_int]),
        "reax_slices": (c_int, [c_int, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp]),
        "reax_b200_status": (c_int, [c_vp]),
    },
    "libreax_howu": {
        "howu3_dense": (c_int, _HOWU),
        "howu3_skip": (c_int, _HOWU),
        "howu3_smem": (c_int, []),
        "reax_howu": (c_int, _HOWU),
        "reax_kkt": (c_int, [c_vp] * 6 + [c_int, c_int, c_int, c_vp]),
        "reax_kkt_smem": (c_int, []),
        "reax_howu_norm": (c_int, [c_vp] * 8 + [c_float, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_ll, c_vp, c_float,
                                                  c_float]),
        "reax_rarn": (c_int, [c_vp, c_int, c_int, c_ll, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_float, c_float, c_vp]),
        "reax_conv_l2": (c_int, [c_vp, c_ll, c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_float, c_int, c_int,
                                 c_int, c_int, c_int, c_vp]),
        "reax_conv_v": (c_int, [c_vp, c_ll, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp]),
        "reax_fmha_b": (c_int, _FMHA_B),
        "reax_fmha_q": (c_int, _FMHA_Q),
        "reax_fmha_q_hd": (c_int, _FMHA_Q[:-1] + [c_int, c_vp]),
        "reax_fmha_b_hd": (c_int, _FMHA_B[:-1] + [c_int, c_vp]),
        "reax_b200_status": (c_int, [c_vp]),
    },
    "libreax_fmha_post": {
        "reax_fmha_b": (c_int, _FMHA_B),
        "reax_fmha_q": (c_int, _FMHA_Q),
        "reax_fmha_qp": (c_int, _FMHA_QP),
        "reax_fmha_q_hd": (c_int, _FMHA_Q[:-1] + [c_int, c_vp]),
        "reax_fmha_b_hd": (c_int, _FMHA_B[:-1] + [c_int, c_vp]),
        "reax_b200_status": (c_int, [c_vp]),
    },
}

_lock = threading.Lock()
_loaded: dict[str, C.CDLL] = {}


def load(name: str) -> C.CDLL:
    """dlopen one library (RTLD_LOCAL, like the engine) and bind every prototype; raise if anything is missing."""
    if name not in LIBRARIES:
        raise ReaxLibraryError(f"unknown library {name}")
    with _lock:
        if name in _loaded:
            return _loaded[name]
        path = lib_path(name)
        if not os.path.exists(path):
            raise ReaxLibraryError(f"{path} is not built (run `python -m reax_engine_kernels_b200.build`)")
        try:
            lib = C.CDLL(path, mode=os.RTLD_LOCAL | os.RTLD_NOW)
        except OSError as e:
            raise ReaxLibraryError(f"cannot load {path}: {e}") from e
        for fn, (res, args) in PROTOTYPES[name].items():
            try:
                f = getattr(lib, fn)
            except AttributeError as e:
                raise ReaxLibraryError(f"{path} does not export {fn}") from e
            f.restype, f.argtypes = res, args
        _loaded[name] = lib
        return lib


def exported_symbols(path: str) -> set[str]:
    """Dynamic text symbols of a shared library (nm -D), used by the symbol-set test."""
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if len(ln.split()) == 3 and ln.split()[1] == "T"}
