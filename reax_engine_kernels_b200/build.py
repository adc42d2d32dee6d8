"""In-tree build of the five sm_100a kernel libraries (and the test oracle).

Each library is one nvcc translation unit compiled with ``-gencode arch=compute_100a,code=sm_100a`` into
``reax_engine_kernels_b200/lib/`` so the built ``.so`` files travel with the source tree.  Builds are
incremental (a library is rebuilt when any of its sources or headers is newer than the ``.so``) and run
in parallel.

    python -m reax_engine_kernels_b200.build          # libraries only
    python -m reax_engine_kernels_b200.build --all    # + oracle (and oracle/_ref when the reference is present)
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-diag-suppress", "177"]

# library -> translation unit
LIBRARIES = {
    "libreax_gv": "gv.cu",
    "libreax_plain": "plain.cu",
    "libreax_slices": "slices.cu",
    "libreax_howu": "howu_lib.cu",
    "libreax_fmha_post": "fmha_post_lib.cu",
}


def lib_path(name: str) -> str:
    return os.path.join(LIBDIR, name + ".so")


def _newest(paths) -> float:
    return max((os.path.getmtime(p) for p in paths if os.path.exists(p)), default=0.0)


def _deps(tu: str):
    return [os.path.join(CSRC, tu)] + glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(ROOT, "include", "reax_abi.h")]


def _run(cmd, what):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build of {what} failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build_library(name: str, force: bool = False, verbose: bool = False) -> str:
    tu = LIBRARIES[name]
    src = os.path.join(CSRC, tu)
    out = lib_path(name)
    if not os.path.exists(src):
        raise FileNotFoundError(src)
    if not force and os.path.exists(out) and os.path.getmtime(out) >= _newest(_deps(tu)):
        return out
    os.makedirs(LIBDIR, exist_ok=True)
    tmp = out + ".tmp"
    cmd = [NVCC] + ARCH + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose else []) + [src, "-o", tmp]
    log = _run(cmd, name)
    os.replace(tmp, out)
    if verbose:
        print(log)
    return out


def build_libraries(force: bool = False, verbose: bool = False, names=None):
    names = list(names or [n for n, tu in LIBRARIES.items() if os.path.exists(os.path.join(CSRC, tu))])
    with cf.ThreadPoolExecutor(max_workers=len(names) or 1) as ex:
        futs = {ex.submit(build_library, n, force, verbose): n for n in names}
        return [f.result() for f in cf.as_completed(futs)]


def build_oracle(force: bool = False):
    """The fp64 CPU oracle (test infrastructure) and, when the reference sources are present, the reference's own
    kernels compiled for sm_100a into oracle/_ref (the GPU cross-check)."""
    sys.path.insert(0, ROOT)
    from oracle import build as ob  # noqa: E402  (test infrastructure, built beside the product)

    ob.build_oracle(force=force)
    ob.build_reference(force=force)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--all", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("libs", nargs="*")
    a = ap.parse_args(argv)
    for p in build_libraries(force=a.force, verbose=a.verbose, names=a.libs or None):
        print("built", p)
    if a.all:
        build_oracle(force=a.force)


if __name__ == "__main__":
    main()
