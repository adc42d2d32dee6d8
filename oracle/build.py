"""Build recipe for the TEST oracle (not product code).

* ``oracle/liboracle.so``: the fp64 C++ restatement (reax_oracle.cpp), built with g++.
* ``oracle/_ref/libreax_*.so``: the reference's own CUDA sources, compiled UNMODIFIED from where they lie under
  the reference checkout for sm_100a (the reference ships sm_120 builds only).  Run on a B200 they are the
  second reference point and the source of the golden fixtures in tests/golden/.  This step needs the
  reference checkout (present in the build container only); the built files travel with the tree.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
REF_OUT = os.path.join(HERE, "_ref")
# The reference checkout: REAX_REFERENCE names its root.  Unset means "not available here" (the GPU box has no
# checkout and uses the prebuilt oracle/_ref files).
REFERENCE = os.environ.get("REAX_REFERENCE", "")
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cutlass_include() -> str:
    """CUTLASS 4.2.1 headers (the version the reference pins): REAX_CUTLASS_INC, else the copy vendored inside the
    installed vllm package (third_party/deep_gemm/include).  Raises when neither exists."""
    p = os.environ.get("REAX_CUTLASS_INC", "")
    if p:
        if not os.path.isdir(os.path.join(p, "cutlass")):
            raise RuntimeError(f"REAX_CUTLASS_INC={p} holds no cutlass/ header tree")
        return p
    import importlib.util

    spec = importlib.util.find_spec("vllm")
    if spec is not None and spec.submodule_search_locations:
        for root in spec.submodule_search_locations:
            cand = os.path.join(root, "third_party", "deep_gemm", "include")
            if os.path.isdir(os.path.join(cand, "cutlass")):
                return cand
    raise RuntimeError("CUTLASS headers not found: set REAX_CUTLASS_INC to a CUTLASS 4.2.1 include directory")

# reference library -> (sources relative to the reference root, extra flags): the reference's own flags
# (build.sh:15-19) with the architecture switched to sm_100a
CUTLASS = "<cutlass>"  # placeholder in the flag lists, resolved by cutlass_include() when a build runs
REF_LIBS = {
    "libreax_gv": (["libreax_gv/gateup_vis2.cu"], ["-std=c++17", "-I", CUTLASS]),
    "libreax_plain": (["libreax_plain/gemm_plain2.cu"], ["-std=c++17", "-I", CUTLASS]),
    "libreax_slices": (["libreax_slices/gemm_slices_v2.cu"], ["-std=c++17", "-I", CUTLASS]),
    "libreax_howu": (["libreax_howu/reax_howu.cu", "libreax_howu/reax_kkt.cu", "libreax_howu/reax_howu_norm_v3.cu",
                      "libreax_howu/reax_rarn_final.cu", "libreax_howu/reax_fmha_v8.cu", "libreax_howu/reax_conv_v2.cu"],
                     ["-fmad=false", "-DRPF=10"]),
    "libreax_fmha_post": (["libreax_fmha_post/reax_fmha_v11.cu"], ["-fmad=false"]),
}


def oracle_path() -> str:
    return os.path.join(HERE, "liboracle.so")


def ref_path(name: str) -> str:
    return os.path.join(REF_OUT, name + ".so")


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "reax_oracle.cpp")
    out = oracle_path()
    if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src):
        return out
    cmd = ["g++", "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-std=c++17", "-shared", "-fPIC", "-pthread",
           "-fvisibility=hidden", src, "-o", out + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"oracle build failed:\n{r.stderr}")
    os.replace(out + ".tmp", out)
    return out


def _build_ref(name: str, force: bool) -> str | None:
    srcs, flags = REF_LIBS[name]
    paths = [os.path.join(REFERENCE, s) for s in srcs]
    out = ref_path(name)
    if not all(os.path.exists(p) for p in paths):
        return None
    if not force and os.path.exists(out) and os.path.getmtime(out) >= max(os.path.getmtime(p) for p in paths):
        return out
    os.makedirs(REF_OUT, exist_ok=True)
    flags = [cutlass_include() if f == CUTLASS else f for f in flags]
    cmd = [NVCC, "-O3"] + ARCH + flags + ["-shared", "-Xcompiler", "-fPIC"] + paths + ["-o", out + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"reference build of {name} failed:\n{' '.join(cmd)}\n{r.stderr[-4000:]}")
    os.replace(out + ".tmp", out)
    return out


def build_reference(force: bool = False):
    """Compile the reference sources for sm_100a into oracle/_ref.  Skipped (with a message) when REAX_REFERENCE is
    unset; an error when it names a directory that does not exist."""
    if not REFERENCE:
        print("oracle/_ref: REAX_REFERENCE is unset; the reference kernels are not rebuilt")
        return []
    if not os.path.isdir(REFERENCE):
        raise RuntimeError(f"REAX_REFERENCE={REFERENCE} is not a directory")
    with cf.ThreadPoolExecutor(max_workers=len(REF_LIBS)) as ex:
        return [f.result() for f in [ex.submit(_build_ref, n, force) for n in REF_LIBS]]


if __name__ == "__main__":
    print(build_oracle(force=True))
    print(build_reference())
