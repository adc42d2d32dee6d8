"""CPU checks of the boundary: every library loads and exports exactly the entry points include/reax_abi.h
declares for it; configuration tables match the reference's (names and counts are ABI data)."""
import os
import re

import pytest

from reax_engine_kernels_b200 import abi, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "reax_abi.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"\b(?:int|const char\*)\s+([a-z_0-9]+)\s*\(", src))


def built_libraries():
    return [n for n in build.LIBRARIES if os.path.exists(build.lib_path(n))]


def test_header_matches_prototype_table():
    declared = header_functions()
    bound = set().union(*[set(p) for p in abi.PROTOTYPES.values()])
    assert declared == bound, (declared ^ bound)


def test_all_five_libraries_built():
    assert sorted(built_libraries()) == sorted(build.LIBRARIES), "missing: " + str(set(build.LIBRARIES) - set(built_libraries()))


@pytest.mark.parametrize("name", sorted(build.LIBRARIES))
def test_library_exports_exactly_its_abi(name):
    path = build.lib_path(name)
    if not os.path.exists(path):
        pytest.fail(f"{path} not built")
    assert abi.exported_symbols(path) == set(abi.PROTOTYPES[name])
    abi.load(name)  # dlopen + bind every prototype (no device call)


def test_reference_export_names_are_covered():
    # the 22 distinct names the reference libraries export (SURVEY boundary table), plus our extensions
    ref = {"reax_gv_ncfg", "reax_gv_cfgname", "reax_gv", "reax_gemm_ncfg", "reax_gemm_cfgname", "reax_gemm",
           "reax_slices_ncfg", "reax_slices_cfgname", "reax_slices", "howu3_dense", "howu3_skip", "howu3_smem",
           "reax_howu", "reax_kkt", "reax_kkt_smem", "reax_howu_norm", "reax_rarn", "reax_conv_l2", "reax_conv_v",
           "reax_fmha_b", "reax_fmha_q", "reax_fmha_qp"}
    assert ref <= header_functions()


GV_NAMES = ["128x256x32 w64x64 s3", "256x128x32 w64x64 s3", "128x128x32 w64x64 s4", "128x256x32 w64x64 s4",
            "128x256x64 w64x64x64 s2", "256x128x64 w64x64x64 s2", "128x128x64 w64x64x64 s3",
            "128x128x64 w64x64x64 s2", "64x256x64 w64x64x64 s2", "128x256x32 w64x64 s2", "128x192x32 w64x48 s3",
            "128x192x32 w64x48 s4", "192x128x32 w48x64 s3", "192x128x32 w48x64 s4", "64x256x32 w64x64 s4",
            "64x256x32 w32x64 s4", "192x192x32 w96x48 s3", "128x128x32 w64x64 s3", "128x128x32 w64x32 s4",
            "256x128x32 w64x64 s4"]


def _names(lib, stem):
    L = abi.load(lib)
    n = getattr(L, stem + "_ncfg")()
    return n, [getattr(L, stem + "_cfgname")(i).decode() for i in range(n)], getattr(L, stem + "_cfgname")


def test_cfg_tables():
    n, names, f = _names("libreax_gv", "reax_gv")
    assert n == 20 and names == GV_NAMES
    assert f(20) == b"?" and f(-1) == b"?"
    n, names, f = _names("libreax_plain", "reax_gemm")
    assert n == 15 and names[0] == "128x256x32 w64x64 s3" and names[14] == "64x128x32 w64x128 s4".replace("w64x128", "w64x64")
    assert f(15) == b"?"
    n, names, f = _names("libreax_slices", "reax_slices")
    assert n == 16 and names[12] == "128x128x32 w64x64 s5" and names[15] == "256x128x32 w64x64 s5"
    assert f(16) == b"?" and f(-3) == b"?"
