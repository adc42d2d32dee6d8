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
    # the 22 distinct names the five reference libraries export, plus this build's extensions
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


PLAIN_NAMES = ["128x256x32 w64x64 s3", "256x128x32 w64x64 s3", "128x128x32 w64x64 s4", "128x256x32 w64x64 s4",
               "128x256x32 w64x64 s2", "192x128x32 w48x64 s3", "192x128x32 w48x64 s4", "64x256x32 w64x64 s4",
               "64x256x32 w32x64 s4", "128x128x32 w64x64 s3", "128x128x32 w64x32 s4", "256x128x32 w64x64 s4",
               "256x64x32 w64x64 s4", "128x64x32 w64x64 s4", "64x128x32 w64x64 s4"]

SLICE_NAMES = ["128x256x32 w64x64 s3", "256x128x32 w64x64 s3", "128x128x32 w64x64 s4", "64x256x32 w64x64 s4",
               "128x128x32 w64x64 s3", "256x128x32 w64x64 s4", "128x256x32 w64x64 s4", "64x128x32 w64x64 s4",
               "128x64x32 w64x64 s4", "64x256x32 w64x64 s3", "64x128x32 w32x64 s4", "256x64x32 w64x64 s3",
               "128x128x32 w64x64 s5", "128x128x32 w64x64 s6", "64x128x32 w32x64 s6", "256x128x32 w64x64 s5"]


def test_cfg_tables():
    for lib, stem, want in (("libreax_gv", "reax_gv", GV_NAMES), ("libreax_plain", "reax_gemm", PLAIN_NAMES),
                            ("libreax_slices", "reax_slices", SLICE_NAMES)):
        n, names, f = _names(lib, stem)
        assert n == len(want) and names == want, lib
        for bad in (n, n + 7, -1, -3, 1 << 30):
            assert f(bad) == b"?", (lib, bad)


def _ref_string_table(path, fn):
    """The string array inside the reference's `fn` (its cfgname function), parsed from the source text."""
    src = open(path).read()
    body = src[src.index(f"const char* {fn}(int c)"):]
    start = body.index("{", body.index("n[] ="))
    arr = body[start + 1:body.index("};", start)]
    return re.findall(r'"([^"]*)"', arr)


@pytest.mark.skipif(not os.environ.get("REAX_REFERENCE"), reason="REAX_REFERENCE (reference checkout) not set")
def test_cfg_tables_match_reference_source():
    """Every name of the three tables equals the reference's own table, read from its source (gateup_vis2.cu:172-181,
    gemm_plain2.cu:32-36, gemm_slices_v2.cu:56-64); the SLICE_CFGS tile macro (gemm_slices_v2.cu:37-53) spells the
    same 16 names in the same order."""
    ref = os.environ["REAX_REFERENCE"]
    assert _ref_string_table(os.path.join(ref, "libreax_gv", "gateup_vis2.cu"), "reax_gv_cfgname") == GV_NAMES
    assert _ref_string_table(os.path.join(ref, "libreax_plain", "gemm_plain2.cu"), "reax_gemm_cfgname") == PLAIN_NAMES
    sl = os.path.join(ref, "libreax_slices", "gemm_slices_v2.cu")
    assert _ref_string_table(sl, "reax_slices_cfgname") == SLICE_NAMES
    rows = re.findall(r"X\((\d+),\s*(\d+),\s*(\d+),\s*(\d+),\s*(\d+),\s*(\d+),\s*(\d+),\s*(\d+)\)", open(sl).read())
    assert [int(r[0]) for r in rows] == list(range(16))
    assert [f"{r[1]}x{r[2]}x{r[3]} w{r[4]}x{r[5]} s{r[7]}" for r in rows] == SLICE_NAMES
