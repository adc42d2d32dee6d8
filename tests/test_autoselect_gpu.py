"""Engine-style start-up cfg selection on the GPU: every cfg index of the three GEMM libraries passes the bit check
on the layer's shape (this build's indices share one K-reduction order), the chosen index is timed fastest among
them, and a later call with the chosen index reproduces the probe's bits and matches the oracle."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import synth
from reax_engine_kernels_b200.autoselect import CfgSelector
from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
bf = synth.bf16_bits_to_f32


@pytest.mark.parametrize("M", [8, 512])
def test_selector_over_all_gemm_libraries(M):
    K, N = 1024, 1536
    x = synth.bf16_normal(1500 + M, (M, K))
    w = synth.bf16_normal(1501 + M, (N, K), 0.02)
    xt, wt = synth.to_torch_bf16(x), synth.to_torch_bf16(w)
    sel = CfgSelector(reps=3)
    for name, ch, n in (("libreax_gv", sel.gv(xt, wt), 20), ("libreax_plain", sel.gemm(xt, wt, ldd=N + 64), 15),
                        ("libreax_slices", sel.slices(xt, wt, 2, K // 2, part_fp32=False), 16)):
        assert ch.valid == list(range(n)), (name, ch.rejected)
        assert ch.cfg in ch.valid and ch.seconds == min(ch.timings.values())
    assert sel.gv(xt, wt) is sel.cache[("libreax_gv", (M, K), (N, K))]  # cached per shape
    d = synth.from_torch_bf16(rk.gemm(xt, wt, cfg=sel.gemm(xt, wt, ldd=N + 64).cfg))
    assert_close(bf(d), bf(orc.gemm(x, w)))
    d0 = synth.from_torch_bf16(rk.gemm(xt, wt, cfg=0))
    assert np.array_equal(d, d0)
