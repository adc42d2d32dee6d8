"""Start-up cfg selection logic (reax_engine_kernels_b200.autoselect.pick_cfg) with fake runs and timings: the
bit check rejects indices whose output differs or whose call fails, and the fastest valid index wins."""
import numpy as np
import pytest

from reax_engine_kernels_b200.autoselect import NoValidCfg, pick_cfg


def _same(a, b):
    return np.array_equal(a, b)


def test_fastest_valid_index_wins():
    base = np.arange(12, dtype=np.uint16)
    outs = {c: base.copy() for c in range(6)}
    outs[2][5] ^= 1  # one flipped bit: rejected
    times = {0: 3.0, 1: 2.0, 2: 0.5, 3: 1.0, 4: 1.0, 5: 4.0}
    ch = pick_cfg(6, lambda c: outs[c], lambda c: times[c], _same)
    assert ch.cfg == 3  # the fastest valid index; 2 was faster but wrong, 4 ties with 3 (lower index kept)
    assert ch.valid == [0, 1, 3, 4, 5]
    assert set(ch.rejected) == {2}
    assert ch.seconds == 1.0


def test_failed_call_is_rejected_and_first_runner_is_reference():
    base = np.zeros(4, np.uint16)

    def run(c):
        if c == 0:
            raise RuntimeError("reax_gv returned 9")
        return base if c != 3 else base + 1

    ch = pick_cfg(4, run, lambda c: float(10 - c), _same)
    assert 0 in ch.rejected and 3 in ch.rejected
    assert ch.valid == [1, 2] and ch.cfg == 2


def test_explicit_reference_and_no_valid():
    ref = np.ones(3, np.uint16)
    ch = pick_cfg(3, lambda c: ref.copy() if c == 1 else ref * 0, lambda c: 1.0, _same, reference=ref)
    assert ch.cfg == 1 and ch.valid == [1]
    with pytest.raises(NoValidCfg):
        pick_cfg(2, lambda c: ref * 0, lambda c: 1.0, _same, reference=ref)
    with pytest.raises(NoValidCfg):
        pick_cfg(0, lambda c: ref, lambda c: 1.0, _same)
