"""The parity tolerance of this project (bf16 outputs, fp32 accumulation):

    rel = |y - r| / max(|r|, 1e-2 * rms(r));   max(rel) <= 1e-2  and  mean(rel) <= 1e-3

Bit-exact checks (tables, masks, write sets, slice mapping) use torch.equal / numpy.array_equal instead.
"""
import numpy as np

MAX_REL = 1e-2
MEAN_REL = 1e-3


def rel_errors(y, r):
    y = np.asarray(y.detach().cpu() if hasattr(y, "detach") else y, dtype=np.float64)
    r = np.asarray(r.detach().cpu() if hasattr(r, "detach") else r, dtype=np.float64)
    assert y.shape == r.shape, (y.shape, r.shape)
    if r.size == 0:
        return np.zeros(0)
    rms = float(np.sqrt(np.mean(r * r)))
    den = np.maximum(np.abs(r), 1e-2 * rms if rms > 0 else 1e-30)
    return np.abs(y - r) / den


def assert_close(y, r, max_rel=MAX_REL, mean_rel=MEAN_REL):
    e = rel_errors(y, r)
    if e.size == 0:
        return
    assert np.all(np.isfinite(e)), "non-finite values"
    mx, mn = float(e.max()), float(e.mean())
    assert mx <= max_rel and mn <= mean_rel, f"max rel {mx:.3g} (<= {max_rel}), mean rel {mn:.3g} (<= {mean_rel})"


def interval_errors(y, r, lo, hi):
    """Relative error of y against the interval [min(lo, hi), max(lo, hi)] of legitimately rounded results
    (r = the primary oracle value, used for the rms floor of the denominator)."""
    f = lambda a: np.asarray(a.detach().cpu() if hasattr(a, "detach") else a, dtype=np.float64)
    y, r, lo, hi = f(y), f(r), f(lo), f(hi)
    a, b = np.minimum(lo, hi), np.maximum(lo, hi)
    dist = np.where(y < a, a - y, np.where(y > b, y - b, 0.0))
    rms = float(np.sqrt(np.mean(r * r))) if r.size else 0.0
    den = np.maximum(np.abs(r), 1e-2 * rms if rms > 0 else 1e-30)
    return dist / den


def assert_close_interval(y, r, lo, hi, max_rel=MAX_REL, mean_rel=MEAN_REL):
    """max/mean bound applied to the distance from the interval of results reachable by the intermediate
    roundings (an element whose exact intermediate is not near a rounding boundary has lo == hi == r)."""
    e = interval_errors(y, r, lo, hi)
    if e.size == 0:
        return
    assert np.all(np.isfinite(e)), "non-finite values"
    mx, mn = float(e.max()), float(e.mean())
    assert mx <= max_rel and mn <= mean_rel, f"max rel {mx:.3g} (<= {max_rel}), mean rel {mn:.3g} (<= {mean_rel})"
