"""The parity tolerance of this project, for the tests (the definitions live beside the oracle, in
oracle/tolerance.py, so the benchmark's CPU-baseline leg reports the same statistics)."""
from oracle.tolerance import *  # noqa: F401,F403
from oracle.tolerance import MAX_REL, MEAN_REL  # noqa: F401
