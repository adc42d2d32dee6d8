"""B200-native (sm_100a) REAX engine kernel libraries.

The product is five shared libraries (``lib/libreax_*.so``) exporting the reference's C ABI
(``include/reax_abi.h``).  This package builds them (``build``), binds them with ctypes exactly as the
engine does (``abi``) and offers a torch-tensor front end (``kernels``).  Host-side helpers above the ABI:
``autoselect`` (start-up cfg choice per layer shape, as the engine makes it), ``seqpar`` (one long sequence's
attention sharded over the ranks of a node, K/V all-gathered over NCCL) and ``dist`` (shard ownership and the
max-over-ranks timing reduction).
"""
from . import abi, build  # noqa: F401

__all__ = ["abi", "build"]
