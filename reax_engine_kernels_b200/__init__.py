"""B200-native (sm_100a) REAX engine kernel libraries.

The product is five shared libraries (``lib/libreax_*.so``) exporting the reference's C ABI
(``include/reax_abi.h``).  This package builds them (``build``), binds them with ctypes exactly as the
engine does (``abi``) and offers a torch-tensor front end (``kernels``).
"""
from . import abi, build  # noqa: F401

__all__ = ["abi", "build"]
