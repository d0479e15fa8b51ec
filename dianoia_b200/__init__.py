"""dianoia_b200: dianoia's Q4_0 / Q8_0 block-quantized linear path on B200.

The product is ``libdianoia_b200.so`` (CUDA, sm_100a) behind the C-ABI in
``include/dianoia_b200.h``; this package holds its build script, a ctypes
loader and a Python mirror of the reference's host-side matrix classes.
"""
from ._lib import LIB_PATH, LibraryMissing, lib  # noqa: F401
from .native import (  # noqa: F401
    ArgumentError,
    NativeKernels,
    NativeQ4Matrix,
    NativeQ8Matrix,
    StateError,
    half_to_double,
)

__version__ = "0.1.0"
