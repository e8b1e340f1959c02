"""h3b: the X-MinimaxH3 DiT-block quantized hot path on B200 (sm_100a).

Kernels live in libh3b.so (C ABI in include/h3b.h); this package is the
torch-facing host side.  Importing it does not need a GPU; calling an operator
does, and raises if the library was not built.
"""

from ._lib import EXPORTED, H3BError, LIB_PATH, device_status, lib  # noqa: F401
from . import ops, kernels, attention  # noqa: F401
from .kernels import h3b_int8_kernel, h3b_w4a8_kernel  # noqa: F401

__all__ = ["ops", "kernels", "attention", "h3b_int8_kernel", "h3b_w4a8_kernel", "lib", "device_status",
           "H3BError", "EXPORTED", "LIB_PATH"]
