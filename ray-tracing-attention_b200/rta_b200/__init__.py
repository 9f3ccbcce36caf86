"""rta_b200 -- B200 (sm_100a) CUDA backend for the decode path of Ray Tracing Attention.

The package is a thin host layer over librta_cuda.so (C-ABI in include/rta.h):
`ops` exposes the decode-path operators on device tensors.
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
