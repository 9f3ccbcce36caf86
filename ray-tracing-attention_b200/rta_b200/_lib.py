"""ctypes binding of librta_cuda.so (the C-ABI declared in include/rta.h).

The CUDA library is the only implementation: if it cannot be built or loaded
this module raises, there is no host fallback.
"""
from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

from . import _build

RTA_OK, RTA_E_ARG, RTA_E_ASSET, RTA_E_CUDA, RTA_E_DEVICE_CHECK, RTA_E_TIMEOUT, RTA_E_STATE = range(7)
F32, F16, BF16, Q4_K, Q6_K = 0, 1, 30, 12, 14
Q4_K_TILED, Q6_K_TILED = 112, 114  # rta_tile_weights re-layouts (same bytes)
Q4_K_PANEL, Q6_K_PANEL = 212, 214  # rta_panel_weights re-layouts for the tensor-core product
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210, Q4_K_TILED: 144, Q6_K_TILED: 210, Q4_K_PANEL: 144, Q6_K_PANEL: 210}
TILED = {Q4_K: Q4_K_TILED, Q6_K: Q6_K_TILED}
PANEL = {Q4_K: Q4_K_PANEL, Q6_K: Q6_K_PANEL}


class RtaError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"rta status {status}: {message}")
        self.status = status


_lib = None

c_u32, c_u64, c_i32, c_sz, c_f, c_p = (ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_size_t,
                                       ctypes.c_float, ctypes.c_void_p)
_SIGNATURES = {
    "rta_last_error": (ctypes.c_char_p, []),
    "rta_version": (ctypes.c_char_p, []),
    "rta_quantize": (c_i32, [c_i32, c_p, c_sz, c_p, c_p]),
    "rta_synthetic_blocks": (c_i32, [c_i32, c_u64, c_f, c_u64, c_sz, c_p, c_p]),
    "rta_synthetic_normal": (c_i32, [c_u64, c_f, c_f, c_sz, c_p, c_p]),
    "rta_dequantize": (c_i32, [c_i32, c_p, c_sz, c_p, c_p]),
    "rta_tile_weights": (c_i32, [c_i32, c_p, c_u32, c_u32, c_p, c_p]),
    "rta_panel_weights": (c_i32, [c_i32, c_p, c_u32, c_u32, c_p, c_p]),
    "rta_gemm_tc_workspace_bytes": (c_sz, [c_i32, c_u32, c_u32]),
    "rta_gemm_tc": (c_i32, [c_i32, c_p, c_u32, c_u32, c_p, c_u32, c_p, c_i32, c_p, c_p, c_p, c_sz, c_p]),
    "rta_mlp_tc_workspace_bytes": (c_sz, [c_i32, c_u32, c_u32, c_u32]),
    "rta_mlp_tc": (c_i32, [c_i32, c_p, c_p, c_p, c_u32, c_u32, c_p, c_u32, c_p, c_p, c_i32, c_p, c_sz, c_p]),
    "rta_team_handle_bytes": (c_sz, []),
    "rta_team_create": (c_i32, [c_u32, c_u32, c_sz, ctypes.POINTER(c_p), c_p]),
    "rta_team_connect": (c_i32, [c_p, c_p]),
    "rta_team_allreduce_f32": (c_i32, [c_p, c_p, c_p, c_p, c_sz, c_p]),
    "rta_team_argmax": (c_i32, [c_p, c_p, c_p, c_u32, c_u32, c_p, c_p, c_p]),
    "rta_team_error": (c_i32, [c_p, c_p, ctypes.POINTER(c_u32)]),
    "rta_team_disconnect": (c_i32, [c_p]),
    "rta_team_destroy": (None, [c_p]),
    "rta_gemv": (c_i32, [c_i32, c_p, c_u32, c_u32, c_p, c_u32, c_p, c_i32, c_p]),
    "rta_gemv_swiglu": (c_i32, [c_i32, c_p, c_p, c_u32, c_u32, c_p, c_u32, c_p, c_p]),
    "rta_mlp_swiglu": (c_i32, [c_i32, c_p, c_p, c_p, c_u32, c_u32, c_p, c_u32, c_p, c_p, c_i32, c_p]),
    "rta_readout_workspace_bytes": (c_sz, [c_u32]),
    "rta_readout": (c_i32, [c_i32, c_p, c_u32, c_u32, c_p, c_u32, c_p, c_p, c_p, c_p, c_p]),
    "rta_attention_workspace_bytes": (c_sz, [c_u32, c_u32, c_u32, c_u32]),
    "rta_attention_default_splits": (c_u32, [c_u32, c_u32]),
    "rta_attention_decode_f16": (c_i32, [c_p, c_p, c_p, c_u32, c_u32, c_u32, c_u32, c_u32, c_u32, c_u32, c_p, c_p,
                                         c_p, c_u32, c_p, c_sz, c_p]),
    "rta_workspace_error": (c_i32, [c_p, c_sz, c_p, ctypes.POINTER(c_u32)]),
    "rta_attention_decode_f16_noalloc": (c_i32, [c_p, c_p, c_p, c_u32, c_u32, c_u32, c_u32, c_u32, c_u32, c_u32, c_p,
                                                 c_p, c_p, c_u32, c_p, c_p]),
    "rta_gated_delta_step": (c_i32, [c_p, c_p, c_p, c_p, c_p, c_p, c_p, c_u32, c_p, c_p, c_p, c_p, c_p, c_u32, c_u32,
                                     c_u32, c_u32, c_f, c_p, c_p]),
}


def header_symbols() -> list[str]:
    """Every function name declared in include/*.h (the boundary contract)."""
    names = []
    for h in sorted(_build.INCLUDE.glob("*.h")):
        text = h.read_text()
        names += re.findall(r"^RTA_API\s+[\w\s\*]+?\b(rta_\w+)\s*\(", text, flags=re.M)
    return names


def load(build: bool = True):
    """Load (building first if stale) the CUDA library; raises on failure."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.build_library() if build else _build.LIBRARY
    if not Path(path).exists():
        raise RtaError(RTA_E_CUDA, f"{path} missing; the CUDA path has no fallback")
    lib = ctypes.CDLL(str(path), mode=os.RTLD_NOW | getattr(os, "RTLD_GLOBAL", 0))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != RTA_OK:
        msg = load().rta_last_error().decode(errors="replace")
        raise RtaError(status, msg)


def library_path() -> Path:
    return _build.LIBRARY
