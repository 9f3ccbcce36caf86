"""TEST INFRASTRUCTURE ONLY -- numpy/ctypes face of the C oracle (rta_oracle.c).

The oracle is the CPU restatement of the reference's decode-path arithmetic
(Winamin/Ray-Tracing-Attention GLSL shaders).  Only tests/, the smoke check in
__graft_entry__.py and bench.py's cpu_baseline leg may import this module, and
only as the checker: the product (ray-tracing-attention_b200/) never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "rta_oracle.c"
LIBRARY = HERE / "liboracle.so"

Q4_K, Q6_K, F32, F16, BF16 = 12, 14, 0, 1, 30
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}
DENSE_BYTES = {F32: 4, F16: 2, BF16: 2}


def row_bytes(fmt: int, cols: int) -> int:
    """Bytes of one row of `cols` coefficients in an exporter format."""
    return cols * DENSE_BYTES[fmt] if fmt in DENSE_BYTES else cols // 256 * BLOCK_BYTES[fmt]


def to_bf16_bits(values) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(values, np.float32).view(np.uint32)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return np.where(np.isnan(np.ascontiguousarray(values, np.float32)), (u >> 16) | 0x40, rounded).astype(np.uint16)


def dense_values(fmt: int, raw) -> np.ndarray:
    """Decode a dense F32 / F16 / BF16 byte run to fp32 (ggufValue's dense branches)."""
    b = np.ascontiguousarray(raw, np.uint8)
    if fmt == F32:
        return b.view(np.float32).copy()
    if fmt == F16:
        return b.view(np.float16).astype(np.float32)
    return (b.view(np.uint16).astype(np.uint32) << 16).view(np.float32)


def build(force: bool = False) -> Path:
    """Compile the oracle with the reference worker's FP rule (-ffp-contract=off)."""
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < SOURCE.stat().st_mtime:
        tmp = LIBRARY.with_suffix(f".{os.getpid()}.tmp")
        subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fopenmp",
                        "-fPIC", "-shared", str(SOURCE), "-o", str(tmp), "-lm"], check=True)
        os.replace(tmp, LIBRARY)
    return LIBRARY


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        f, u32, i32, sz, p = ctypes.c_float, ctypes.c_uint32, ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p
        sig = {
            "rta_oracle_half_to_float": (f, [ctypes.c_uint16]),
            "rta_oracle_float_to_half": (ctypes.c_uint16, [f]),
            "rta_oracle_dequant": (None, [i32, p, sz, p]),
            "rta_oracle_quantize": (None, [i32, p, sz, p]),
            "rta_oracle_gemv": (None, [i32, p, u32, u32, p, u32, p]),
            "rta_oracle_mlp": (None, [i32, p, p, p, u32, u32, p, u32, p, p]),
            "rta_oracle_mlp_fmt": (None, [i32, i32, p, p, p, u32, u32, p, u32, p, p]),
            "rta_oracle_rmsnorm": (None, [p, p, u32, f, p]),
            "rta_oracle_lmhead": (None, [i32, p, u32, u32, p, u32, p, p, p]),
            "rta_oracle_attention": (None, [p, p, p, p, u32, u32, u32, u32, u32, u32, u32, u32, i32, p, p]),
            "rta_oracle_gdn": (None, [p, p, p, p, p, p, p, p, p, p, u32, u32, u32, u32, f, i32, p, p, p]),
            "rta_oracle_rope": (None, [p, u32, u32, u32, p, u32]),
            "rta_oracle_head_norm": (None, [p, p, u32, u32, f]),
            "rta_oracle_sigmoid": (f, [f]),
            "rta_oracle_threads": (i32, []),
            "rta_oracle_set_threads": (None, [i32]),
            "rta_oracle_inv_freq": (None, [f, u32, u32, p]),
            "rta_oracle_synthetic_value": (f, [ctypes.c_uint64, ctypes.c_uint64]),
            "rta_oracle_synthetic_blocks": (None, [i32, ctypes.c_uint64, f, ctypes.c_uint64, sz, p]),
            "rta_oracle_synthetic_normal": (None, [ctypes.c_uint64, f, f, sz, p]),
            "rta_oracle_synthetic_half": (None, [ctypes.c_uint64, f, ctypes.c_uint64, sz, p]),
            "rta_oracle_synthetic_range": (None, [ctypes.c_uint64, f, ctypes.c_uint64, sz, p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(_lib, name)
            fn.restype, fn.argtypes = res, args
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def threads() -> int:
    return int(lib().rta_oracle_threads())


def use_all_cores() -> int:
    """Run the OpenMP loops on every core this process may use (its CPU affinity),
    whatever OMP_NUM_THREADS a launcher set; returns the thread count."""
    import os
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    lib().rta_oracle_set_threads(n)
    return threads()


def quantize(fmt: int, values) -> np.ndarray:
    """fp32 [..., 256*k] -> raw blocks (uint8), the reference packet quantizer."""
    v = _c(values, np.float32).reshape(-1)
    assert v.size % 256 == 0
    n = v.size // 256
    out = np.zeros(n * BLOCK_BYTES[fmt], np.uint8)
    lib().rta_oracle_quantize(fmt, _p(v), n, _p(out))
    return out


def dequantize(fmt: int, blocks) -> np.ndarray:
    b = _c(blocks, np.uint8).reshape(-1)
    n = b.size // BLOCK_BYTES[fmt]
    out = np.empty(n * 256, np.float32)
    lib().rta_oracle_dequant(fmt, _p(b), n, _p(out))
    return out


def gemv(fmt: int, W, rows_out: int, cols: int, x) -> np.ndarray:
    x = _c(x, np.float32).reshape(-1, cols)
    W = _c(W, np.uint8).reshape(-1) if fmt != F32 or np.asarray(W).dtype == np.uint8 else _c(W, np.float32)
    y = np.empty((x.shape[0], rows_out), np.float32)
    lib().rta_oracle_gemv(fmt, _p(W), rows_out, cols, _p(x), x.shape[0], _p(y))
    return y


def mlp(fmt: int, wg, wu, wd, D: int, F: int, x, down_fmt: int | None = None):
    """SwiGLU MLP (op 2 kind 3 then op 2); down_fmt: the down rows' format when it differs."""
    x = _c(x, np.float32).reshape(-1, D)
    act = np.empty((x.shape[0], F), np.float32)
    y = np.empty((x.shape[0], D), np.float32)
    lib().rta_oracle_mlp_fmt(fmt, fmt if down_fmt is None else down_fmt, _p(_c(wg, np.uint8)), _p(_c(wu, np.uint8)),
                             _p(_c(wd, np.uint8)), D, F, _p(x), x.shape[0], _p(act), _p(y))
    return act, y


def rmsnorm(x, w, eps: float) -> np.ndarray:
    x = _c(x, np.float32).reshape(-1)
    out = np.empty_like(x)
    lib().rta_oracle_rmsnorm(_p(x), _p(_c(w, np.float32)), x.size, eps, _p(out))
    return out


def lmhead(fmt: int, W, V: int, D: int, x, want_logits: bool = True):
    x = _c(x, np.float32).reshape(-1, D)
    B = x.shape[0]
    logits = np.empty((B, V), np.float32) if want_logits else None
    arg = np.empty(B, np.uint32)
    best = np.empty(B, np.float32)
    lib().rta_oracle_lmhead(fmt, _p(_c(W, np.uint8)), V, D, _p(x), B,
                            _p(logits) if logits is not None else None, _p(arg), _p(best))
    return logits, arg, best


def attention(q, keys, values, gate, query_start: int, history_start: int, capacity: int, gated: bool = True):
    """q/gate [rows, heads, hd]; keys/values [count, kvh, hd] (index = age - history_start)."""
    q = _c(q, np.float32)
    rows, heads, hd = q.shape
    keys = _c(keys, np.float32)
    values = _c(values, np.float32)
    count, kvh, _ = keys.shape
    g = _c(np.zeros_like(q) if gate is None else gate, np.float32)
    out = np.empty_like(q)
    phys = np.empty((rows, heads, 2), np.float32)
    lib().rta_oracle_attention(_p(q), _p(keys), _p(values), _p(g), rows, heads, kvh, hd, count,
                               query_start, history_start, capacity, int(gated), _p(out), _p(phys))
    return out, phys


def gdn(x, qk, v, z, wa, wb, a_log, dt_bias, conv_w, norm_w, H: int, KH: int, eps: float,
        state, conv, use_past: bool = True):
    """Recurrent layer detector; `state` [H,128,128] and `conv` [3S,3] are updated in place.
    With norm_w None (z unused) the output is the detector before the gated RMSNorm (op 15)."""
    x = _c(x, np.float32)
    rows, D = x.shape
    S = H * 128
    out = np.empty((rows, S), np.float32)
    assert state.dtype == np.float32 and state.flags.c_contiguous
    assert conv.dtype == np.float32 and conv.flags.c_contiguous
    args = [None if a is None else _c(a, np.float32) for a in (qk, v, z, wa, wb, a_log, dt_bias, conv_w, norm_w)]
    lib().rta_oracle_gdn(_p(x), *[None if a is None else _p(a) for a in args], rows, D, H, KH, eps, int(use_past),
                         _p(state), _p(conv), _p(out))
    return out


def rope(v, heads: int, hd: int, rotary: int, inv_freq, time: int):
    v = _c(v, np.float32).copy()
    lib().rta_oracle_rope(_p(v), heads, hd, rotary, _p(_c(inv_freq, np.float32)), time)
    return v


def head_norm(v, w, heads: int, hd: int, eps: float):
    v = _c(v, np.float32).copy()
    lib().rta_oracle_head_norm(_p(v), _p(_c(w, np.float32)), heads, hd, eps)
    return v


def inv_freq(theta: float, rotary: int, hd: int) -> np.ndarray:
    out = np.zeros(hd // 2, np.float32)
    lib().rta_oracle_inv_freq(theta, rotary, hd, _p(out))
    return out


def sigmoid(x: float) -> float:
    return float(lib().rta_oracle_sigmoid(x))


# ------------------------------------------------- synthetic model values
def synthetic_blocks(fmt: int, seed: int, sigma: float, nblocks: int, first_block: int = 0) -> np.ndarray:
    """Host restatement of rta_synthetic_blocks: bit-identical packed blocks."""
    out = np.empty(nblocks * BLOCK_BYTES[fmt], np.uint8)
    lib().rta_oracle_synthetic_blocks(fmt, seed, sigma, first_block, nblocks, _p(out))
    return out


def synthetic_normal(seed: int, sigma: float, n: int, mean: float = 0.0) -> np.ndarray:
    """Host restatement of rta_synthetic_normal (fp32, bit-identical)."""
    out = np.empty(n, np.float32)
    lib().rta_oracle_synthetic_normal(seed, sigma, mean, n, _p(out))
    return out


def synthetic_range(seed: int, sigma: float, first: int, n: int, half: bool = False) -> np.ndarray:
    """Elements [first, first + n) of the generator's stream times sigma: fp32, or
    rounded to fp16 (returned as float32 values) like the seeded fp16 histories."""
    if half:
        out = np.empty(n, np.uint16)
        lib().rta_oracle_synthetic_half(seed, sigma, first, n, _p(out))
        return out.view(np.float16).astype(np.float32)
    out = np.empty(n, np.float32)
    lib().rta_oracle_synthetic_range(seed, sigma, first, n, _p(out))
    return out
