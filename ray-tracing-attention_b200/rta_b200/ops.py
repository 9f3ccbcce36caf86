"""Torch-tensor face of the decode-path operators (device memory plumbing only).

Every function forwards device pointers of CUDA tensors to librta_cuda.so and
raises RtaError on any failure.  Tensors must be contiguous and on the current
CUDA device; calls are asynchronous on torch's current stream.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import BLOCK_BYTES, PANEL, Q4_K, Q6_K, TILED, check


def _stream():
    return ctypes_ptr(torch.cuda.current_stream().cuda_stream)


def ctypes_ptr(v: int):
    import ctypes
    return ctypes.c_void_p(v)


def _ptr(t: torch.Tensor | None):
    if t is None:
        return None
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("operator tensors must be contiguous CUDA tensors")
    return ctypes_ptr(t.data_ptr())


def nblocks(fmt: int, numel_or_rows: int, cols: int | None = None) -> int:
    n = numel_or_rows * (cols or 1)
    if n % 256:
        raise ValueError("coefficient count must be a multiple of 256")
    return n // 256


def quantize(fmt: int, values: torch.Tensor) -> torch.Tensor:
    nb = values.numel() // 256
    out = torch.empty(nb * BLOCK_BYTES[fmt], dtype=torch.uint8, device=values.device)
    check(_lib.load().rta_quantize(fmt, _ptr(values), nb, _ptr(out), _stream()))
    return out


def synthetic_blocks(fmt: int, rows: int, cols: int, seed: int, sigma: float = 0.02, device=None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    nb = rows * cols // 256
    if out is None:
        out = torch.empty(nb * BLOCK_BYTES[fmt], dtype=torch.uint8, device=device or "cuda")
    check(_lib.load().rta_synthetic_blocks(fmt, seed, sigma, 0, nb, _ptr(out), _stream()))
    return out


def synthetic_normal(n: int, seed: int, sigma: float = 1.0, mean: float = 0.0, device=None) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float32, device=device or "cuda")
    check(_lib.load().rta_synthetic_normal(seed, sigma, mean, n, _ptr(out), _stream()))
    return out


def dequantize(fmt: int, blocks: torch.Tensor) -> torch.Tensor:
    nb = blocks.numel() // BLOCK_BYTES[fmt]
    out = torch.empty(nb * 256, dtype=torch.float32, device=blocks.device)
    check(_lib.load().rta_dequantize(fmt, _ptr(blocks), nb, _ptr(out), _stream()))
    return out


def tile_weights(fmt: int, w: torch.Tensor, rows: int, cols: int) -> tuple[int, torch.Tensor]:
    """Re-lay a row-major Q4_K / Q6_K matrix into the tiled GEMV order.
    Returns (tiled format code, tiled bytes); the input is left unchanged."""
    out = torch.empty_like(w)
    check(_lib.load().rta_tile_weights(fmt, _ptr(w), rows, cols, _ptr(out), _stream()))
    return TILED[fmt], out


def panel_weights(fmt: int, w: torch.Tensor, rows: int, cols: int) -> tuple[int, torch.Tensor]:
    """Re-lay a row-major Q4_K / Q6_K matrix (rows % 128 == 0) into the panel order
    of the tensor-core product.  Returns (panel format code, panel bytes)."""
    out = torch.empty_like(w)
    check(_lib.load().rta_panel_weights(fmt, _ptr(w), rows, cols, _ptr(out), _stream()))
    return PANEL[fmt], out


def gemm_tc(fmt: int, w: torch.Tensor, rows: int, cols: int, x: torch.Tensor, y: torch.Tensor | None = None,
            accumulate: bool = False, argmax: bool = False, store: bool = True,
            workspace: torch.Tensor | None = None, split: bool = False):
    """Tensor-core batched product with panel weights: returns (y, argmax ids, best)
    (ids / best None unless argmax; y None when store is False).  split: x enters
    as two fp16 operands (fp16(x) + fp16(x - fp16(x)))."""
    x = x.reshape(-1, cols)
    B = x.shape[0]
    lib = _lib.load()
    if workspace is None:
        workspace = torch.empty(lib.rta_gemm_tc_workspace_bytes(fmt, B, cols), dtype=torch.uint8, device=x.device)
    if store and y is None:
        y = torch.empty(B, rows, dtype=torch.float32, device=x.device)
    ids = torch.empty(B, dtype=torch.int32, device=x.device) if argmax else None
    best = torch.empty(B, dtype=torch.float32, device=x.device) if argmax else None
    flags = (1 if accumulate else 0) | (2 if split else 0)  # RTA_GEMM_ACCUMULATE, RTA_GEMM_SPLIT_ACTIVATIONS
    check(lib.rta_gemm_tc(fmt, _ptr(w), rows, cols, _ptr(x), B, _ptr(y if store else None), flags,
                          _ptr(ids), _ptr(best), _ptr(workspace), workspace.numel(), _stream()))
    return (y if store else None), ids, best


def gemv(fmt: int, w: torch.Tensor, rows: int, cols: int, x: torch.Tensor, y: torch.Tensor | None = None,
         accumulate: bool = False) -> torch.Tensor:
    x = x.reshape(-1, cols)
    if y is None:
        y = torch.empty(x.shape[0], rows, dtype=torch.float32, device=x.device)
    check(_lib.load().rta_gemv(fmt, _ptr(w), rows, cols, _ptr(x), x.shape[0], _ptr(y), int(accumulate), _stream()))
    return y


def gemv_swiglu(fmt: int, wg, wu, rows: int, cols: int, x: torch.Tensor, act: torch.Tensor | None = None):
    x = x.reshape(-1, cols)
    act = torch.empty(x.shape[0], rows, dtype=torch.float32, device=x.device) if act is None else act
    check(_lib.load().rta_gemv_swiglu(fmt, _ptr(wg), _ptr(wu), rows, cols, _ptr(x), x.shape[0], _ptr(act), _stream()))
    return act


def mlp_swiglu(fmt: int, wg, wu, wd, hidden: int, middle: int, x: torch.Tensor, y: torch.Tensor | None = None,
               act: torch.Tensor | None = None, accumulate: bool = False):
    x = x.reshape(-1, hidden)
    B = x.shape[0]
    act = torch.empty(B, middle, dtype=torch.float32, device=x.device) if act is None else act
    y = torch.empty(B, hidden, dtype=torch.float32, device=x.device) if y is None else y
    check(_lib.load().rta_mlp_swiglu(fmt, _ptr(wg), _ptr(wu), _ptr(wd), hidden, middle, _ptr(x), B, _ptr(act),
                                     _ptr(y), int(accumulate), _stream()))
    return act, y


def mlp_tc(fmt: int, wg, wu, wd, hidden: int, middle: int, x: torch.Tensor, y: torch.Tensor | None = None,
           act: torch.Tensor | None = None, accumulate: bool = False, workspace: torch.Tensor | None = None):
    """SwiGLU MLP on the tensor cores (panel weights): returns y; act receives
    the activation rows when given."""
    x = x.reshape(-1, hidden)
    B = x.shape[0]
    lib = _lib.load()
    if workspace is None:
        workspace = torch.empty(lib.rta_mlp_tc_workspace_bytes(fmt, B, hidden, middle), dtype=torch.uint8,
                                device=x.device)
    y = torch.empty(B, hidden, dtype=torch.float32, device=x.device) if y is None else y
    check(lib.rta_mlp_tc(fmt, _ptr(wg), _ptr(wu), _ptr(wd), hidden, middle, _ptr(x), B, _ptr(act), _ptr(y),
                         int(accumulate), _ptr(workspace), workspace.numel(), _stream()))
    return y


def readout(fmt: int, w: torch.Tensor, vocab: int, hidden: int, x: torch.Tensor, logits: bool = True,
            workspace: torch.Tensor | None = None):
    x = x.reshape(-1, hidden)
    B = x.shape[0]
    lib = _lib.load()
    if workspace is None:
        workspace = torch.empty(lib.rta_readout_workspace_bytes(B), dtype=torch.uint8, device=x.device)
    lg = torch.empty(B, vocab, dtype=torch.float32, device=x.device) if logits else None
    arg = torch.empty(B, dtype=torch.int32, device=x.device)
    best = torch.empty(B, dtype=torch.float32, device=x.device)
    check(lib.rta_readout(fmt, _ptr(w), vocab, hidden, _ptr(x), B, _ptr(lg), _ptr(arg), _ptr(best), _ptr(workspace),
                          _stream()))
    return lg, arg, best


def attention_workspace(heads: int, kv_heads: int, head_dim: int, splits: int, device=None) -> torch.Tensor:
    n = _lib.load().rta_attention_workspace_bytes(heads, kv_heads, head_dim, splits)
    return torch.empty(n, dtype=torch.uint8, device=device or "cuda")


def attention_decode_f16(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, time: int, capacity: int,
                         pos_stride: int, kv_stride: int, gate: torch.Tensor | None = None, splits: int | None = None,
                         workspace: torch.Tensor | None = None, phys: bool = True):
    heads, head_dim = q.shape[-2], q.shape[-1]
    kv_heads = heads // 4
    lib = _lib.load()
    if splits is None:
        splits = lib.rta_attention_default_splits(min(time + 1, capacity), kv_heads)
    if workspace is None:
        workspace = attention_workspace(heads, kv_heads, head_dim, splits, q.device)
    out = torch.empty(heads, head_dim, dtype=torch.float32, device=q.device)
    ph = torch.empty(heads, 2, dtype=torch.float32, device=q.device) if phys else None
    check(lib.rta_attention_decode_f16(_ptr(q), _ptr(k), _ptr(v), time, capacity, heads, kv_heads, head_dim,
                                       pos_stride, kv_stride, _ptr(gate), _ptr(out), _ptr(ph), splits,
                                       _ptr(workspace), workspace.numel(), _stream()))
    return out, ph, workspace


def workspace_error(workspace: torch.Tensor) -> int:
    import ctypes
    word = ctypes.c_uint32(0)
    st = _lib.load().rta_workspace_error(_ptr(workspace), workspace.numel(), _stream(), ctypes.byref(word))
    if st not in (_lib.RTA_OK, _lib.RTA_E_DEVICE_CHECK, _lib.RTA_E_TIMEOUT):
        check(st)
    return int(word.value)


def gated_delta_step(x: torch.Tensor, attn_norm: torch.Tensor, w_alpha: torch.Tensor, w_beta: torch.Tensor,
                     a_log: torch.Tensor, dt_bias: torch.Tensor, proj: torch.Tensor, conv_w: torch.Tensor,
                     conv_state: torch.Tensor, state: torch.Tensor, positions: torch.Tensor, heads: int,
                     key_heads: int, eps: float = 1e-6, error_word: torch.Tensor | None = None) -> torch.Tensor:
    """One token of the recurrent gated-delta layer for a batch of sequences
    (rta_gated_delta_step).  x [B, D]; proj [B, >= 2*key_heads*128 + heads*128];
    conv_state [B, 2, 3*heads*128, 3] and state [B, heads, 128, 128] are updated in
    place; positions [B] int32/uint32.  Returns the detector output [B, heads*128]."""
    B, D = x.shape
    out = torch.empty(B, heads * 128, dtype=torch.float32, device=x.device)
    check(_lib.load().rta_gated_delta_step(_ptr(x), _ptr(attn_norm), _ptr(w_alpha), _ptr(w_beta), _ptr(a_log),
                                           _ptr(dt_bias), _ptr(proj), proj.shape[1], _ptr(conv_w),
                                           _ptr(conv_state), _ptr(state), _ptr(out), _ptr(positions), D, heads,
                                           key_heads, B, eps, _ptr(error_word), _stream()))
    return out


__all__ = ["gated_delta_step", "quantize", "dequantize", "synthetic_blocks", "synthetic_normal", "gemv", "gemv_swiglu", "mlp_swiglu", "readout",
           "attention_decode_f16", "attention_workspace", "workspace_error", "Q4_K", "Q6_K", "BLOCK_BYTES"]
