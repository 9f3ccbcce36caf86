"""Tensor parallelism of the MLP and the vocabulary readout over the GPUs of one box.

The reference decodes on one GPU with whole matrices per layer
(ray_tracing/compiler/export.py:87-91); it has no collective.  Here one process
per GPU holds a slice of each split matrix:

* MLP (executeMLP, ray_tracing/native/src/optical_resident.cpp:484-491): the
  gate / up rows and the down projection's columns are divided in matching
  contiguous slices of the middle dimension.  Rank r forms
  act_r = swiglu(Wg_r x, Wu_r x) and the partial product Wd[:, r] act_r; the
  partials plus the residual are summed on every rank, in rank order, by ONE
  kernel of the library (rta_team_allreduce_f32) over NVLink peer memory.
* Readout (ops 16/17, ray_tracing/native/shaders/resident_math.comp:117-127):
  the vocabulary rows are divided; every rank finds its best row and one
  kernel (rta_team_argmax) agrees on the best of the bests, ties -> lowest id.

Slices are whole units: 256 middle rows (one Q4_K / Q6_K block column of the
down projection, two 128-row tiles of the tensor-core product) and 128
vocabulary rows.  A plan is a pure function of (size, unit, world), so every
rank derives the same plan locally.  Batches of 16 rows or more run on the
tensor cores (panel weights), smaller ones on the GEMV (tiled weights).

The team's handles travel through torch.distributed.all_gather_object, so any
backend carries them (gloo in the CPU tests); the data never does.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import BLOCK_BYTES, PANEL, TILED, check

MIDDLE_UNIT = 256
VOCAB_UNIT = 128
TC_MIN_BATCH = 16  # batches at or above this use the tensor-core product


def split_units(total: int, unit: int, world: int) -> list[tuple[int, int]]:
    """Contiguous (start, count) slices of `total` rows, each a multiple of
    `unit`; the first (total / unit) % world ranks get one unit more."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if total <= 0 or total % unit:
        raise ValueError(f"{total} rows is not a positive multiple of {unit}")
    units = total // unit
    if units < world:
        raise ValueError(f"{units} units of {unit} rows cannot feed {world} ranks")
    base, extra = divmod(units, world)
    out, start = [], 0
    for r in range(world):
        n = (base + (1 if r < extra else 0)) * unit
        out.append((start, n))
        start += n
    return out


def _contiguous(a):
    return np.ascontiguousarray(a) if isinstance(a, np.ndarray) else a.contiguous()


def slice_rows(fmt: int, w, rows: int, cols: int, start: int, count: int):
    """Rows [start, start + count) of a row-major Q4_K / Q6_K matrix (flat bytes)."""
    if start < 0 or count <= 0 or start + count > rows or cols % 256:
        raise ValueError("row slice out of range")
    row_bytes = cols // 256 * BLOCK_BYTES[fmt]
    return _contiguous(w.reshape(-1)[start * row_bytes:(start + count) * row_bytes])


def slice_columns(fmt: int, w, rows: int, cols: int, start: int, count: int):
    """Columns [start, start + count) (whole 256-wide blocks) of every row of a
    row-major Q4_K / Q6_K matrix: a [rows x count] matrix, flat bytes."""
    if start % 256 or count % 256 or start < 0 or count <= 0 or start + count > cols:
        raise ValueError("column slice must cover whole 256-column blocks inside the matrix")
    bb = BLOCK_BYTES[fmt]
    blocks = w.reshape(rows, cols // 256, bb)[:, start // 256:(start + count) // 256, :]
    return _contiguous(blocks).reshape(-1)


class Team:
    """Peer exchange among the ranks of a torch.distributed group (or a team of
    one without it).  Each rank must be on its own GPU (torch.cuda.set_device)."""

    def __init__(self, capacity_bytes: int, group=None):
        import torch.distributed as dist
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if dist_on else 0
        self.world = dist.get_world_size(group) if dist_on else 1
        lib = _lib.load()
        hb = lib.rta_team_handle_bytes()
        handle = ctypes.create_string_buffer(hb)
        ptr = ctypes.c_void_p()
        check(lib.rta_team_create(self.rank, self.world, capacity_bytes, ctypes.byref(ptr), handle))
        self._ptr = ptr
        if self.world > 1:
            handles: list = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            if any(len(h) != hb for h in handles):
                raise ValueError("team handles of unexpected size")
            joined = ctypes.create_string_buffer(b"".join(handles), hb * self.world)
            check(lib.rta_team_connect(ptr, joined))
            dist.barrier(group=group)

    def _stream(self):
        import torch
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def allreduce(self, partial, addend=None, out=None):
        """out = addend + sum over ranks of partial (same bits on every rank)."""
        import torch
        from .ops import _ptr
        out = torch.empty_like(partial) if out is None else out
        check(_lib.load().rta_team_allreduce_f32(self._ptr, _ptr(partial), _ptr(addend), _ptr(out),
                                                 partial.numel(), self._stream()))
        return out

    def argmax(self, ids, best, id_base: int):
        """Global (ids, best) from every rank's local argmax over rows starting at id_base."""
        import torch
        from .ops import _ptr
        out_ids = torch.empty_like(ids)
        out_best = torch.empty_like(best)
        check(_lib.load().rta_team_argmax(self._ptr, _ptr(ids), _ptr(best), id_base, ids.numel(), _ptr(out_ids),
                                          _ptr(out_best), self._stream()))
        return out_ids, out_best

    def error(self) -> int:
        """Device error word of the exchanges so far (synchronizes; cleared after reading)."""
        word = ctypes.c_uint32(0)
        check(_lib.load().rta_team_error(self._ptr, self._stream(), ctypes.byref(word)))
        return int(word.value)

    def close(self) -> None:
        if self._ptr is None:
            return
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        lib = _lib.load()
        status = lib.rta_team_disconnect(self._ptr)
        if self.world > 1:
            dist.barrier(group=self.group)  # no peer still maps this rank's buffer
        lib.rta_team_destroy(self._ptr)
        self._ptr = None
        check(status)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class ShardedMLP:
    """One SwiGLU MLP layer split over a team: y = residual + Wd swiglu(Wg x, Wu x).
    wg, wu [middle x hidden] and wd [hidden x middle] are the whole row-major
    GGUF matrices (uint8 tensors, on any device); each rank keeps its slice."""

    def __init__(self, team: Team, fmt: int, wg, wu, wd, hidden: int, middle: int, batch: int):
        import torch
        from . import ops
        self.team, self.fmt, self.hidden, self.batch = team, fmt, hidden, batch
        self.start, self.count = split_units(middle, MIDDLE_UNIT, team.world)[team.rank]
        dev = torch.device("cuda", torch.cuda.current_device())
        g = slice_rows(fmt, wg, middle, hidden, self.start, self.count).to(dev)
        u = slice_rows(fmt, wu, middle, hidden, self.start, self.count).to(dev)
        d = slice_columns(fmt, wd, hidden, middle, self.start, self.count).to(dev)
        self.tc = batch >= TC_MIN_BATCH
        relay = ops.panel_weights if self.tc else ops.tile_weights
        self.code, self.wg = relay(fmt, g, self.count, hidden)
        _, self.wu = relay(fmt, u, self.count, hidden)
        _, self.wd = relay(fmt, d, hidden, self.count)
        self.partial = torch.empty(batch, hidden, dtype=torch.float32, device=dev)
        self.act = None if self.tc else torch.empty(batch, self.count, dtype=torch.float32, device=dev)
        lib = _lib.load()
        self.workspace = (torch.empty(lib.rta_mlp_tc_workspace_bytes(self.code, batch, hidden, self.count),
                                      dtype=torch.uint8, device=dev) if self.tc else None)

    def __call__(self, x, residual=None, out=None):
        from . import ops
        x = x.reshape(self.batch, self.hidden)
        if self.tc:
            ops.mlp_tc(self.code, self.wg, self.wu, self.wd, self.hidden, self.count, x, y=self.partial,
                       workspace=self.workspace)
        else:
            ops.mlp_swiglu(self.code, self.wg, self.wu, self.wd, self.hidden, self.count, x, y=self.partial,
                           act=self.act)
        return self.team.allreduce(self.partial, residual, out)


class ShardedReadout:
    """The vocabulary readout split over a team: per batch row the id of the
    largest logit (ties -> lowest id) and its value, on every rank."""

    def __init__(self, team: Team, fmt: int, w, vocab: int, hidden: int, batch: int):
        import torch
        from . import ops
        self.team, self.hidden, self.batch = team, hidden, batch
        self.start, self.count = split_units(vocab, VOCAB_UNIT, team.world)[team.rank]
        dev = torch.device("cuda", torch.cuda.current_device())
        part = slice_rows(fmt, w, vocab, hidden, self.start, self.count).to(dev)
        self.tc = batch >= TC_MIN_BATCH
        self.code, self.w = (ops.panel_weights if self.tc else ops.tile_weights)(fmt, part, self.count, hidden)
        lib = _lib.load()
        nbytes = (lib.rta_gemm_tc_workspace_bytes(self.code, batch, hidden) if self.tc
                  else lib.rta_readout_workspace_bytes(batch))
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def local(self, x):
        """This rank's best row (local ids) and value per batch row."""
        from . import ops
        x = x.reshape(self.batch, self.hidden)
        if self.tc:
            _, ids, best = ops.gemm_tc(self.code, self.w, self.count, self.hidden, x, argmax=True, store=False,
                                       workspace=self.workspace)
        else:
            _, ids, best = ops.readout(self.code, self.w, self.count, self.hidden, x, logits=False,
                                       workspace=self.workspace)
        return ids, best

    def __call__(self, x):
        ids, best = self.local(x)
        return self.team.argmax(ids, best, self.start)


__all__ = ["split_units", "slice_rows", "slice_columns", "Team", "ShardedMLP", "ShardedReadout",
           "MIDDLE_UNIT", "VOCAB_UNIT", "TC_MIN_BATCH", "TILED", "PANEL"]
