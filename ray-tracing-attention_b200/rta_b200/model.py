"""ResidentModel: Python handle over the rta_model_* C-ABI (one model, one GPU)."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import _lib, assets


class ModelSpecC(ctypes.Structure):
    """Mirror of rta_model_spec (include/rta.h)."""
    _fields_ = [("hidden_size", ctypes.c_uint32), ("middle_size", ctypes.c_uint32),
                ("vocabulary_size", ctypes.c_uint32), ("depth", ctypes.c_uint32),
                ("attention_heads", ctypes.c_uint32), ("kv_heads", ctypes.c_uint32),
                ("attention_head_dim", ctypes.c_uint32), ("rotary_dim", ctypes.c_uint32),
                ("state_heads", ctypes.c_uint32), ("state_key_heads", ctypes.c_uint32),
                ("state_head_dim", ctypes.c_uint32), ("attention_gate", ctypes.c_uint32),
                ("qk_norm", ctypes.c_uint32), ("rope_theta", ctypes.c_float), ("norm_epsilon", ctypes.c_float),
                ("layer_kinds", ctypes.c_uint8 * 256)]

    @classmethod
    def from_spec(cls, s: assets.Spec) -> "ModelSpecC":
        c = cls(s.hidden_size, s.middle_size, s.vocabulary_size, s.depth, s.attention_heads, s.kv_heads,
                s.attention_head_dim, s.rotary_dim, s.state_heads, s.state_key_heads, s.state_head_dim,
                int(s.attention_gate), int(s.qk_norm), float(s.rope_theta), float(s.norm_epsilon))
        for i, k in enumerate(s.layer_types):
            c.layer_kinds[i] = 1 if k == "full" else 2
        return c


_P, _U32, _SZ, _I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_size_t, ctypes.c_int
_SIGS = {
    "rta_model_last_error": (ctypes.c_char_p, []),
    "rta_model_open": (_I, [ctypes.POINTER(ModelSpecC), _P, _SZ, _P, _SZ, _P, _SZ, _U32, _I, ctypes.POINTER(_P)]),
    "rta_model_open_batch": (_I, [ctypes.POINTER(ModelSpecC), _P, _SZ, _P, _SZ, _P, _SZ, _U32, _U32, _I,
                                  ctypes.POINTER(_P)]),
    "rta_model_open_team": (_I, [ctypes.POINTER(ModelSpecC), _P, _SZ, _P, _SZ, _P, _SZ, _U32, _U32, _P, _P, _U32,
                                 _I, ctypes.POINTER(_P)]),
    "rta_model_open_ex": (_I, [ctypes.POINTER(ModelSpecC), _P, _SZ, _P, _SZ, _P, _SZ, _U32, _U32, _U32, _I,
                               ctypes.POINTER(_P)]),
    "rta_model_attention": (_I, [_P, _U32, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _P, _P, _P, _P,
                                 ctypes.POINTER(_U32), ctypes.POINTER(ctypes.c_double)]),
    "rta_model_debug_attention": (_I, [_P, _U32, _P, _P, _P, _P, ctypes.POINTER(_U32)]),
    "rta_model_prefill_batch": (_I, [_P, _P, _P, _U32, _P, ctypes.POINTER(ctypes.c_double)]),
    "rta_model_seed_history": (_I, [_P, _P, ctypes.c_uint64]),
    "rta_model_generate_batch": (_I, [_P, _U32, _P, _P, ctypes.POINTER(ctypes.c_double)]),
    "rta_model_open_files": (_I, [ctypes.POINTER(ModelSpecC), ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                  _U32, _I, ctypes.POINTER(_P)]),
    "rta_model_close": (None, [_P]),
    "rta_model_prefill": (_I, [_P, _P, _U32, _P, ctypes.POINTER(ctypes.c_double)]),
    "rta_model_generate": (_I, [_P, _U32, _P, ctypes.POINTER(_U32), ctypes.POINTER(ctypes.c_double)]),
    "rta_model_prefill_capture": (_I, [_P, _P, _U32, _P, _P, _P, ctypes.POINTER(ctypes.c_double)]),
    "rta_model_profile_step": (_I, [_P, _P, _P, _P, _SZ, ctypes.POINTER(_SZ)]),
    "rta_model_mlp": (_I, [_P, _U32, _P, _U32, _P, _P]),
    "rta_model_vocabulary": (_I, [_P, _P, _P, ctypes.POINTER(_U32), ctypes.POINTER(ctypes.c_float)]),
    "rta_model_state": (_I, [_P, _P, ctypes.POINTER(_U32)]),
    "rta_model_resources": (_I, [_P, _P, _SZ]),
    "rta_model_prefill_checkpoint": (_I, [_P, _P, _U32, _P, _U32, ctypes.POINTER(ctypes.c_double)]),
    "rta_model_cache_info": (_I, [_P, _P, _SZ, _P]),
    "rta_model_finish_history": (_I, [_P, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                      ctypes.POINTER(ctypes.c_uint64)]),
    "rta_model_cache_limit": (_I, [_P, ctypes.c_uint64]),
    "rta_model_state_address": (_I, [_P, _P, ctypes.POINTER(_U32)]),
}
PACKET_HISTORY = 1  # RTA_MODEL_PACKET_HISTORY
TOKEN_PREFILL = 2   # RTA_MODEL_TOKEN_PREFILL
TC_PREFILL = 4      # RTA_MODEL_TC_PREFILL
SPLIT_ACTIVATIONS = 8  # RTA_MODEL_SPLIT_ACTIVATIONS
CACHE = 16             # RTA_MODEL_CACHE
# RTA_CACHE_* counters (include/rta.h), in index order
CACHE_INFO_NAMES = ("prefill_hit", "reused_tokens", "stable_tokens", "snapshot_kind", "shared_blocks",
                    "saved_boundaries", "boundaries", "lookups", "computed_tokens", "evictions", "address_hit",
                    "replayed_tokens", "tree_queries", "tree_nodes", "tree_capacity", "tree_leaf", "restored_tokens",
                    "checkpoint_restored", "finish_saved", "finish_tokens", "bytes", "digests")
PROFILE_KINDS = ("start", "readout", "embed", "qkv", "attention_prep", "attention", "o_proj", "in_proj",
                 "gated_delta", "out_proj", "gate_up", "down", "exchange")  # RTA_PROF_* (include/rta.h)
RESOURCE_NAMES = ("payload_bytes", "derived_layer_bytes", "history_bytes", "recurrent_state_bytes", "capacity",
                  "attention_splits", "kernels_per_decode_step", "kernels_per_prefill_step", "position",
                  "sequences", "tensor_core_matrices")


def _lib_model():
    lib = _lib.load()
    if not getattr(lib, "_model_sigs", False):
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
        lib._model_sigs = True
    return lib


def _check(status: int):
    if status != 0:
        raise _lib.RtaError(status, _lib_model().rta_model_last_error().decode(errors="replace"))


def _np_ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _current_device() -> int:
    """The caller's current CUDA device (one process per GPU sets it before opening a model)."""
    try:
        import torch
        if torch.cuda.is_available():
            return int(torch.cuda.current_device())
    except ImportError:
        pass
    return 0


class ResidentModel:
    """One resident model on one GPU (prefill / generate / mlp / vocabulary).
    With sequences > 1 the handle decodes that many sequences side by side
    (prefill_batch / seed_history / generate_batch)."""

    def __init__(self, handle, spec: assets.Spec, capacity: int, device: int, sequences: int = 1):
        self._h = handle
        self.spec = spec
        self.capacity = capacity
        self.device = device
        self.sequences = sequences
        self.last_gpu_ms = 0.0

    # ---------------------------------------------------------------- open
    @classmethod
    def from_payloads(cls, spec: assets.Spec, params, matrices, basis, capacity: int, device: int | None = None,
                      sequences: int = 1, history: str = "fp16", token_prefill: bool = False,
                      tc_prefill: bool = False, split_activations: bool = False, cache: bool = False):
        """history: "fp16" K/V rings, or "packet" (the reference's Q4_K/Q6_K history packets).
        token_prefill: prefill one position per step instead of 64-position chunks;
        tc_prefill: the chunks' products on the tensor cores (panel copies of the weights);
        split_activations: batched decode products take x as two fp16 operands;
        cache: prefix boundaries and the reply tree (single sequence; RTA_MODEL_CACHE).
        params: uint32 numpy; matrices/basis: uint8 numpy (host) or torch CUDA tensors (device).
        device: CUDA ordinal (default: the caller's current device)."""
        device = _current_device() if device is None else device
        lib = _lib_model()
        params = np.ascontiguousarray(params, np.uint32)

        def addr(buf):
            if isinstance(buf, np.ndarray):
                b = np.ascontiguousarray(buf, np.uint8)
                return _np_ptr(b), b.nbytes, b
            return ctypes.c_void_p(buf.data_ptr()), buf.numel() * buf.element_size(), buf
        mp, mb, mkeep = addr(matrices)
        bp, bb, bkeep = addr(basis)
        cs = ModelSpecC.from_spec(spec)
        h = ctypes.c_void_p()
        if history not in ("fp16", "packet"):
            raise ValueError("history must be 'fp16' or 'packet'")
        flags = ((PACKET_HISTORY if history == "packet" else 0) | (TOKEN_PREFILL if token_prefill else 0)
                 | (TC_PREFILL if tc_prefill else 0) | (SPLIT_ACTIVATIONS if split_activations else 0)
                 | (CACHE if cache else 0))
        _check(lib.rta_model_open_ex(ctypes.byref(cs), _np_ptr(params), params.size, mp, mb, bp, bb, capacity,
                                     sequences, flags, device, ctypes.byref(h)))
        del mkeep, bkeep
        model = cls(h, spec, capacity, device, sequences)
        model.history = history
        return model

    @classmethod
    def with_team(cls, spec: assets.Spec, params, matrices, basis, capacity: int, sequence_starts, team,
                  device: int | None = None, history: str = "fp16"):
        """Tensor-parallel hybrid handle (rta_model_open_team): this rank decodes the
        attention / recurrent layers of sequences [starts[rank], starts[rank + 1]) and
        a 1/world slice of every MLP and of the vocabulary readout for all of them.
        team: a connected tensor_parallel.Team whose exchanges this handle owns."""
        device = _current_device() if device is None else device
        lib = _lib_model()
        params = np.ascontiguousarray(params, np.uint32)
        starts = np.ascontiguousarray(sequence_starts, np.uint32)

        def addr(buf):
            if isinstance(buf, np.ndarray):
                b = np.ascontiguousarray(buf, np.uint8)
                return _np_ptr(b), b.nbytes, b
            return ctypes.c_void_p(buf.data_ptr()), buf.numel() * buf.element_size(), buf
        mp, mb, mkeep = addr(matrices)
        bp, bb, bkeep = addr(basis)
        cs = ModelSpecC.from_spec(spec)
        h = ctypes.c_void_p()
        flags = PACKET_HISTORY if history == "packet" else 0
        sequences = int(starts[-1])
        _check(lib.rta_model_open_team(ctypes.byref(cs), _np_ptr(params), params.size, mp, mb, bp, bb, capacity,
                                       sequences, _np_ptr(starts), team._ptr, flags, device, ctypes.byref(h)))
        del mkeep, bkeep
        model = cls(h, spec, capacity, device, sequences)
        model.history = history
        model.team = team
        return model

    @classmethod
    def synthetic_team(cls, spec: assets.Spec, seed: int, capacity: int, sequence_starts, team,
                       device: int | None = None, history: str = "fp16"):
        """Random-init model of `spec` (same weights on every rank: generated from the seed)
        opened as a tensor-parallel hybrid handle."""
        import torch
        device = _current_device() if device is None else device
        torch.cuda.set_device(device)
        layout = assets.plan(spec, seed)
        mats, basis = assets.generate_device(layout, seed)
        model = cls.with_team(spec, layout.params(), mats, basis, capacity, sequence_starts, team, device, history)
        model.layout = layout
        del mats, basis
        torch.cuda.empty_cache()
        return model

    @classmethod
    def from_directory(cls, directory, capacity: int, device: int | None = None):
        device = _current_device() if device is None else device
        directory = Path(directory)
        import json
        spec = assets.Spec.from_dict(json.loads((directory / "model.json").read_text())["model_spec"])
        lib = _lib_model()
        cs = ModelSpecC.from_spec(spec)
        h = ctypes.c_void_p()
        _check(lib.rta_model_open_files(ctypes.byref(cs), str(directory / "optical_model.bin").encode(),
                                        str(directory / "geometry_weights.bin").encode(),
                                        str(directory / "vocabulary.bin").encode(), capacity, device,
                                        ctypes.byref(h)))
        return cls(h, spec, capacity, device)

    @classmethod
    def synthetic(cls, spec: assets.Spec, seed: int = 0, capacity: int = 1024, device: int | None = None,
                  sequences: int = 1, history: str = "fp16", token_prefill: bool = False,
                  tc_prefill: bool = False, split_activations: bool = False, cache: bool = False):
        """Random-init model of `spec` generated on the GPU (payloads in the exporter's layout)."""
        import torch
        device = _current_device() if device is None else device
        torch.cuda.set_device(device)
        layout = assets.plan(spec, seed)
        mats, basis = assets.generate_device(layout, seed)
        model = cls.from_payloads(spec, layout.params(), mats, basis, capacity, device, sequences, history,
                                  token_prefill, tc_prefill, split_activations, cache)
        model.layout = layout
        del mats, basis
        torch.cuda.empty_cache()
        return model

    # ----------------------------------------------------------- operations
    def close(self):
        if self._h is not None:
            _lib_model().rta_model_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, ids, stops=(), checkpoint: int | None = None):
        """checkpoint: the stable prefix of worker op 11 (default: the whole prompt)."""
        ids = np.ascontiguousarray(ids, np.uint32)
        st = (list(stops)[:2] + [0xFFFFFFFF] * 2)[:2]
        st = np.array(st, np.uint32)
        ms = ctypes.c_double(0)
        boundary = ids.size if checkpoint is None else int(checkpoint)
        _check(_lib_model().rta_model_prefill_checkpoint(self._h, _np_ptr(ids), ids.size, _np_ptr(st), boundary,
                                                         ctypes.byref(ms)))
        self.last_gpu_ms = ms.value
        return ms.value

    # ------------------------------------------------------------ caches
    def cache_info(self):
        """Counters of the caches' last prefill / generate / finish_history (RTA_CACHE_*),
        plus lookup_ms, tree_ms and restore_ms."""
        out = np.zeros(len(CACHE_INFO_NAMES), np.uint64)
        ms = np.zeros(3, np.float64)
        _check(_lib_model().rta_model_cache_info(self._h, _np_ptr(out), out.size, _np_ptr(ms)))
        info = dict(zip(CACHE_INFO_NAMES, map(int, out)))
        info.update(lookup_ms=float(ms[0]), tree_ms=float(ms[1]), restore_ms=float(ms[2]))
        return info

    def finish_history(self):
        """Save prompt + reply as a prefix boundary (worker op 13): (saved, tokens, boundaries)."""
        a, b, c = ctypes.c_uint64(0), ctypes.c_uint64(0), ctypes.c_uint64(0)
        _check(_lib_model().rta_model_finish_history(self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)))
        return int(a.value), int(b.value), int(c.value)

    def cache_limit(self, nbytes: int):
        _check(_lib_model().rta_model_cache_limit(self._h, int(nbytes)))

    def state_address(self):
        """The 256-bit address of the current decode state (8 uint32) and the position."""
        out = np.zeros(8, np.uint32)
        pos = ctypes.c_uint32(0)
        _check(_lib_model().rta_model_state_address(self._h, _np_ptr(out), ctypes.byref(pos)))
        return out, int(pos.value)

    def prefill_capture(self, ids, stops=(), layers: bool = False):
        """Debug prefill (worker op 1 with debug = 1): returns the final-normed residual
        row of every position [n, D] and, with layers=True, every layer's output rows
        [depth, n, D] (else None)."""
        ids = np.ascontiguousarray(ids, np.uint32)
        st = np.array((list(stops)[:2] + [0xFFFFFFFF] * 2)[:2], np.uint32)
        D = self.spec.hidden_size
        states = np.zeros((ids.size, D), np.float32)
        lay = np.zeros((self.spec.depth, ids.size, D), np.float32) if layers else None
        ms = ctypes.c_double(0)
        _check(_lib_model().rta_model_prefill_capture(self._h, _np_ptr(ids), ids.size, _np_ptr(st), _np_ptr(states),
                                                      _np_ptr(lay) if lay is not None else None, ctypes.byref(ms)))
        self.last_gpu_ms = ms.value
        return states, lay

    def generate(self, count: int):
        out = np.zeros(count, np.uint32)
        n = ctypes.c_uint32(0)
        ms = ctypes.c_double(0)
        _check(_lib_model().rta_model_generate(self._h, count, _np_ptr(out), ctypes.byref(n), ctypes.byref(ms)))
        self.last_gpu_ms = ms.value
        return out[:n.value].copy()

    # ------------------------------------------------------ several sequences
    def prefill_batch(self, prompts, stops=()):
        """prompts: one id sequence per handle sequence (empty = idle)."""
        if len(prompts) != self.sequences:
            raise ValueError("one prompt per sequence")
        lengths = np.array([len(p) for p in prompts], np.uint32)
        stride = max(1, int(lengths.max()))
        ids = np.zeros((self.sequences, stride), np.uint32)
        for z, p in enumerate(prompts):
            ids[z, :len(p)] = np.asarray(p, np.uint32)
        st = np.array((list(stops)[:2] + [0xFFFFFFFF] * 2)[:2], np.uint32)
        ms = ctypes.c_double(0)
        _check(_lib_model().rta_model_prefill_batch(self._h, _np_ptr(ids), _np_ptr(lengths), stride, _np_ptr(st),
                                                    ctypes.byref(ms)))
        self.last_gpu_ms = ms.value
        return ms.value

    def seed_history(self, lengths, seed: int = 0):
        lengths = np.ascontiguousarray(lengths, np.uint32)
        if lengths.size != self.sequences:
            raise ValueError("one history length per sequence")
        _check(_lib_model().rta_model_seed_history(self._h, _np_ptr(lengths), seed))

    def generate_batch(self, count: int):
        """Returns one id array per sequence (shorter where a stop id ended it)."""
        out = np.zeros((self.sequences, count), np.uint32)
        n = np.zeros(self.sequences, np.uint32)
        ms = ctypes.c_double(0)
        _check(_lib_model().rta_model_generate_batch(self._h, count, _np_ptr(out), _np_ptr(n), ctypes.byref(ms)))
        self.last_gpu_ms = ms.value
        return [out[z, :n[z]].copy() for z in range(self.sequences)]

    def profile_step(self, capacity: int = 4096):
        """One decode step of every running sequence with each launch group timed on
        its own: a list of (kind, ms, algorithmic bytes) in launch order."""
        kinds = np.zeros(capacity, np.uint32)
        ms = np.zeros(capacity, np.float64)
        nbytes = np.zeros(capacity, np.float64)
        n = ctypes.c_size_t(0)
        _check(_lib_model().rta_model_profile_step(self._h, _np_ptr(kinds), _np_ptr(ms), _np_ptr(nbytes), capacity,
                                                   ctypes.byref(n)))
        k = min(n.value, capacity)
        return [(PROFILE_KINDS[int(kinds[i])], float(ms[i]), float(nbytes[i])) for i in range(k)]

    def attention(self, query, keys, values, gate=None, *, layer=None, query_start=None, history_start=0,
                  block=128):
        """Full-attention diagnostic (worker op 14): the detector of a full layer over a
        supplied compact history; returns output, physical, history_packets and dense
        receipts shaped like ResidentRuntime.attention's result."""
        s = self.spec
        H, KVH, hd = s.attention_heads, s.kv_heads, s.attention_head_dim
        q = np.ascontiguousarray(query, np.float32).reshape(-1, H, hd)
        k = np.ascontiguousarray(keys, np.float32).reshape(-1, KVH, hd)
        v = np.ascontiguousarray(values, np.float32).reshape(-1, KVH, hd)
        g = np.zeros_like(q) if gate is None else np.ascontiguousarray(gate, np.float32).reshape(q.shape)
        if layer is None:
            layer = s.full_layers[0]
        if query_start is None:
            query_start = history_start + len(k) - len(q)
        rows, count = len(q), len(k)
        vis = [min(query_start - history_start + r + 1, self.capacity) for r in range(rows)]
        records = H * sum((n + block - 1) // block for n in vis)
        stride = hd + 8 + block // 32
        out = np.zeros((rows, H, hd), np.float32)
        phys = np.zeros((rows, H, 2), np.float32)
        pbytes = KVH * (144 + 210)
        packets = np.zeros((count, pbytes), np.uint8)
        receipts = np.zeros((records, stride), np.uint32)
        n = ctypes.c_uint32(0)
        ms = ctypes.c_double(0)
        _check(_lib_model().rta_model_attention(self._h, layer, _np_ptr(q), _np_ptr(k), _np_ptr(v), _np_ptr(g), rows,
                                                count, query_start, history_start, block, _np_ptr(out),
                                                _np_ptr(phys), _np_ptr(packets), _np_ptr(receipts), ctypes.byref(n),
                                                ctypes.byref(ms)))
        assert n.value == records
        return dict(output=out, physical=phys, history_packets=packets, receipts=receipts, block=block,
                    stride=stride, query_start=query_start, history_start=history_start, gpu_ms=ms.value,
                    legacy_available=history_start == 0)

    def debug_attention(self, seq: int = 0):
        """Test hook (packet history): q, gate, detector output of the last full layer of the
        last step and that layer's visible history packets, oldest first."""
        s = self.spec
        Q = s.attention_heads * s.attention_head_dim
        q, gate, att = (np.zeros(Q, np.float32) for _ in range(3))
        packets = np.zeros((self.capacity, s.kv_heads * (144 + 210)), np.uint8)
        n = ctypes.c_uint32(0)
        _check(_lib_model().rta_model_debug_attention(self._h, seq, _np_ptr(q), _np_ptr(gate), _np_ptr(att),
                                                      _np_ptr(packets), ctypes.byref(n)))
        return q, gate, att, packets[:n.value].copy()

    def mlp(self, x, layer: int):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.spec.hidden_size)
        y = np.zeros_like(x)
        act = np.zeros((x.shape[0], self.spec.middle_size), np.float32)
        _check(_lib_model().rta_model_mlp(self._h, layer, _np_ptr(x), x.shape[0], _np_ptr(y), _np_ptr(act)))
        return y, act

    def vocabulary(self, hidden, logits: bool = False):
        h = np.ascontiguousarray(hidden, np.float32).reshape(self.spec.hidden_size)
        lg = np.zeros(self.spec.vocabulary_size, np.float32) if logits else None
        arg = ctypes.c_uint32(0)
        best = ctypes.c_float(0)
        _check(_lib_model().rta_model_vocabulary(self._h, _np_ptr(h), _np_ptr(lg) if lg is not None else None,
                                                 ctypes.byref(arg), ctypes.byref(best)))
        return int(arg.value), float(best.value), lg

    def state(self):
        s = np.zeros(self.spec.hidden_size, np.float32)
        pos = ctypes.c_uint32(0)
        _check(_lib_model().rta_model_state(self._h, _np_ptr(s), ctypes.byref(pos)))
        return s, int(pos.value)

    def resources(self):
        out = np.zeros(len(RESOURCE_NAMES), np.uint64)
        _check(_lib_model().rta_model_resources(self._h, _np_ptr(out), out.size))
        return dict(zip(RESOURCE_NAMES, map(int, out)))
