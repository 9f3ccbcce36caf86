"""WorkerClient: a Python client of the native worker's pipe protocol, for rta_worker.

The reference drives its native worker through ray_tracing.runtime.ResidentRuntime
(resident_runtime.py:10): a subprocess spoken to over stdin/stdout with a 5-word
hello, <3I op,count,debug> requests and <2I status,size> replies
(optical_resident.cpp:964-971).  rta_worker serves that protocol from the B200
library; this client speaks it too, so tests and tools can exercise the worker
exactly as the runtime does without importing the reference.  Reply layouts
follow the runtime's parsers (resident_runtime.py:116-345).
"""
from __future__ import annotations

import json
import os
import struct
import subprocess
from pathlib import Path

import numpy as np

from . import assets

HELLO_MAGIC = 0x5254523A
ATTENTION_MAGIC = 0x41545231


def worker_path() -> Path:
    return Path(__file__).with_name("rta_worker")


class WorkerError(RuntimeError):
    pass


class WorkerClient:
    """One rta_worker process serving one model directory (model.json + payloads)."""

    def __init__(self, directory, capacity: int = 300, attention_block: int = 128, worker=None, cache: bool = True):
        directory = Path(directory)
        self.spec = assets.Spec.from_dict(json.loads((directory / "model.json").read_text())["model_spec"])
        self.capacity = capacity
        self.attention_block = attention_block
        env = dict(os.environ, RT_ATTENTION_BLOCK=str(attention_block))
        self._p = subprocess.Popen([str(worker or worker_path()), str(directory / "optical_model.bin"),
                                    str(directory / "vocabulary.bin"), str(capacity), str(int(cache))],
                                   stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.PIPE, env=env)
        hello = self._read(20)
        magic, depth, blocks, middle, mode = struct.unpack("<5I", hello)
        if magic != HELLO_MAGIC or depth != self.spec.depth or middle != self.spec.middle_size:
            raise WorkerError(f"unexpected hello {hello.hex()}")
        self.mode = mode

    # ------------------------------------------------------------ framing
    def _read(self, n: int) -> bytes:
        data = self._p.stdout.read(n)
        if data is None or len(data) != n:
            raise WorkerError("worker closed its output: " + self._p.stderr.read().decode(errors="replace")[-400:])
        return data

    def request(self, op: int, count: int = 0, debug: int = 0, body: bytes = b"") -> bytes:
        self._p.stdin.write(struct.pack("<3I", op, count, debug) + body)
        self._p.stdin.flush()
        status, size = struct.unpack("<2I", self._read(8))
        payload = self._read(size) if size else b""
        if status:
            raise WorkerError(f"worker op {op} failed (status {status})")
        return payload

    def close(self):
        if self._p.poll() is None:
            try:
                self._p.stdin.write(struct.pack("<3I", 0, 0, 0))
                self._p.stdin.flush()
                self._p.wait(timeout=60)
            except Exception:
                self._p.kill()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -------------------------------------------------------- operations
    def prefill(self, ids, stops=()):
        ids = np.ascontiguousarray(ids, "<u4")
        st = np.array((list(stops)[:2] + [0xFFFFFFFF] * 2)[:2], "<u4")
        payload = self.request(1, ids.size, 0, ids.tobytes() + st.tobytes())
        timing = np.frombuffer(payload, "<f8", count=6)
        control = np.frombuffer(payload, "<u4", count=8, offset=48)
        # history-cache counters after the batch and feature words (resident_runtime.py:134-147)
        c = np.frombuffer(payload, "<u8", count=10, offset=80 + 32 + 16)
        return dict(gpu_ms=float(timing[1]), wall_ms=float(timing[2]), control=control,
                    cache_hit=bool(timing[4]), cached_prefix_tokens=int(timing[5]), stable_prefix_tokens=int(c[0]),
                    snapshot_kind=int(c[1]), shared_blocks=int(c[2]), saved_boundaries=int(c[3]),
                    boundaries=int(c[4]), computed_tokens=int(c[6]), address_hit=int(
                        np.frombuffer(payload, "<u8", count=2, offset=80 + 32 + 16 + 64 + 8)[1]))

    def generate(self, count: int):
        """Op 2: one GenerationPacket (optical_resident.cpp:63-71)."""
        payload = self.request(2, count)
        control = np.frombuffer(payload, "<u4", count=8, offset=18 * 8)
        n = int(control[1])
        ids = np.frombuffer(payload, "<u4", count=64, offset=18 * 8 + 32)[:n].copy()
        time = np.frombuffer(payload, "<f8", count=18)
        cache = np.frombuffer(payload, "<u4", count=4, offset=18 * 8 + 32 + 256 + 20 + 32)
        return dict(ids=ids, running=bool(control[2]), gpu_ms=float(time[0]), reply_cache_hit=bool(time[5]),
                    cached_tokens=int(cache[0]), tree_queries=int(cache[1]), cache_nodes=int(cache[2]))

    def finish_history(self):
        """Op 13: (saved, tokens, boundaries)."""
        payload = self.request(13, 0)
        v = np.frombuffer(payload, "<u8", count=3)
        return int(v[0]), int(v[1]), int(v[2])

    def mlp(self, x, layer: int = 0):
        x = np.ascontiguousarray(x, "<f4").reshape(-1, self.spec.hidden_size)
        rows, D, F = x.shape[0], self.spec.hidden_size, self.spec.middle_size
        payload = self.request(6, rows, layer, x.tobytes())
        out = np.frombuffer(payload, "<f4", count=rows * D).reshape(rows, D)
        act = np.frombuffer(payload, "<f4", count=rows * F, offset=rows * D * 4).reshape(rows, F)
        hits = np.frombuffer(payload, "<u4", count=rows, offset=rows * (D + F) * 4)
        return dict(output=out.copy(), activation=act.copy(), feature_hits=hits.copy())

    def resources(self):
        return np.frombuffer(self.request(8), "<u8").copy()

    def grow(self, capacity: int):
        payload = self.request(10, capacity)
        self.capacity = capacity
        return np.frombuffer(payload, "<f8", count=3)

    def attention(self, query, keys, values, gate=None, *, layer=None, query_start=None, history_start=0):
        """Op 14 with the runtime's request body and reply checks (resident_runtime.py:265-345)."""
        s = self.spec
        H, KVH, hd = s.attention_heads, s.kv_heads, s.attention_head_dim
        q = np.ascontiguousarray(query, "<f4").reshape(-1, H, hd)
        k = np.ascontiguousarray(keys, "<f4").reshape(-1, KVH, hd)
        v = np.ascontiguousarray(values, "<f4").reshape(-1, KVH, hd)
        g = np.zeros_like(q) if gate is None else np.ascontiguousarray(gate, "<f4").reshape(q.shape)
        layer = s.full_layers[0] if layer is None else layer
        if query_start is None:
            query_start = history_start + len(k) - len(q)
        if len(k) > self.capacity:
            self.grow(len(k))
        body = struct.pack("<4I", len(k), query_start, history_start, 0) + q.tobytes() + k.tobytes() + \
            v.tobytes() + g.tobytes()
        payload = self.request(14, len(q), layer, body)
        header = np.frombuffer(payload, "<u4", count=12)
        magic, rows, count, heads, kvh, dim, pbytes, block, stride, records, legacy, error = map(int, header)
        blk = self.attention_block
        want_records = heads * sum((min(query_start - history_start + r + 1, self.capacity) + blk - 1) // blk
                                   for r in range(len(q)))
        if (magic, rows, count, heads, kvh, dim, block, stride) != (ATTENTION_MAGIC, len(q), len(k), H, KVH, hd, blk,
                                                                    hd + 8 + blk // 32):
            raise WorkerError("full-attention diagnostic protocol mismatch")
        if records != want_records or legacy != int(history_start == 0) or error:
            raise WorkerError("full-attention diagnostic coverage mismatch")
        timing = np.frombuffer(payload, "<f8", count=4, offset=48)
        offset = 80

        def take(dtype, shape):
            nonlocal offset
            a = np.frombuffer(payload, dtype, count=int(np.prod(shape)), offset=offset).copy().reshape(shape)
            offset += a.nbytes
            return a
        result = dict(output=take("<f4", (rows, heads, dim)), physical=take("<f4", (rows, heads, 2)),
                      legacy_output=take("<f4", (rows, heads, dim)), legacy_physical=take("<f4", (rows, heads, 2)),
                      history_packets=take("u1", (count, pbytes)), receipts=take("<u4", (records, stride)),
                      gpu_ms=float(timing[0]))
        if offset != len(payload):
            raise WorkerError("unexpected full-attention diagnostic payload size")
        return result
