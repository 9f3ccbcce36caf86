"""The reference's own runtime parses rta_worker's replies (drop-in boundary).

tests/golden/worker_session.npz holds one rta_worker session recorded on a B200
(tests/golden/make_worker_session.py): the exact request bytes the reference's
ResidentRuntime writes for a session of prefill (plain, checkpointed op 11,
boundary-marked op 12, layer capture), generate, stream, finish_history, mlp,
vocabulary, resources, attention, grow and quit, and every reply byte the
worker sent back.  Here the unmodified ray_tracing.runtime.ResidentRuntime is
run against a fake worker process that replays those replies: the runtime's
build step is patched to name a worker (as the reference's own verifier does
with a pinned worker, verify_attention_receipts.py:364-375), every byte the
runtime writes must equal the recorded request, and every reply must parse
into the values the recording holds.

The reference package must be importable: a checkout named "reference" beside
this repository, or the directory in the RTA_REFERENCE environment variable.
Without it the test is skipped.  CPU only; nothing here launches GPU work.
"""
import json
import os
import struct
import sys
from pathlib import Path
from unittest import mock

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

SESSION = GOLDEN / "worker_session.npz"


def _reference_root():
    cand = os.environ.get("RTA_REFERENCE")
    root = Path(cand) if cand else ROOT.parent / "reference"
    return root if (root / "ray_tracing" / "runtime" / "resident_runtime.py").exists() else None


REFERENCE = _reference_root()
pytestmark = pytest.mark.skipif(REFERENCE is None or not SESSION.exists(),
                                reason="reference checkout or recorded worker session not available")


class ReplayWorker:
    """subprocess.Popen stand-in: checks every byte the runtime writes against the
    recorded requests, and releases a request's recorded reply once the request is
    complete."""

    def __init__(self, argv, hello, requests, replies):
        self.argv = argv
        self.expected = b"".join(requests) + struct.pack("<I", 0)
        self.ends = list(np.cumsum([len(r) for r in requests]))
        self.replies = replies
        self.written = bytearray()
        self.out = bytearray(hello)
        self.served = 0
        self.returncode = None
        worker = self

        class In:
            def write(self, b):
                worker.written += b
                n = len(worker.written)
                assert worker.expected.startswith(bytes(worker.written)), (
                    f"request bytes diverge from the recording within byte {n}")
                while worker.served < len(worker.ends) and n >= worker.ends[worker.served]:
                    worker.out += worker.replies[worker.served]
                    worker.served += 1
                if bytes(worker.written) == worker.expected:
                    worker.returncode = 0  # quit received
                return len(b)

            def flush(self):
                pass

            def close(self):
                pass

        class Out:
            def read(self, n):
                assert len(worker.out) >= n, "the runtime reads a reply the worker never sent"
                data = bytes(worker.out[:n])
                del worker.out[:n]
                return data

            def close(self):
                pass

        self.stdin, self.stdout = In(), Out()

    def poll(self):
        return self.returncode

    def wait(self, timeout=None):
        return 0

    def kill(self):
        self.returncode = -9


def test_reference_runtime_parses_every_worker_reply(tmp_path):
    sys.dont_write_bytecode = True
    if str(REFERENCE) not in sys.path:
        sys.path.insert(0, str(REFERENCE))
    from ray_tracing.runtime import resident_runtime as rr
    sys.path.insert(0, str(GOLDEN))
    import make_worker_session as mws

    g = np.load(SESSION)
    names = [str(n) for n in g["names"]]
    reqs = [g[f"request_{i}"].tobytes() for i in range(len(names))]
    reps = [g[f"reply_{i}"].tobytes() for i in range(len(names))]
    (tmp_path / "model.json").write_text(str(g["model_json"]))
    asset = tmp_path / "optical_model.bin"
    asset.write_bytes(b"")  # the runtime only passes the path on to the worker
    spec = mws.session_spec()
    x = mws.session_inputs(spec)
    stop_id = int(g["stop_id"])
    launched = []

    def popen(argv, **kwargs):
        launched.append(argv)
        return ReplayWorker(argv, g["hello"].tobytes(), reqs, reps)

    with mock.patch("ray_tracing.compiler.build.build", return_value=tmp_path / "rta_worker"), \
            mock.patch.object(rr.subprocess, "Popen", side_effect=popen):
        rt = rr.ResidentRuntime(asset, capacity=mws.CAPACITY)
    assert Path(launched[0][0]).name == "rta_worker" and launched[0][3] == str(mws.CAPACITY)
    assert rt.metadata["depth"] == spec.depth and rt.metadata["mlp_backend"] == "standard"
    assert rt.metadata["detector_mode"] == "ordered"

    def reply_payload(i, frame=0):
        data, at = reps[i], 0
        for _ in range(frame + 1):
            status, size = struct.unpack_from("<2I", data, at)
            payload = data[at + 8:at + 8 + size]
            at += 8 + size
        return payload

    r = rt.prefill(x["prompt"])
    assert r["control"][4] == 0xFFFFFFFF and r["prefill_query_positions"] == 12
    assert r["prefill_cache_hit"] is False and r["history_saved_boundaries"] == 1
    assert r["prefill_computed_tokens"] == 12 and r["stable_prefix_tokens"] == 12
    gen = rt.generate(8)
    ids8 = np.frombuffer(reply_payload(names.index("generate")), "<u4", count=8, offset=176)
    assert np.array_equal(gen["ids"], ids8) and len(gen["ids"]) == 8 and rt.position == 20
    assert gen["cached_tokens"] == 0 and gen["compute_tokens"] == 8 and gen["cache_nodes"] == 8
    # the reference's cache check (benchmark_attention_receipts.py:130-150)
    hit = rt.prefill(x["prompt"])
    assert hit["prefill_cache_hit"] is True and hit["cached_prefix_tokens"] == 12
    assert hit["history_address_hit"] == 1 and hit["prefill_computed_tokens"] == 0 and hit["prefill_snapshot_kind"] == 1
    replay = rt.generate(8)
    assert np.array_equal(replay["ids"], gen["ids"]) and replay["reply_cache_hit"] is True
    assert replay["cached_tokens"] == 8 and replay["compute_tokens"] == 0 and replay["tree_cache_hits"] == 8
    stream = list(rt.stream_generate(4))
    assert [len(s["ids"]) for s in stream] == [1, 1, 1, 1] and rt.position == 24
    assert stream[0]["cache_state_tokens"] == 8  # the replayed reply is computed before the stream goes on
    r = rt.prefill(x["prompt_ckpt"], stops=(stop_id,), checkpoint_tokens=5)
    assert r["stable_prefix_tokens"] == 5 and r["prefill_cache_hit"] is False
    gen = rt.generate(6)
    assert len(gen["ids"]) == 3 and int(gen["ids"][-1]) == stop_id and gen["control"][2] == 0
    fh = rt.finish_history()  # prompt + reply, the stop id left out
    assert fh["history_output_saved"] == 1 and fh["history_output_tokens"] == 9 + 2
    r = rt.prefill(x["prompt_marks"], checkpoint_boundaries=[(3, 1), (6, 2)])
    assert r["prefill_computed_tokens"] == 7 and r["stable_prefix_tokens"] == 3
    r = rt.prefill(x["prompt_debug"], debug=True)
    assert r["state"].shape == (6, spec.hidden_size) and r["layers"].shape == (spec.depth, 6, spec.hidden_size)
    assert np.all(np.isfinite(r["state"])) and np.all(np.isfinite(r["layers"]))
    # the final-normed rows have unit RMS times the output norm weight: not all zero, not raw residuals
    assert np.all(np.linalg.norm(r["state"], axis=1) > 0)
    fh = rt.finish_history()
    assert fh["history_output_saved"] == 0
    m = rt.mlp(x["mlp_x"], layer=1)
    assert m["output"].shape == (3, spec.hidden_size) and m["activation"].shape == (3, spec.middle_size)
    assert np.all(m["feature_hits"] == spec.middle_size)
    voc = rt.vocabulary(x["hidden"])
    assert voc["hit_count"] == spec.vocabulary_size and 0 <= voc["token"] < spec.vocabulary_size
    assert np.array_equal(voc["restored_query"], x["hidden"])  # the query packets are its bits
    res = rt.resources()
    assert res["attention_block"] == 128 and res["history_path_packet_bytes"] > 0
    att = rt.attention(x["q"], x["k"], x["v"], x["gate"], layer=1)
    assert att["output"].shape == (2, spec.attention_heads, spec.attention_head_dim)
    assert att["receipt_format"] == "dense" and att["legacy_available"]
    assert att["history_packets"].shape == (20, spec.kv_heads * (144 + 210))
    r = rt.prefill(x["prompt_long"])  # beyond capacity 32: grows to 64 first (op 10), then prefills
    assert rt.capacity == 64 and rt.growth_events[-1]["previous"] == 32
    gen = rt.generate(3)
    assert len(gen["ids"]) == 3 and rt.position == 43
    rt.close()
    assert launched and rt.process.served == len(names) and rt.process.returncode == 0
