"""Record one rta_worker session for the protocol replay test (needs a GPU).

    python tests/golden/make_worker_session.py [--out tests/golden/worker_session.npz]

rta_worker is started with the argv the reference runtime uses
(ray_tracing/runtime/resident_runtime.py:37-39: asset, vocabulary, capacity,
cache, routing, aperture, word tile, feature tile, readout unroll, readout
words, prefill batch, matrix rows) on a small synthetic model, and driven with
the exact request bytes that ResidentRuntime's methods write for the session
listed in SESSION (resident_runtime.py:110-392: prefill with and without
checkpoints and layer capture, a repeated prefill and its replayed reply (the
worker runs with its caches on, as the runtime starts it), generate, stream,
grow, finish_history, mlp, vocabulary, attention, resources, quit).  Every request and every reply byte is
stored, with the model.json the runtime reads.  tests/test_runtime_replay.py
then runs the unmodified ResidentRuntime against a replay of these bytes: it
must write the same requests and parse every reply.
"""
from __future__ import annotations

import argparse
import json
import os
import struct
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "ray-tracing-attention_b200"))

SEED = 57
CAPACITY = 32  # ResidentRuntime raises capacity to at least 32


def session_spec():
    from rta_b200 import assets
    return assets.Spec("qwen35", 512, 1024, 4096, ("recurrent", "full"), 16, 4, 256, 64, state_heads=16,
                       state_key_heads=16)


def session_inputs(spec):
    """Seeded inputs of every call of the session (the replay test rebuilds them)."""
    rng = np.random.default_rng(SEED)
    V, D = spec.vocabulary_size, spec.hidden_size
    H, KVH, hd = spec.attention_heads, spec.kv_heads, spec.attention_head_dim
    return dict(
        prompt=rng.integers(0, V, 12).astype(np.uint32),
        prompt_ckpt=rng.integers(0, V, 9).astype(np.uint32),
        prompt_marks=rng.integers(0, V, 7).astype(np.uint32),
        prompt_debug=rng.integers(0, V, 6).astype(np.uint32),
        prompt_long=rng.integers(0, V, 40).astype(np.uint32),   # beyond capacity 32: the runtime grows first
        mlp_x=rng.normal(0, 0.25, (3, D)).astype(np.float32),
        hidden=rng.normal(0, 1, D).astype(np.float32),
        q=rng.normal(0, 1, (2, H, hd)).astype(np.float32),
        k=rng.normal(0, 1, (20, KVH, hd)).astype(np.float32),
        v=rng.normal(0, 1, (20, KVH, hd)).astype(np.float32),
        gate=rng.normal(0, 1, (2, H, hd)).astype(np.float32),
    )


def requests(spec, x, stop_id):
    """(name, request bytes, reply frames) in session order, encoded as the runtime's
    methods encode them."""
    req = lambda op, count, debug=0, body=b"": struct.pack("<3I", op, count, debug) + body
    stops = lambda s: struct.pack("<2I", *((list(s)[:2] + [0xFFFFFFFF] * 2)[:2]))
    out = [
        ("prefill", req(1, 12, 0, x["prompt"].tobytes() + stops(())), 1),
        ("generate", req(2, 8, 0), 1),
        # the same prompt again: a boundary hit, then the reply replayed from the reply tree
        ("prefill_again", req(1, 12, 0, x["prompt"].tobytes() + stops(())), 1),
        ("generate_replay", req(2, 8, 0), 1),
        ("stream", req(9, 4, 3), 4),
        ("prefill_checkpoint", req(11, 9, 0, x["prompt_ckpt"].tobytes() + stops((stop_id,)) + struct.pack("<I", 5)),
         1),
        ("generate_to_stop", req(2, 6, 0), 1),
        ("finish_after_stop", req(13, 0), 1),
        ("prefill_boundaries", req(12, 7, 0, x["prompt_marks"].tobytes() + stops(()) +
                                   struct.pack("<I", 2) + struct.pack("<4I", 3, 1, 6, 2)), 1),
        ("prefill_layers", req(1, 6, 1, x["prompt_debug"].tobytes() + stops(())), 1),
        ("finish_history", req(13, 0), 1),
        ("mlp", req(6, 3, 1, x["mlp_x"].tobytes()), 1),
        ("vocabulary", req(4, 1, 0, x["hidden"].tobytes()), 1),
        ("resources", req(8, 0), 1),
        ("attention", req(14, 2, 1, struct.pack("<4I", 20, 18, 0, 0) + x["q"].tobytes() + x["k"].tobytes() +
                          x["v"].tobytes() + x["gate"].tobytes()), 1),
        ("grow", req(10, 64), 1),
        ("prefill_long", req(1, 40, 0, x["prompt_long"].tobytes() + stops(())), 1),
        ("generate_after_grow", req(2, 3, 0), 1),
    ]
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE / "worker_session.npz"))
    args = ap.parse_args()
    import torch
    from rta_b200 import _build, assets
    from rta_b200.model import ResidentModel
    _build.build_all()
    spec = session_spec()
    layout = assets.plan(spec, SEED)
    mats, basis = assets.generate_device(layout, SEED)
    x = session_inputs(spec)
    with tempfile.TemporaryDirectory() as tmp:
        d = Path(tmp)
        asset = assets.write_files(d, layout, mats.cpu().numpy(), basis.cpu().numpy())
        # a stop id the checkpointed prompt's continuation reaches (its third token)
        lib = ResidentModel.from_payloads(spec, layout.params(), mats, basis, CAPACITY, history="packet")
        lib.prefill(x["prompt_ckpt"])
        stop_id = int(lib.generate(6)[2])
        lib.close()
        del mats, basis
        torch.cuda.empty_cache()
        argv = [str(_build.WORKER), str(asset.resolve()), str((d / "vocabulary.bin").resolve()), str(CAPACITY), "1",
                "rt_full", "0.08", "32", "8", "1", "4", "512", "8"]
        env = dict(os.environ, RT_ATTENTION_BACKEND="standard", RT_ATTENTION_BLOCK="128", RT_ATTENTION_STATS="0",
                   RT_MLP_BACKEND="standard", RT_ATTENTION_V_MEMBERS="0")
        p = subprocess.Popen(argv, stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.PIPE, env=env)

        def read(n):
            data = p.stdout.read(n)
            if len(data) != n:
                raise RuntimeError("worker ended: " + p.stderr.read().decode(errors="replace"))
            return data
        hello = read(20)
        names, reqs, replies = [], [], []
        for name, blob, frames in requests(spec, x, stop_id):
            p.stdin.write(blob)
            p.stdin.flush()
            got = b""
            for _ in range(frames):
                head = read(8)
                status, size = struct.unpack("<2I", head)
                if status:
                    raise RuntimeError(f"{name}: status {status}: " + p.stderr.read1().decode(errors="replace"))
                got += head + read(size)
            names.append(name)
            reqs.append(np.frombuffer(blob, np.uint8))
            replies.append(np.frombuffer(got, np.uint8))
        p.stdin.write(struct.pack("<I", 0))
        p.stdin.flush()
        p.wait(timeout=30)
        model_json = (d / "model.json").read_text()
    np.savez_compressed(args.out, names=np.array(names), hello=np.frombuffer(hello, np.uint8),
                        model_json=np.array(model_json), stop_id=stop_id,
                        **{f"request_{i}": r for i, r in enumerate(reqs)},
                        **{f"reply_{i}": r for i, r in enumerate(replies)})
    print(f"recorded {len(names)} requests -> {args.out}")


if __name__ == "__main__":
    main()
