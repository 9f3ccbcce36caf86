"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in the build container, where the reference checkout is importable:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <path-to-reference>

It imports the reference's own CPU code unmodified and records its outputs:
  * gguf-py 0.19.0 gguf.quants.dequantize (the reference's decode dependency,
    ray_tracing/compiler/sources.py:37-40) on Q4_K / Q6_K blocks;
  * verify_attention_receipts.full_attention (FP64 GQA detector oracle,
    ray_tracing/verification/verify_attention_receipts.py:84-114) on the
    reference's own adversarial case generator `cases` (:206-281);
  * the FP64 SwiGLU oracle expression of verify_rt_mlp.py:85-89 on the same
    seeded input rows the reference uses (:63-67);
  * cpu_selftest (:333-361) and ModelSpec geometry (compiler/spec.py) for the
    2B and 9B shapes.
The fixtures land next to this script; the GPU box never needs the reference.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import oracle  # noqa: E402  (test infrastructure: the C restatement)

# Attention cases kept as fixtures (history counts <= 129 keep the files small).
ATTENTION_CASES = ("boundary_1", "boundary_15", "boundary_16", "boundary_17", "boundary_33", "boundary_64",
                   "boundary_65", "zero_q_uniform", "subnormal_and_signed_zero_q",
                   "tiny_q_with_nontrivial_scores", "extreme_scores_and_gates", "gqa_head_identity")


def spec_2b(ModelSpec):
    return ModelSpec("qwen35", 2048, 6144, 151936, ("recurrent", "recurrent", "recurrent", "full") * 6, 16, 4, 256,
                     64, 10000000.0, 1e-6, True, True, 16, 16, 128).validate()


def spec_9b(ModelSpec):
    return ModelSpec("qwen35", 4096, 12288, 151936, ("recurrent", "recurrent", "recurrent", "full") * 8, 16, 4, 256,
                     64, 10000000.0, 1e-6, True, True, 32, 16, 128).validate()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of a checkout of the reference project (holds the ray_tracing package)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    import gguf
    from gguf import GGMLQuantizationType, dequantize
    from ray_tracing.compiler.spec import ModelSpec
    from ray_tracing.verification import verify_attention_receipts as var

    manifest = {"gguf_version": getattr(gguf, "__version__", None) or _dist_version("gguf"),
                "sources": {}}

    # 1. Q4_K / Q6_K blocks from the oracle quantizer, decoded by gguf.
    rng = np.random.default_rng(20261201)
    values = np.concatenate([
        rng.normal(0, 0.02, 64 * 256),
        rng.normal(0, 1.0, 32 * 256),
        rng.uniform(-1e3, 1e3, 16 * 256),
        np.zeros(256), np.full(256, -0.5), np.full(256, 3.0),
        np.where(np.arange(256) % 2, 1e-3, -7.0),
        np.linspace(-4, 4, 256),
    ]).astype(np.float32)
    blocks = {}
    for fmt in (12, 14):
        b = oracle.quantize(fmt, values)
        ref = dequantize(b.reshape(-1, oracle.BLOCK_BYTES[fmt]), GGMLQuantizationType(fmt)).reshape(-1)
        blocks[f"blocks_{fmt}"] = b
        blocks[f"gguf_{fmt}"] = ref.astype(np.float32)
    np.savez_compressed(HERE / "quant_blocks.npz", values=values, **blocks)
    manifest["sources"]["quant_blocks.npz"] = "gguf.quants.dequantize on oracle-quantized blocks"

    # 2. Attention: the reference's adversarial cases through its FP64 oracle.
    spec = spec_2b(ModelSpec)
    out = {}
    names = []
    for case in var.cases(spec, 256):
        if case["name"] not in ATTENTION_CASES:
            continue
        count = len(case["keys"])
        capacity = max(32, 1 << max(0, (count - 1)).bit_length())
        # keep the last (up to) four query rows; each row's oracle is independent
        keep = min(4, len(case["query"]))
        query, gate = case["query"][-keep:], case["gate"][-keep:]
        query_start = case["query_start"] + len(case["query"]) - keep
        dense = var.full_attention(query, case["keys"], case["values"], gate, query_start,
                                   case["history_start"], capacity, spec.attention_gate)
        n = case["name"]
        names.append(n)
        out[f"{n}/query"], out[f"{n}/gate"] = query, gate
        out[f"{n}/keys"], out[f"{n}/values"] = case["keys"], case["values"]
        out[f"{n}/meta"] = np.array([query_start, case["history_start"], capacity], np.int64)
        out[f"{n}/output"] = dense["output"].astype(np.float32)
        out[f"{n}/maximum"] = dense["maximum"].astype(np.float32)
        out[f"{n}/reference"] = dense["reference"].astype(np.float32)
    np.savez_compressed(HERE / "attention_cases.npz", names=np.array(names), **out)
    manifest["sources"]["attention_cases.npz"] = ("verify_attention_receipts.cases(spec_2b, 256) -> "
                                                   "full_attention (FP64)")
    manifest["cpu_selftest"] = {k: (list(v) if isinstance(v, tuple) else v) for k, v in var.cpu_selftest().items()}

    # 3. MLP: FP64 SwiGLU oracle expression on a small Q4_K MLP.
    D, F = 512, 1024
    rng = np.random.default_rng(20261110)
    x = rng.normal(0, 0.25, (32, D)).astype(np.float32)
    x[1] = 0
    x[2] = -x[0]
    x[3] = np.where(np.arange(D) % 2, -0.5, 0.5)
    wrng = np.random.default_rng(7)
    mats = {}
    for name, shape in (("gate", (F, D)), ("up", (F, D)), ("down", (D, F))):
        w = wrng.normal(0, 0.02, shape).astype(np.float32)
        mats[name] = oracle.quantize(12, w)
    deq = {k: dequantize(v.reshape(-1, 144), GGMLQuantizationType.Q4_K).reshape(s).astype(np.float64)
           for (k, v), s in zip(mats.items(), ((F, D), (F, D), (D, F)))}
    xd = x.astype(np.float64)
    gate = xd @ deq["gate"].T
    up = xd @ deq["up"].T
    sig = np.where(gate >= 0, 1 / (1 + np.exp(-np.abs(gate))), np.exp(-np.abs(gate)) / (1 + np.exp(-np.abs(gate))))
    act = gate * sig * up
    y = act @ deq["down"].T
    np.savez_compressed(HERE / "mlp_q4k.npz", x=x, w_gate=mats["gate"], w_up=mats["up"], w_down=mats["down"],
                        activation=act, output=y, shape=np.array([D, F]))
    manifest["sources"]["mlp_q4k.npz"] = "verify_rt_mlp.py:85-89 expression, FP64, gguf-decoded Q4_K weights"

    # 4. Geometry of the benchmark shapes.
    manifest["spec_2b"] = {"history_bytes": spec.history_bytes, "fingerprint": spec.fingerprint,
                           "feed_forward_stride": spec.feed_forward_stride, "working_width": spec.working_width}
    s9 = spec_9b(ModelSpec)
    manifest["spec_9b"] = {"history_bytes": s9.history_bytes, "fingerprint": s9.fingerprint,
                           "feed_forward_stride": s9.feed_forward_stride, "working_width": s9.working_width}
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True))
    print(json.dumps(manifest, indent=1))


def _dist_version(name):
    try:
        from importlib.metadata import version
        return version(name)
    except Exception:
        return None


if __name__ == "__main__":
    main()
