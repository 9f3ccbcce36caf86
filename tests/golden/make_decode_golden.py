"""Generate the model-level decode fixtures at the benchmark sizes.

Run in the build container (CPU only, no reference checkout needed):

    python tests/golden/make_decode_golden.py [--only config4|config5]

The fixtures pin the CUDA engine to the model oracle (oracle/model.py, the C
restatement of the reference's shader math in the reference worker's per-token
schedule) on exactly the models the benchmark decodes.  The models are rebuilt
on the host by oracle.model.synthetic_payloads, which restates the engine's GPU
weight generator bit for bit (a GPU test checks the bytes), so the GPU tests
regenerate the same weights on the device instead of loading gigabytes.

  decode_config4.npz  benchmark config 4: the 2B-shape hybrid (seed 20261201,
      capacity 2048, fp16 history), the benchmark's 512-token prompt, then 256
      greedy tokens with their top-2 relative logit margins, and the oracle's
      final-normed state at a few positions of prompt + generated ids (the
      GPU test replays that sequence teacher-forced).
  ragged_config5.npz  benchmark config 5: the 9B-shape hybrid (seed 20261205),
      64 sequences with the benchmark's seeded histories (U[128, 8192], seeded
      rings / states / residual rows, seed 20261206), three greedy steps per
      sequence with margins.
"""
from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "ray-tracing-attention_b200"))

from oracle import oracle as O  # noqa: E402  (test infrastructure)
from oracle.model import OracleModel, seed_sequence, synthetic_payloads  # noqa: E402
from rta_b200 import assets, sharding  # noqa: E402  (layout planning only: pure Python)

CONFIG4_SEED, CONFIG4_PROMPT, CONFIG4_TOKENS, CONFIG4_CAPACITY = 20261201, 512, 256, 2048
CONFIG4_CHECKPOINTS = (0, 63, 127, 255, 511, 600, 700, CONFIG4_PROMPT + CONFIG4_TOKENS - 2)
CONFIG5_SEED, CONFIG5_STEPS = 20261205, 3


def margin(logits) -> float:
    top2 = np.sort(logits)[-2:]
    return float((top2[1] - top2[0]) / max(abs(top2[1]), 1e-30))


def config4(out: Path):
    spec = assets.spec_2b()
    layout = assets.plan(spec, CONFIG4_SEED)
    t0 = time.time()
    mats, basis = synthetic_payloads(layout, CONFIG4_SEED)
    ref = OracleModel(spec, layout.params(), mats, basis, CONFIG4_CAPACITY, kv="fp16")
    prompt = np.random.default_rng(CONFIG4_SEED).integers(0, spec.vocabulary_size, CONFIG4_PROMPT)
    out_norm = ref.f32(ref.p[4], spec.hidden_size)
    states, where = [], []

    def record():
        if ref.pos - 1 in CONFIG4_CHECKPOINTS:
            where.append(ref.pos - 1)
            states.append(O.rmsnorm(ref.state, out_norm, ref.eps))

    ref.reset()
    for t in prompt:
        ref.forward(int(t))
        record()
    tokens, margins = [], []
    for i in range(CONFIG4_TOKENS):
        tok, lg = ref.readout()
        tokens.append(tok)
        margins.append(margin(lg))
        if i + 1 < CONFIG4_TOKENS:
            ref.forward(tok)
            record()
        if i % 32 == 0:
            print(f"config4: token {i} ({time.time() - t0:.0f} s)", flush=True)
    np.savez_compressed(out, seed=CONFIG4_SEED, capacity=CONFIG4_CAPACITY, prompt=prompt.astype(np.uint32),
                        tokens=np.array(tokens, np.uint32), margins=np.array(margins, np.float64),
                        state_positions=np.array(where, np.uint32), states=np.array(states, np.float32))
    print(f"config4 written in {time.time() - t0:.0f} s", flush=True)


def config5(out: Path):
    spec = assets.spec_9b()
    lengths = sharding.config5_histories(CONFIG5_SEED)
    capacity = (int(lengths.max()) + 256 + 255) // 256 * 256  # the benchmark's ring size
    layout = assets.plan(spec, CONFIG5_SEED)
    t0 = time.time()
    mats, basis = synthetic_payloads(layout, CONFIG5_SEED)
    ref = OracleModel(spec, layout.params(), mats, basis, capacity, kv="fp16")
    nseq = len(lengths)
    tokens = np.zeros((nseq, CONFIG5_STEPS), np.uint32)
    margins = np.zeros((nseq, CONFIG5_STEPS), np.float64)
    for z in range(nseq):
        seed_sequence(ref, nseq, z, int(lengths[z]), CONFIG5_SEED + 1)
        for i in range(CONFIG5_STEPS):
            tok, lg = ref.readout()
            tokens[z, i] = tok
            margins[z, i] = margin(lg)
            if i + 1 < CONFIG5_STEPS:
                ref.forward(tok)
        print(f"config5: sequence {z} ({time.time() - t0:.0f} s)", flush=True)
    np.savez_compressed(out, seed=CONFIG5_SEED, history_seed=CONFIG5_SEED + 1, capacity=capacity,
                        lengths=lengths, tokens=tokens, margins=margins)
    print(f"config5 written in {time.time() - t0:.0f} s", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", choices=("config4", "config5"))
    args = ap.parse_args()
    if args.only in (None, "config4"):
        config4(HERE / "decode_config4.npz")
    if args.only in (None, "config5"):
        config5(HERE / "ragged_config5.npz")


if __name__ == "__main__":
    main()
