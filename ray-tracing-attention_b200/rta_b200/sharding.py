"""Sequence sharding of a ragged decode batch over the GPUs of one box.

benchmark config 5 decodes 64 independent sequences whose histories are drawn
uniformly from [128, 8192].  Sequences share nothing but the weights, so the
batch shards by sequence with no collective on the data path: every rank owns
a disjoint set of sequences on its own GPU, with the weights replicated.  The
plan is a pure function of (history lengths, world size), so every rank derives
the same plan locally; the per-step cost of a sequence grows with its history
(attention reads every visible position), so sequences are dealt longest first
to the least-loaded rank (LPT), which also keeps the per-rank sequence counts
within one of each other.
"""
from __future__ import annotations

import numpy as np

CONFIG5_SEQUENCES = 64
CONFIG5_HISTORY = (128, 8192)  # inclusive bounds of the uniform history draw


def config5_histories(seed: int, sequences: int = CONFIG5_SEQUENCES, lo: int = CONFIG5_HISTORY[0],
                      hi: int = CONFIG5_HISTORY[1]) -> np.ndarray:
    """Seeded history lengths of the ragged batch (uint32)."""
    return np.random.default_rng(seed).integers(lo, hi + 1, sequences).astype(np.uint32)


def shard_sequences(lengths, world: int, cost_per_sequence: float = 1024.0) -> list[list[int]]:
    """Deal sequence indices to `world` ranks, longest history first, each to the
    rank whose load (sum of history + cost_per_sequence, the fixed per-token
    cost of a sequence in the same units) is smallest; ties go to the rank with
    fewer sequences, then to the lower rank.  Deterministic."""
    lengths = np.asarray(lengths, dtype=np.int64)
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    load = [0.0] * world
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], len(shards[k]), k))
        shards[r].append(i)
        load[r] += float(lengths[i]) + cost_per_sequence
    return [sorted(s) for s in shards]


def shard_balance(lengths, shards) -> float:
    """max rank load / mean rank load (1.0 = perfect)."""
    lengths = np.asarray(lengths, dtype=np.float64)
    loads = [float(lengths[s].sum()) + 1024.0 * len(s) for s in shards]
    return max(loads) / (sum(loads) / len(loads))
