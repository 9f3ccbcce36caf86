"""Host logic of the multi-GPU paths, on CPU: the sequence-sharding plan of the
ragged batch (benchmark config 5) and the max-over-ranks timing reduction of
bench.py, including a world_size-2 run over the gloo backend."""
import os

import numpy as np
import pytest

from rta_b200 import sharding


def test_plan_covers_every_sequence_once_and_balances():
    lengths = sharding.config5_histories(20261201)
    assert lengths.size == 64 and lengths.min() >= 128 and lengths.max() <= 8192
    for world in (1, 2, 4, 8):
        shards = sharding.shard_sequences(lengths, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(64))
        counts = [len(s) for s in shards]
        assert max(counts) - min(counts) <= 1
        assert sharding.shard_balance(lengths, shards) < 1.05, world
    assert sharding.shard_sequences(lengths, 4) == sharding.shard_sequences(lengths.copy(), 4)


def test_plan_edge_cases():
    assert sharding.shard_sequences([5], 1) == [[0]]
    assert sharding.shard_sequences([5, 5], 4) == [[0], [1], [], []]
    with pytest.raises(ValueError):
        sharding.shard_sequences([1], 0)


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lengths = sharding.config5_histories(7)
    mine = sharding.shard_sequences(lengths, world)[rank]
    plans = [None] * world
    dist.all_gather_object(plans, mine)
    worst = bench.max_over_ranks(float(len(mine) * 10 + rank), world)
    out.put((rank, plans, worst))
    dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_the_plan_and_the_max():
    import multiprocessing as mp
    import socket
    ctx = mp.get_context("spawn")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    lengths = sharding.config5_histories(7)
    want = sharding.shard_sequences(lengths, 2)
    for rank, plans, worst in results:
        assert plans == want
        assert worst == max(len(s) * 10 + r for r, s in enumerate(want))
