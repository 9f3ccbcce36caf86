"""Host logic of the tensor-parallel MLP and vocabulary readout, on CPU.

The split plans and the weight slicing of rta_b200.tensor_parallel are checked
against the oracle: the sum of the ranks' partial MLPs equals the whole MLP
(executeMLP, optical_resident.cpp:484-491), the best of the ranks' local argmax
equals the whole readout's (ops 16/17, resident_math.comp:117-127), and two gloo
ranks that exchange their partials agree on the sum."""
import os

import numpy as np
import pytest

from conftest import rel_l2
from oracle import oracle
from rta_b200 import tensor_parallel as tp


def test_split_units_cover_balance_and_align():
    for total, unit in ((6144, 256), (12288, 256), (151936, 128), (768, 256)):
        for world in range(1, 9):
            if total // unit < world:
                continue
            plan = tp.split_units(total, unit, world)
            assert len(plan) == world
            assert plan[0][0] == 0 and sum(n for _, n in plan) == total
            for (s0, n0), (s1, _) in zip(plan, plan[1:]):
                assert s0 + n0 == s1
            counts = [n for _, n in plan]
            assert all(n % unit == 0 and n > 0 for n in counts)
            assert max(counts) - min(counts) <= unit
    # the benchmark vocabulary: 1187 tiles of 128 rows, uneven over 2 and 8 ranks
    assert [n for _, n in tp.split_units(151936, 128, 2)] == [594 * 128, 593 * 128]
    assert tp.split_units(6144, 256, 8) == [(768 * r, 768) for r in range(8)]


def test_split_units_rejects_bad_plans():
    with pytest.raises(ValueError):
        tp.split_units(6144, 256, 0)
    with pytest.raises(ValueError):
        tp.split_units(6000, 256, 2)
    with pytest.raises(ValueError):
        tp.split_units(512, 256, 3)


@pytest.mark.parametrize("fmt", [12, 14])
def test_slices_are_the_matrix_blocks(fmt):
    rows, cols = 32, 1024
    rng = np.random.default_rng(fmt)
    W = oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    dense = oracle.dequantize(fmt, W).reshape(rows, cols)
    r = tp.slice_rows(fmt, W, rows, cols, 8, 16)
    assert np.array_equal(oracle.dequantize(fmt, r).reshape(16, cols), dense[8:24])
    c = tp.slice_columns(fmt, W, rows, cols, 256, 512)
    assert c.flags.c_contiguous and c.size == rows * 2 * (144 if fmt == 12 else 210)
    assert np.array_equal(oracle.dequantize(fmt, c).reshape(rows, 512), dense[:, 256:768])
    with pytest.raises(ValueError):
        tp.slice_columns(fmt, W, rows, cols, 128, 256)
    with pytest.raises(ValueError):
        tp.slice_rows(fmt, W, rows, cols, 24, 16)


def _mlp_mats(D, F, seed):
    rng = np.random.default_rng(seed)
    wg, wu = (oracle.quantize(12, rng.normal(0, 0.02, F * D).astype(np.float32)) for _ in range(2))
    wd = oracle.quantize(12, rng.normal(0, 0.02, D * F).astype(np.float32))
    x = rng.normal(0, 1, (3, D)).astype(np.float32)
    return wg, wu, wd, x


def _partial_mlp(wg, wu, wd, D, F, x, start, count):
    g = tp.slice_rows(12, wg, F, D, start, count)
    u = tp.slice_rows(12, wu, F, D, start, count)
    d = tp.slice_columns(12, wd, D, F, start, count)
    return oracle.mlp(12, g, u, d, D, count, x)


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_split_mlp_sums_to_the_whole(world):
    D, F = 512, 1536
    wg, wu, wd, x = _mlp_mats(D, F, world)
    act, y = oracle.mlp(12, wg, wu, wd, D, F, x)
    total = np.zeros_like(y, dtype=np.float64)
    for start, count in tp.split_units(F, tp.MIDDLE_UNIT, world):
        a_r, y_r = _partial_mlp(wg, wu, wd, D, F, x, start, count)
        assert np.array_equal(a_r, act[:, start:start + count])  # each activation row is the whole MLP's
        total += y_r
    assert rel_l2(total, y) < 1e-5


@pytest.mark.parametrize("world", [1, 2, 5])
def test_split_readout_picks_the_whole_argmax(world):
    V, D = 128 * 7, 512
    rng = np.random.default_rng(11 + world)
    W = oracle.quantize(14, rng.normal(0, 0.02, V * D).astype(np.float32))
    x = rng.normal(0, 1, (4, D)).astype(np.float32)
    x[3] = 0.0  # all logits 0: ties everywhere -> id 0
    _, want_arg, want_best = oracle.lmhead(14, W, V, D, x, want_logits=False)
    best = np.full(4, -np.inf, np.float32)
    arg = np.full(4, -1, np.int64)
    for start, count in tp.split_units(V, tp.VOCAB_UNIT, world):
        _, a, b = oracle.lmhead(14, tp.slice_rows(14, W, V, D, start, count), count, D, x, want_logits=False)
        for i in range(4):  # larger value wins; on a tie the earlier (lower id) rank keeps it
            if b[i] > best[i]:
                best[i], arg[i] = b[i], int(a[i]) + start
    assert np.array_equal(arg, want_arg.astype(np.int64)) and np.array_equal(best, want_best)
    assert arg[3] == 0


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch
    D, F = 512, 1536
    wg, wu, wd, x = _mlp_mats(D, F, 77)
    start, count = tp.split_units(F, tp.MIDDLE_UNIT, world)[rank]
    _, y_r = _partial_mlp(wg, wu, wd, D, F, x, start, count)
    t = torch.from_numpy(y_r.copy())
    dist.all_reduce(t)
    out.put((rank, t.numpy()))
    dist.destroy_process_group()


def test_two_gloo_ranks_sum_their_partials():
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
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    D, F = 512, 1536
    wg, wu, wd, x = _mlp_mats(D, F, 77)
    _, y = oracle.mlp(12, wg, wu, wd, D, F, x)
    assert np.array_equal(results[0], results[1])
    assert rel_l2(results[0], y) < 1e-5
