"""Tensor-parallel MLP and readout on the GPU: the tensor-core MLP operator
(rta_mlp_tc), a team of one on one GPU, and two ranks on two GPUs exchanging
through NVLink peer memory (skipped with fewer than two GPUs).

Tolerance: 1e-3 relative L2 against the oracle (the decode path's floating-point
bar); ranks must agree bit for bit (the exchange sums in rank order); argmax ids
must equal the oracle's wherever the top-2 logit margin exceeds 1e-3 of the
largest |logit|."""
import os

import numpy as np
import pytest

from conftest import rel_l2
from oracle import oracle

TOL = 1e-3


@pytest.fixture(scope="module")
def tp():
    import torch
    from rta_b200 import _lib
    from rta_b200 import tensor_parallel
    _lib.load()
    torch.cuda.set_device(0)
    return tensor_parallel


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _np(t):
    return t.detach().cpu().numpy()


def _mats(D, F, seed):
    rng = np.random.default_rng(seed)
    wg, wu = (oracle.quantize(12, rng.normal(0, 0.02, F * D).astype(np.float32)) for _ in range(2))
    wd = oracle.quantize(12, rng.normal(0, 0.02, D * F).astype(np.float32))
    return wg, wu, wd


def _check_argmax(ids, best, W, V, D, x):
    want_lg, _, _ = oracle.lmhead(14, W, V, D, x)
    compared = 0
    for b in range(x.shape[0]):
        assert abs(best[b] - want_lg[b, ids[b]]) <= 1e-3 * max(1.0, np.abs(want_lg[b]).max())
        top2 = np.sort(want_lg[b])[-2:]
        if top2[1] - top2[0] > 1e-3 * np.abs(want_lg[b]).max():
            assert ids[b] == int(np.argmax(want_lg[b])), b
            compared += 1
    return compared


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,hidden,middle,batch,with_act", [
    (12, 2048, 6144, 16, False), (12, 2048, 6144, 64, True), (14, 1024, 2048, 33, False), (12, 4096, 1536, 100, True),
])
def test_mlp_tc_matches_the_oracle(tp, fmt, hidden, middle, batch, with_act):
    import torch
    from rta_b200 import ops
    rng = np.random.default_rng(hidden + middle + batch)
    wg, wu = (oracle.quantize(fmt, rng.normal(0, 0.02, middle * hidden).astype(np.float32)) for _ in range(2))
    wd = oracle.quantize(fmt, rng.normal(0, 0.02, hidden * middle).astype(np.float32))
    x = rng.normal(0, 1, (batch, hidden)).astype(np.float32)
    y0 = rng.normal(0, 1, (batch, hidden)).astype(np.float32)
    code, g = ops.panel_weights(fmt, _t(wg), middle, hidden)
    _, u = ops.panel_weights(fmt, _t(wu), middle, hidden)
    _, d = ops.panel_weights(fmt, _t(wd), hidden, middle)
    act = torch.empty(batch, middle, device="cuda") if with_act else None
    y = _t(y0)
    ops.mlp_tc(code, g, u, d, hidden, middle, _t(x), y=y, act=act, accumulate=True)
    want_act, want_y = oracle.mlp(fmt, wg, wu, wd, hidden, middle, x)
    assert rel_l2(_np(y), y0 + want_y) < TOL
    assert rel_l2(_np(y) - y0, want_y) < TOL
    if with_act:
        assert rel_l2(_np(act), want_act) < TOL


@pytest.mark.gpu
def test_team_of_one_sums_exactly(tp):
    import torch
    with tp.Team(capacity_bytes=64 * 4096 * 4) as team:
        assert (team.rank, team.world) == (0, 1)
        g = torch.Generator(device="cuda").manual_seed(3)
        for n in (4, 2048, 64 * 4096, 5000 * 4):
            p = torch.randn(n, device="cuda", generator=g)
            a = torch.randn(n, device="cuda", generator=g)
            assert torch.equal(team.allreduce(p, a), a + p)
            assert torch.equal(team.allreduce(p), p)
        assert team.error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 24])
def test_team_of_one_mlp(tp, batch):
    from rta_b200 import ops
    D, F = 2048, 6144
    wg, wu, wd = _mats(D, F, batch)
    rng = np.random.default_rng(batch + 1)
    x = rng.normal(0, 1, (batch, D)).astype(np.float32)
    res = rng.normal(0, 1, (batch, D)).astype(np.float32)
    with tp.Team(capacity_bytes=batch * D * 4) as team:
        mlp = tp.ShardedMLP(team, 12, _t(wg), _t(wu), _t(wd), D, F, batch)
        assert mlp.tc == (batch >= 16) and (mlp.start, mlp.count) == (0, F)
        y = _np(mlp(_t(x), residual=_t(res)))
        _, want = oracle.mlp(12, wg, wu, wd, D, F, x)
        assert rel_l2(y - res, want) < TOL
        if not mlp.tc:  # the GEMV path's residual add is the same single rounding as the exchange's
            _, t_g = ops.tile_weights(12, _t(wg), F, D)
            _, t_u = ops.tile_weights(12, _t(wu), F, D)
            code, t_d = ops.tile_weights(12, _t(wd), D, F)
            _, whole = ops.mlp_swiglu(code, t_g, t_u, t_d, D, F, _t(x), y=_t(res), accumulate=True)
            assert np.array_equal(_np(whole), y)
        assert team.error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 16])
def test_team_of_one_readout(tp, batch):
    V, D = 128 * 148, 2048
    rng = np.random.default_rng(40 + batch)
    W = oracle.quantize(14, rng.normal(0, 0.02, V * D).astype(np.float32))
    x = rng.normal(0, 1, (batch, D)).astype(np.float32)
    with tp.Team(capacity_bytes=8 * batch) as team:
        head = tp.ShardedReadout(team, 14, _t(W), V, D, batch)
        ids, best = head(_t(x))
        ids, best = _np(ids).astype(np.int64), _np(best)
        assert _check_argmax(ids, best, W, V, D, x) >= max(1, batch // 2)
        assert team.error() == 0


# ------------------------------------------------------------------ two GPUs
def _rank_main(rank, world, port, out):
    import torch
    import torch.distributed as dist
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))

    def ready():  # both ranks' set-up done before the first exchange (its wait is bounded by about a second)
        torch.cuda.synchronize()
        dist.barrier()

    from rta_b200 import tensor_parallel as tp
    res = {}
    try:
        D, F = 2048, 6144
        wg, wu, wd = _mats(D, F, 5)
        for batch in (1, 32):
            rng = np.random.default_rng(batch)
            x = rng.normal(0, 1, (batch, D)).astype(np.float32)
            r0 = rng.normal(0, 1, (batch, D)).astype(np.float32)
            with tp.Team(capacity_bytes=batch * D * 4) as team:
                mlp = tp.ShardedMLP(team, 12, _t(wg), _t(wu), _t(wd), D, F, batch)
                ready()
                y = mlp(_t(x), residual=_t(r0))
                y2 = mlp(_t(x), residual=y)  # a second exchange on the other slot parity
                res[f"mlp{batch}"] = (_np(y), _np(y2), team.error(), mlp.count)
        V = 128 * 148
        rng = np.random.default_rng(9)
        W = oracle.quantize(14, rng.normal(0, 0.02, V * D).astype(np.float32))
        for batch in (1, 16):
            x = np.random.default_rng(batch + 50).normal(0, 1, (batch, D)).astype(np.float32)
            with tp.Team(capacity_bytes=8 * batch) as team:
                head = tp.ShardedReadout(team, 14, _t(W), V, D, batch)
                ready()
                ids, best = head(_t(x))
                res[f"head{batch}"] = (_np(ids), _np(best), team.error())
        # a peer that never arrives: rank 0 exchanges alone, its bounded wait runs
        # out (about a second) and the team's error word says so
        with tp.Team(capacity_bytes=4096) as team:
            if rank == 0:
                import time
                t0 = time.perf_counter()
                team.allreduce(torch.ones(1024, device="cuda"))
                res["timeout"] = (team.error(), time.perf_counter() - t0)
            dist.barrier()
        out.put((rank, res, None))
    except Exception as e:  # reported to the parent, which fails the test
        out.put((rank, res, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_ranks_on_two_gpus(tp):
    import multiprocessing as mp
    import socket
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in procs:
            rank, res, err = q.get(timeout=600)
            assert err is None, (rank, err)
            got[rank] = res
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    D, F = 2048, 6144
    wg, wu, wd = _mats(D, F, 5)
    for batch in (1, 32):
        rng = np.random.default_rng(batch)
        x = rng.normal(0, 1, (batch, D)).astype(np.float32)
        r0 = rng.normal(0, 1, (batch, D)).astype(np.float32)
        _, want = oracle.mlp(12, wg, wu, wd, D, F, x)
        y, y2, err0, count0 = got[0][f"mlp{batch}"]
        y_1, y2_1, err1, count1 = got[1][f"mlp{batch}"]
        assert err0 == 0 and err1 == 0 and count0 + count1 == F
        assert np.array_equal(y, y_1) and np.array_equal(y2, y2_1)  # every rank holds the same bits
        assert rel_l2(y - r0, want) < TOL
        assert rel_l2(y2 - y, want) < TOL
    V = 128 * 148
    W = oracle.quantize(14, np.random.default_rng(9).normal(0, 0.02, V * D).astype(np.float32))
    for batch in (1, 16):
        x = np.random.default_rng(batch + 50).normal(0, 1, (batch, D)).astype(np.float32)
        ids, best, e0 = got[0][f"head{batch}"]
        ids1, best1, e1 = got[1][f"head{batch}"]
        assert e0 == 0 and e1 == 0
        assert np.array_equal(ids, ids1) and np.array_equal(best, best1)
        _check_argmax(ids.astype(np.int64), best, W, V, D, x)
    word, seconds = got[0]["timeout"]
    assert word & 1 and seconds < 30
