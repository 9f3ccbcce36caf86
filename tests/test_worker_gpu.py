"""rta_worker over its pipe protocol (the runtime-facing boundary), on the GPU.

The worker is the drop-in for the reference's native worker: the reference's
ResidentRuntime spawns it and speaks <3I op,count,debug> / <2I status,size>
frames.  rta_b200.runtime.WorkerClient speaks the same protocol; these tests run
a synthetic model directory (exporter layout) through it and require the
worker's replies to equal the in-process C-ABI results on the same payloads
bit for bit (prefill + generate, MLP, the attention diagnostic), plus the
protocol's error behaviour (status 1 on an unserved op, the session survives).
"""
import numpy as np
import pytest

from test_model_gpu import small_spec

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    import torch
    from rta_b200 import assets
    spec = small_spec(kinds=("recurrent", "full"))
    layout = assets.plan(spec, 31)
    mats, basis = assets.generate_device(layout, 31)
    d = tmp_path_factory.mktemp("model")
    assets.write_files(d, layout, mats.cpu().numpy(), basis.cpu().numpy())
    del mats, basis
    torch.cuda.empty_cache()
    return d


def test_worker_serves_the_protocol_like_the_library(model_dir):
    from rta_b200 import assets
    from rta_b200.model import ResidentModel
    from rta_b200.runtime import WorkerClient, WorkerError
    spec, params, mats, basis = assets.read_files(model_dir)
    lib = ResidentModel.from_payloads(spec, params, mats, basis, 64, history="packet")
    rng = np.random.default_rng(31)
    prompt = rng.integers(0, spec.vocabulary_size, 12)
    with WorkerClient(model_dir, capacity=64) as w:
        assert w.mode & 4
        w.prefill(prompt)
        got = w.generate(6)["ids"]
        lib.prefill(prompt)
        assert np.array_equal(got, lib.generate(6))

        x = rng.normal(0, 0.25, (5, spec.hidden_size)).astype(np.float32)
        x[1] = 0
        r = w.mlp(x, layer=1)
        y, act = lib.mlp(x, 1)
        assert np.array_equal(r["output"], y) and np.array_equal(r["activation"], act)
        assert np.all(r["output"][1] == 0) and np.all(r["feature_hits"] == spec.middle_size)
        for rows in (1, 3):   # row-prefix identity (verify_rt_mlp.py:96-98)
            assert np.array_equal(w.mlp(x[:rows], layer=1)["output"], r["output"][:rows])

        H, KVH, hd = spec.attention_heads, spec.kv_heads, spec.attention_head_dim
        q = rng.normal(0, 1, (2, H, hd)).astype(np.float32)
        k = rng.normal(0, 1, (40, KVH, hd)).astype(np.float32)
        v = rng.normal(0, 1, (40, KVH, hd)).astype(np.float32)
        g = rng.normal(0, 1, (2, H, hd)).astype(np.float32)
        a = w.attention(q, k, v, g, layer=1)
        b = lib.attention(q, k, v, g, layer=1, block=128)
        for key in ("output", "physical", "history_packets", "receipts"):
            assert np.array_equal(a[key], b[key]), key
        assert np.array_equal(a["legacy_output"], a["output"])

        with pytest.raises(WorkerError):
            w.request(5)                       # codec: not served -> status 1
        res = w.resources()                    # the session survives an error reply
        assert res.size == 61 and res[38] == 128
    lib.close()


def test_worker_caches_replay_a_reply(model_dir):
    """The worker's cache argument (on by default, as ResidentRuntime starts it):
    a repeated prompt restores its boundary and the reply is replayed from the
    reply tree with the same ids; with the argument 0 nothing is cached."""
    from rta_b200 import assets
    from rta_b200.runtime import WorkerClient
    spec, _params, _mats, _basis = assets.read_files(model_dir)
    prompt = np.random.default_rng(32).integers(0, spec.vocabulary_size, 20)
    with WorkerClient(model_dir, capacity=64) as w:
        first = w.prefill(prompt)
        assert not first["cache_hit"] and first["saved_boundaries"] == 1 and first["computed_tokens"] == 20
        a = w.generate(10)
        again = w.prefill(prompt)
        assert again["cache_hit"] and again["cached_prefix_tokens"] == 20 and again["address_hit"] == 1
        assert again["computed_tokens"] == 0
        b = w.generate(10)
        assert np.array_equal(a["ids"], b["ids"]) and b["reply_cache_hit"] and b["cached_tokens"] == 10
        assert w.finish_history()[0] == 0  # the replayed reply has no computed state yet
        c = w.generate(2)
        assert not c["reply_cache_hit"] and c["cached_tokens"] == 0
        saved, tokens, _ = w.finish_history()
        assert saved == 1 and tokens == 20 + 12
    with WorkerClient(model_dir, capacity=64, cache=False) as w:
        w.prefill(prompt)
        x = w.generate(10)
        assert np.array_equal(x["ids"], a["ids"])
        r = w.prefill(prompt)
        assert not r["cache_hit"] and r["computed_tokens"] == 20
        assert not w.generate(10)["reply_cache_hit"]
        assert w.finish_history() == (0, 0, 0)
