"""GPU tests of the multi-sequence engine (ragged batch, benchmark config 5).

A handle with S sequences decodes one token per running sequence per step.
Below 16 sequences every batched kernel runs the single-sequence arithmetic for
each sequence, so each sequence must produce exactly the tokens and the
residual state of a single-sequence handle fed the same prompt: compared bit
for bit here, with ragged prompt lengths, a per-sequence stop, more than 8
sequences (several GEMV launches per step) and seeded synthetic histories.
From 16 sequences on the products run on the tensor cores (fp16-rounded
activations, fp32 accumulation): those handles are held to the oracle within
the north-star tolerance, tokens compared wherever the top-2 margin exceeds it.
"""
import numpy as np
import pytest

from test_model_gpu import small_spec

pytestmark = pytest.mark.gpu


def open_pair(spec, seed, capacity, sequences):
    import torch
    from rta_b200 import assets
    from rta_b200.model import ResidentModel
    layout = assets.plan(spec, seed)
    mats, basis = assets.generate_device(layout, seed)
    params = layout.params()
    batch = ResidentModel.from_payloads(spec, params, mats, basis, capacity, sequences=sequences)
    single = ResidentModel.from_payloads(spec, params, mats, basis, capacity)
    del mats, basis
    torch.cuda.empty_cache()
    return batch, single


def single_run(single, prompt, count, stops=()):
    single.prefill(prompt, stops)
    return single.generate(count)


@pytest.mark.parametrize("kinds", [("recurrent", "recurrent", "recurrent", "full"), ("full", "recurrent")])
def test_batch_tokens_equal_single_sequence_runs(kinds):
    spec = small_spec(kinds=kinds)
    batch, single = open_pair(spec, 3, capacity=64, sequences=3)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, spec.vocabulary_size, n) for n in (5, 17, 1)]
    batch.prefill_batch(prompts)
    got = batch.generate_batch(12)
    for z, p in enumerate(prompts):
        want = single_run(single, p, 12)
        assert np.array_equal(got[z], want), (z, got[z], want)
    res = batch.resources()
    assert res["sequences"] == 3
    batch.close()
    single.close()


def test_batch_stop_ends_one_sequence_only():
    spec = small_spec()
    batch, single = open_pair(spec, 4, capacity=64, sequences=2)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, spec.vocabulary_size, 6), rng.integers(0, spec.vocabulary_size, 9)]
    free = [single_run(single, p, 8) for p in prompts]
    stop = int(free[0][2])                      # sequence 0 stops at its third token
    if stop in free[1].tolist():
        pytest.skip("both sequences emit the stop id; pick another seed")
    batch.prefill_batch(prompts, stops=(stop,))
    got = batch.generate_batch(8)
    assert np.array_equal(got[0], free[0][:3])
    assert np.array_equal(got[1], free[1])
    batch.close()
    single.close()


def test_batch_more_than_eight_sequences():
    """10 sequences: each GEMV runs as two launches (8 + 2 rows)."""
    spec = small_spec(kinds=("recurrent", "full"))
    batch, single = open_pair(spec, 6, capacity=32, sequences=10)
    rng = np.random.default_rng(6)
    prompts = [rng.integers(0, spec.vocabulary_size, int(n)) for n in rng.integers(1, 12, 10)]
    batch.prefill_batch(prompts)
    got = batch.generate_batch(6)
    for z in (0, 7, 8, 9):
        want = single_run(single, prompts[z], 6)
        assert np.array_equal(got[z], want), (z, got[z], want)
    batch.close()
    single.close()


def test_seeded_histories_decode():
    """Synthetic histories (throughput runs): every sequence decodes, positions advance."""
    spec = small_spec(kinds=("recurrent", "full"))
    batch, single = open_pair(spec, 8, capacity=256, sequences=4)
    single.close()
    lengths = np.array([100, 7, 255, 300], np.uint32)   # 300 > capacity: the ring holds the newest 256
    batch.seed_history(lengths, seed=11)
    got = batch.generate_batch(5)
    assert all(len(g) == 5 for g in got)
    assert all(int(t) < spec.vocabulary_size for g in got for t in g)
    res = batch.resources()
    assert res["position"] == 105
    again = batch.generate_batch(3)
    assert all(len(g) == 3 for g in again)
    batch.close()


TOL = 1e-3  # relative L2


@pytest.mark.parametrize("sequences,split", [(18, False), (20, False), (20, True)])
def test_tensor_core_batch_tracks_the_oracle(sequences, split):
    """18 or 20 sequences: every matrix on the tensor cores (with `split`, each
    activation row as two fp16 operands, RTA_MODEL_SPLIT_ACTIVATIONS); at
    20 x 16 heads the gated delta runs the persistent (head, sequence) walk (at
    18, eight CTAs per head).  Per sequence: greedy tokens equal the oracle's
    wherever the oracle's top-2 margin exceeds the tolerance (the first
    legitimate near-tie flip ends the comparison, as in the single-sequence
    tests)."""
    import torch
    from oracle.model import OracleModel
    from rta_b200 import assets
    from rta_b200.model import ResidentModel
    spec = small_spec(kinds=("recurrent", "full"))
    layout = assets.plan(spec, 9)
    mats, basis = assets.generate_device(layout, 9)
    params = layout.params()
    batch = ResidentModel.from_payloads(spec, params, mats, basis, 32, sequences=sequences, split_activations=split)
    m, b = mats.cpu().numpy(), basis.cpu().numpy()
    del mats, basis
    torch.cuda.empty_cache()
    res = batch.resources()
    assert res["tensor_core_matrices"] == 2 * 5 + 1  # (in/qkvg, out/o, gate, up, down) x 2 layers + LM head
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, spec.vocabulary_size, int(n)) for n in rng.integers(1, 10, sequences)]
    batch.prefill_batch(prompts)
    got = batch.generate_batch(6)
    compared = 0
    for z in (0, 1, 9, sequences - 1):
        ref = OracleModel(spec, params, m, b, 32)
        ref.prefill(prompts[z])
        want, margins = ref.generate(6)
        for i in range(min(len(got[z]), len(want))):
            if margins[i] > TOL:
                assert got[z][i] == want[i], (z, i, got[z], want, margins)
                compared += 1
            if got[z][i] != want[i]:
                break
    assert compared >= 8
    batch.close()


def test_tensor_core_batch_diagnostics_match_the_oracle():
    """mlp (worker op 6) and vocabulary (op 4) on a tensor-core handle."""
    import torch
    from conftest import rel_l2
    from oracle import oracle
    from rta_b200 import assets
    from rta_b200.model import ResidentModel
    spec = small_spec(kinds=("recurrent", "full"))
    layout = assets.plan(spec, 10)
    mats, basis = assets.generate_device(layout, 10)
    params = layout.params()
    batch = ResidentModel.from_payloads(spec, params, mats, basis, 32, sequences=16)
    m = mats.cpu().numpy()
    del mats, basis
    torch.cuda.empty_cache()
    t = {x.name: x for x in layout.matrices}
    rng = np.random.default_rng(10)
    x = rng.normal(0, 0.5, (5, spec.hidden_size)).astype(np.float32)
    y, act = batch.mlp(x, 1)
    g, u, d = (t[f"blk.1.ffn_{n}.weight"] for n in ("gate", "up", "down"))
    wg, wu, wd = (m[w.offset:w.offset + w.nbytes] for w in (g, u, d))
    want_act, want_y = oracle.mlp(g.fmt, wg, wu, wd, spec.hidden_size, spec.middle_size, x)
    assert rel_l2(act, want_act) < TOL and rel_l2(y, want_y) < TOL
    batch.close()


def test_tensor_core_batch_at_9b_layer_shapes():
    """The 9B layer shapes on the tensor cores (hidden 4096, intermediate 12288,
    32 state heads over 16 key heads, 16q/4kv x 256) in four layers [rec, rec,
    rec, full], 16 sequences with ragged prompts, against the oracle per
    sequence (vocabulary cut to 32768 rows to keep the host oracle quick; the
    full 151936-row model at 64 sequences is checked against recorded
    fixtures in test_model_golden_gpu.py)."""
    import torch
    from oracle.model import OracleModel
    from rta_b200 import assets
    from rta_b200.model import ResidentModel
    spec = assets.Spec("qwen35", 4096, 12288, 32768, ("recurrent", "recurrent", "recurrent", "full"), 16, 4, 256,
                       64, state_heads=32, state_key_heads=16)
    layout = assets.plan(spec, 41)
    mats, basis = assets.generate_device(layout, 41)
    params = layout.params()
    batch = ResidentModel.from_payloads(spec, params, mats, basis, 32, sequences=16)
    m, b = mats.cpu().numpy(), basis.cpu().numpy()
    del mats, basis
    torch.cuda.empty_cache()
    assert batch.resources()["tensor_core_matrices"] > 0
    rng = np.random.default_rng(41)
    prompts = [rng.integers(0, spec.vocabulary_size, int(n)) for n in rng.integers(1, 6, 16)]
    batch.prefill_batch(prompts)
    got = batch.generate_batch(3)
    ref = OracleModel(spec, params, m, b, 32)
    compared = 0
    for z in (0, 5, 10, 15):
        ref.prefill(prompts[z])
        want, margins = ref.generate(3)
        for i in range(min(len(got[z]), len(want))):
            if margins[i] > TOL:
                assert got[z][i] == want[i], (z, i, got[z], want, margins)
                compared += 1
            if got[z][i] != want[i]:
                break
    assert compared >= 6
    batch.close()
