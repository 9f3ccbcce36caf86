"""The decode caches of a single-sequence handle (RTA_MODEL_CACHE) on the GPU.

What the reference's own cache check asserts (benchmark_attention_receipts.py:
130-150): after prefill(prompt) + generate(32), a second prefill(prompt) is a
boundary hit with the state address (no position computed), the following
generate(32) replays every token from the reply tree (no token computed), the
ids are the first reply's.  Here, in addition, every cached result is compared
with an uncached handle of the same weights:
* replayed tokens, and the tokens decoded after a replay (the device state
  catches up one step per token, the decode step's kernels), equal the
  uncached handle's, and the states are bit-identical;
* a prefill that restores a shorter boundary and computes the rest equals a
  full prefill (bit-identical with one position per step; within the chunked
  prefill's own rounding with 64-position chunks);
* finish_history saves prompt + reply, a later prompt that extends it restores
  it; a stop id ends a replay as it ended the decode; the byte limit evicts the
  least recently used boundaries; the state address is a deterministic digest
  of the state that changes with every consumed token.
"""
import numpy as np
import pytest

from conftest import rel_l2
from test_model_gpu import small_spec

pytestmark = pytest.mark.gpu


def pair(seed, capacity=256, **kw):
    """A cached and an uncached handle of the same synthetic weights."""
    from rta_b200.model import ResidentModel
    spec = small_spec()
    c = ResidentModel.synthetic(spec, seed, capacity, cache=True, **kw)
    u = ResidentModel.synthetic(spec, seed, capacity, **kw)
    return spec, c, u


@pytest.mark.parametrize("history", ["fp16", "packet"])
def test_prefill_hit_and_reply_replay(history):
    spec, c, u = pair(41, history=history)
    rng = np.random.default_rng(41)
    prompt = rng.integers(0, spec.vocabulary_size, 40)

    c.prefill(prompt)
    info = c.cache_info()
    assert (info["prefill_hit"], info["computed_tokens"], info["saved_boundaries"], info["boundaries"]) == (0, 40, 1, 1)
    assert info["digests"] == 1 and info["stable_tokens"] == 40
    first = c.generate(16)
    info = c.cache_info()
    assert info["replayed_tokens"] == 0 and info["digests"] == 16 and info["tree_nodes"] == 16
    u.prefill(prompt)
    assert np.array_equal(first, u.generate(16))

    c.prefill(prompt)  # the same prompt: restored, nothing computed, the address known
    info = c.cache_info()
    assert info["prefill_hit"] == 1 and info["reused_tokens"] == 40 and info["computed_tokens"] == 0
    assert info["address_hit"] == 1 and info["snapshot_kind"] == 1 and info["digests"] == 0
    assert info["shared_blocks"] == 3 and info["saved_boundaries"] == 0
    replay = c.generate(16)
    info = c.cache_info()
    assert np.array_equal(replay, first)
    assert info["replayed_tokens"] == 16 and info["digests"] == 0 and info["tree_queries"] == 16
    assert info["tree_leaf"] < info["tree_capacity"] == 65536

    more = c.generate(8)  # past the tree: the state catches up on the 16 replayed tokens first
    info = c.cache_info()
    assert info["replayed_tokens"] == 0 and info["restored_tokens"] == 16 and info["checkpoint_restored"] == 0
    assert np.array_equal(more, u.generate(8))
    sc, pc = c.state()
    su, pu = u.state()
    assert pc == pu == 40 + 24 and np.array_equal(sc, su)
    c.close()
    u.close()


def test_prefix_reuse_equals_full_prefill_per_position():
    spec, c, u = pair(43, token_prefill=True)
    rng = np.random.default_rng(43)
    prompt = rng.integers(0, spec.vocabulary_size, 90)
    c.prefill(prompt[:50])
    c.prefill(prompt, checkpoint=50)
    info = c.cache_info()
    assert info["prefill_hit"] == 1 and info["reused_tokens"] == 50 and info["computed_tokens"] == 40
    assert info["snapshot_kind"] == 2 and info["shared_blocks"] == 4 and info["boundaries"] == 2
    u.prefill(prompt)
    sc, _ = c.state()
    su, _ = u.state()
    assert np.array_equal(sc, su)
    assert np.array_equal(c.generate(12), u.generate(12))
    c.close()
    u.close()


def test_prefix_reuse_with_chunks():
    spec, c, u = pair(44)
    rng = np.random.default_rng(44)
    prompt = rng.integers(0, spec.vocabulary_size, 150)
    c.prefill(prompt[:70])
    c.prefill(prompt)
    info = c.cache_info()
    assert info["reused_tokens"] == 70 and info["computed_tokens"] == 80 and info["snapshot_kind"] == 3
    u.prefill(prompt)
    sc, _ = c.state()
    su, _ = u.state()
    assert rel_l2(sc, su) < 1e-4, rel_l2(sc, su)
    c.close()
    u.close()


def test_finish_history_then_extended_prompt():
    spec, c, u = pair(45, token_prefill=True)
    rng = np.random.default_rng(45)
    prompt = rng.integers(0, spec.vocabulary_size, 30)
    c.prefill(prompt)
    reply = c.generate(12)
    saved, tokens, boundaries = c.finish_history()
    assert (saved, tokens, boundaries) == (1, 42, 2)
    assert c.finish_history() == (0, 42, 2)  # held already
    follow = rng.integers(0, spec.vocabulary_size, 10)
    convo = np.concatenate([prompt, reply, follow])
    c.prefill(convo)
    info = c.cache_info()
    assert info["reused_tokens"] == 42 and info["computed_tokens"] == 10
    # the restored reply's state came from decode steps; the uncached handle
    # prefills the same ids one position per step with the same kernels
    u.prefill(convo)
    sc, _ = c.state()
    su, _ = u.state()
    assert np.array_equal(sc, su)
    # a replayed reply has no computed state: nothing is saved until it is
    c.prefill(prompt)
    assert np.array_equal(c.generate(12), reply)
    assert c.cache_info()["replayed_tokens"] == 12
    assert c.finish_history()[0] == 0
    c.close()
    u.close()


def test_stop_id_ends_replay():
    spec, c, u = pair(46)
    rng = np.random.default_rng(46)
    prompt = rng.integers(0, spec.vocabulary_size, 24)
    u.prefill(prompt)
    free = u.generate(12)
    stop = int(free[5])
    first_at = int(np.argmax(free == stop))
    c.prefill(prompt, stops=(stop,))
    got = c.generate(12)
    assert got[-1] == stop and len(got) == first_at + 1
    assert np.array_equal(got, free[:first_at + 1])
    c.prefill(prompt, stops=(stop,))
    again = c.generate(12)
    assert np.array_equal(again, got) and c.cache_info()["replayed_tokens"] == len(got)
    c.close()
    u.close()


def test_byte_limit_evicts_least_recent():
    spec, c, _u = pair(47)
    _u.close()
    rng = np.random.default_rng(47)
    prompts = [rng.integers(0, spec.vocabulary_size, 20) for _ in range(4)]
    c.prefill(prompts[0])
    one = c.cache_info()["bytes"]
    c.cache_limit(int(one * 2.5))
    for p in prompts[1:]:
        c.prefill(p)
    info = c.cache_info()
    assert info["boundaries"] == 2 and info["evictions"] == 2 and info["bytes"] <= one * 2.5
    c.prefill(prompts[3])
    assert c.cache_info()["prefill_hit"] == 1
    c.prefill(prompts[0])
    assert c.cache_info()["prefill_hit"] == 0
    c.close()


def test_state_address_is_a_digest_of_the_state():
    spec, c, u = pair(48)
    u.close()
    from rta_b200.model import ResidentModel
    d = ResidentModel.synthetic(spec, 48, 256, cache=True)
    rng = np.random.default_rng(48)
    prompt = rng.integers(0, spec.vocabulary_size, 33)
    c.prefill(prompt)
    d.prefill(prompt)
    a, pa = c.state_address()
    b, pb = d.state_address()
    assert pa == pb == 33 and np.array_equal(a, b)
    other = prompt.copy()
    other[-1] = (other[-1] + 1) % spec.vocabulary_size
    d.prefill(other)
    assert not np.array_equal(d.state_address()[0], a)
    c.generate(1)
    assert not np.array_equal(c.state_address()[0], a)
    c.close()
    d.close()
