"""The reference's history format on the GPU: Q4_K key / Q6_K value packets.

* The decode engine with packet history (RTA_MODEL_PACKET_HISTORY) against the
  model oracle keeping the same packets (OracleModel(kv="packet")): state after
  prefill within 1e-3, greedy tokens identical wherever the margin allows,
  across a history-ring wrap.
* The full-attention diagnostic (worker op 14): its history packets bit-exact
  with the oracle's packet quantizer on the same K/V rows; its outputs and dense
  receipts against an FP64 restatement of the reference's verifier
  (verify_attention_receipts.py:84-203: full_attention, receipt_reference,
  check_receipts) on the decoded packets, within the reference's bound
  3e-6 * max(1, peak).
"""
import numpy as np
import pytest

from conftest import ref_bound, rel_l2
from oracle import oracle
from test_model_gpu import check_generation, small_spec

pytestmark = pytest.mark.gpu


def build_packet(spec, seed, capacity, token_prefill=False):
    import torch
    from oracle.model import OracleModel
    from rta_b200 import assets
    from rta_b200.model import ResidentModel
    layout = assets.plan(spec, seed)
    mats, basis = assets.generate_device(layout, seed)
    params = layout.params()
    model = ResidentModel.from_payloads(spec, params, mats, basis, capacity, history="packet",
                                        token_prefill=token_prefill)
    ref = OracleModel(spec, params, mats.cpu().numpy(), basis.cpu().numpy(), capacity, kv="packet")
    del mats, basis
    torch.cuda.empty_cache()
    return model, ref


def test_engine_packet_history_tracks_the_oracle_closely():
    """Whole-model: quantizing K to 4 bits makes a random-init model's state depend
    on code-boundary flips, so the bar is relative: the GPU packet path must sit
    far closer to the packet oracle than the packet history sits to fp16 history."""
    spec = small_spec(kinds=("full", "recurrent", "full", "recurrent"))
    model, ref = build_packet(spec, 12, 64)
    from oracle.model import OracleModel
    prompt = np.random.default_rng(12).integers(0, spec.vocabulary_size, 4)
    model.prefill(prompt)
    ref.prefill(prompt)
    fp16 = OracleModel(spec, ref.p, ref.m, ref.b, 64, kv="fp16")
    fp16.prefill(prompt)
    state = model.state()[0]
    gap = rel_l2(ref.state, fp16.state)
    assert rel_l2(state, ref.state) < 0.25 * gap, (rel_l2(state, ref.state), gap)
    res = model.resources()
    assert res["history_bytes"] == 2 * 64 * 1416   # 2 full layers x capacity x 1416-byte packets
    model.close()


@pytest.mark.parametrize("seed,capacity,prompt_len", [(14, 64, 20), (15, 16, 14), (16, 512, 300), (17, 128, 126)])
def test_engine_packet_attention_step_matches_fp64(seed, capacity, prompt_len):
    """Teacher-forced: the decode step's own q, gate and ring packets, read back,
    give the FP64 detector output the step produced (prefill and decode graphs,
    with the ring wrapping in the second and fourth cases; the last two split
    the history over several CTAs per KV head, some of them empty).  The
    prefill runs one position per step here so that its last step leaves the
    decode step's own buffers to read back; the chunked prefill's packet rows
    are checked through the history it leaves (test_model_gpu.py)."""
    spec = small_spec(kinds=("recurrent", "full"))
    model, _ = build_packet(spec, seed, capacity, token_prefill=True)
    H, KVH, hd = spec.attention_heads, spec.kv_heads, spec.attention_head_dim
    R = spec.rotary_dim
    prompt = np.random.default_rng(seed).integers(0, spec.vocabulary_size, prompt_len)
    model.prefill(prompt)
    assert model.resources()["attention_splits"] == max(1, capacity // 64)
    for step in range(3):   # after prefill, then after 3 and 6 decode steps (16-slot ring wraps at 16)
        q, gate, att, packets = model.debug_attention()
        assert len(packets) == min(model.state()[1], capacity)
        keys, values = decode_packets(packets, KVH, hd)
        t = len(packets) - 1
        dense = full_attention(q.reshape(1, H, hd), keys, values, gate.reshape(1, H, hd), t, 0, capacity,
                               bool(spec.attention_gate))
        out = dense["output"][0]
        want = out.copy()
        d = np.arange(R)
        want[:, (d % 2) * (R // 2) + d // 2] = out[:, :R]   # o-projection axis order (row mode 4)
        ok, err, limit = ref_bound(att.reshape(H, hd), want)
        assert ok, (step, err, limit)
        model.generate(3)
    model.close()


def sigmoid(x):
    x = np.asarray(x, np.float64)
    light = np.exp(-np.abs(x))
    return np.where(x >= 0, 1 / (1 + light), light / (1 + light))


def decode_packets(packets, kvh, hd):
    count = len(packets)
    keys = oracle.dequantize(12, np.ascontiguousarray(packets[:, :kvh * 144]).reshape(-1))
    values = oracle.dequantize(14, np.ascontiguousarray(packets[:, kvh * 144:]).reshape(-1))
    return (keys.reshape(count, kvh, hd).astype(np.float64), values.reshape(count, kvh, hd).astype(np.float64))


def full_attention(q, keys, values, gate, query_start, history_start, capacity, gated):
    """FP64 dense GQA restatement (verify_attention_receipts.py:84-114)."""
    rows, heads, d = q.shape
    mapping = np.arange(heads) // (heads // keys.shape[1])
    ek, ev = keys[:, mapping, :], values[:, mapping, :]
    scores = np.einsum("rhd,nhd->rhn", q.astype(np.float64), ek) / np.sqrt(float(d))
    ages = history_start + np.arange(len(keys))
    times = query_start + np.arange(rows)
    visible = (ages[None, :] <= times[:, None]) & (times[:, None] - ages[None, :] < capacity)
    masked = np.where(visible[:, None, :], scores, -np.inf)
    m = masked.max(axis=2)
    e = np.exp(masked - m[:, :, None])
    z = e.sum(axis=2)
    out = np.einsum("rhn,nhd->rhd", e, ev) / z[:, :, None]
    if gated:
        out = out * sigmoid(gate)
    return dict(output=out, maximum=m, reference=z, scores=scores, visible=visible, values=ev, times=times)


def receipt_reference(dense, block, history_start):
    """Expected groups from time identities (verify_attention_receipts.py:117-139)."""
    rows, heads, _ = dense["scores"].shape
    records = []
    for row in range(rows):
        available = int(np.count_nonzero(dense["visible"][row]))
        time = int(dense["times"][row])
        for group in range((available + block - 1) // block):
            count = min(block, available - group * block)
            idx = time - history_start - group * block - np.arange(count)
            for head in range(heads):
                s = dense["scores"][row, head, idx]
                m = float(s.max())
                e = np.exp(s - m)
                records.append(dict(count=count, maximum=m, reference=float(e.sum()),
                                    numerator=np.einsum("n,nd->d", e, dense["values"][idx, head, :]), head=head))
    return records


@pytest.mark.parametrize("rows,count,history_start,block", [(3, 300, 0, 128), (2, 200, 100, 256), (1, 64, 5, 512)])
def test_attention_diagnostic_packets_receipts_and_output(rows, count, history_start, block):
    spec = small_spec(kinds=("recurrent", "full"))
    from rta_b200 import assets
    from rta_b200.model import ResidentModel
    layout = assets.plan(spec, 21)
    mats, basis = assets.generate_device(layout, 21)
    model = ResidentModel.from_payloads(spec, layout.params(), mats, basis, 512, history="packet")
    H, KVH, hd = spec.attention_heads, spec.kv_heads, spec.attention_head_dim
    rng = np.random.default_rng(rows * 1000 + count)
    q = rng.normal(0, 1, (rows, H, hd)).astype(np.float32)
    k = rng.normal(0, 1, (count, KVH, hd)).astype(np.float32)
    v = rng.normal(0, 1, (count, KVH, hd)).astype(np.float32)
    g = rng.normal(0, 1, (rows, H, hd)).astype(np.float32)
    query_start = history_start + count - rows
    got = model.attention(q, k, v, g, query_start=query_start, history_start=history_start, block=block)

    # packets: bit-exact with the oracle's packet quantizer on the same rows
    want_k = oracle.quantize(12, k.reshape(-1)).reshape(count, KVH * 144)
    want_v = oracle.quantize(14, v.reshape(-1)).reshape(count, KVH * 210)
    assert np.array_equal(got["history_packets"], np.concatenate([want_k, want_v], axis=1))

    keys, values = decode_packets(got["history_packets"], KVH, hd)
    dense = full_attention(q, keys, values, g, query_start, history_start, 512, bool(spec.attention_gate))
    for actual, expected in ((got["output"], dense["output"]), (got["physical"][..., 0] - 20.0, dense["maximum"])):
        ok, err, limit = ref_bound(actual, expected)
        assert ok, (err, limit)
    rel_z = np.abs(got["physical"][..., 1] - dense["reference"]) / dense["reference"]
    assert rel_z.max() < 1e-5

    expected = receipt_reference(dense, block, history_start)
    raw = got["receipts"]
    assert raw.shape == (len(expected), hd + 8 + block // 32)
    assert np.all((raw[:, 7] & 3) == 3) and np.all((raw[:, 7] & ~np.uint32(15)) == 0)
    nums = raw.view(np.float32)
    for rec, e in zip(raw, expected):
        cnt = e["count"]
        assert int(rec[2]) == cnt
        mask = [((1 << min(32, max(0, cnt - 32 * w))) - 1) & 0xFFFFFFFF for w in range(block // 32)]
        assert list(map(int, rec[8:8 + block // 32])) == mask
        assert 1 <= int(rec[3]) <= cnt + (cnt + 3) // 4 - 1
        assert 1 <= int(rec[4]) <= cnt and int(rec[5]) == cnt
        assert bool(int(rec[7]) & 8) == (int(rec[4]) < cnt)
        assert int(rec[6]) == (2 + (cnt + 15) // 16 if e["head"] == 0 else 0)
    wm = np.array([e["maximum"] for e in expected])
    wz = np.array([e["reference"] for e in expected])
    wu = np.array([e["numerator"] for e in expected])
    for actual, expected in ((nums[:, 0], wm), (nums[:, 1], wz), (nums[:, 8 + block // 32:], wu)):
        ok, err, limit = ref_bound(actual, expected)   # check_receipts' error_metrics bound
        assert ok, (err, limit)
    model.close()
