"""GPU parity tests of the decode-path operators (CUDA path vs the oracle).

Bars (from the north star): dequantization and quantization bit-exact;
GEMV / MLP / readout / attention within 1e-3 relative L2 of the oracle
(fp32 accumulation); argmax identical wherever the top-2 margin exceeds it.
"""
import numpy as np
import pytest

from conftest import ref_bound, rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-3  # relative L2


@pytest.fixture(scope="module")
def ops():
    import torch
    from rta_b200 import ops as rops
    torch.cuda.init()
    return rops


def _t(a, dtype=None):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda() if dtype is None else \
        torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("fmt", [12, 14])
def test_quantize_bit_exact(ops, golden, fmt):
    rng = np.random.default_rng(21)
    values = np.concatenate([golden("quant_blocks.npz")["values"],
                             rng.normal(0, 0.02, 4096 * 256).astype(np.float32)])
    mine = _np(ops.quantize(fmt, _t(values)))
    assert np.array_equal(mine, oracle.quantize(fmt, values))


@pytest.mark.parametrize("fmt", [12, 14])
def test_dequantize_bit_exact_with_gguf(ops, golden, fmt):
    g = golden("quant_blocks.npz")
    mine = _np(ops.dequantize(fmt, _t(g[f"blocks_{fmt}"])))
    assert np.array_equal(mine.view(np.uint32), g[f"gguf_{fmt}"].view(np.uint32))


@pytest.mark.parametrize("fmt,rows,cols,batch", [
    (12, 48, 256, 1), (12, 6144, 2048, 1), (12, 2048, 6144, 1), (12, 1024, 4096, 3), (12, 256, 12288, 1),
    (12, 512, 2048, 8), (12, 128, 512, 32), (14, 64, 2048, 1), (14, 4096, 4096, 2), (14, 160, 2048, 5),
])
def test_gemv_parity(ops, fmt, rows, cols, batch):
    import torch
    rng = np.random.default_rng(rows * 7 + cols + batch)
    W = oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    x[0, :7] = 0.0
    y = _np(ops.gemv(fmt, _t(W), rows, cols, _t(x)))
    want = oracle.gemv(fmt, W, rows, cols, x)
    assert rel_l2(y, want) < TOL, rel_l2(y, want)
    # accumulate epilogue: y += W x
    base = rng.normal(0, 1, (batch, rows)).astype(np.float32)
    acc = _t(base.copy())
    ops.gemv(fmt, _t(W), rows, cols, _t(x), y=acc, accumulate=True)
    torch.cuda.synchronize()
    assert rel_l2(_np(acc), base + want) < TOL


def test_gemv_rejects_bad_shapes(ops):
    from rta_b200._lib import RtaError
    W = _t(np.zeros(144 * 8, np.uint8))
    x = _t(np.zeros((1, 256), np.float32))
    with pytest.raises(RtaError):
        ops.gemv(12, W, 8, 256, x)          # rows not a multiple of 16
    with pytest.raises(RtaError):
        ops.gemv(13, W, 16, 256, x)         # unknown format


def test_mlp_config1_parity(ops):
    """benchmark config 1: SwiGLU MLP, hidden 2048, intermediate 6144, Q4_K, batch 1."""
    D, F = 2048, 6144
    rng = np.random.default_rng(20261110)
    mats = [oracle.quantize(12, rng.normal(0, 0.02, n).astype(np.float32)) for n in (F * D, F * D, D * F)]
    x = rng.normal(0, 1, (1, D)).astype(np.float32)
    act, y = ops.mlp_swiglu(12, _t(mats[0]), _t(mats[1]), _t(mats[2]), D, F, _t(x))
    want_act, want_y = oracle.mlp(12, *mats, D, F, x)
    assert rel_l2(_np(act), want_act) < TOL
    assert rel_l2(_np(y), want_y) < TOL


def test_mlp_matches_reference_fp64_expression(ops, golden):
    """The reference's own SwiGLU oracle (verify_rt_mlp.py:85-89), rows 1/7/8/17/32."""
    g = golden("mlp_q4k.npz")
    D, F = (int(v) for v in g["shape"])
    previous = None
    for rows in (1, 7, 8, 17, 32):
        act, y = ops.mlp_swiglu(12, _t(g["w_gate"]), _t(g["w_up"]), _t(g["w_down"]), D, F, _t(g["x"][:rows]))
        act, y = _np(act), _np(y)
        assert rel_l2(act, g["activation"][:rows]) < TOL
        assert rel_l2(y, g["output"][:rows]) < TOL
        if rows > 1:
            assert np.all(y[1] == 0) and np.all(act[1] == 0)   # zero input row -> zero output
        if previous is not None:                               # row-prefix consistency (bit-identical)
            np.testing.assert_array_equal(y[:len(previous)], previous)
        previous = y


@pytest.mark.parametrize("batch", [1, 4])
def test_readout_config3_parity(ops, batch):
    """benchmark config 3: LM head 151936 x 2048 Q6_K, logits + argmax."""
    V, D = 151936, 2048
    rng = np.random.default_rng(31 + batch)
    W = oracle.quantize(14, rng.normal(0, 0.02, V * D).astype(np.float32))
    x = rng.normal(0, 1, (batch, D)).astype(np.float32)
    logits, arg, best = ops.readout(14, _t(W), V, D, _t(x))
    want_logits, want_arg, want_best = oracle.lmhead(14, W, V, D, x)
    logits, arg = _np(logits), _np(arg)
    assert rel_l2(logits, want_logits) < TOL
    for b in range(batch):
        top2 = np.sort(want_logits[b])[-2:]
        margin = (top2[1] - top2[0]) / max(abs(top2[1]), 1e-30)
        if margin > TOL:
            assert arg[b] == want_arg[b]
        assert logits[b, arg[b]] == _np(best)[b]


def test_readout_tie_goes_to_lowest_id(ops):
    V, D = 4096, 2048
    w = np.zeros((V, D), np.float32)
    w[[77, 1033, 4000], 5] = 0.5
    W = oracle.quantize(14, w)
    x = np.zeros((1, D), np.float32)
    x[0, 5] = 1.0
    _, arg, _ = ops.readout(14, _t(W), V, D, _t(x), logits=False)
    assert int(_np(arg)[0]) == 77


def _attention_case(ops, q, keys, values, gate, time, capacity, layout="LHD", splits=None):
    """Run the CUDA kernel with fp16 K/V; return (out, phys, oracle_out, oracle_phys)."""
    import torch
    count = keys.shape[0]
    kvh = keys.shape[1]
    k16 = keys.astype(np.float16)
    v16 = values.astype(np.float16)
    # ring layout: position p in slot p % capacity
    slots = np.zeros((capacity, kvh, 256), np.float16), np.zeros((capacity, kvh, 256), np.float16)
    for p in range(count):
        slots[0][p % capacity] = k16[p]
        slots[1][p % capacity] = v16[p]
    if layout == "LHD":
        kd, vd = _t(slots[0]), _t(slots[1])
        pos_stride, kv_stride = kvh, 1
    else:  # [kvh][capacity][hd]
        kd, vd = _t(np.ascontiguousarray(slots[0].transpose(1, 0, 2))), \
            _t(np.ascontiguousarray(slots[1].transpose(1, 0, 2)))
        pos_stride, kv_stride = 1, capacity
    out, phys, ws = ops.attention_decode_f16(_t(q), kd, vd, time, capacity, pos_stride, kv_stride,
                                             gate=None if gate is None else _t(gate), splits=splits)
    torch.cuda.synchronize()
    assert ops.workspace_error(ws) == 0
    want, want_phys = oracle.attention(q[None], k16.astype(np.float32), v16.astype(np.float32),
                                       None if gate is None else gate[None], time, 0, capacity, gate is not None)
    return _np(out), _np(phys), want[0], want_phys[0]


@pytest.mark.parametrize("L", [1, 17, 64, 65, 512, 4096, 32768])
def test_attention_config2_parity(ops, L):
    """Benchmark config 2 at every history length it names (512 / 4096 / 32768,
    default splits) against the oracle, plus short edge lengths."""
    rng = np.random.default_rng(L)
    q = rng.normal(0, 1, (16, 256)).astype(np.float32)
    keys = rng.normal(0, 1, (L, 4, 256)).astype(np.float32)
    values = rng.normal(0, 1, (L, 4, 256)).astype(np.float32)
    out, phys, want, want_phys = _attention_case(ops, q, keys, values, None, L - 1, L)
    assert rel_l2(out, want) < TOL
    np.testing.assert_allclose(phys, want_phys, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("L,splits", [(4096, 64), (5000, 48), (300, 40)])
def test_attention_many_splits(ops, L, splits):
    """More split CTAs than SMs (64 x 4 KV heads, 48 x 4, 40 x 4): the four-stage
    kernel that runs several CTAs per SM; 300 positions over 40 splits leaves
    most of them empty."""
    rng = np.random.default_rng(L + splits)
    q = rng.normal(0, 1, (16, 256)).astype(np.float32)
    keys = rng.normal(0, 1, (L, 4, 256)).astype(np.float32)
    values = rng.normal(0, 1, (L, 4, 256)).astype(np.float32)
    gate = rng.normal(0, 2, (16, 256)).astype(np.float32)
    out, phys, want, want_phys = _attention_case(ops, q, keys, values, gate, L - 1, L, splits=splits)
    assert rel_l2(out, want) < TOL
    np.testing.assert_allclose(phys, want_phys, rtol=1e-4, atol=1e-4)


def test_attention_ring_wrap_and_gate(ops):
    rng = np.random.default_rng(9)
    count, capacity = 700, 256           # only the newest 256 positions are visible
    q = rng.normal(0, 1, (16, 256)).astype(np.float32)
    keys = rng.normal(0, 1, (count, 4, 256)).astype(np.float32)
    values = rng.normal(0, 1, (count, 4, 256)).astype(np.float32)
    gate = rng.normal(0, 2, (16, 256)).astype(np.float32)
    for layout in ("LHD", "HLD"):
        out, phys, want, want_phys = _attention_case(ops, q, keys, values, gate, count - 1, capacity, layout)
        assert rel_l2(out, want) < TOL


def test_attention_reference_adversarial_cases(ops, golden):
    """The reference's own case generator (verify_attention_receipts.cases) through the
    fp16 cache.  Keys beyond the fp16 range (the 1e6 ramp case) need the packet
    format and are excluded here."""
    g = golden("attention_cases.npz")
    for name in g["names"]:
        if str(name) == "tiny_q_with_nontrivial_scores":
            continue
        qs, hs, cap = (int(v) for v in g[f"{name}/meta"])
        q, gate = g[f"{name}/query"], g[f"{name}/gate"]
        keys, values = g[f"{name}/keys"], g[f"{name}/values"]
        for r in range(q.shape[0]):
            t = qs + r
            out, phys, want, _ = _attention_case(ops, q[r], keys[:t + 1], values[:t + 1], gate[r], t, cap)
            ok, err, limit = ref_bound(out, want, 2e-5)
            assert ok or rel_l2(out, want) < 1e-5, (str(name), r, err, limit)
            # and against the reference's FP64 oracle on the fp32 inputs (fp16 storage error only)
            assert rel_l2(out, g[f"{name}/output"][r]) < TOL, (str(name), r)


def test_attention_long_history_properties(ops):
    """L = 32768, size-independent properties on top of the oracle comparison:
    constant V gives that constant; a dominant key selects its value."""
    import torch
    L = 32768
    rng = np.random.default_rng(4)
    q = rng.normal(0, 1, (16, 256)).astype(np.float32)
    k = torch.randn(L, 4, 256, device="cuda").half()
    v = torch.full((L, 4, 256), 0.375, device="cuda").half()
    out, phys, ws = ops.attention_decode_f16(_t(q), k, v, L - 1, L, 4, 1)
    torch.cuda.synchronize()
    assert np.allclose(_np(out), 0.375, rtol=1e-5)
    # one position with a huge score dominates: its value row is returned
    kk = torch.zeros(L, 4, 256, device="cuda").half()
    vv = torch.randn(L, 4, 256, device="cuda").half()
    q2 = np.zeros((16, 256), np.float32)
    q2[:, 0] = 8.0
    kk[12345, :, 0] = 60.0
    out, _, _ = ops.attention_decode_f16(_t(q2), kk, vv, L - 1, L, 4, 1)
    torch.cuda.synchronize()
    want = _np(vv[12345].float()).repeat(4, axis=0)
    assert rel_l2(_np(out), want) < 1e-4
