"""CPU tests: the oracle (C restatement of the reference shader math) pinned
against the reference's own CPU code through the committed golden fixtures."""
import json

import numpy as np
import pytest

from conftest import GOLDEN, ref_bound, rel_l2
from oracle import oracle


def test_half_conversion_matches_ieee_rne():
    rng = np.random.default_rng(1)
    f = np.concatenate([
        rng.normal(0, 1, 20000), rng.normal(0, 1e-5, 5000), rng.normal(0, 1e-7, 5000),
        rng.normal(0, 3e4, 5000), [0.0, -0.0, 65504.0, 65520.0, 65519.99, 1e10, -1e10, 2 ** -24, 2 ** -25,
                                   3 * 2 ** -26, 2 ** -14, np.inf, -np.inf],
    ]).astype(np.float32)
    lib = oracle.lib()
    mine = np.array([lib.rta_oracle_float_to_half(float(v)) for v in f], dtype=np.uint16)
    ref = f.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref)
    back = np.array([lib.rta_oracle_half_to_float(int(h)) for h in range(0, 65536, 7)], np.float32)
    want = np.arange(0, 65536, 7, dtype=np.uint16).view(np.float16).astype(np.float32)
    ok = ~np.isnan(want)
    assert np.array_equal(back[ok].view(np.uint32), want[ok].view(np.uint32))


@pytest.mark.parametrize("fmt", [12, 14])
def test_dequant_bit_exact_with_gguf(golden, fmt):
    g = golden("quant_blocks.npz")
    blocks = g[f"blocks_{fmt}"]
    mine = oracle.dequantize(fmt, blocks)
    assert np.array_equal(mine.view(np.uint32), g[f"gguf_{fmt}"].view(np.uint32))


@pytest.mark.parametrize("fmt", [12, 14])
def test_quantizer_reproduces_fixture_blocks(golden, fmt):
    g = golden("quant_blocks.npz")
    assert np.array_equal(oracle.quantize(fmt, g["values"]), g[f"blocks_{fmt}"])


@pytest.mark.parametrize("fmt", [12, 14])
def test_quantizer_error_bound(fmt):
    rng = np.random.default_rng(3)
    v = rng.normal(0, 0.02, 256 * 256).astype(np.float32)
    d = oracle.dequantize(fmt, oracle.quantize(fmt, v))
    # per-block error is bounded by half a quantization step of the block range
    assert rel_l2(d, v) < (0.08 if fmt == 12 else 0.02)


def test_attention_oracle_matches_reference_fp64(golden):
    g = golden("attention_cases.npz")
    worst = 0.0
    for name in g["names"]:
        qs, hs, cap = (int(v) for v in g[f"{name}/meta"])
        out, phys = oracle.attention(g[f"{name}/query"], g[f"{name}/keys"], g[f"{name}/values"], g[f"{name}/gate"],
                                     qs, hs, cap, True)
        ok, err, limit = ref_bound(out, g[f"{name}/output"])
        assert ok, (str(name), err, limit)
        np.testing.assert_allclose(phys[..., 0] - 20.0, g[f"{name}/maximum"], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(phys[..., 1], g[f"{name}/reference"], rtol=2e-5)
        worst = max(worst, err / limit)
    assert worst <= 1.0


def test_mlp_oracle_matches_reference_fp64(golden):
    g = golden("mlp_q4k.npz")
    D, F = (int(v) for v in g["shape"])
    act, y = oracle.mlp(12, g["w_gate"], g["w_up"], g["w_down"], D, F, g["x"])
    ok, err, limit = ref_bound(act, g["activation"])
    assert ok, (err, limit)
    ok, err, limit = ref_bound(y, g["output"])
    assert ok, (err, limit)
    # zero rows stay exactly zero (verify_rt_mlp.py: rows of x[1] = 0)
    assert np.all(y[1] == 0) and np.all(act[1] == 0)


def test_gemv_matches_fp64_dot():
    rng = np.random.default_rng(5)
    rows, cols = 48, 768
    for fmt in (12, 14):
        W = oracle.quantize(fmt, rng.normal(0, 0.05, rows * cols).astype(np.float32))
        x = rng.normal(0, 1, (3, cols)).astype(np.float32)
        y = oracle.gemv(fmt, W, rows, cols, x)
        dense = oracle.dequantize(fmt, W).reshape(rows, cols).astype(np.float64)
        assert rel_l2(y, x.astype(np.float64) @ dense.T) < 1e-6


def test_lmhead_argmax_ties_go_to_lowest_id():
    V, D = 64, 256
    w = np.zeros((V, D), np.float32)
    w[[5, 9, 40], 0] = 1.0          # three identical best rows
    w[7, 0] = -1.0
    W = oracle.quantize(14, w)
    x = np.zeros((1, D), np.float32)
    x[0, 0] = 2.0
    logits, arg, best = oracle.lmhead(14, W, V, D, x)
    assert arg[0] == 5 and best[0] == logits[0, 5]


def _gdn_fp64(x, qk, v, z, wa, wb, a_log, dt_bias, conv_w, norm_w, H, KH, eps, state, conv):
    """Independent FP64 statement of the gated delta rule (rows = 1)."""
    S, K, HD = H * 128, KH * 128, 128
    sig = lambda t: 1 / (1 + np.exp(-t))
    raw = np.concatenate([np.tile(qk[:K], H // KH), np.tile(qk[K:], H // KH), v]).astype(np.float64)
    hist = np.concatenate([conv.astype(np.float64), raw[:, None]], 1)          # [3S, 4] oldest..current
    sig_in = (hist * conv_w.astype(np.float64)).sum(1)
    frame = sig_in * sig(sig_in)
    a = wa.astype(np.float64) @ x.astype(np.float64)
    b = wb.astype(np.float64) @ x.astype(np.float64)
    decay = np.exp(-np.exp(a_log.astype(np.float64)) * np.log1p(np.exp(a + dt_bias)))
    beta = sig(b)
    out = np.zeros(S)
    st = state.astype(np.float64).copy()
    for h in range(H):
        q = frame[h * HD:(h + 1) * HD]
        k = frame[S + h * HD:S + (h + 1) * HD]
        q = q / np.sqrt((q * q).sum() + eps)
        k = k / np.sqrt((k * k).sum() + eps)
        vv = frame[2 * S + h * HD:2 * S + (h + 1) * HD]
        s = st[h] * decay[h]
        r = s @ k
        s = s + np.outer((vv - r) * beta[h], k)
        o = s @ (q / np.sqrt(HD))
        st[h] = s
        zz = z[h * HD:(h + 1) * HD].astype(np.float64)
        o = o / np.sqrt((o * o).mean() + eps) * norm_w[h * HD:(h + 1) * HD] * zz * sig(zz)
        out[h * HD:(h + 1) * HD] = o
    return out, st, hist[:, 1:]


@pytest.mark.parametrize("H,KH", [(2, 2), (4, 2)])
def test_gdn_oracle_matches_fp64_statement(H, KH):
    rng = np.random.default_rng(11)
    D, S, K = 256, H * 128, KH * 128
    x = rng.normal(0, 1, (1, D)).astype(np.float32)
    qk = rng.normal(0, 1, (1, 2 * K)).astype(np.float32)
    v = rng.normal(0, 1, (1, S)).astype(np.float32)
    z = rng.normal(0, 1, (1, S)).astype(np.float32)
    wa = rng.normal(0, 0.05, (H, D)).astype(np.float32)
    wb = rng.normal(0, 0.05, (H, D)).astype(np.float32)
    a_log = rng.normal(0, 0.5, H).astype(np.float32)
    dt_bias = rng.normal(0, 0.5, H).astype(np.float32)
    conv_w = rng.normal(0, 0.5, (3 * S, 4)).astype(np.float32)
    norm_w = rng.normal(1, 0.1, S).astype(np.float32)
    state = rng.normal(0, 0.1, (H, 128, 128)).astype(np.float32)
    conv = rng.normal(0, 1, (3 * S, 3)).astype(np.float32)
    want, want_state, want_conv = _gdn_fp64(x[0], qk[0], v[0], z[0], wa, wb, a_log, dt_bias, conv_w, norm_w, H, KH,
                                            1e-6, state, conv)
    st, cv = state.copy(), conv.copy()
    out = oracle.gdn(x, qk, v, z, wa, wb, a_log, dt_bias, conv_w, norm_w, H, KH, 1e-6, st, cv)
    assert rel_l2(out[0], want) < 1e-5
    assert rel_l2(st, want_state) < 1e-5
    assert np.allclose(cv, want_conv)


def test_reference_geometry_manifest():
    m = json.loads((GOLDEN / "manifest.json").read_text())
    assert m["spec_2b"]["history_bytes"] == 1416 and m["spec_2b"]["fingerprint"] == "d1b9251ad05ff9b6"
    assert m["cpu_selftest"]["group_merge_FP64"] is True
    assert m["gguf_version"] == "0.19.0"


@pytest.mark.parametrize("fmt", [0, 1, 30])
def test_dense_formats_decode_and_gemv(fmt):
    """Dense F32 / F16 / BF16 rows (ggufValue's first branches): the oracle's decode
    equals numpy's conversion of the same bits, and its octet-order GEMV equals an
    FP64 matrix product of the decoded weights within fp32 rounding."""
    rng = np.random.default_rng(fmt + 3)
    rows, cols = 48, 512
    w = rng.normal(0, 0.02, rows * cols).astype(np.float32)
    raw = {0: w.view(np.uint8), 1: w.astype(np.float16).view(np.uint8),
           30: oracle.to_bf16_bits(w).view(np.uint8)}[fmt]
    dec = oracle.dense_values(fmt, raw)
    want_dec = {0: w, 1: w.astype(np.float16).astype(np.float32),
                30: (oracle.to_bf16_bits(w).astype(np.uint32) << 16).view(np.float32)}[fmt]
    assert np.array_equal(dec.view(np.uint32), want_dec.view(np.uint32))
    assert oracle.row_bytes(fmt, cols) * rows == raw.size
    x = rng.normal(0, 1, (3, cols)).astype(np.float32)
    y = oracle.gemv(fmt, raw, rows, cols, x)
    want = x.astype(np.float64) @ dec.reshape(rows, cols).astype(np.float64).T
    assert rel_l2(y, want) < 1e-6
    if fmt == 30:  # bf16 rounds to nearest even: halfway cases go to the even neighbour
        assert oracle.to_bf16_bits(np.float32([1.00390625, 1.01171875])).tolist() == [0x3F80, 0x3F82]
