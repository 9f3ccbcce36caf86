"""The tiled weight layout and the GEMV that streams it (CUDA path vs the oracle).

The engine re-lays every Q4_K / Q6_K matrix once at load (rta_tile_weights):
16-row x 256-column tiles, codes in mma fragment order.  These tests pin the
byte layout against a host restatement of it, then check the tiled GEMV, SwiGLU
MLP and vocabulary readout against the oracle on the untiled (GGUF-order)
blocks, at the same shapes and tolerance as the GGUF-layout operators.
"""
import numpy as np
import pytest

from conftest import rel_l2
from oracle import oracle

TOL = 1e-3  # relative L2


def q6_codes(blocks):
    """[..., 210] Q6_K blocks -> [..., 256] 6-bit codes (GGUF bit layout)."""
    n = np.arange(256)
    part, within = n // 128, n % 128
    ql = blocks[..., part * 64 + within % 64] >> (4 * (within // 64))
    qh = blocks[..., 128 + part * 32 + within % 32] >> (2 * (within // 32))
    return (ql & 15) | ((qh & 3) << 4)


def tile_host(fmt, blocks, rows, cols):
    """Host restatement of the tiled order (see include/rta.h, rta_tile_weights)."""
    bb = 144 if fmt == 12 else 210
    kb = cols // 256
    w = blocks.reshape(rows // 16, 16, kb, bb).transpose(0, 2, 1, 3)  # [tile row][block][row][byte]
    lane = np.arange(32)
    g, t = lane >> 2, lane & 3
    if fmt == 12:
        out = np.zeros(w.shape[:2] + (2304,), np.uint8)
        for pl in range(4):
            for wi in range(4):
                row = g + 8 * (wi & 1)
                for bi in range(4):
                    src = 16 + 32 * pl + 16 * (wi >> 1) + 4 * t + bi
                    out[..., pl * 512 + lane * 16 + wi * 4 + bi] = w[..., row, src]
        out[..., 2048:] = w[..., :16].reshape(w.shape[:2] + (256,))
    else:
        code = q6_codes(w)  # [tile row][block][row][256]
        out = np.zeros(w.shape[:2] + (3360,), np.uint8)
        for j in range(8):
            for e in range(4):
                k0 = 32 * j + 4 * t + e
                k1 = k0 + 16
                c0, c08 = code[..., g, k0], code[..., g + 8, k0]
                c1, c18 = code[..., g, k1], code[..., g + 8, k1]
                for word, val in enumerate([(c0 & 15) | ((c08 & 15) << 4), (c1 & 15) | ((c18 & 15) << 4),
                                            (c0 >> 4) | ((c08 >> 4) << 2) | ((c1 >> 4) << 4) | ((c18 >> 4) << 6)]):
                    lb = 12 * j + 4 * word + e          # lane byte 0..95
                    o = (lb // 16) * 512 + lane * 16 + lb % 16
                    out[..., o] = val
        out[..., 3072:3328] = w[..., 192:208].reshape(w.shape[:2] + (256,))
        out[..., 3328:3360] = w[..., 208:210].reshape(w.shape[:2] + (32,))
    return out.reshape(-1)


def test_host_tiling_unpacks_to_the_gguf_codes():
    """The kernel's fragment unpack of a tiled block gives back every GGUF code."""
    rng = np.random.default_rng(3)
    rows, cols = 32, 512
    lane = np.arange(32)
    g, t = lane >> 2, lane & 3
    for fmt in (12, 14):
        W = oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
        bb = 144 if fmt == 12 else 210
        T = tile_host(fmt, W, rows, cols).reshape(rows // 16, cols // 256, -1)
        blocks = W.reshape(rows // 16, 16, cols // 256, bb).transpose(0, 2, 1, 3)
        if fmt == 12:
            # Q4_K: plane p word i of lane (g,t); group 2p + nib at k = 4t..4t+3 (+16 for words 2, 3)
            for p in range(4):
                words = T[..., p * 512 + lane[:, None] * 16 + np.arange(16)]  # [.., lane, 16 bytes]
                for wi in range(4):
                    row = g + 8 * (wi & 1)
                    for nib in range(2):
                        got = (words[..., 4 * wi:4 * wi + 4] >> (4 * nib)) & 15
                        src = 16 + 32 * p + 16 * (wi >> 1) + 4 * t[:, None] + np.arange(4)
                        want = (blocks[..., row[:, None], src] >> (4 * nib)) & 15
                        assert np.array_equal(got, want)
            assert np.array_equal(T[..., 2048:].reshape(blocks.shape[:2] + (16, 16)), blocks[..., :16])
        else:
            codes = q6_codes(blocks)
            lanebytes = np.stack([T[..., (b // 16) * 512 + lane * 16 + b % 16] for b in range(96)], -1)
            for j in range(8):
                L0, L1, Hh = (lanebytes[..., 12 * j + 4 * w:12 * j + 4 * w + 4].astype(np.int64) for w in range(3))
                a = [(L0 & 15) | (((Hh >> 0) & 3) << 4), (L0 >> 4) | (((Hh >> 2) & 3) << 4),
                     (L1 & 15) | (((Hh >> 4) & 3) << 4), (L1 >> 4) | (((Hh >> 6) & 3) << 4)]
                k0 = 32 * j + 4 * t[:, None] + np.arange(4)
                for i, (row, k) in enumerate([(g, k0), (g + 8, k0), (g, k0 + 16), (g + 8, k0 + 16)]):
                    assert np.array_equal(a[i], codes[..., row[:, None], k]), (j, i)
            assert np.array_equal(T[..., 3072:3328].reshape(blocks.shape[:2] + (16, 16)), blocks[..., 192:208])
            assert np.array_equal(T[..., 3328:].reshape(blocks.shape[:2] + (16, 2)), blocks[..., 208:210])


@pytest.fixture(scope="module")
def ops():
    import torch
    from rta_b200 import ops as rops
    torch.cuda.init()
    return rops


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,rows,cols", [(12, 64, 512), (14, 48, 768), (12, 32, 2048), (14, 16, 4096)])
def test_tile_layout_bit_exact(ops, fmt, rows, cols):
    rng = np.random.default_rng(rows + cols)
    W = oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    code, T = ops.tile_weights(fmt, _t(W), rows, cols)
    assert code == fmt + 100
    assert np.array_equal(_np(T), tile_host(fmt, W, rows, cols))


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,rows,cols,batch", [
    (12, 48, 256, 1), (12, 6144, 2048, 1), (12, 2048, 6144, 1), (12, 1024, 4096, 3), (12, 256, 12288, 1),
    (12, 512, 2048, 8), (12, 128, 512, 32), (14, 64, 2048, 1), (14, 4096, 4096, 2), (14, 160, 2048, 5),
    (14, 2048, 6144, 1), (14, 96, 1280, 8),
])
def test_tiled_gemv_parity(ops, fmt, rows, cols, batch):
    import torch
    rng = np.random.default_rng(rows * 7 + cols + batch)
    W = oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    x[0, :7] = 0.0
    code, T = ops.tile_weights(fmt, _t(W), rows, cols)
    y = _np(ops.gemv(code, T, rows, cols, _t(x)))
    want = oracle.gemv(fmt, W, rows, cols, x)
    assert rel_l2(y, want) < TOL, rel_l2(y, want)
    base = rng.normal(0, 1, (batch, rows)).astype(np.float32)
    acc = _t(base.copy())
    ops.gemv(code, T, rows, cols, _t(x), y=acc, accumulate=True)
    torch.cuda.synchronize()
    assert rel_l2(_np(acc), base + want) < TOL


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,cols", [(12, 2048), (14, 2048), (12, 6144), (14, 4096)])
def test_tiled_batch_rows_equal_batch_one(ops, fmt, cols):
    """Every batch row runs the batch-1 arithmetic, in both batch layouts (lanes
    carrying groups for 2 rows, MMA columns carrying rows for 3..16 rows per
    launch): identical bits at any batch size, SwiGLU pairs included."""
    rng = np.random.default_rng(11 + fmt + cols)
    rows = 256
    W = oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    U = oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    x = rng.normal(0, 1, (29, cols)).astype(np.float32)
    x[3] = 0.0
    code, T = ops.tile_weights(fmt, _t(W), rows, cols)
    _, TU = ops.tile_weights(fmt, _t(U), rows, cols)
    one = np.stack([_np(ops.gemv(code, T, rows, cols, _t(x[b:b + 1])))[0] for b in range(29)])
    one_act = np.stack([_np(ops.gemv_swiglu(code, T, TU, rows, cols, _t(x[b:b + 1])))[0] for b in range(29)])
    for batch in (2, 3, 5, 8, 13, 16, 29):
        full = _np(ops.gemv(code, T, rows, cols, _t(x[:batch])))
        assert np.array_equal(full.view(np.uint32), one[:batch].view(np.uint32)), batch
        act = _np(ops.gemv_swiglu(code, T, TU, rows, cols, _t(x[:batch])))
        assert np.array_equal(act.view(np.uint32), one_act[:batch].view(np.uint32)), batch


@pytest.mark.gpu
def test_tiled_mlp_config1_parity(ops):
    rng = np.random.default_rng(20261110)
    D, F = 2048, 6144
    Wg, Wu = (oracle.quantize(12, rng.normal(0, 0.02, F * D).astype(np.float32)) for _ in range(2))
    Wd = oracle.quantize(12, rng.normal(0, 0.02, D * F).astype(np.float32))
    x = rng.normal(0, 1, (2, D)).astype(np.float32)
    tg, tu, td = (ops.tile_weights(12, _t(w), r, c)[1] for w, r, c in ((Wg, F, D), (Wu, F, D), (Wd, D, F)))
    act, y = ops.mlp_swiglu(112, tg, tu, td, D, F, _t(x))
    want_act, want_y = oracle.mlp(12, Wg, Wu, Wd, D, F, x)
    assert rel_l2(_np(act), want_act) < TOL, rel_l2(_np(act), want_act)
    assert rel_l2(_np(y), want_y) < TOL, rel_l2(_np(y), want_y)


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 4, 64])
def test_tiled_readout_parity(ops, batch):
    rng = np.random.default_rng(77 + batch)
    V, D = 4096, 2048
    W = oracle.quantize(14, rng.normal(0, 0.02, V * D).astype(np.float32))
    x = rng.normal(0, 1, (batch, D)).astype(np.float32)
    code, T = ops.tile_weights(14, _t(W), V, D)
    logits, arg, best = ops.readout(code, T, V, D, _t(x))
    lg, want_arg, _ = oracle.lmhead(14, W, V, D, x, want_logits=True)
    assert rel_l2(_np(logits), lg) < TOL
    got = _np(arg)
    for b in range(batch):
        top = np.sort(lg[b])[-2:]
        if top[1] - top[0] > 1e-3 * max(1.0, abs(top[1])):
            assert got[b] == want_arg[b]
