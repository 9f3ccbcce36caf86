"""The tensor-core batched product (qgemm.cu): panel layout, dequantizer and
block algebra, restated on the host and checked against the GGUF decode.

The kernel expands each panel row into fp16 integers A = sc*(q-8) (Q4_K:
one mask-and-or puts a nibble under the exponent byte, 0x6400 | 16q is
1024 + 16q, and one fp16 FMA (1024 + 16q)(sc/16) - 72 sc is exact; the panel
stores each code word as bytes (0, 2, 1, 3) so that the pairs come out in K
order) or sc*(q-32) (Q6_K: byte permutes and a bit-select), and multiplies by
the row's block scale times 2^6 (one fp16 rounding), so the accumulator sums
whole K ranges; the Q4_K mins enter as one more K=16 product of
fp16(2^6 (8 d sc - dmin m)) against the group sums, into the same
accumulator, and the epilogue scales by 2^-6.
These host tests emulate exactly those bit operations (an fp16 FMA is the
exact product-sum rounded once, which float64 reproduces for these integers)
and the block algebra, so the index math is pinned before any GPU run.  The
GPU tests compare the kernel with the oracle GEMV / readout.
"""
import numpy as np
import pytest

from conftest import rel_l2
from oracle import oracle

TOL = 1e-3  # relative L2


# ----------------------------------------------------------- host layout
def panel_host(fmt, blocks, rows, cols):
    """GGUF rows -> panel order (qgemm.cu header: one panel per 128-row tile and block column)."""
    bb = 144 if fmt == 12 else 210
    kb = cols // 256
    w = blocks.reshape(rows // 128, 128, kb, bb).transpose(0, 2, 1, 3)  # [tile][block col][row][byte]
    if fmt == 12:
        swap = np.array([0, 2, 1, 3, 4, 6, 5, 7, 8, 10, 9, 11, 12, 14, 13, 15])  # each code word as bytes (0, 2, 1, 3)
        codes = w[..., 16:].reshape(w.shape[:3] + (4, 2, 16))[..., swap].transpose(0, 1, 3, 4, 2, 5)  # [.., pl, part, row, 16]
        out = np.concatenate([codes.reshape(w.shape[:2] + (16384,)), w[..., :16].reshape(w.shape[:2] + (2048,))], -1)
    else:
        parts = []
        for h in range(2):
            ql = w[..., 64 * h:64 * h + 64].reshape(w.shape[:3] + (2, 2, 16)).transpose(0, 1, 3, 4, 2, 5)
            qh = w[..., 128 + 32 * h:160 + 32 * h].reshape(w.shape[:3] + (2, 16)).transpose(0, 1, 3, 2, 4)
            parts += [ql.reshape(w.shape[:2] + (8192,)), qh.reshape(w.shape[:2] + (4096,))]
        parts += [w[..., 192:208].reshape(w.shape[:2] + (2048,)), w[..., 208:210].reshape(w.shape[:2] + (256,))]
        out = np.concatenate(parts, -1)
    return np.ascontiguousarray(out).reshape(-1)


# ------------------------------------------------------ bit-level emulation
def byte_perm(x, y, s):
    src = [(x >> (8 * i)) & 0xFF for i in range(4)] + [(y >> (8 * i)) & 0xFF for i in range(4)]
    return sum(src[(s >> (4 * i)) & 7] << (8 * i) for i in range(4))


def halves(u):
    return np.array([u & 0xFFFF, u >> 16], np.uint16).view(np.float16).astype(np.float64)


def hfma2(u, s, k):
    """__hfma2 on the two halves of u: exact a*s+k rounded once to fp16."""
    a = halves(u)
    return (a * np.float64(np.float16(s)) + np.float64(np.float16(k))).astype(np.float16).astype(np.float64)


def words(b):
    return [int.from_bytes(bytes(b[4 * i:4 * i + 4]), "little") for i in range(len(b) // 4)]


def q4_scale_min(hdr, G):
    if G < 4:
        return hdr[4 + G] & 63, hdr[8 + G] & 63
    mixed = hdr[12 + G - 4]
    return (mixed & 15) | ((hdr[G] >> 6) << 4), (mixed >> 4) | ((hdr[4 + G] >> 6) << 4)


def q4_scales_host(hdr, j):
    """Emulates q4_scales: the 6-bit (sc, m) of groups 2j, 2j+1, 4+2j, 5+2j from
    the three 16-bit header fields at bytes 4+2j, 8+2j, 12+2j."""
    w = words(np.asarray(hdr, np.uint8))
    Y, Z, W = (w[1] >> (16 * j)) & 0xFFFF, (w[2] >> (16 * j)) & 0xFFFF, (w[3] >> (16 * j)) & 0xFFFF
    sc = [Y & 63, (Y >> 8) & 63, (W & 15) | ((Y >> 2) & 48), ((W >> 8) & 15) | ((Y >> 10) & 48)]
    mn = [Z & 63, (Z >> 8) & 63, ((W >> 4) & 15) | ((Z >> 2) & 48), ((W >> 12) & 15) | ((Z >> 10) & 48)]
    return sc, mn


def dequant_q4_host(P, m, h, j):
    """Emulates dequant_q4: 32 tensor-memory columns (64 fp16 sc*(q-8), before
    the block scale) of row m."""
    hdr = P[16384 + 16 * m:16384 + 16 * m + 16].astype(np.int64)
    pl = 2 * h + j
    c = np.concatenate([P[((pl * 2 + p) * 128 + m) * 16:((pl * 2 + p) * 128 + m) * 16 + 16] for p in range(2)])
    sc, _ = q4_scales_host(hdr, j)
    sc0, sc1 = sc[2 * h], sc[2 * h + 1]
    mask, magic = 0x00F000F0, 0x64006400
    lo, hi = [], []
    for x in words(c):
        lo += list(hfma2((((x << 4) & 0xFFFFFFFF) & mask) | magic, sc0 * 0.0625, -72.0 * sc0))
        lo += list(hfma2(((x >> 4) & mask) | magic, sc0 * 0.0625, -72.0 * sc0))
        hi += list(hfma2((x & mask) | magic, sc1 * 0.0625, -72.0 * sc1))
        hi += list(hfma2(((x >> 8) & mask) | magic, sc1 * 0.0625, -72.0 * sc1))
    return np.array(lo + hi)  # coefficient order 64j + 0..63 of the half-step


def dequant_q6_host(P, m, h, j):
    """Emulates dequant_q6: columns 16j.. (low run) and 32 + 16j.. (high run) of row m
    (bit-select of the ql permute and the permute of the pre-shifted qh word)."""
    base = 12288 * h
    ql = np.concatenate([P[base + ((j * 2 + p) * 128 + m) * 16:base + ((j * 2 + p) * 128 + m) * 16 + 16]
                         for p in range(2)])
    qh = np.concatenate([P[base + 8192 + (p * 128 + m) * 16:base + 8192 + (p * 128 + m) * 16 + 16] for p in range(2)])
    s4 = words(P[24576 + 16 * m:24576 + 16 * m + 16])
    wl, wh = (s4[2], s4[3]) if h else (s4[0], s4[1])
    int8 = lambda word, i: ((word >> (8 * i)) & 0xFF) - 256 * (((word >> (8 * i)) & 0xFF) > 127)
    qlw, qhw = words(ql), words(qh)
    sel = 0xFCF0FCF0
    lo, hi = [], []
    for w in range(8):
        u = w // 4
        a, b = int8(wl, 2 * j + u), int8(wh, 2 * j + u)
        qs = (qlw[w] << 4) & 0xFFFFFFFF
        hl, hh = qhw[w] >> (2 * j), qhw[w] >> (4 + 2 * j)
        for sel_l, sel_h in ((0x5140, 0x1404), (0x5342, 0x3424)):
            al, ah = byte_perm(qs, 0x64646464, sel_l), byte_perm(qlw[w], 0x64646464, sel_l)
            bl, bh = byte_perm(hl, 0, sel_h), byte_perm(hh, 0, sel_h)
            lo += list(hfma2((al & sel) | (bl & ~sel & 0xFFFFFFFF), a * 0.0625, -96.0 * a))
            hi += list(hfma2((ah & sel) | (bh & ~sel & 0xFFFFFFFF), b * 0.0625, -96.0 * b))
    return np.array(lo), np.array(hi)


def gguf_q4(block):
    """(d, dmin, sc*q per coefficient, m per group) of one Q4_K block."""
    d = np.frombuffer(bytes(block[0:2]), np.float16)[0]
    dmin = np.frombuffer(bytes(block[2:4]), np.float16)[0]
    hdr = block[:16].astype(np.int64)
    k = np.arange(256)
    q = (block[16 + (k // 64) * 32 + k % 32].astype(np.int64) >> (4 * ((k % 64) // 32))) & 15
    sm = np.array([q4_scale_min(hdr, G) for G in range(8)])
    return float(d), float(dmin), sm[k // 32, 0] * q, sm[:, 1]


def gguf_q6(block):
    d = np.frombuffer(bytes(block[208:210]), np.float16)[0]
    k = np.arange(256)
    half, local = k // 128, k % 128
    ql = (block[half * 64 + local % 64].astype(np.int64) >> (4 * (local // 64))) & 15
    qh = (block[128 + half * 32 + local % 32].astype(np.int64) >> (2 * (local // 32))) & 3
    sc = block[192:208].view(np.int8).astype(np.int64)
    return float(d), sc[k // 16] * ((ql | (qh << 4)) - 32)


def _matrix(fmt, rows, cols, seed):
    rng = np.random.default_rng(seed)
    return oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))


@pytest.mark.parametrize("fmt", [12, 14])
def test_dequantizer_emulation_gives_exact_block_integers(fmt):
    rows, cols = 128, 512
    W = _matrix(fmt, rows, cols, 5 + fmt)
    bb = 144 if fmt == 12 else 210
    P = panel_host(fmt, W, rows, cols).reshape(cols // 256, -1)  # one tile: [block col][panel bytes]
    blocks = W.reshape(rows, cols // 256, bb)
    for kb in range(cols // 256):
        for m in (0, 1, 31, 64, 127):
            if fmt == 12:
                _, _, A, mins = gguf_q4(blocks[m, kb])
                hdr = blocks[m, kb][:16].astype(np.int64)
                scs = np.array([q4_scale_min(hdr, G)[0] for G in range(8)])
                for h in range(2):
                    for j in range(2):
                        got = dequant_q4_host(P[kb], m, h, j)
                        k = np.arange(128 * h + 64 * j, 128 * h + 64 * j + 64)
                        want = A[k] - 8 * scs[k // 32]
                        assert np.array_equal(got, want.astype(np.float64)), (kb, m, h, j)
                    sc, mn = q4_scales_host(P[kb][16384 + 16 * m:16384 + 16 * m + 16].astype(np.int64), h)
                    groups = [2 * h, 2 * h + 1, 4 + 2 * h, 5 + 2 * h]  # thread j = h here
                    assert sc == [q4_scale_min(hdr, G)[0] for G in groups]
                    assert mn == [int(mins[G]) for G in groups]
            else:
                _, A = gguf_q6(blocks[m, kb])
                for h in range(2):
                    for j in range(2):
                        lo, hi = dequant_q6_host(P[kb], m, h, j)
                        wl = A[128 * h + 32 * j:128 * h + 32 * j + 32].astype(np.float64)
                        wh = A[128 * h + 64 + 32 * j:128 * h + 96 + 32 * j].astype(np.float64)
                        # fp16 holds |A| <= 2048 exactly and rounds larger values to even
                        assert np.array_equal(lo, wl.astype(np.float16).astype(np.float64)), (kb, m, h, j)
                        assert np.array_equal(hi, wh.astype(np.float16).astype(np.float64)), (kb, m, h, j)


@pytest.mark.parametrize("fmt", [12, 14])
def test_block_algebra_matches_the_oracle_gemv(fmt):
    """The folded operand fp16(2^6 d * sc (q - 8)) (and, for Q4_K, fp16(2^6 (8 d sc -
    dmin m)) against the hi / lo sums of the fp16-rounded x, so the mins cancel
    against the same x the codes see), accumulated over blocks in fp32 and scaled
    by 2^-6, is the oracle GEMV well within the north-star tolerance (centring the
    codes keeps the two rounded terms small next to the weight they sum to)."""
    rows, cols, batch = 128, 768, 3
    W = _matrix(fmt, rows, cols, 11 + fmt)
    rng = np.random.default_rng(fmt)
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    bb = 144 if fmt == 12 else 210
    blocks = W.reshape(rows, cols // 256, bb)
    xh = x.astype(np.float16).astype(np.float64)
    h16 = lambda a: np.asarray(a, np.float64).astype(np.float16).astype(np.float64)
    y = np.zeros((batch, rows), np.float32)
    for r in range(rows):
        acc = np.zeros(batch, np.float32)
        for kb in range(cols // 256):
            xs = xh[:, 256 * kb:256 * kb + 256]
            if fmt == 12:
                d, dmin, A, mins = gguf_q4(blocks[r, kb])
                hdr = blocks[r, kb][:16].astype(np.int64)
                scs = np.array([q4_scale_min(hdr, G)[0] for G in range(8)], np.float64)
                XG = xs.astype(np.float32).reshape(batch, 8, 32).sum(-1, dtype=np.float32)  # sums of the fp16 x
                Xhi = XG.astype(np.float16).astype(np.float64)
                Xlo = (XG - Xhi).astype(np.float16).astype(np.float64)
                Af = h16(h16(64.0 * d) * h16(A - 8.0 * scs[np.arange(256) // 32]))
                Mf = h16(64.0 * (8.0 * d * scs - dmin * mins.astype(np.float64)))
                acc = (acc + (xs @ Af).astype(np.float32) + ((Xhi + Xlo) @ Mf).astype(np.float32)).astype(np.float32)
            else:
                d, A = gguf_q6(blocks[r, kb])
                Af = h16(h16(64.0 * d) * h16(A))
                acc = (acc + (xs @ Af).astype(np.float32)).astype(np.float32)
        y[:, r] = acc / np.float32(64.0)
    want = oracle.gemv(fmt, W, rows, cols, x)
    err = rel_l2(y, want)
    assert err < 5e-4, err
    print(f"fmt {fmt}: folded-operand algebra rel-L2 {err:.2e}")


# ---------------------------------------------------------------- GPU
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
@pytest.mark.parametrize("fmt,rows,cols", [(12, 128, 512), (14, 256, 768), (12, 384, 2048), (14, 128, 4096)])
def test_panel_layout_bit_exact(ops, fmt, rows, cols):
    W = _matrix(fmt, rows, cols, rows + cols)
    code, P = ops.panel_weights(fmt, _t(W), rows, cols)
    assert code == fmt + 200
    assert np.array_equal(_np(P), panel_host(fmt, W, rows, cols))


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,rows,cols,batch", [
    (12, 128, 256, 16), (12, 256, 2048, 1), (12, 384, 2048, 17), (12, 2048, 6144, 64), (12, 1024, 4096, 33),
    (12, 512, 12288, 8), (12, 256, 2048, 100), (14, 128, 2048, 16), (14, 640, 2048, 64), (14, 256, 4096, 5),
    (14, 2048, 6144, 32), (14, 384, 1280, 130),
])
def test_gemm_tc_parity(ops, fmt, rows, cols, batch):
    rng = np.random.default_rng(rows * 3 + cols + batch)
    W = oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    x[0, :7] = 0.0
    if batch > 2:
        x[2] = 0.0
    code, P = ops.panel_weights(fmt, _t(W), rows, cols)
    y, _, _ = ops.gemm_tc(code, P, rows, cols, _t(x))
    y = _np(y)
    want = oracle.gemv(fmt, W, rows, cols, x)
    assert rel_l2(y, want) < TOL, rel_l2(y, want)
    for b in range(batch):  # every batch row on its own, not only in aggregate
        if b == 2:
            assert np.all(y[b] == 0)
            continue
        assert rel_l2(y[b], want[b]) < TOL, (b, rel_l2(y[b], want[b]))


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,rows,cols,batch", [(12, 384, 2048, 64), (12, 256, 4096, 20), (14, 128, 2048, 33),
                                                 (14, 640, 2048, 64), (12, 512, 12288, 16)])
def test_gemm_tc_split_activations(ops, fmt, rows, cols, batch):
    """RTA_GEMM_SPLIT_ACTIVATIONS: x enters as fp16(x) + fp16(x - fp16(x)) (twice
    the MMA columns: 32, 64 or 128), so only the weight operand's rounding is
    left -- within the tolerance, and no farther from the oracle than the one
    fp16 rounding of x; stores and residual adds alike."""
    rng = np.random.default_rng(rows + cols + batch + 7)
    W = oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    x[1] = 0.0
    code, P = ops.panel_weights(fmt, _t(W), rows, cols)
    want = oracle.gemv(fmt, W, rows, cols, x)
    y_plain, _, _ = ops.gemm_tc(code, P, rows, cols, _t(x))
    y_split, _, _ = ops.gemm_tc(code, P, rows, cols, _t(x), split=True)
    e_plain, e_split = rel_l2(_np(y_plain), want), rel_l2(_np(y_split), want)
    assert e_split < TOL and e_split <= e_plain, (e_split, e_plain)
    assert np.all(_np(y_split)[1] == 0)
    y0 = rng.normal(0, 1, (batch, rows)).astype(np.float32)
    y = _t(y0)
    ops.gemm_tc(code, P, rows, cols, _t(x), y=y, accumulate=True, split=True)
    assert rel_l2(_np(y) - y0, want) < TOL


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,rows,cols", [(12, 256, 2048), (14, 256, 2048), (12, 1024, 4096), (14, 512, 12288)])
def test_gemm_tc_accumulates_into_the_residual(ops, fmt, rows, cols):
    """K-split schedules (8 slices of 1, 2 or 6 blocks here) add their partial
    sums into the residual."""
    batch = 24
    rng = np.random.default_rng(fmt + 40)
    W = oracle.quantize(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    y0 = rng.normal(0, 1, (batch, rows)).astype(np.float32)
    code, P = ops.panel_weights(fmt, _t(W), rows, cols)
    y = _t(y0)
    ops.gemm_tc(code, P, rows, cols, _t(x), y=y, accumulate=True)
    want = y0 + oracle.gemv(fmt, W, rows, cols, x)
    assert rel_l2(_np(y), want) < TOL


@pytest.mark.gpu
@pytest.mark.parametrize("batch,split", [(16, False), (64, False), (64, True)])
def test_gemm_tc_readout_argmax(ops, batch, split):
    """Config 3 shape class: Q6_K vocabulary rows with the per-row argmax (also
    with split activations: 128 MMA columns, whole tiles per CTA)."""
    V, D = 151936 // 8, 2048  # 18992 rows (a multiple of 128 would be needed: trimmed below)
    V = V // 128 * 128
    rng = np.random.default_rng(batch)
    W = oracle.quantize(14, rng.normal(0, 0.02, V * D).astype(np.float32))
    x = rng.normal(0, 1, (batch, D)).astype(np.float32)
    code, P = ops.panel_weights(14, _t(W), V, D)
    lg, ids, best = ops.gemm_tc(code, P, V, D, _t(x), argmax=True, split=split)
    want_lg, want_arg, want_best = oracle.lmhead(14, W, V, D, x)
    lg, ids, best = _np(lg), _np(ids).astype(np.int64), _np(best)
    assert rel_l2(lg, want_lg) < TOL
    for b in range(batch):
        assert best[b] == lg[b, ids[b]] and ids[b] == int(np.argmax(lg[b]))
        top2 = np.sort(want_lg[b])[-2:]
        if top2[1] - top2[0] > 1e-3 * np.abs(want_lg[b]).max():
            assert ids[b] == int(want_arg[b]), b
    # argmax only (no logits written)
    _, ids2, best2 = ops.gemm_tc(code, P, V, D, _t(x), argmax=True, store=False, split=split)
    assert np.array_equal(_np(ids2).astype(np.int64), ids) and np.array_equal(_np(best2), best)
