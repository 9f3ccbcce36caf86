"""TEST INFRASTRUCTURE ONLY -- model-level oracle of the reference decode loop.

Composes the C restatement (rta_oracle.c) in the reference worker's per-token
schedule, reading the same payloads the product loads:

  word()    readout of the final-normed state + argmax   (optical_resident.cpp:528-530)
  forward() op 0 embedding, layer() x depth, op 1 index 2 (optical_resident.cpp:521)
  layer()   op 1, op 2 kind 5, [full: op 14, op 3, history, detector | recurrent:
            ops 18-21, 15], op 2 kind 2 (+residual), op 1, executeMLP (optical_resident.cpp:455-491)

Row modes of the packed projections follow quantizedWeight
(ray_tracing/native/shaders/resident_quant.glsl:21-27).  The history of a
full-attention layer is kept either in fp16 (kv="fp16", the format the CUDA
engine stores) or as the reference's Q4_K key / Q6_K value packets
(kv="packet", resident_history_quant.glsl:9-41).
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

BLOCK = {O.Q4_K: 144, O.Q6_K: 210}


class OracleModel:
    def __init__(self, spec, params, matrices, basis, capacity: int, kv: str = "fp16"):
        self.s = spec
        self.p = np.asarray(params, np.uint32)
        self.m = np.asarray(matrices, np.uint8)
        self.b = np.asarray(basis, np.uint8)
        self.capacity = capacity
        self.kv = kv
        s = spec
        self.D, self.F, self.V = s.hidden_size, s.middle_size, s.vocabulary_size
        self.hd, self.H, self.KVH = s.attention_head_dim, s.attention_heads, s.kv_heads
        self.R = s.rotary_dim
        self.eps = np.float32(s.norm_epsilon)
        self.inv_freq = O.inv_freq(s.rope_theta, self.R, self.hd)
        self.layers = [self._layer(l) for l in range(s.depth)]
        self.reset()

    # ------------------------------------------------------------ payload
    def f32(self, off, n):
        return self.p[off:off + n].view(np.float32)

    def _desc(self, l, i, rows, cols):
        base = 32 + l * 64
        field = base + 32 if i == 8 else base + 9 + 2 * i
        at = int(self.p[base + 27] + self.p[field]) * 4
        meta = int(self.p[field + 1])
        fmt, mode = meta & 255, meta >> 8
        nbytes = rows * O.row_bytes(fmt, cols)
        return self.m[at:at + nbytes], fmt, mode

    def _orig(self, a):
        return np.where(a < self.R, (a % 2) * (self.R // 2) + a // 2, a)

    def _rows(self, raw, fmt, cols, rows_src, idx):
        rb = O.row_bytes(fmt, cols)
        return raw.reshape(rows_src, rb)[idx].reshape(-1)

    def _mode_rows(self, mode, n):
        r = np.arange(n)
        hd = self.hd
        if mode == 1:
            return (r // hd) * 2 * hd + self._orig(r % hd)
        if mode == 2:
            return (r // hd) * 2 * hd + hd + self._orig(r % hd)
        if mode == 3:
            return (r // hd) * hd + self._orig(r % hd)
        if mode == 5:
            return r % (self.s.state_key_heads * 128)
        return r

    def _layer(self, l):
        s, D = self.s, self.D
        base = 32 + l * 64
        full = int(self.p[base + 26]) == 1
        L = {"full": full, "attn_norm": self.f32(self.p[base], D), "post_norm": self.f32(self.p[base + 1], D)}
        if full:
            Q, KV = s.query_width, s.kv_width
            gated = bool(s.attention_gate)
            rawq, fq, mq = self._desc(l, 0, Q * (2 if gated else 1), D)
            rawk, fk, mk = self._desc(l, 1, KV, D)
            rawv, fv, mv = self._desc(l, 8, KV, D)
            qrows = Q * (2 if gated else 1)
            L["fmt"] = fq
            L["q"] = self._rows(rawq, fq, D, qrows, self._mode_rows(mq, Q))
            L["k"] = self._rows(rawk, fk, D, KV, self._mode_rows(mk, KV))
            L["v"] = self._rows(rawv, fv, D, KV, self._mode_rows(mv, KV))
            if gated:
                rawg, fg, mg = self._desc(l, 6, qrows, D)
                L["gate"] = self._rows(rawg, fg, D, qrows, self._mode_rows(mg, Q))
            L["o"], L["o_fmt"], mo = self._desc(l, 2, D, Q)
            L["o_unpair"] = mo == 4
            L["qnorm"] = self.f32(self.p[base + 24], Q)
            L["knorm"] = self.f32(self.p[base + 25], Q)
        else:
            K, S = s.state_key_heads * 128, s.state_width
            raw, f, _ = self._desc(l, 0, 2 * K + S, D)
            L["fmt"] = f
            L["qkv"] = raw
            L["z"], L["z_fmt"], _ = self._desc(l, 6, S, D)
            L["out"], L["out_fmt"], _ = self._desc(l, 2, D, S)
            at_b = int(self.p[base + 27] + self.p[base + 35]) * 4
            at_a = int(self.p[base + 27] + self.p[base + 36]) * 4
            L["wb"] = self.m[at_b:at_b + s.state_heads * D * 4].view(np.float32).reshape(s.state_heads, D)
            L["wa"] = self.m[at_a:at_a + s.state_heads * D * 4].view(np.float32).reshape(s.state_heads, D)
            L["dt_bias"] = self.f32(self.p[base + 37], s.state_heads)
            L["a_log"] = self.f32(self.p[base + 38], s.state_heads)
            L["conv_w"] = self.f32(self.p[base + 34], 3 * S * 4).reshape(3 * S, 4)
            L["ssm_norm"] = self.f32(self.p[base + 31], S)
        L["g"], L["mlp_fmt"], _ = self._desc(l, 3, self.F, D)
        L["u"], _, _ = self._desc(l, 5, self.F, D)
        L["d"], L["down_fmt"], _ = self._desc(l, 4, D, self.F)
        return L

    # ------------------------------------------------------------- state
    def reset(self):
        s = self.s
        self.state = np.zeros(self.D, np.float32)
        self.pos = 0
        self.hist = {l: [] for l, L in enumerate(self.layers) if L["full"]}
        S = s.state_width
        self.rec = {l: np.zeros((s.state_heads, 128, 128), np.float32) for l, L in enumerate(self.layers)
                    if not L["full"]}
        self.conv = {l: np.zeros((3 * S, 3), np.float32) for l in self.rec}

    def _embed(self, token):
        fmt = int(self.p[13])
        rb = O.row_bytes(fmt, self.D)
        off = int(self.p[14]) * 4 + token * rb
        if fmt in O.DENSE_BYTES:
            return O.dense_values(fmt, self.b[off:off + rb])
        return O.dequantize(fmt, self.b[off:off + rb])

    def readout(self, logits=True):
        fmt = int(self.p[15])
        rb = O.row_bytes(fmt, self.D)
        off = int(self.p[16]) * 4
        W = self.b[off:off + rb * self.V]
        x = O.rmsnorm(self.state, self.f32(self.p[4], self.D), self.eps)
        lg, arg, best = O.lmhead(fmt, W, self.V, self.D, x, want_logits=True)
        return int(arg[0]), lg[0]

    def _history_kv(self, k, v):
        if self.kv == "fp16":
            return k.astype(np.float16).astype(np.float32), v.astype(np.float16).astype(np.float32)
        kq = O.dequantize(O.Q4_K, O.quantize(O.Q4_K, k)).reshape(k.shape)
        vq = O.dequantize(O.Q6_K, O.quantize(O.Q6_K, v)).reshape(v.shape)
        return kq, vq

    def _full(self, l, L):
        D, hd, H, KVH = self.D, self.hd, self.H, self.KVH
        xn = O.rmsnorm(self.state, L["attn_norm"], self.eps)
        f = L["fmt"]
        q = O.gemv(f, L["q"], H * hd, D, xn)[0]
        k = O.gemv(f, L["k"], KVH * hd, D, xn)[0]
        v = O.gemv(f, L["v"], KVH * hd, D, xn)[0]
        gate = O.gemv(f, L["gate"], H * hd, D, xn)[0] if "gate" in L else None
        if self.s.qk_norm:
            q = O.head_norm(q, L["qnorm"], H, hd, self.eps)
            kn = L["knorm"].reshape(H, hd)[::H // KVH].reshape(-1)
            k = O.head_norm(k, kn, KVH, hd, self.eps)
        q = O.rope(q, H, hd, self.R, self.inv_freq, self.pos)
        k = O.rope(k, KVH, hd, self.R, self.inv_freq, self.pos)
        kh, vh = self._history_kv(k.reshape(KVH, hd), v.reshape(KVH, hd))
        self.hist[l].append((kh, vh))
        keys = np.stack([e[0] for e in self.hist[l]])
        values = np.stack([e[1] for e in self.hist[l]])
        out, _ = O.attention(q.reshape(1, H, hd), keys, values, None if gate is None else gate.reshape(1, H, hd),
                             self.pos, 0, self.capacity, gate is not None)
        det = out.reshape(-1)
        if L["o_unpair"]:  # mode 4: column axis -> original axis (resident_quant.glsl:26)
            a = np.arange(H * hd)
            src = (a // hd) * hd + self._orig(a % hd)
            un = np.empty_like(det)
            un[src] = det
            det = un
        self.state = self.state + O.gemv(L["o_fmt"], L["o"], D, H * hd, det)[0]

    def _recurrent(self, l, L):
        s, D = self.s, self.D
        K, S = s.state_key_heads * 128, s.state_width
        xn = O.rmsnorm(self.state, L["attn_norm"], self.eps)
        qkv = O.gemv(L["fmt"], L["qkv"], 2 * K + S, D, xn)[0]
        z = O.gemv(L["z_fmt"], L["z"], S, D, xn)[0]
        out = O.gdn(xn[None], qkv[None, :2 * K], qkv[None, 2 * K:], z[None], L["wa"], L["wb"], L["a_log"],
                    L["dt_bias"], L["conv_w"], L["ssm_norm"], s.state_heads, s.state_key_heads, self.eps,
                    self.rec[l], self.conv[l], True)[0]
        self.state = self.state + O.gemv(L["out_fmt"], L["out"], D, S, out)[0]

    def _mlp(self, L):
        xn = O.rmsnorm(self.state, L["post_norm"], self.eps)
        act, y = O.mlp(L["mlp_fmt"], L["g"], L["u"], L["d"], self.D, self.F, xn, L["down_fmt"])
        self.state = self.state + y[0]

    def forward(self, token):
        self.state = self._embed(token)
        for l, L in enumerate(self.layers):
            if L["full"]:
                self._full(l, L)
            else:
                self._recurrent(l, L)
            self._mlp(L)
        self.pos += 1

    def prefill(self, ids):
        self.reset()
        for t in ids:
            self.forward(int(t))

    def generate(self, count, stops=()):
        ids, margins = [], []
        for _ in range(count):
            tok, lg = self.readout()
            top2 = np.sort(lg)[-2:]
            margins.append(float((top2[1] - top2[0]) / max(abs(top2[1]), 1e-30)))
            ids.append(tok)
            if tok in stops:
                break
            self.forward(tok)
        return np.array(ids, np.uint32), np.array(margins)


# ------------------------------------------------------------ synthetic models
def synthetic_payloads(layout, seed: int, sigma: float = 0.02):
    """Host restatement of the product's GPU model generator (assets.generate_device):
    tensor i of the layout (matrices, then vocabulary rows) is drawn with the seed
    seed * 1000003 + i -- packed blocks through the synthetic block generator, F32
    tensors as sigma * N -- so the returned (matrices, basis) bytes equal the GPU's
    bit for bit."""
    mats = np.zeros(layout.matrix_words * 4, np.uint8)
    basis = np.zeros(layout.basis_words * 4, np.uint8)
    for i, t in enumerate(layout.matrices + layout.basis):
        buf = mats if i < len(layout.matrices) else basis
        tseed = seed * 1000003 + i
        if t.fmt == O.F32:
            buf[t.offset:t.offset + t.nbytes] = O.synthetic_normal(tseed, sigma, t.rows * t.cols).view(np.uint8)
        elif t.fmt == O.F16:
            v = O.synthetic_normal(tseed, sigma, t.rows * t.cols)
            buf[t.offset:t.offset + t.nbytes] = v.astype(np.float16).view(np.uint8)
        elif t.fmt == O.BF16:
            v = O.synthetic_normal(tseed, sigma, t.rows * t.cols)
            buf[t.offset:t.offset + t.nbytes] = O.to_bf16_bits(v).view(np.uint8)
        else:
            buf[t.offset:t.offset + t.nbytes] = O.synthetic_blocks(t.fmt, tseed, sigma, t.rows * t.cols // 256)
    return mats, basis


def seed_sequence(ref: "OracleModel", nseq: int, z: int, length: int, seed: int):
    """Put `ref` in the state rta_model_seed_history gives sequence z of an nseq-sequence
    fp16-history handle: history positions 0..length-1 of every full layer from the
    seeded K (seed) and V (seed + 1) rings [full layer][sequence][kv head][capacity][hd],
    recurrent states sigma 0.02 (seed + 2) [layer][sequence][head][128][128], the conv
    taps (seed + 3) [layer][sequence][parity][3S][3] of the buffer the next position's
    parity reads, and the residual row (seed + 4) [sequence][D]; next position `length`."""
    s = ref.s
    cap, hd, kvh = ref.capacity, ref.hd, ref.KVH
    assert length <= cap, "seeded histories here never wrap the ring"
    ref.reset()
    full = [l for l, L in enumerate(ref.layers) if L["full"]]
    rec = [l for l, L in enumerate(ref.layers) if not L["full"]]
    for fi, l in enumerate(full):
        k = np.empty((length, kvh, hd), np.float32)
        v = np.empty((length, kvh, hd), np.float32)
        for h in range(kvh):
            first = (((fi * nseq + z) * kvh + h) * cap) * hd
            k[:, h, :] = O.synthetic_range(seed, 1.0, first, length * hd, half=True).reshape(length, hd)
            v[:, h, :] = O.synthetic_range(seed + 1, 1.0, first, length * hd, half=True).reshape(length, hd)
        ref.hist[l] = [(k[p], v[p]) for p in range(length)]
    H, S = s.state_heads, s.state_width
    for ri, l in enumerate(rec):
        n = H * 128 * 128
        ref.rec[l] = O.synthetic_range(seed + 2, 0.02, (ri * nseq + z) * n, n).reshape(H, 128, 128).copy()
        per = 2 * 3 * S * 3
        par = length & 1
        ref.conv[l] = O.synthetic_range(seed + 3, 1.0, (ri * nseq + z) * per + par * 3 * S * 3,
                                        3 * S * 3).reshape(3 * S, 3).copy()
    ref.state = O.synthetic_range(seed + 4, 1.0, z * ref.D, ref.D).copy()
    ref.pos = length
