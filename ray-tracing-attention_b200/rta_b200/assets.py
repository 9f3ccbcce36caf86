"""Model payloads in the reference compiler's layout.

The resident model consumes the three payloads the reference exporter writes
(ray_tracing/compiler/export.py:51-150):

  optical_model.bin    'RTRES004' + <9I d, depth, depth, middle, V, 4, n_params, matrix_words, 0>
                       + parameter words (32-word global header, 64 words per layer,
                       then small fp32 tensors appended in export order)
  geometry_weights.bin per-layer packed matrices, 4-byte padded, export order
  vocabulary.bin       'RTBASQ01' + <2I V, D> + token_embd rows (+ output rows when untied)

`Layout` restates the exporter's placement rules (which header word points
where, in which order tensors are appended) so that a synthetic model built
here is byte-compatible with what `rt-compile` produces; a CPU test compares
both writers.  Synthetic weights are generated on the GPU (counter-based
N(0, sigma) -> Q4_K/Q6_K) straight into the matrix payload.
"""
from __future__ import annotations

import json
import struct
from dataclasses import asdict, dataclass, field
from pathlib import Path

import numpy as np

Q4_K, Q6_K, F32, F16, BF16 = 12, 14, 0, 1, 30
FORMAT_BYTES = {F32: 4.0, F16: 2.0, BF16: 2.0, Q4_K: 144 / 256, Q6_K: 210 / 256}
STRIDE = 64


@dataclass(frozen=True)
class Spec:
    """The compiler's ModelSpec fields (ray_tracing/compiler/spec.py:9-26)."""
    architecture: str
    hidden_size: int
    middle_size: int
    vocabulary_size: int
    layer_types: tuple
    attention_heads: int
    kv_heads: int
    attention_head_dim: int
    rotary_dim: int
    rope_theta: float = 10000000.0
    norm_epsilon: float = 1e-6
    attention_gate: bool = True
    qk_norm: bool = True
    state_heads: int = 1
    state_key_heads: int = 1
    state_head_dim: int = 128
    version: int = 1

    @property
    def depth(self): return len(self.layer_types)
    @property
    def query_width(self): return self.attention_heads * self.attention_head_dim
    @property
    def kv_width(self): return self.kv_heads * self.attention_head_dim
    @property
    def state_width(self): return self.state_heads * self.state_head_dim
    @property
    def full_layers(self): return tuple(i for i, k in enumerate(self.layer_types) if k == "full")
    @property
    def recurrent_layers(self): return tuple(i for i, k in enumerate(self.layer_types) if k == "recurrent")

    def to_dict(self):
        d = asdict(self)
        d["layer_types"] = list(self.layer_types)
        return d

    @classmethod
    def from_dict(cls, d):
        d = dict(d)
        d["layer_types"] = tuple(d["layer_types"])
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})


def spec_2b() -> Spec:
    """benchmark config 4: 24 layers [rec, rec, rec, full] x 6, D 2048, F 6144, 16q/4kv x 256,
    16 recurrent heads (16 key heads) x 128, V 151936; rotary 64 of 256 (Qwen3.5 partial rotary)."""
    return Spec("qwen35", 2048, 6144, 151936, ("recurrent", "recurrent", "recurrent", "full") * 6, 16, 4, 256, 64,
                state_heads=16, state_key_heads=16)


def spec_9b() -> Spec:
    """benchmark config 5: 32 layers (3:1), D 4096, F 12288, 16q/4kv x 256, 32 recurrent heads
    over 16 key heads x 128, V 151936."""
    return Spec("qwen35", 4096, 12288, 151936, ("recurrent", "recurrent", "recurrent", "full") * 8, 16, 4, 256, 64,
                state_heads=32, state_key_heads=16)


@dataclass
class Tensor:
    name: str
    rows: int
    cols: int
    fmt: int
    offset: int = 0      # byte offset within its payload
    words: int = 0       # 4-byte words incl. padding

    @property
    def nbytes(self):
        return int(self.rows * self.cols * FORMAT_BYTES[self.fmt])


@dataclass
class Layout:
    """Placement of every tensor of a model in the three payloads (export.py order)."""
    spec: Spec
    header: np.ndarray
    small: list = field(default_factory=list)          # (name, float32 array) appended after the header
    matrices: list = field(default_factory=list)       # Tensor, byte offset in geometry_weights
    basis: list = field(default_factory=list)          # Tensor, byte offset in vocabulary payload
    matrix_words: int = 0
    basis_words: int = 0

    def params(self) -> np.ndarray:
        return np.concatenate([self.header] + [np.ascontiguousarray(v, "<f4").ravel().view("<u4")
                                               for _, v in self.small]).astype("<u4")


def _plan(spec: Spec, small_values, formats) -> Layout:
    """Restates export.py:160-230: header words, small-tensor order, matrix order."""
    d, depth, middle = spec.hidden_size, spec.depth, spec.middle_size
    header = np.zeros(32 + depth * STRIDE, np.uint32)
    header[:4] = [depth, depth, middle, 4]
    header[11:13] = [1, 1]
    lay = Layout(spec, header)
    count = [len(header)]

    def add(name, value):
        v = np.asarray(value, np.float32).ravel()
        lay.small.append((name, v))
        start = count[0]
        count[0] += v.size
        return start

    header[4] = add("output_norm.weight", small_values("output_norm.weight", (d,)))
    header[7] = add("lens", np.zeros(8))
    mw = 0
    for layer, kind in enumerate(spec.layer_types):
        base = 32 + layer * STRIDE
        prefix = f"blk.{layer}."
        start = mw
        written = {}

        def packed(name, rows, cols):
            nonlocal mw
            if name in written:
                return written[name]
            fmt = formats(prefix + name)
            t = Tensor(prefix + name, rows, cols, fmt, offset=mw * 4)
            t.words = (t.nbytes + 3) // 4
            lay.matrices.append(t)
            written[name] = (mw - start, fmt, t)
            mw += t.words
            return written[name]

        def descriptor(index, name, rows, cols, mode=0, offset_rows=0):
            at, fmt, _ = packed(name, rows, cols)
            row_bytes = int(d * FORMAT_BYTES[fmt])
            assert offset_rows * row_bytes % 4 == 0
            offset = base + 32 if index == 8 else base + 9 + index * 2
            header[offset] = at + offset_rows * row_bytes // 4
            header[offset + 1] = fmt | (mode << 8)

        header[base] = add(prefix + "attn_norm.weight", small_values(prefix + "attn_norm.weight", (d,)))
        header[base + 1] = add(prefix + "post_attention_norm.weight",
                               small_values(prefix + "post_attention_norm.weight", (d,)))
        header[base + 5] = add(prefix + "lens", np.zeros(8))
        Q, KV, hd = spec.query_width, spec.kv_width, spec.attention_head_dim
        if kind == "full":
            qrows = Q * (2 if spec.attention_gate else 1)
            descriptor(0, "attn_q.weight", qrows, d, 1 if spec.attention_gate else 3)
            descriptor(1, "attn_k.weight", KV, d, 3)
            descriptor(8, "attn_v.weight", KV, d, 3)
            descriptor(2, "attn_output.weight", d, Q, 4)
            if spec.attention_gate:
                descriptor(6, "attn_q.weight", qrows, d, 2)
            perm = np.arange(hd)
            r = spec.rotary_dim
            perm[:r] = np.stack((np.arange(r // 2), np.arange(r // 2) + r // 2), -1).ravel()
            header[base + 2] = add(prefix + "rope_phase", np.zeros(Q // 2))
            for name, fieldno in (("attn_q_norm.weight", 24), ("attn_k_norm.weight", 25)):
                norm = small_values(prefix + name, (hd,))[perm] if spec.qk_norm else np.ones(hd)
                header[base + fieldno] = add(prefix + name, np.tile(norm, spec.attention_heads))
            header[base + 23] = spec.attention_heads
            header[base + 29] = spec.rotary_dim
        else:
            key, s = spec.state_key_heads * 128, spec.state_width
            descriptor(0, "attn_qkv.weight", 2 * key + s, d, 5)
            descriptor(1, "attn_qkv.weight", 2 * key + s, d, 5, key)
            descriptor(8, "attn_qkv.weight", 2 * key + s, d, 0, 2 * key)
            descriptor(2, "ssm_out.weight", d, s)
            descriptor(6, "attn_gate.weight", s, d)
            conv = small_values(prefix + "ssm_conv1d.weight", (2 * key + s, 4))
            repeat = spec.state_heads // spec.state_key_heads
            header[base + 34] = add(prefix + "ssm_conv1d.weight",
                                    np.concatenate((np.tile(conv[:key], (repeat, 1)),
                                                    np.tile(conv[key:2 * key], (repeat, 1)), conv[2 * key:]), 0))
            header[base + 35], header[base + 39], _ = packed("ssm_beta.weight", spec.state_heads, d)
            header[base + 36], header[base + 40], _ = packed("ssm_alpha.weight", spec.state_heads, d)
            header[base + 37] = add(prefix + "ssm_dt.bias", small_values(prefix + "ssm_dt.bias", (spec.state_heads,)))
            header[base + 38] = add(prefix + "ssm_a", small_values(prefix + "ssm_a", (spec.state_heads,)))
            header[base + 24] = add(prefix + "q_ones", np.ones(s))
            header[base + 25] = add(prefix + "k_ones", np.ones(s))
            header[base + 31] = add(prefix + "ssm_norm.weight",
                                    np.tile(small_values(prefix + "ssm_norm.weight", (128,)), spec.state_heads))
            header[base + 23] = spec.state_heads
        descriptor(3, "ffn_gate.weight", middle, d)
        descriptor(4, "ffn_down.weight", d, middle)
        descriptor(5, "ffn_up.weight", middle, d)
        header[base + 26] = header[base + 30] = 1 if kind == "full" else 2
        header[base + 27] = start
        header[base + 28] = mw - start
    lay.matrix_words = mw
    # vocabulary payload: token_embd then output (untied)
    bw = 0
    for name, kind_field, off_field in (("token_embd.weight", 13, 14), ("output.weight", 15, 16)):
        fmt = formats(name)
        t = Tensor(name, spec.vocabulary_size, d, fmt, offset=bw * 4)
        t.words = (t.nbytes + 3) // 4
        header[kind_field] = fmt
        header[off_field] = bw
        lay.basis.append(t)
        bw += t.words
    lay.basis_words = bw
    return lay


def synthetic_small_values(seed: int):
    """Seeded values for the small fp32 tensors of a random-init model."""
    rng = np.random.default_rng(seed)

    def value(name, shape):
        if name.endswith("norm.weight"):
            return (1.0 + rng.normal(0, 0.05, shape)).astype(np.float32)
        if name.endswith("ssm_conv1d.weight"):
            return rng.normal(0, 0.3, shape).astype(np.float32)
        if name.endswith("ssm_dt.bias"):
            dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), shape))
            return (dt + np.log(-np.expm1(-dt))).astype(np.float32)     # softplus^-1(dt)
        if name.endswith("ssm_a"):
            return np.log(rng.uniform(1, 16, shape)).astype(np.float32)  # A_log (positive decay rate)
        return rng.normal(0, 0.02, shape).astype(np.float32)
    return value


def default_formats(name: str) -> int:
    if name.endswith(("ssm_alpha.weight", "ssm_beta.weight")):
        return F32
    if name in ("token_embd.weight", "output.weight"):
        return Q6_K
    return Q4_K


def plan(spec: Spec, seed: int = 0, formats=default_formats) -> Layout:
    return _plan(spec, synthetic_small_values(seed), formats)


def generate_device(layout: Layout, seed: int, sigma: float = 0.02, device="cuda"):
    """Synthetic matrix and vocabulary payloads generated on the GPU."""
    import torch
    from . import _lib
    from .ops import _ptr, _stream
    lib = _lib.load()
    mats = torch.zeros(layout.matrix_words * 4, dtype=torch.uint8, device=device)
    basis = torch.zeros(layout.basis_words * 4, dtype=torch.uint8, device=device)
    for i, t in enumerate(layout.matrices + layout.basis):
        buf = mats if i < len(layout.matrices) else basis
        view = buf[t.offset:t.offset + t.nbytes]
        tseed = seed * 1000003 + i
        if t.fmt == F32:
            out = view.view(torch.float32)
            _lib.check(lib.rta_synthetic_normal(tseed, sigma, 0.0, t.rows * t.cols, _ptr(out), _stream()))
        elif t.fmt in (F16, BF16):  # the same fp32 draws, rounded to nearest even
            tmp = torch.empty(t.rows * t.cols, dtype=torch.float32, device=device)
            _lib.check(lib.rta_synthetic_normal(tseed, sigma, 0.0, t.rows * t.cols, _ptr(tmp), _stream()))
            view.view(torch.float16 if t.fmt == F16 else torch.bfloat16).copy_(
                tmp.to(torch.float16 if t.fmt == F16 else torch.bfloat16))
            del tmp
        else:
            _lib.check(lib.rta_synthetic_blocks(t.fmt, tseed, sigma, 0, t.rows * t.cols // 256, _ptr(view),
                                                _stream()))
    torch.cuda.synchronize()
    return mats, basis


def generate_host(layout: Layout, seed: int):
    """Host-side payloads of a layout: random valid packed blocks (numpy, seeded) for
    every matrix, N(0, 0.02) for the F32 ones.  Returns (params, matrices, basis)."""
    rng = np.random.default_rng(seed)
    mats = np.zeros(layout.matrix_words * 4, np.uint8)
    basis = np.zeros(layout.basis_words * 4, np.uint8)
    for i, t in enumerate(layout.matrices + layout.basis):
        buf = mats if i < len(layout.matrices) else basis
        if t.fmt == F32:
            buf[t.offset:t.offset + t.nbytes] = rng.normal(0, 0.02, t.rows * t.cols).astype(np.float32).view(np.uint8)
            continue
        bs = 144 if t.fmt == Q4_K else 210
        nb = t.rows * t.cols // 256
        blk = rng.integers(0, 256, (nb, bs), dtype=np.uint8)
        d = rng.uniform(1e-4, 6e-4, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
        if t.fmt == Q4_K:
            blk[:, 0:2] = d
            blk[:, 2:4] = rng.uniform(1e-4, 6e-4, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
        else:
            blk[:, 208:210] = d
        buf[t.offset:t.offset + t.nbytes] = blk.reshape(-1)
    return layout.params(), mats, basis


def write_files(directory, layout: Layout, matrices: np.ndarray, basis: np.ndarray) -> Path:
    """Write optical_model.bin / geometry_weights.bin / vocabulary.bin / model.json."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    spec = layout.spec
    params = layout.params()
    (directory / "geometry_weights.bin").write_bytes(np.ascontiguousarray(matrices, np.uint8).tobytes())
    with (directory / "vocabulary.bin").open("wb") as f:
        f.write(b"RTBASQ01")
        f.write(struct.pack("<2I", spec.vocabulary_size, spec.hidden_size))
        f.write(np.ascontiguousarray(basis, np.uint8).tobytes())
    with (directory / "optical_model.bin").open("wb") as f:
        f.write(b"RTRES004")
        f.write(struct.pack("<9I", spec.hidden_size, spec.depth, spec.depth, spec.middle_size,
                            spec.vocabulary_size, 4, len(params), layout.matrix_words, 0))
        f.write(params.tobytes())
    meta = {"architecture": spec.architecture, "model_spec": spec.to_dict(), "depth": spec.depth,
            "hidden_size": spec.hidden_size, "middle": spec.middle_size, "vocabulary": spec.vocabulary_size,
            "precision": "original coefficient formats", "source_model": "synthetic (seeded random init)"}
    (directory / "model.json").write_text(json.dumps(meta, indent=1))
    return directory / "optical_model.bin"


def read_files(directory):
    """(spec, params u32, matrices u8, basis u8) from an exported model directory."""
    directory = Path(directory)
    meta = json.loads((directory / "model.json").read_text())
    spec = Spec.from_dict(meta["model_spec"])
    raw = (directory / "optical_model.bin").read_bytes()
    if raw[:8] != b"RTRES004":
        raise ValueError("optical_model.bin: bad magic")
    hdr = struct.unpack_from("<9I", raw, 8)
    params = np.frombuffer(raw, "<u4", count=hdr[6], offset=44)
    matrices = np.fromfile(directory / "geometry_weights.bin", np.uint8)
    voc = (directory / "vocabulary.bin").read_bytes()
    if voc[:8] != b"RTBASQ01":
        raise ValueError("vocabulary.bin: bad magic")
    basis = np.frombuffer(voc, np.uint8, offset=16)
    return spec, params, matrices, basis
