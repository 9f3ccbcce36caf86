"""Pin rta_b200.assets (our payload writer) to the reference's own exporter.

Run in the build container, where the reference checkout is importable:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_export_golden.py --reference <path-to-reference>

For a tiny hybrid model it builds our layout and seeded host payloads
(rta_b200.assets.plan / generate_host), hands the very same tensors to the
reference's unmodified exporter (ray_tracing/compiler/export.py:51-150) through
a source object with the interface export() reads (shape / packed / floating /
norm / actual; a non-GGUF source, so no value transforms apply), and records
the SHA-256 of the three payloads it writes (optical_model.bin,
geometry_weights.bin, vocabulary.bin).  It checks that our writer produces the
same bytes and stores the digests in export_tiny.json; tests/test_assets_export.py
then re-derives our payloads on any machine and compares with those digests.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "ray-tracing-attention_b200"))

from rta_b200 import assets  # noqa: E402

SEED = 20261203
TINY = dict(architecture="qwen35", hidden_size=256, middle_size=512, vocabulary_size=512,
            layer_types=("recurrent", "full"), attention_heads=16, kv_heads=4, attention_head_dim=256,
            rotary_dim=64, state_heads=16, state_key_heads=16)
PAYLOADS = ("optical_model.bin", "geometry_weights.bin", "vocabulary.bin")


def tiny_spec() -> assets.Spec:
    t = TINY
    return assets.Spec(t["architecture"], t["hidden_size"], t["middle_size"], t["vocabulary_size"], t["layer_types"],
                       t["attention_heads"], t["kv_heads"], t["attention_head_dim"], t["rotary_dim"],
                       state_heads=t["state_heads"], state_key_heads=t["state_key_heads"])


def our_payloads(directory):
    """(digests, layout, raw small values) of our writer for the tiny model."""
    spec = tiny_spec()
    raw = {}
    values = assets.synthetic_small_values(SEED)

    def recording(name, shape):
        v = values(name, shape)
        raw[name] = v
        return v
    layout = assets._plan(spec, recording, assets.default_formats)
    params, mats, basis = assets.generate_host(layout, SEED)
    assets.write_files(directory, layout, mats, basis)
    digests = {n: hashlib.sha256((Path(directory) / n).read_bytes()).hexdigest() for n in PAYLOADS}
    return digests, layout, raw, mats, basis


class LayoutSource:
    """The interface export() reads from a source, served from our layout's tensors."""

    def __init__(self, spec, layout, raw, mats, basis, path):
        self.spec, self.path = spec, path
        self._packed = {}
        for t in layout.matrices:
            self._packed[t.name] = (mats[t.offset:t.offset + t.nbytes], t.fmt, t.rows, t.cols)
        for t in layout.basis:
            self._packed[t.name] = (basis[t.offset:t.offset + t.nbytes], t.fmt, t.rows, t.cols)
        self._raw = raw

    def actual(self, name):
        return name

    def has(self, name):
        return name in self._packed or name in self._raw

    def shape(self, name):
        _, _, rows, cols = self._packed[name]
        return (rows, cols)

    def packed(self, name):
        data, fmt, _, _ = self._packed[name]
        return np.ascontiguousarray(data), fmt, {12: "Q4_K", 14: "Q6_K", 0: "F32"}[fmt]

    def floating(self, name):
        return np.asarray(self._raw[name], np.float32)

    def norm(self, name):
        return self.floating(name)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of a checkout of the reference project (holds the ray_tracing package)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    from ray_tracing.compiler import export as ref_export
    from ray_tracing.compiler.spec import ModelSpec

    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        ours, layout, raw, mats, basis = our_payloads(tmp / "ours")
        src_dir = tmp / "source"
        src_dir.mkdir()
        (src_dir / "tokenizer.json").write_text("{}")
        (src_dir / "chat_template.jinja").write_text("{{ messages }}")
        (src_dir / "generation_config.json").write_text("{}")
        spec = ModelSpec(**TINY).validate()
        ref_export.export(LayoutSource(spec, layout, raw, mats, basis, src_dir), tmp / "reference")
        ref = {n: hashlib.sha256((tmp / "reference" / n).read_bytes()).hexdigest() for n in PAYLOADS}
    if ours != ref:
        raise SystemExit(f"our writer differs from the reference exporter: ours={ours} reference={ref}")
    out = {"seed": SEED, "spec": {k: list(v) if isinstance(v, tuple) else v for k, v in TINY.items()},
           "reference_export_sha256": ref,
           "generator": "tests/golden/make_export_golden.py (reference ray_tracing/compiler/export.py:51-150)"}
    (HERE / "export_tiny.json").write_text(json.dumps(out, indent=1))
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
