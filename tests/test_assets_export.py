"""Our payload writer against the reference's exporter (CPU).

tests/golden/make_export_golden.py ran the reference's unmodified export()
(ray_tracing/compiler/export.py:51-150) on the tensors of a tiny seeded hybrid
model and stored the SHA-256 of the three payloads it wrote.  Here our writer
(rta_b200.assets) re-derives the same model and must produce the same bytes:
header words, descriptors, row modes, small-tensor order and placement,
matrix and vocabulary payloads.
"""
import hashlib
import json
from pathlib import Path

from golden.make_export_golden import PAYLOADS, our_payloads

HERE = Path(__file__).resolve().parent


def test_writer_matches_reference_exporter_bytes(tmp_path):
    want = json.loads((HERE / "golden" / "export_tiny.json").read_text())["reference_export_sha256"]
    got, _, _, _, _ = our_payloads(tmp_path)
    assert got == want
    for name in PAYLOADS:
        assert hashlib.sha256((tmp_path / name).read_bytes()).hexdigest() == want[name]
