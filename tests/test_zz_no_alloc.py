"""The allocation-free attention entry point (rta_attention_decode_f16_noalloc).

Callers that may not allocate device memory while decoding (a serving loop
living inside another framework's allocator, a latency-critical path that must
not hit cudaMalloc's implicit synchronisation) use this variant: its split
records live in a fixed array inside the library's device image instead of a
caller workspace.  This test calls it through the C-ABI and checks it against
the workspace variant, rta_attention_decode_f16, on two calls in a row (the
second call reuses the array the first one left behind): both run the same
kernels with the same splits, so the outputs must agree bit for bit.  It also
checks the outputs against the attention oracle (1e-3 relative L2), the
optional outputs left out (no error word, no physical pair), and the argument
checks (the scratch limit, misaligned K/V).  It is collected last so that a run
stopping at the first failure has already run every other test; it also passes
alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3  # relative L2 against the oracle, the tolerance of the other attention tests


def _call_noalloc(lib, q, k, v, time, capacity, splits, gate=None, err=None, with_phys=True):
    import torch
    out = torch.empty(16, 256, dtype=torch.float32, device="cuda")
    phys = torch.empty(16, 2, dtype=torch.float32, device="cuda") if with_phys else None
    ptr = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
    status = lib.rta_attention_decode_f16_noalloc(
        ptr(q), ptr(k), ptr(v), time, capacity, 16, 4, 256, 4, 1, ptr(gate), ptr(out), ptr(phys), splits,
        ptr(err), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return status, out, phys


def test_noalloc_matches_workspace_variant_on_consecutive_calls():
    import torch
    from oracle import oracle
    from rta_b200 import _lib, ops
    lib = _lib.load()
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(1234)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    cases = [(700, 1024, 11, True), (4096, 4096, 37, False)]  # (history, capacity, splits, gated)
    for L, cap, splits, gated in cases:
        q = torch.randn(16, 256, device="cuda", generator=g)
        k = torch.randn(L, 4, 256, device="cuda", generator=g).half()
        v = torch.randn(L, 4, 256, device="cuda", generator=g).half()
        gate = torch.randn(16, 256, device="cuda", generator=g) if gated else None
        status, out, phys = _call_noalloc(lib, q, k, v, L - 1, cap, splits, gate, err)
        assert status == _lib.RTA_OK, lib.rta_last_error()
        want, want_phys, ws = ops.attention_decode_f16(q, k, v, L - 1, cap, 4, 1, gate=gate, splits=splits)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert ops.workspace_error(ws) == 0
        assert torch.equal(out, want), f"rel-L2 {rel_l2(out.cpu().numpy(), want.cpu().numpy())}"
        assert torch.equal(phys, want_phys)
        qn = q.cpu().numpy()
        ref, _ = oracle.attention(qn[None], k.float().cpu().numpy(), v.float().cpu().numpy(),
                                  None if gate is None else gate.cpu().numpy()[None], L - 1, 0, cap, gated)
        assert rel_l2(out.cpu().numpy(), ref[0]) < TOL


def test_noalloc_without_optional_outputs():
    """No device error word and no physical pair: the documented optional path."""
    import torch
    from rta_b200 import _lib, ops
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(99)
    L = 1500
    q = torch.randn(16, 256, device="cuda", generator=g)
    k = torch.randn(L, 4, 256, device="cuda", generator=g).half()
    v = torch.randn(L, 4, 256, device="cuda", generator=g).half()
    status, out, _ = _call_noalloc(lib, q, k, v, L - 1, 2048, 20, err=None, with_phys=False)
    assert status == _lib.RTA_OK, lib.rta_last_error()
    want, _, ws = ops.attention_decode_f16(q, k, v, L - 1, 2048, 4, 1, splits=20)
    torch.cuda.synchronize()
    assert ops.workspace_error(ws) == 0
    assert torch.equal(out, want)


def test_noalloc_rejects_bad_arguments_before_launching():
    import torch
    from rta_b200 import _lib
    lib = _lib.load()
    q = torch.zeros(16, 256, device="cuda")
    kv = torch.zeros(65, 4, 256, device="cuda").half()
    status, _, _ = _call_noalloc(lib, q, kv, kv, 63, 64, 65)   # 16 heads x 65 splits > 1024 records
    assert status == _lib.RTA_E_ARG
    assert b"static scratch limit" in lib.rta_last_error()
    # K starting 8 bytes into the buffer is rejected before any launch; 16 bytes in is fine
    # (positions 0..60 stay inside the 65-position buffer either way)
    status, _, _ = _call_noalloc(lib, q, kv.view(-1)[4:], kv, 60, 64, 4)
    assert status == _lib.RTA_E_ARG
    assert b"16-byte aligned" in lib.rta_last_error()
    shifted = kv.view(-1)[8:]
    status, _, _ = _call_noalloc(lib, q, shifted, shifted, 60, 64, 4)
    assert status == _lib.RTA_OK, lib.rta_last_error()
    torch.cuda.synchronize()
