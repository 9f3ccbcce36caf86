"""Kernel-level parity of the recurrent gated-delta layer (rta_gated_delta_step)
against the oracle's restatement of ops 18-21 (rta_oracle_gdn,
ray_tracing/native/shaders/resident_math.comp:131-148).

Both head layouts of the benchmark shapes are covered: 16 state heads over 16
key heads at hidden 2048 (2B) and 32 state heads over 16 key heads at hidden
4096 (9B), at batch 1 (16-row CTAs, eight per head) and at batches of 64
(head, sequence) units and more (one persistent CTA per SM walking a range of
units, whole states staged by bulk copies; fewer units than SMs leave CTAs
without work; at 40 sequences the ranges cross head boundaries).  Three
consecutive positions run, so both conv-history buffers are read and written.
Bars: detector output and recurrent state within 1e-3 relative L2 of the oracle
after every step; the rolled convolution taps are copies and must be exact.
"""
import numpy as np
import pytest

from conftest import rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _inputs(rng, B, D, H, KH):
    S, K = H * 128, KH * 128
    return dict(
        x=rng.normal(0, 1, (B, D)).astype(np.float32),
        attn_norm=(1 + rng.normal(0, 0.1, D)).astype(np.float32),
        wa=rng.normal(0, 0.02, (H, D)).astype(np.float32),
        wb=rng.normal(0, 0.02, (H, D)).astype(np.float32),
        a_log=rng.normal(0, 0.5, H).astype(np.float32),
        dt_bias=rng.normal(0, 0.5, H).astype(np.float32),
        proj=rng.normal(0, 1, (B, 2 * K + 2 * S)).astype(np.float32),
        conv_w=rng.normal(0, 0.5, (3 * S, 4)).astype(np.float32),
    )


@pytest.mark.parametrize("D,H,KH,B", [(2048, 16, 16, 1), (4096, 32, 16, 1), (4096, 32, 16, 16), (2048, 16, 16, 24),
                                     (4096, 32, 16, 40), (4096, 32, 16, 2), (4096, 32, 16, 8), (2048, 16, 16, 4)])
def test_gated_delta_matches_oracle(D, H, KH, B):
    import torch
    from rta_b200 import ops
    rng = np.random.default_rng(D + H + B)
    S, K = H * 128, KH * 128
    eps = 1e-6
    state = rng.normal(0, 0.02, (B, H, 128, 128)).astype(np.float32)
    conv = rng.normal(0, 1, (B, 2, 3 * S, 3)).astype(np.float32)
    ref_state = state.copy()
    start = np.array([7 + 3 * z for z in range(B)], np.uint32)  # mixed parities across the batch
    ref_conv = [conv[z, start[z] & 1].copy() for z in range(B)]
    d_state = torch.from_numpy(state).cuda()
    d_conv = torch.from_numpy(conv).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for step in range(3):
        inp = _inputs(rng, B, D, H, KH)
        pos = start + step
        dev = {k: torch.from_numpy(v).cuda() for k, v in inp.items()}
        out = ops.gated_delta_step(dev["x"], dev["attn_norm"], dev["wa"], dev["wb"], dev["a_log"], dev["dt_bias"],
                                   dev["proj"], dev["conv_w"], d_conv, d_state,
                                   torch.from_numpy(pos.astype(np.int32)).cuda(), H, KH, eps, error_word=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got_out, got_state, got_conv = out.cpu().numpy(), d_state.cpu().numpy(), d_conv.cpu().numpy()
        for z in range(B):
            xn = oracle.rmsnorm(inp["x"][z], inp["attn_norm"], eps)
            p = inp["proj"][z]
            want = oracle.gdn(xn[None], p[None, :2 * K], p[None, 2 * K:2 * K + S], None, inp["wa"], inp["wb"],
                              inp["a_log"], inp["dt_bias"], inp["conv_w"], None, H, KH, eps, ref_state[z],
                              ref_conv[z], True)[0]
            assert rel_l2(got_out[z], want) < TOL, (step, z, rel_l2(got_out[z], want))
            assert rel_l2(got_state[z], ref_state[z]) < TOL, (step, z, rel_l2(got_state[z], ref_state[z]))
            nxt = got_conv[z, (pos[z] & 1) ^ 1]
            assert np.array_equal(nxt, ref_conv[z]), (step, z)


def test_gated_delta_rejects_misaligned_inputs():
    import torch
    from rta_b200 import _lib, ops
    D, H, KH = 2048, 16, 16
    rng = np.random.default_rng(5)
    dev = {k: torch.from_numpy(v).cuda() for k, v in _inputs(rng, 1, D, H, KH).items()}
    state = torch.zeros(1, H, 128, 128, device="cuda")
    conv = torch.zeros(1, 2, 3 * H * 128, 3, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    xs = torch.zeros(D + 1, device="cuda")[1:].view(1, D)  # 4 bytes off a 16-byte boundary
    with pytest.raises(_lib.RtaError) as e:
        ops.gated_delta_step(xs, dev["attn_norm"], dev["wa"], dev["wb"], dev["a_log"], dev["dt_bias"], dev["proj"],
                             dev["conv_w"], conv, state, pos, H, KH)
    assert e.value.status == _lib.RTA_E_ARG
