"""Dense coefficient formats (F32 / F16 / BF16, the exporter's codes 0 / 1 / 30)
on the GPU: a real rt-compile of safetensors weights emits BF16 projections
(compiler/export.py:12), so every projection, the embedding and the output rows
may be dense.  Checked against the oracle's restatement of ggufValue's dense
branches and op 2's octet order: the GEMV operator and its SwiGLU / readout
forms within 1e-3 relative L2, and whole models whose matrices are dense (one
sequence on the CUDA-core GEMVs, and a batch whose packed matrices run on the
tensor cores) with greedy tokens equal to the oracle's wherever the top-2
margin exceeds 1e-3."""
import numpy as np
import pytest

from conftest import rel_l2
from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _raw(fmt, w):
    return {0: w.view(np.uint8), 1: w.astype(np.float16).view(np.uint8),
            30: oracle.to_bf16_bits(w).view(np.uint8)}[fmt]


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("fmt,rows,cols,batch", [(0, 48, 512, 1), (1, 160, 2048, 3), (30, 2048, 4096, 8),
                                                 (30, 512, 12288, 5), (1, 64, 256, 17)])
def test_dense_gemv_matches_the_oracle(fmt, rows, cols, batch):
    from rta_b200 import ops
    rng = np.random.default_rng(rows + cols + fmt)
    raw = _raw(fmt, rng.normal(0, 0.02, rows * cols).astype(np.float32))
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    y = ops.gemv(fmt, _t(raw), rows, cols, _t(x)).cpu().numpy()
    assert rel_l2(y, oracle.gemv(fmt, raw, rows, cols, x)) < TOL
    y0 = rng.normal(0, 1, (batch, rows)).astype(np.float32)
    yd = _t(y0)
    ops.gemv(fmt, _t(raw), rows, cols, _t(x), y=yd, accumulate=True)
    assert rel_l2(yd.cpu().numpy() - y0, oracle.gemv(fmt, raw, rows, cols, x)) < TOL


@pytest.mark.parametrize("fmt", [1, 30])
def test_dense_mlp_and_readout(fmt):
    from rta_b200 import ops
    rng = np.random.default_rng(fmt)
    D, F = 1024, 2048
    wg, wu, wd = (_raw(fmt, rng.normal(0, 0.02, n).astype(np.float32)) for n in (F * D, F * D, D * F))
    x = rng.normal(0, 1, (2, D)).astype(np.float32)
    act, y = ops.mlp_swiglu(fmt, _t(wg), _t(wu), _t(wd), D, F, _t(x))
    want_act, want_y = oracle.mlp(fmt, wg, wu, wd, D, F, x)
    assert rel_l2(act.cpu().numpy(), want_act) < TOL and rel_l2(y.cpu().numpy(), want_y) < TOL
    V = 4096
    W = _raw(fmt, rng.normal(0, 0.02, V * D).astype(np.float32))
    logits, arg, _ = ops.readout(fmt, _t(W), V, D, _t(x))
    want_lg, want_arg, _ = oracle.lmhead(fmt, W, V, D, x)
    assert rel_l2(logits.cpu().numpy(), want_lg) < TOL
    for b in range(2):
        top2 = np.sort(want_lg[b])[-2:]
        if top2[1] - top2[0] > TOL * abs(top2[1]):
            assert int(arg.cpu()[b]) == int(want_arg[b])


def _dense_formats(name):
    from rta_b200 import assets
    if name.endswith(("ssm_alpha.weight", "ssm_beta.weight")):
        return assets.F32
    if name == "token_embd.weight":
        return assets.F16
    if name == "output.weight":
        return assets.BF16
    if ".ffn_down" in name:
        return assets.F32
    return assets.BF16


@pytest.mark.parametrize("sequences", [1, 18])
def test_dense_model_decodes_like_the_oracle(sequences):
    """BF16 attention / recurrent / gate / up projections, F32 down projections,
    an F16 embedding and a BF16 vocabulary."""
    import torch
    from oracle.model import OracleModel
    from rta_b200 import assets
    from rta_b200.model import ResidentModel
    from test_model_gpu import small_spec
    spec = small_spec(kinds=("recurrent", "full"))
    layout = assets.plan(spec, 61, formats=_dense_formats)
    mats, basis = assets.generate_device(layout, 61)
    params = layout.params()
    model = ResidentModel.from_payloads(spec, params, mats, basis, 32, sequences=sequences)
    m, b = mats.cpu().numpy(), basis.cpu().numpy()
    del mats, basis
    torch.cuda.empty_cache()
    rng = np.random.default_rng(61)
    prompts = [rng.integers(0, spec.vocabulary_size, int(n)) for n in rng.integers(2, 8, sequences)]
    ref = OracleModel(spec, params, m, b, 32)
    if sequences == 1:
        model.prefill(prompts[0])
        state, _ = model.state()  # after the prompt, before any generated token
        ref.prefill(prompts[0])
        assert rel_l2(state, ref.state) < TOL, rel_l2(state, ref.state)
        got = [model.generate(6)]
        ref.reset()
    else:
        model.prefill_batch(prompts)
        got = model.generate_batch(6)
    compared = 0
    for z in sorted({0, sequences - 1}):
        ref.prefill(prompts[z])
        want, margins = ref.generate(6)
        for i in range(min(len(got[z]), len(want))):
            if margins[i] > TOL:
                assert got[z][i] == want[i], (z, i, got[z], want, margins)
                compared += 1
            if got[z][i] != want[i]:
                break
    assert compared >= 3
    model.close()
