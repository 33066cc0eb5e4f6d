"""The LayerNorm folded into the up_conv GEMM (``granite::conv_module_lnfold``): the weight fold and the row
statistics against numpy, and the folded module against the reference goldens and the oracle, including inputs
whose rows have a large mean relative to their spread (the folded form subtracts mean * colsum after the GEMM)."""
import os

import numpy as np
import pytest
import torch

from granite_conv_b200 import ConvModuleStack, ops, synth
from granite_conv_b200.weights import fold_layernorm_, glu_interleave, prepare_from_params
from oracle import conv_module as O
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).to(DEV)


def test_fold_weights_match_numpy():
    p = prepare_from_params(synth.make_params(301), device=DEV, ln_fold=True)
    w = p.w1_glu.float().cpu().numpy()
    g = p.ln_w.float().cpu().numpy()
    bt = p.ln_b.float().cpu().numpy()
    b1 = p.b1_glu.cpu().numpy().astype(np.float64)
    wg = O.bf16_round((w * g[None, :]).astype(np.float32))
    np.testing.assert_array_equal(p.w1g_glu.float().cpu().numpy(), wg)
    np.testing.assert_allclose(p.b1g_glu.cpu().numpy(), b1 + w.astype(np.float64) @ bt.astype(np.float64),
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(p.c1_glu.cpu().numpy(), wg.astype(np.float64).sum(axis=1), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("M,D,masked", [(300, 1024, False), (512, 1024, True), (256, 2048, False), (128, 512, True)])
def test_layernorm_stats(M, D, masked):
    rng = np.random.default_rng(M + D)
    x = O.bf16_round((rng.normal(0.3, 2.0, (M, D))).astype(np.float32))
    T = 128
    lens = None
    if masked:
        lens = np.array([(97 * b) % T + 1 for b in range(M // T)], dtype=np.int32)
    st = ops.layernorm_stats(_t(x), 1e-5, None if lens is None else torch.from_numpy(lens).to(DEV), T)
    st = st.cpu().numpy()
    xd = x.astype(np.float64)
    mean = xd.mean(axis=1)
    rstd = 1.0 / np.sqrt(xd.var(axis=1) + 1e-5)
    valid = np.ones(M, bool) if lens is None else (np.arange(M) % T < np.repeat(lens, T))
    np.testing.assert_allclose(st[valid, 0], rstd[valid], rtol=2e-6)
    np.testing.assert_allclose(st[valid, 1], (rstd * mean)[valid], rtol=2e-5, atol=1e-6)


@pytest.mark.parametrize("tag,seed,w_std", [("w002", 1003, 0.02), ("w006", 2003, 0.06)])
def test_lnfold_vs_reference_golden(tag, seed, w_std):
    """The test-fire goldens (B=2, T=37) placed in a 128-frame grid with lengths: valid frames against the
    reference module run on the trimmed utterances."""
    g = np.load(os.path.join(GOLDEN, f"module_bf16_b2t37_{tag}.npz"))
    p = prepare_from_params(synth.make_params(seed, w_std=w_std), device=DEV, ln_fold=True)
    x = O.bf16_round(synth.make_activations(seed + 500, (2, 37, synth.D_MODEL)))
    xp = np.zeros((2, 128, synth.D_MODEL), np.float32)
    xp[:, :37] = x
    lens = g["lengths"]
    y = ops.run_conv_module(_t(xp), p, lengths=torch.from_numpy(lens).to(DEV)).float().cpu().numpy()
    valid = np.concatenate([y[b, :L] for b, L in enumerate(lens)])
    assert_bf16_close(valid, O.from_bf16_bits(g["trimmed"]), f"lnfold module {tag} vs trimmed reference")


@pytest.mark.parametrize("B,T,masked,loc,scale", [(2, 128, False, 0.0, 1.0), (3, 256, True, 0.0, 1.0),
                                                  (4, 384, True, 0.5, 3.0), (2, 256, False, 5.0, 1.0),
                                                  (2, 128, True, -3.0, 0.5), (3, 512, False, 0.0, 30.0)])
def test_lnfold_vs_oracle(B, T, masked, loc, scale):
    params = synth.make_params(400 + T, w_std=0.05)
    p = prepare_from_params(params, device=DEV, ln_fold=True)
    rng = np.random.default_rng(B * T)
    x = O.bf16_round(rng.normal(loc, scale, (B, T, synth.D_MODEL)).astype(np.float32))
    lens = None
    if masked:
        lens = np.maximum(1, (np.arange(B) * 113 + T // 3) % (T + 1)).astype(np.int32)
        lens[0] = T
    lt = None if lens is None else torch.from_numpy(lens).to(DEV)
    y = ops.run_conv_module(_t(x), p, lengths=lt)
    ref = O.conv_module(x, O.prepare_bf16(params), lengths=lens, mode="fused")
    assert_bf16_close(y, ref, f"lnfold B={B} T={T} loc={loc} scale={scale}")
    # the module output alone (no residual), where the folded LayerNorm's rounding is not hidden by x
    y0 = ops.run_conv_module(_t(x), p, lengths=lt, add_residual=False)
    ref0 = O.conv_module(x, O.prepare_bf16(params), lengths=lens, mode="fused", residual=False)
    assert_bf16_close(y0, ref0, f"lnfold no residual B={B} T={T} loc={loc} scale={scale}")
    if lens is not None:        # padded frames are x + b2 up to one bf16 rounding, as in the unfolded module
        yn = y.float().cpu().numpy()
        b2 = O.bf16_round(params.down_bias)
        for b, L in enumerate(lens):
            np.testing.assert_allclose(yn[b, L:], O.bf16_round(x[b, L:] + b2), atol=0, rtol=0)


def test_lnfold_close_to_unfolded_module():
    """Folded and unfolded modules on the same weights differ only by where bf16 rounding happens."""
    params = synth.make_params(77, w_std=0.05)
    p = prepare_from_params(params, device=DEV, ln_fold=True)
    x = _t(O.bf16_round(synth.make_activations(78, (4, 640, synth.D_MODEL))))
    lt = torch.tensor([640, 600, 300, 129], dtype=torch.int32, device=DEV)
    y_fold = ops.run_conv_module(x, p, lengths=lt, ln_fold=True)
    y_ref = ops.run_conv_module(x, p, lengths=lt, ln_fold=False)
    assert_bf16_close(y_fold, y_ref.float().cpu().numpy(), "folded vs unfolded")


def test_lnfold_stack_and_fold_in_place():
    layers = [prepare_from_params(synth.make_params(900 + i), device=DEV) for i in range(2)]
    for q in layers:
        fold_layernorm_(q)
    stack = ConvModuleStack(layers)
    x = _t(O.bf16_round(synth.make_activations(901, (3, 256, synth.D_MODEL))))
    lt = torch.tensor([256, 200, 17], dtype=torch.int32, device=DEV)
    y = stack(x, lt)
    y0 = x
    for q in layers:
        y0 = ops.run_conv_module(y0, q, lengths=lt, ln_fold=False)
    assert_bf16_close(y, y0.float().cpu().numpy(), "folded stack vs unfolded stack")


def test_glu_interleave_roundtrip_on_folded():
    """The folded weights keep the GLU-interleaved row order of W1."""
    p = prepare_from_params(synth.make_params(55), device=DEV, ln_fold=True)
    g = p.ln_w.float()
    w_plain = synth.make_params(55).up_weight
    wb = torch.from_numpy(w_plain).to(torch.bfloat16).to(DEV).float()
    expect = glu_interleave((wb * g[None, :]).to(torch.bfloat16))
    assert torch.equal(p.w1g_glu, expect)
