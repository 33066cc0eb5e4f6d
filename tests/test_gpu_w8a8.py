"""The W8A8 conv module (``granite::conv_module_w8a8``, ``gsn_conv_module_w8a8``): int8 weights and per-row int8
activations on kind::i8 tensor-core MMAs, against the W8A8 oracle and the dequantised-weight bf16 oracle."""
import numpy as np
import pytest
import torch

from granite_conv_b200 import _lib, ops, synth
from granite_conv_b200.weights import prepare_from_params
from oracle import conv_module as O
from parity import assert_bf16_close, stats

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).to(DEV)


@pytest.mark.parametrize("M,K,masked", [(1, 8, False), (300, 1024, False), (256, 2048, True), (37, 264, False)])
def test_quant_rows_bit_exact(M, K, masked):
    g = np.random.default_rng(M + K)
    x = O.bf16_round(g.normal(0, 1.5, (M, K)).astype(np.float32))
    x[M // 2] = 0.0                                   # an all-zero row: q = 0, scale = 0
    if M > 3:
        x[1, 5] = 40.0                                # a row with one large value
    lens, T = None, 0
    ref_x = x
    if masked:
        T = 128
        lens = np.array([100, 1], dtype=np.int32)
        valid = (np.arange(M) % T) < np.repeat(lens, T)
        ref_x = x * valid[:, None]
    q, s = ops.quant_rows(_t(x), None if lens is None else torch.from_numpy(lens).to(DEV), T)
    rq, rs = O.quantize_rows(ref_x)
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)


def _refs(params, x, lens):
    prep = O.prepare_bf16(params)
    q1, s1 = O.quantize_per_channel(prep["w1"])
    q2, s2 = O.quantize_per_channel(prep["w2"])
    w8a8 = O.conv_module_w8a8(x, prep, q1, s1, q2, s2, lengths=lens)
    prep_q = dict(prep, w1=q1.astype(np.float32) * s1[:, None], w2=q2.astype(np.float32) * s2[:, None])
    deq = O.conv_module(x, prep_q, lengths=lens, mode="fused")
    return w8a8, deq


@pytest.mark.parametrize("B,T,lens", [(3, 256, [256, 150, 64]), (2, 200, None), (2, 384, [384, 1])])
def test_module_w8a8_vs_oracles(B, T, lens):
    """Against the W8A8 oracle (the same quantisation, exact integer sums) and against the bf16-activation module
    with the same int8 weights (the activation quantisation error only), both within 2e-2 / rel-L2 1e-2."""
    params = synth.make_params(1004 + T)
    p = prepare_from_params(params, device=DEV, int8=True)
    x = O.bf16_round(synth.make_activations(1504 + T, (B, T, synth.D_MODEL)))
    lens_np = None if lens is None else np.array(lens, dtype=np.int32)
    y = ops.run_conv_module(_t(x), p, lengths=None if lens is None else torch.from_numpy(lens_np).to(DEV),
                            w8a8=True)
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    w8a8, deq = _refs(params, x, lens_np)
    assert_bf16_close(y, w8a8, f"W8A8 module B={B} T={T} vs W8A8 oracle")
    assert_bf16_close(y, deq, f"W8A8 module B={B} T={T} vs dequantised-weight oracle")
    if lens_np is not None:
        yn = y.float().cpu().numpy()
        for b, L in enumerate(lens_np):     # padded frames: x + b2, as every module entry point writes them
            np.testing.assert_array_equal(yn[b, L:], O.bf16_round(x[b, L:] + O.bf16_round(params.down_bias)))


def test_module_w8a8_delta_tracks_bf16_weights():
    """The module's own contribution (output minus residual) stays within rel-L2 3e-2 of the int8-weight module with
    bf16 activations at w_std 0.06, where the contribution is not dwarfed by the residual."""
    params = synth.make_params(2006, w_std=0.06)
    p = prepare_from_params(params, device=DEV, int8=True)
    x = O.bf16_round(synth.make_activations(2506, (2, 256, synth.D_MODEL)))
    xt = _t(x)
    y8 = ops.run_conv_module(xt, p, w8a8=True).float()
    yw = ops.run_conv_module(xt, p, int8=True).float()
    s = stats(y8 - xt.float(), (yw - xt.float()).cpu().numpy())
    assert s["rel_l2"] <= 3e-2, s


def test_module_w8a8_compile_fullgraph():
    p = prepare_from_params(synth.make_params(7), device=DEV, int8=True)
    x = torch.randn((2, 128, synth.D_MODEL), device=DEV).bfloat16()
    f = lambda x: ops.run_conv_module(x, p, w8a8=True)  # noqa: E731
    assert torch.equal(torch.compile(f, fullgraph=True)(x), f(x))


def test_module_w8a8_fused_equals_unfused():
    """T on the 128 grid runs GLU, depthwise and SiLU inside the kind::i8 up_conv kernel; T off the grid runs the
    int8 GEMM, then the depthwise kernel.  The same utterances through both (T = 256 and the same frames padded to
    T = 257, equal lengths) give bit-identical valid frames."""
    params = synth.make_params(3001)
    p = prepare_from_params(params, device=DEV, int8=True)
    x = O.bf16_round(synth.make_activations(3501, (3, 257, synth.D_MODEL)))
    lens = torch.tensor([256, 201, 77], dtype=torch.int32, device=DEV)
    y_grid = ops.run_conv_module(_t(x[:, :256]), p, lengths=lens, w8a8=True).float().cpu().numpy()
    y_off = ops.run_conv_module(_t(x), p, lengths=lens, w8a8=True).float().cpu().numpy()
    for b, L in enumerate(lens.tolist()):
        np.testing.assert_array_equal(y_grid[b, :L], y_off[b, :L])
