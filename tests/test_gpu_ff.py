"""The feed-forward halves of the Conformer block (``granite::feed_forward_half``) and its post LayerNorm
(``granite::layer_norm``) against the reference goldens and the oracle; the SiLU-epilogue GEMM and the scaled
residual GEMM against torch fp32."""
import os

import numpy as np
import pytest
import torch

from granite_conv_b200 import _lib, ops, synth
from granite_conv_b200.weights import prepare_ff_from_params
from oracle import conv_module as O
from oracle import feed_forward as FF
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).to(DEV)


@pytest.mark.parametrize("tag,seed,w_std", [("w002", 1101, 0.02), ("w006", 1102, 0.06)])
def test_ff_half_vs_reference_golden(tag, seed, w_std):
    g = np.load(os.path.join(GOLDEN, f"ff_half_b2t37_{tag}.npz"))
    p = prepare_ff_from_params(synth.make_ff_params(seed, w_std=w_std), device=DEV)
    x = O.bf16_round(synth.make_activations(seed + 500, (2, 37, synth.D_MODEL)))
    y = ops.run_feed_forward_half(_t(x), p)
    assert_bf16_close(y, O.from_bf16_bits(g["bf16"]), f"ff half {tag} vs reference")


@pytest.mark.parametrize("B,T,masked", [(1, 1, False), (2, 300, False), (3, 256, True), (4, 640, True)])
def test_ff_half_vs_oracle(B, T, masked):
    params = synth.make_ff_params(500 + T, w_std=0.05)
    p = prepare_ff_from_params(params, device=DEV)
    x = O.bf16_round(synth.make_activations(501 + T, (B, T, synth.D_MODEL)))
    lens = None
    if masked:
        lens = np.maximum(1, (np.arange(B) * 97 + T // 2) % (T + 1)).astype(np.int32)
        lens[0] = T
    y = ops.run_feed_forward_half(_t(x), p, None if lens is None else torch.from_numpy(lens).to(DEV))
    ref = FF.feed_forward_half(x, FF.prepare_ff_bf16(params), lengths=lens, mode="reference")
    assert_bf16_close(y, ref, f"ff half B={B} T={T} masked={masked}")
    if lens is not None:       # padded frames: x + 0.5 * b_down, one bf16 rounding
        yn = y.float().cpu().numpy()
        hb = 0.5 * O.bf16_round(params.down_bias)
        for b, L in enumerate(lens):
            np.testing.assert_allclose(yn[b, L:], O.bf16_round(x[b, L:] + hb), atol=0, rtol=0)


def test_gemm_silu_vs_torch():
    M, K, N = 300, 1024, 4096
    g = torch.Generator(device=DEV).manual_seed(7)
    a = torch.randn((M, K), generator=g, device=DEV).bfloat16()
    w = (torch.randn((N, K), generator=g, device=DEV) * 0.03).bfloat16()
    b = torch.randn((N,), generator=g, device=DEV) * 0.1
    h = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    _lib.call("gsn_gemm_silu_bf16", a.data_ptr(), w.data_ptr(), b.data_ptr(), h.data_ptr(), M, K, N, None, 0,
              torch.cuda.current_stream().cuda_stream)
    ref = torch.nn.functional.silu(a.float() @ w.float().t() + b)
    assert_bf16_close(h, ref.cpu().numpy(), "gemm silu")


@pytest.mark.parametrize("scale", [0.5, 1.0, -2.0])
def test_gemm_residual_scaled_vs_torch(scale):
    M, K, N = 257, 4096, 1024
    g = torch.Generator(device=DEV).manual_seed(8)
    d = torch.randn((M, K), generator=g, device=DEV).bfloat16()
    w = (torch.randn((N, K), generator=g, device=DEV) * 0.02).bfloat16()
    b = torch.randn((N,), generator=g, device=DEV) * 0.1
    r = torch.randn((M, N), generator=g, device=DEV).bfloat16()
    out = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    _lib.call("gsn_gemm_residual_scaled_bf16", d.data_ptr(), w.data_ptr(), b.data_ptr(), r.data_ptr(), N,
              out.data_ptr(), N, M, K, N, float(scale), None, 0, torch.cuda.current_stream().cuda_stream)
    ref = scale * (d.float() @ w.float().t() + b) + r.float()
    assert_bf16_close(out, ref.cpu().numpy(), f"gemm residual scale {scale}")


def test_layer_norm_op_and_compile():
    D = 1024
    x = torch.randn((3, 77, D), device=DEV).bfloat16() * 2 + 0.3
    w = (1 + 0.05 * torch.randn(D, device=DEV)).bfloat16()
    b = (0.05 * torch.randn(D, device=DEV)).bfloat16()
    y = torch.ops.granite.layer_norm(x, w, b, 1e-5)
    ref = torch.nn.functional.layer_norm(x.float(), (D,), w.float(), b.float(), 1e-5)
    assert_bf16_close(y, ref.cpu().numpy(), "layer_norm op")
    p = prepare_ff_from_params(synth.make_ff_params(3), device=DEV)

    def f(x):
        return torch.ops.granite.layer_norm(ops.run_feed_forward_half(x, p), w, b, 1e-5)

    xx = torch.randn((2, 128, D), device=DEV).bfloat16()
    assert torch.equal(torch.compile(f, fullgraph=True)(xx), f(xx))
