"""Conv modules chained in a stack (``gsn_conv_module_lnfold_chain_bf16``, ``ConvModuleStack`` with LayerNorm-folded
weights): each layer's down_conv + residual writes its output rows' statistics as per-256-column (mean, M2) blocks
and the next layer's folded LayerNorm merges them, instead of a statistics launch.  The row blocks are checked
against float64 statistics of the bf16 output, the chained stack against the same layers run one module call at
a time and against the oracle applied layer by layer."""
import numpy as np
import pytest
import torch

from granite_conv_b200 import ConvModuleStack, _lib, dispatch, ops, synth
from granite_conv_b200.weights import prepare_from_params
from oracle import conv_module as O
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _x(seed, shape, scale=1.0, shift=0.0):
    return O.bf16_round(synth.make_activations(seed, shape) * scale + shift)


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).to(DEV)


@pytest.mark.parametrize("M,K,N,shift", [(256, 2048, 1024, 0.0), (384, 1024, 512, 5.0), (128, 512, 256, 0.0)])
def test_residual_gemm_row_blocks(M, K, N, shift):
    """The down_conv + residual output is the plain entry point's bit for bit, and each (mean, M2) block matches
    float64 statistics of that bf16 output (the residual shifted by `shift` gives rows with a mean far from 0)."""
    rng = np.random.default_rng(M + K + N)
    d = _t(rng.standard_normal((M, K)).astype(np.float32))
    w = _t((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    b = torch.from_numpy((rng.standard_normal(N) * 0.1).astype(np.float32)).to(DEV)
    res = _t((rng.standard_normal((M, N)) + shift).astype(np.float32))
    out_ref = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    out = torch.empty_like(out_ref)
    parts = torch.full((M, N // 256, 2), float("nan"), dtype=torch.float32, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("gsn_gemm2_residual_bf16", d.data_ptr(), w.data_ptr(), b.data_ptr(), res.data_ptr(), N,
              out_ref.data_ptr(), N, M, K, N, None, 0, st)
    _lib.call("gsn_gemm2_residual_stats_bf16", d.data_ptr(), w.data_ptr(), b.data_ptr(), res.data_ptr(), N,
              out.data_ptr(), N, M, K, N, None, 0, parts.data_ptr(), st)
    torch.cuda.synchronize()
    assert torch.equal(out, out_ref)
    y = out.float().cpu().numpy().astype(np.float64).reshape(M, N // 256, 256)
    mean = y.mean(axis=2)
    m2 = ((y - mean[..., None]) ** 2).sum(axis=2)
    p = parts.cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(p[..., 0], mean, rtol=1e-6, atol=1e-6 * (1 + abs(shift)))
    np.testing.assert_allclose(p[..., 1], m2, rtol=2e-5, atol=1e-3)


@pytest.mark.parametrize("d_model,d_inner", [(1024, 2048), (512, 1024)])
def test_chained_stack_vs_module_calls(d_model, d_inner):
    """Four layers over a chunk plan with ragged lengths: the chained stack against the same layers run one
    LayerNorm-folded module call at a time (their statistics from the statistics kernel); its first two layers
    against the oracle applied layer by layer (deeper, single bf16 ulps of the two rounding chains compound)."""
    lens = synth.sample_lengths(6006, 20) // 4 + 1
    chunks = dispatch.plan_chunks(lens, exec_batch=8, logical_batch=16)
    params = [synth.make_params(7300 + i, w_std=0.04, d_model=d_model, d_inner=d_inner) for i in range(4)]
    layers = [prepare_from_params(q, device=DEV, ln_fold=True) for q in params]
    stack = ConvModuleStack(layers)
    stack2 = ConvModuleStack(layers[:2])
    preps = [O.prepare_bf16(q) for q in params[:2]]
    for c in chunks:
        x = _x(int(c.index[0]) + 60, (c.B, c.T, d_model))
        xt = _t(x)
        lt = torch.from_numpy(c.lengths).to(DEV)
        assert stack.chained(xt)
        y = stack(xt, lt)
        ref = xt
        for p in layers:
            ref = ops.run_conv_module(ref, p, lengths=lt, ln_fold=True)
        torch.cuda.synchronize()
        for b in range(c.B):
            L = int(c.lengths[b])
            assert_bf16_close(y[b, :L], ref[b, :L], f"chain vs module calls D={d_model} B={c.B} T={c.T} utt {b}")
        y2 = stack2(xt, lt)
        oref = x
        for pr in preps:
            oref = O.conv_module(oref, pr, lengths=c.lengths, mode="fused")
        torch.cuda.synchronize()
        for b in range(c.B):
            L = int(c.lengths[b])
            assert_bf16_close(y2[b, :L], oref[b, :L], f"2-layer chain vs oracle D={d_model} B={c.B} T={c.T} utt {b}")
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0


def test_chained_first_layer_is_the_module_call():
    """A one-layer chain computes its statistics with the statistics kernel: the same bits as the module op."""
    p = prepare_from_params(synth.make_params(7400, w_std=0.05), device=DEV, ln_fold=True)
    x = _t(_x(7401, (3, 256, synth.D_MODEL), scale=3.0, shift=2.0))
    lt = torch.tensor([256, 130, 7], dtype=torch.int32, device=DEV)
    y = ConvModuleStack([p])(x, lt)
    ref = ops.run_conv_module(x, p, lengths=lt, ln_fold=True)
    torch.cuda.synchronize()
    for b, L in enumerate([256, 130, 7]):
        assert torch.equal(y[b, :L], ref[b, :L])


def test_chain_entry_point_rejects_misaligned_statistics():
    p = prepare_from_params(synth.make_params(7500), device=DEV, ln_fold=True)
    B, T, D, inner = 1, 128, synth.D_MODEL, p.d_inner
    x = torch.zeros((B, T, D), dtype=torch.bfloat16, device=DEV)
    out = torch.empty_like(x)
    L = _lib.lib()
    nbytes = int(L.gsn_conv_module_workspace_bytes(B, T, D, inner))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    stats = torch.empty(B * T * (D // 256) * 2 + 1, dtype=torch.float32, device=DEV)
    rc = L.gsn_conv_module_lnfold_chain_bf16(x.data_ptr(), p.w1g_glu.data_ptr(), p.b1g_glu.data_ptr(),
                                             p.c1_glu.data_ptr(), p.dw_w.data_ptr(), p.dw_b.data_ptr(),
                                             p.w2.data_ptr(), p.b2.data_ptr(), None, 1, out.data_ptr(), B, T, D,
                                             inner, p.ln_eps, stats.data_ptr() + 4, None, ws.data_ptr(), nbytes,
                                             torch.cuda.current_stream().cuda_stream)
    assert rc != 0 and "8-byte" in _lib.last_error()
