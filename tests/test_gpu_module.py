"""The whole conv module (``granite::conv_module``, ``granite::conv_module_i8w``) and the 16-layer stack against the
reference goldens, the oracle and size-independent properties at the benchmark sizes."""
import os

import numpy as np
import pytest
import torch

from granite_conv_b200 import ConvModuleStack, dispatch, ops, synth
from granite_conv_b200.weights import prepare_from_params
from oracle import conv_module as O
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def _x(seed, shape):
    return O.bf16_round(synth.make_activations(seed, shape))


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).to(DEV)


@pytest.mark.parametrize("tag,seed,w_std", [("w002", 1003, 0.02), ("w006", 2003, 0.06)])
def test_module_vs_reference_golden(tag, seed, w_std):
    """B=2, T=37 (the test-fire shape): against the reference module's own bf16 output, full and trimmed."""
    g = np.load(os.path.join(GOLDEN, f"module_bf16_b2t37_{tag}.npz"))
    params = synth.make_params(seed, w_std=w_std)
    p = prepare_from_params(params, device=DEV)
    assert np.array_equal(O.bf16_bits(p.dw_w.float().cpu().numpy()), g["dw_weight_folded"])
    x = _x(seed + 500, (2, 37, synth.D_MODEL))
    y = ops.run_conv_module(_t(x), p)
    ref_full = O.from_bf16_bits(g["full"])
    assert_bf16_close(y, ref_full, f"module {tag} vs reference")
    # the module part alone (residual removed) must agree in rel-L2 too when it is not dwarfed by the residual;
    # element-wise it carries the final bf16 rounding of x + delta, so only the L2 gate applies to it
    if w_std >= 0.06:
        dy, dr = y.float().cpu().numpy() - x, ref_full - x
        assert np.linalg.norm(dy - dr) / np.linalg.norm(dr) <= 2e-2
    lens = g["lengths"]
    ym = ops.run_conv_module(_t(x), p, lengths=torch.from_numpy(lens).to(DEV)).float().cpu().numpy()
    valid = np.concatenate([ym[b, :L] for b, L in enumerate(lens)])
    assert_bf16_close(valid, O.from_bf16_bits(g["trimmed"]), f"masked module {tag} vs trimmed reference")


@pytest.mark.parametrize("B,T,masked", [(1, 1, False), (2, 37, True), (3, 128, True), (2, 300, False),
                                        (4, 256, True)])
def test_module_vs_oracle(B, T, masked):
    params = synth.make_params(31 + T, w_std=0.05)
    p = prepare_from_params(params, device=DEV)
    x = _x(77 + T, (B, T, synth.D_MODEL))
    lens = None
    if masked:
        lens = np.maximum(1, (np.arange(B) * 97 + T // 2) % (T + 1)).astype(np.int32)
        lens[0] = T
    y = ops.run_conv_module(_t(x), p, lengths=None if lens is None else torch.from_numpy(lens).to(DEV))
    ref = O.conv_module(x, O.prepare_bf16(params), lengths=lens, mode="fused")
    assert_bf16_close(y, ref, f"module B={B} T={T} masked={masked}")
    if lens is not None:        # padded frames are x + b2 exactly up to one bf16 rounding
        yn = y.float().cpu().numpy()
        b2 = O.bf16_round(params.down_bias)
        for b, L in enumerate(lens):
            np.testing.assert_allclose(yn[b, L:], O.bf16_round(x[b, L:] + b2), atol=0, rtol=0)


def test_module_without_residual():
    params = synth.make_params(5, w_std=0.05)
    p = prepare_from_params(params, device=DEV)
    x = _x(6, (2, 64, synth.D_MODEL))
    y = ops.run_conv_module(_t(x), p, add_residual=False)
    ref = O.conv_module(x, O.prepare_bf16(params), mode="fused", residual=False)
    assert_bf16_close(y, ref, "module no residual")


def test_module_int8_weights():
    params = synth.make_params(1004)
    p = prepare_from_params(params, device=DEV, int8=True)
    x = _x(1504, (3, 200, synth.D_MODEL))
    lens = np.array([200, 150, 64], dtype=np.int32)
    y = ops.run_conv_module(_t(x), p, lengths=torch.from_numpy(lens).to(DEV), int8=True)
    prep = O.prepare_bf16(params)
    q1, s1 = O.quantize_per_channel(prep["w1"])
    q2, s2 = O.quantize_per_channel(prep["w2"])
    prep_q = dict(prep, w1=q1.astype(np.float32) * s1[:, None], w2=q2.astype(np.float32) * s2[:, None])
    ref = O.conv_module(x, prep_q, lengths=lens, mode="fused")
    assert_bf16_close(y, ref, "int8 module vs dequantised oracle")
    # and close to the bf16-weight module (quantisation error only)
    assert_bf16_close(y, O.conv_module(x, prep, lengths=lens, mode="fused"), "int8 vs bf16 weights")


@pytest.mark.parametrize("masked", [False, True])
def test_module_int8_widened_weights_equal_staged(masked):
    """The int8 module with room in the workspace (weights widened to bf16 once, GEMMs on bf16 tiles) and with the
    minimum workspace (int8 W tiles widened in shared memory) give bit-identical outputs."""
    from granite_conv_b200 import _lib
    params = synth.make_params(1010)
    p = prepare_from_params(params, device=DEV, int8=True)
    B, T = 3, 256
    x = _t(_x(1510, (B, T, synth.D_MODEL)))
    lens = torch.tensor([256, 130, 7], dtype=torch.int32, device=DEV) if masked else None
    L = _lib.lib()
    D, inner = synth.D_MODEL, p.d_inner
    small = int(L.gsn_conv_module_workspace_bytes(B, T, D, inner))
    big = int(L.gsn_conv_module_i8w_workspace_bytes(B, T, D, inner))
    assert big == small + 2 * inner * D * 2 + D * inner * 2
    outs = []
    for nbytes in (small, big):
        ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
        out = torch.empty_like(x)
        _lib.call("gsn_conv_module_i8w", x.data_ptr(), p.ln_w.data_ptr(), p.ln_b.data_ptr(), p.w1q_glu.data_ptr(),
                  p.s1_glu.data_ptr(), p.b1_glu.data_ptr(), p.dw_w.data_ptr(), p.dw_b.data_ptr(), p.w2q.data_ptr(),
                  p.s2.data_ptr(), p.b2.data_ptr(), None if lens is None else lens.data_ptr(), 1, out.data_ptr(),
                  B, T, D, inner, float(p.ln_eps), ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream)
        outs.append(out)
    # the weights widened once at prepare time (PreparedConvModule.w1w_glu / w2w): no widening per call, the same bits
    ws = torch.empty(small, dtype=torch.uint8, device=DEV)
    out = torch.empty_like(x)
    _lib.call("gsn_conv_module_i8w_widened", x.data_ptr(), p.ln_w.data_ptr(), p.ln_b.data_ptr(), p.w1w_glu.data_ptr(),
              p.s1_glu.data_ptr(), p.b1_glu.data_ptr(), p.dw_w.data_ptr(), p.dw_b.data_ptr(), p.w2w.data_ptr(),
              p.s2.data_ptr(), p.b2.data_ptr(), None if lens is None else lens.data_ptr(), 1, out.data_ptr(),
              B, T, D, inner, float(p.ln_eps), ws.data_ptr(), small, torch.cuda.current_stream().cuda_stream)
    outs.append(out)
    outs.append(ops.run_conv_module(x, p, lengths=lens, int8=True))      # the op takes the widened copies
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(outs[0], o)


def test_module_full_size_batch_independence():
    """Config-3 shape (B=48, lognormal lengths, T on the 128 grid): every utterance of the padded batch equals the
    same module run on that utterance alone, trimmed to its length (size-independent property), and two
    utterances are checked against the oracle."""
    lens = synth.sample_lengths(1003, 48)
    T = synth.round_up(int(lens.max()), synth.FRAME_GRID)
    params = synth.make_params(1003)
    p = prepare_from_params(params, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(1003)
    x = torch.randn((48, T, synth.D_MODEL), generator=g, device=DEV).to(torch.bfloat16)
    lt = torch.from_numpy(lens).to(DEV)
    y = ops.run_conv_module(x, p, lengths=lt)
    for b in range(0, 48, 5):
        L = int(lens[b])
        yb = ops.run_conv_module(x[b:b + 1, :L].contiguous(), p)
        assert_bf16_close(y[b, :L], yb[0], f"batch independence utt {b} (len {L})")
    prep = O.prepare_bf16(params)
    for b in (int(np.argmin(lens)), int(np.argmax(lens))):
        L = int(lens[b])
        xb = x[b:b + 1, :L].float().cpu().numpy()
        assert_bf16_close(y[b:b + 1, :L], O.conv_module(xb, prep, mode="fused"), f"oracle utt {b}")


def test_stack_on_chunks():
    """Two-layer stack over the chunk plan of 20 utterances vs the oracle applied layer by layer."""
    lens = synth.sample_lengths(5005, 20) // 4 + 1
    chunks = dispatch.plan_chunks(lens, exec_batch=8, logical_batch=16)
    layers = [synth.make_params(7000 + i, w_std=0.04) for i in range(2)]
    stack = ConvModuleStack([prepare_from_params(q, device=DEV) for q in layers])
    preps = [O.prepare_bf16(q) for q in layers]
    for c in chunks:
        x = _x(int(c.index[0]) + 10, (c.B, c.T, synth.D_MODEL))
        y = stack(_t(x), torch.from_numpy(c.lengths).to(DEV))
        ref = x
        for pr in preps:
            ref = O.conv_module(ref, pr, lengths=c.lengths, mode="fused")
        assert_bf16_close(y, ref, f"stack chunk B={c.B} T={c.T}")


def test_stack_run_chunks_two_streams():
    """ConvModuleStack.run_chunks (chunks alternating between two streams) equals running them one by one."""
    lens = synth.sample_lengths(5105, 40)
    chunks = dispatch.plan_chunks(lens, exec_batch=12, logical_batch=24)
    stack = ConvModuleStack([prepare_from_params(synth.make_params(7100 + i), device=DEV) for i in range(3)])
    xs = [_t(_x(int(c.index[0]) + 40, (c.B, c.T, synth.D_MODEL))) for c in chunks]
    ls = [torch.from_numpy(c.lengths).to(DEV) for c in chunks]
    seq = [stack(x, l) for x, l in zip(xs, ls)]
    par = stack.run_chunks(list(zip(xs, ls)))
    torch.cuda.synchronize()
    assert len(par) == len(seq)
    for a, b in zip(seq, par):
        assert torch.equal(a, b)


def test_torch_compile_fullgraph():
    params = synth.make_params(9)
    p = prepare_from_params(params, device=DEV)
    x = _t(_x(10, (2, 128, synth.D_MODEL)))
    lens = torch.tensor([128, 100], dtype=torch.int32, device=DEV)

    def f(x, lens):
        y = ops.run_conv_module(x, p, lengths=lens)
        z = torch.ops.granite.dwconv_silu(y.transpose(1, 2)[:, :256], p.dw_w[:256, None, :], p.dw_b[:256])
        return y, z

    cf = torch.compile(f, fullgraph=True)
    y1, z1 = cf(x, lens)
    y0, z0 = f(x, lens)
    assert torch.equal(y0, y1) and torch.equal(z0, z1)
    assert z1.stride() == z0.stride()


@pytest.mark.parametrize("d_model,d_inner,ln_fold", [(512, 1024, False), (512, 1024, True), (2048, 4096, True),
                                                     (256, 256, False)])
def test_module_other_widths(d_model, d_inner, ln_fold):
    """Widths other than the Granite encoder's: the fused kernel, the LayerNorm fold and the residual GEMM are
    generic in D (a LayerNorm width) and inner (a multiple of 128)."""
    params = synth.make_params(600 + d_model, d_model=d_model, d_inner=d_inner, w_std=0.05)
    p = prepare_from_params(params, device=DEV, ln_fold=ln_fold)
    B, T = 3, 256
    x = O.bf16_round(synth.make_activations(601 + d_model, (B, T, d_model)))
    lens = np.array([256, 131, 40], dtype=np.int32)
    y = ops.run_conv_module(_t(x), p, lengths=torch.from_numpy(lens).to(DEV))
    ref = O.conv_module(x, O.prepare_bf16(params), lengths=lens, mode="fused")
    assert_bf16_close(y, ref, f"module D={d_model} inner={d_inner} ln_fold={ln_fold}")
