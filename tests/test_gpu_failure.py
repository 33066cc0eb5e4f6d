"""Failure detection without a GPU fault: every spin-wait in the kernels is bounded; a wait that runs out records
a code in the device status word and the kernel returns, leaving the context usable."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from granite_conv_b200 import _lib
from oracle import conv_module as O
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives():
    s = torch.cuda.current_stream().cuda_stream
    _lib.device_status(s, clear=True)
    _lib.call("gsn_selftest_bounded_wait", 50_000_000, s)          # 50 ms on an mbarrier nothing completes
    assert _lib.device_status(s, clear=True) == 0x1FF
    assert _lib.device_status(s, clear=False) == 0
    # the context still runs kernels correctly afterwards
    x = O.bf16_round(np.random.default_rng(0).normal(size=(1, 64, 256)).astype(np.float32))
    w = O.bf16_round(np.random.default_rng(1).normal(0, 0.05, (256, 15)).astype(np.float32))
    b = O.bf16_round(np.random.default_rng(2).normal(0, 0.02, 256).astype(np.float32))
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    y = torch.ops.granite.dwconv_silu(xt.transpose(1, 2), torch.from_numpy(w).to(torch.bfloat16).cuda()[:, None],
                                      torch.from_numpy(b).to(torch.bfloat16).cuda())
    assert_bf16_close(y.transpose(1, 2), O.dwconv_silu(x, w, b), "dw after timeout")
    assert _lib.device_status(s) == 0


def test_selftest_argument_checks():
    with pytest.raises(RuntimeError, match="limit_ns"):
        _lib.call("gsn_selftest_bounded_wait", 0, 0)
    with pytest.raises(RuntimeError, match="limit_ns"):
        _lib.call("gsn_selftest_bounded_wait", 3_000_000_000, 0)


# ---- the unwind path of the production kernels: one copy per CTA armed but never issued --------------------------
def _after_abort_module_still_correct():
    """A full-size module call (B=48 lognormal chunk, T on the 128 grid: LayerNorm statistics, the fused
    up_conv + GLU + depthwise kernel, the residual GEMM) right after the unwind: utterances checked against the
    oracle, and the status word stays clear."""
    from granite_conv_b200 import ops, synth
    from granite_conv_b200.weights import prepare_from_params
    s = torch.cuda.current_stream().cuda_stream
    lens = synth.sample_lengths(1003, 48)
    T = synth.round_up(int(lens.max()), 128)
    params = synth.make_params(1005, w_std=0.05)
    p = prepare_from_params(params, device="cuda", ln_fold=True)
    x = O.bf16_round(synth.make_activations(4321, (48, T, synth.D_MODEL)))
    y = ops.run_conv_module(torch.from_numpy(x).to(torch.bfloat16).cuda(), p,
                            lengths=torch.from_numpy(lens).cuda()).float().cpu().numpy()
    prep = O.prepare_bf16(params)
    for b in (0, int(np.argmax(lens)), 47):
        L = int(lens[b])
        ref = O.conv_module(x[b:b + 1, :L], prep, mode="fused")
        assert_bf16_close(y[b:b + 1, :L], ref, f"module utterance {b} after the unwind", rel_l2=1e-2)
    assert _lib.device_status(s) == 0


@pytest.mark.parametrize("layout", ["channels_last", "channels_first"])
def test_depthwise_unwinds_after_withheld_copy(layout):
    """The depthwise kernels with every CTA's first tile armed but never loaded: the bounded wait runs out, the
    kernel records a timeout and returns (the tensor-core kernel also frees its TMEM), and the context then runs the
    whole module correctly."""
    s = torch.cuda.current_stream().cuda_stream
    B, C, T = 4, 256, 512
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((B, T, C), generator=g, device="cuda").to(torch.bfloat16)
    w = (0.05 * torch.randn((C, 15), generator=g, device="cuda")).to(torch.bfloat16)
    b = (0.02 * torch.randn((C,), generator=g, device="cuda")).to(torch.bfloat16)
    if layout == "channels_last":
        xin = x.transpose(1, 2)                                     # (B, C, T) view, C innermost
        y = torch.empty_strided((B, C, T), (T * C, 1, C), dtype=torch.bfloat16, device="cuda")
    else:
        xin = x.transpose(1, 2).contiguous()                        # (B, C, T), T innermost
        y = torch.empty((B, C, T), dtype=torch.bfloat16, device="cuda")
    _lib.device_status(s, clear=True)
    _lib.call("gsn_selftest_dwconv_withheld_bf16", xin.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), B, C, T,
              *xin.stride(), *y.stride(), s)
    # the channels-last kernel's wait (0x104); the channels-first one runs on the tensor cores, where the producer,
    # the MMA issuer or the epilogue may give up first (0x101 - 0x103)
    assert _lib.device_status(s, clear=True) in ((0x104,) if layout == "channels_last" else (0x101, 0x102, 0x103))
    ref = torch.ops.granite.dwconv_silu(xin, w[:, None, :], b)      # the same launch without the withheld copy
    want = F.silu(F.conv1d(xin.float(), w[:, None, :].float(), b.float(), padding=7, groups=C))
    assert_bf16_close(ref.float(), want, f"dw {layout} after the unwind")
    _after_abort_module_still_correct()


def test_gemm_unwinds_after_withheld_copy():
    """The down_conv + residual GEMM with every CTA's second operand load armed but never issued: one K-block of
    MMAs has run into TMEM when the MMA warp's wait runs out; every role unwinds (the producer lets its copies land,
    the epilogue its residual copies, TMEM is freed) and the status word reads a timeout.  A following full-size
    module call, whose kernels allocate TMEM again on every SM, must pass the oracle."""
    s = torch.cuda.current_stream().cuda_stream
    M, K, N = 2048, 2048, 1024
    g = torch.Generator(device="cuda").manual_seed(4)
    d = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn((N, K), generator=g, device="cuda")).to(torch.bfloat16)
    bias = (0.02 * torch.randn((N,), generator=g, device="cuda")).float()
    res = torch.randn((M, N), generator=g, device="cuda").to(torch.bfloat16)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    _lib.device_status(s, clear=True)
    _lib.call("gsn_selftest_gemm_withheld_bf16", d.data_ptr(), w.data_ptr(), bias.data_ptr(), res.data_ptr(),
              out.data_ptr(), M, K, N, s)
    assert _lib.device_status(s, clear=True) in (0x101, 0x102, 0x103)
    assert _lib.device_status(s, clear=False) == 0
    _lib.call("gsn_gemm2_residual_bf16", d.data_ptr(), w.data_ptr(), bias.data_ptr(), res.data_ptr(), N,
              out.data_ptr(), N, M, K, N, None, 0, s)
    want = d.float() @ w.float().t() + bias + res.float()
    assert_bf16_close(out.float(), want, "residual GEMM after the unwind")
    _after_abort_module_still_correct()

