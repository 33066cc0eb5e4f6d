"""The conv-module entry point for callers that cannot allocate device memory (a plugin inside a host application
that owns the GPU memory budget, a latency-critical path where cudaMalloc would synchronise the device):
gsn_conv_module_bf16_noalloc runs the whole module in the library's fixed 32 MiB scratch.  Its results must
match the entry point that takes a caller workspace, call after call, and oversized problems must be refused.

This file is collected last so that a run stopping at the first failure has already run every other test; it
also passes on its own in a fresh process."""
import numpy as np
import pytest
import torch

from granite_conv_b200 import _lib, synth
from granite_conv_b200.weights import prepare_from_params
from oracle import conv_module as O
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _args(p, x, lens, out):
    return (x.data_ptr(), p.ln_w.data_ptr(), p.ln_b.data_ptr(), p.w1_glu.data_ptr(), p.b1_glu.data_ptr(),
            p.dw_w.data_ptr(), p.dw_b.data_ptr(), p.w2.data_ptr(), p.b2.data_ptr(),
            None if lens is None else lens.data_ptr(), 1, out.data_ptr())


def _with_workspace(p, x, lens):
    """The existing entry point, given a workspace allocated by torch."""
    L = _lib.lib()
    B, T, D = x.shape
    out = torch.empty_like(x)
    nbytes = int(L.gsn_conv_module_workspace_bytes(B, T, D, p.d_inner))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    _lib.check(L.gsn_conv_module_bf16(*_args(p, x, lens, out), B, T, D, p.d_inner, p.ln_eps, ws.data_ptr(), nbytes,
                                      torch.cuda.current_stream().cuda_stream), "gsn_conv_module_bf16")
    return out


def _no_alloc(p, x, lens):
    L = _lib.lib()
    B, T, D = x.shape
    out = torch.empty_like(x)
    _lib.check(L.gsn_conv_module_bf16_noalloc(*_args(p, x, lens, out), B, T, D, p.d_inner, p.ln_eps,
                                              torch.cuda.current_stream().cuda_stream), "gsn_conv_module_bf16_noalloc")
    return out


def test_no_alloc_matches_workspace_entry_point_twice():
    """Two calls in a row: a dense call that fills the whole scratch (4096 frames), then a smaller masked one that
    starts from the first call's leftovers in the shared array.  The two entry points run the same kernels on the
    same inputs, so each output must equal the workspace entry point's bit for bit."""
    p = prepare_from_params(synth.make_params(4242, w_std=0.05), device=DEV)
    cases = [
        ((4, 1024), None),
        ((3, 256), np.array([256, 200, 37], dtype=np.int32)),
    ]
    for i, ((B, T), lens) in enumerate(cases):
        x = torch.from_numpy(O.bf16_round(synth.make_activations(777 + i, (B, T, synth.D_MODEL)))).to(
            torch.bfloat16).to(DEV)
        lt = None if lens is None else torch.from_numpy(lens).to(DEV)
        y = _no_alloc(p, x, lt)
        ref = _with_workspace(p, x, lt)
        torch.cuda.synchronize()
        assert torch.equal(y, ref), f"no-alloc call {i} differs from the workspace entry point"
        assert_bf16_close(y, ref, f"no-alloc call {i} vs workspace entry point")
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0


def test_no_alloc_refuses_problems_above_its_scratch():
    L = _lib.lib()
    x = torch.zeros((2, 4096, synth.D_MODEL), dtype=torch.bfloat16, device=DEV)    # 8192 frames: 64 MiB needed
    p = prepare_from_params(synth.make_params(1), device=DEV)
    out = torch.empty_like(x)
    rc = L.gsn_conv_module_bf16_noalloc(*_args(p, x, None, out), 2, 4096, synth.D_MODEL, p.d_inner, p.ln_eps,
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == 5 and "33554432" in _lib.last_error()
    # an unsupported width is reported as unsupported (GSN_ERR_UNSUPPORTED = 2), not as a scratch-size problem
    rc = L.gsn_conv_module_bf16_noalloc(*_args(p, x, None, out), 2, 4096, 768, p.d_inner, p.ln_eps,
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == 2, (rc, _lib.last_error())
