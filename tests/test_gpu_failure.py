"""Failure detection without a GPU fault: every spin-wait in the kernels is bounded; a wait that runs out records
a code in the device status word and the kernel returns, leaving the context usable."""
import numpy as np
import pytest
import torch

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
