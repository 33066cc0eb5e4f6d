"""The enable switch (row a7): ``enable_dwconv_silu`` against the contract of the reference's
``script/models/granite_speech_nar/conv_kernel.py:63-116`` -- fold BN, require a CUDA bf16 model, test-fire, set
``_fused_conv`` on every eligible module and return how many were switched -- in all four modes, with a module whose
``forward`` restates ``ConformerConvModule.forward`` (``conformer.py:175-189``) including its ``_fused_conv``
branches, so the reference modes run the ``granite::`` ops exactly where the reference calls them."""
import copy

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from granite_conv_b200.conv_kernel import enable_dwconv_silu
from granite_conv_b200.weights import fold_conv_bn_
from parity import assert_bf16_close, stats

pytestmark = pytest.mark.gpu
DEV = "cuda"


class _DepthWise(nn.Module):
    """``DepthWiseConv1d`` (conformer.py:134-155) for an odd kernel: the zero padding folded into the conv."""

    def __init__(self, c, k=15):
        super().__init__()
        self._symmetric = True
        self.conv = nn.Conv1d(c, c, k, groups=c, bias=False, padding=k // 2)

    def forward(self, x):
        return self.conv(x)


class _ConvModule(nn.Module):
    """Attribute layout and forward of ``ConformerConvModule`` (conformer.py:158-189)."""

    def __init__(self, d=1024, inner=2048):
        super().__init__()
        self.norm = nn.LayerNorm(d)
        self.up_conv = nn.Conv1d(d, 2 * inner, 1)
        self.glu = nn.GLU(dim=1)
        self.depth_conv = _DepthWise(inner)
        self.silu = nn.SiLU()
        self.batch_norm = nn.BatchNorm1d(inner)
        self.down_conv = nn.Conv1d(inner, d, 1)
        self._fused_conv = False

    def forward(self, x):
        x = self.norm(x)
        x = self.up_conv(x.permute(0, 2, 1))
        if self._fused_conv == "dwconv_silu_glu":
            x = torch.ops.granite.dwconv_silu_glu(x, self.depth_conv.conv.weight, self.depth_conv.conv.bias)
        else:
            x = self.glu(x)
            if self._fused_conv:
                x = torch.ops.granite.dwconv_silu(x, self.depth_conv.conv.weight, self.depth_conv.conv.bias)
            else:
                x = self.depth_conv(x)
                x = self.silu(self.batch_norm(x))
        return self.down_conv(x).permute(0, 2, 1)


class _Encoder(nn.Module):
    """Three conv modules with a linear layer between two of them (a module the switch must leave alone)."""

    def __init__(self, n=3, d=1024, inner=2048, w_std=0.05):
        super().__init__()
        self.layers = nn.ModuleList([_ConvModule(d, inner) for _ in range(n)])
        self.mix = nn.Linear(d, d)
        g = torch.Generator().manual_seed(11)
        with torch.no_grad():
            for m in self.layers:
                for conv in (m.up_conv, m.down_conv, m.depth_conv.conv):
                    conv.weight.normal_(0.0, w_std, generator=g)
                bn = m.batch_norm
                bn.running_mean.normal_(0.0, 0.1, generator=g)
                bn.running_var.uniform_(0.5, 1.5, generator=g)
                bn.weight.uniform_(0.8, 1.2, generator=g)
                bn.bias.normal_(0.0, 0.05, generator=g)

    def forward(self, x):
        for i, m in enumerate(self.layers):
            x = m(x) + x                                 # the block's residual (conformer.py:207)
            if i == 0:
                x = self.mix(x)
        return x


def _models():
    base = _Encoder().eval()
    switched = copy.deepcopy(base).to(DEV, torch.bfloat16)
    eager = copy.deepcopy(base).to(DEV, torch.bfloat16)
    fold_conv_bn_(eager)                                  # the reference's eager path after its own fold
    return switched, eager


def _ops_called(model, x):
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU], acc_events=True) as prof:
        y = model(x)
    torch.cuda.synchronize()
    return y, {e.name for e in prof.events() if e.name.startswith("granite::")}


@pytest.mark.parametrize("mode", ["dwconv_silu", "dwconv_silu_glu", "conv_module", "conv_module_i8w"])
def test_enable_modes_match_eager(mode):
    """Every switched module equals its eager twin (the reference's forward after the fold) on the same input within
    the element gate; the whole three-module chain, where bf16 rounding differences compound through the residual
    adds and the linear layer, within rel-L2 1e-2."""
    switched, eager = _models()
    n = enable_dwconv_silu(switched, mode=mode)
    assert n == 3
    for m in switched.layers:
        assert m._fused_conv == mode
        assert isinstance(m.batch_norm, nn.Identity)
        assert m.depth_conv.conv.bias is not None
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn((2, 256, 1024), generator=g, device=DEV).to(torch.bfloat16)
    expect = {"dwconv_silu": "granite::dwconv_silu", "dwconv_silu_glu": "granite::dwconv_silu_glu",
              "conv_module": "granite::conv_module", "conv_module_i8w": "granite::conv_module_i8w"}[mode]
    with torch.no_grad():
        h = x
        for i, (ms, me) in enumerate(zip(switched.layers, eager.layers)):
            y, called = _ops_called(ms, h)
            ref = me(h)
            assert expect in called, f"{mode}: {expect} not called ({sorted(called)})"
            if mode == "conv_module_i8w":
                # int8 weights change the module's output by the weight quantisation: 4x the element gate (the
                # test-fire's allowance for this mode) and rel-L2 2e-2
                s = stats(y, ref)
                assert s["worst_ratio"] <= 4.0 and s["rel_l2"] <= 2e-2, s
            else:
                s = assert_bf16_close(y, ref, f"switched {mode} module {i} vs eager")
            print(f"{mode} module {i}: max|d| {s['max_abs']:.3e}, worst/gate {s['worst_ratio']:.3f}, "
                  f"rel-L2 {s['rel_l2']:.2e}")
            h = ref + h
            if i == 0:
                h = eager.mix(h)
        whole = stats(switched(x), eager(x))
    assert whole["rel_l2"] <= (2e-2 if mode == "conv_module_i8w" else 1e-2), whole
    print(f"{mode} chain of 3: rel-L2 {whole['rel_l2']:.2e}")


def test_enable_refusals():
    enc = _Encoder(n=1).eval()
    with pytest.raises(ValueError):
        enable_dwconv_silu(copy.deepcopy(enc).to(DEV, torch.bfloat16), mode="dwconv")       # unknown mode
    with pytest.raises(RuntimeError, match="CUDA bf16"):
        enable_dwconv_silu(copy.deepcopy(enc), mode="dwconv_silu")                         # CPU fp32 model
    with pytest.raises(RuntimeError, match="CUDA bf16"):
        enable_dwconv_silu(copy.deepcopy(enc).to(DEV), mode="dwconv_silu")                 # CUDA fp32 model
    assert enable_dwconv_silu(nn.Sequential(nn.Linear(8, 8)).eval(), mode="dwconv_silu") == 0
    train = _Encoder(n=1).to(DEV, torch.bfloat16)                                           # training mode
    with pytest.raises(RuntimeError, match="eval"):
        enable_dwconv_silu(train, mode="dwconv_silu")
    m = copy.deepcopy(enc).to(DEV, torch.bfloat16)
    assert enable_dwconv_silu(m, mode="dwconv_silu") == 1
    assert enable_dwconv_silu(m, mode="dwconv_silu") == 1          # the fold is idempotent; switching again is fine
