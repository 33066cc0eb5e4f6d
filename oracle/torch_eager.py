"""Torch CPU restatement of the reference's eager conv module (test infrastructure only).

Only the tests and the benchmark's CPU-baseline legs (``cpu_baseline``, ``--impl reference``) use this file; the
product path never calls it.  It is the CPU side the B200 kernels are measured against: the op calls the
reference's eager path makes, in the same order, on the host cores.

* ``ConformerConvModule.forward`` after the BN fold (``script/models/granite_speech_nar/conformer.py:175-189`` with
  ``_fused_conv`` unset and ``batch_norm`` an ``Identity``): ``F.layer_norm`` (``:176``), the 1x1 ``up_conv`` as
  ``F.conv1d`` on ``x.permute(0, 2, 1)`` (``:177``), ``F.glu(dim=1)`` (``:181``), the depthwise ``F.conv1d`` with
  ``groups=C`` and the symmetric zero padding folded into the conv (``DepthWiseConv1d``, ``:134-155``),
  ``F.silu`` (``:186``), the 1x1 ``down_conv`` and the permute back (``:187``);
* the residual add of ``ConformerBlock.forward`` (``conformer.py:207``);
* the fold of ``fold_conv_bn_`` (``script/models/granite_speech_nar/fold_bn.py:51-64``): fp32
  ``scale = gamma * rsqrt(var + eps)``, ``W' = W * scale``, ``b' = beta - mean * scale``, cast to the weight dtype.

Like the reference module it has no length mask: a chunk is processed as its padded ``(B, T, D)`` tensor.
"""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.nn.functional as F

K_DW = 15


def host_threads() -> int:
    """Every core this process may run on (``torch.set_num_threads`` of the CPU baseline)."""
    return len(os.sched_getaffinity(0))


class EagerConvModule:
    """The reference's eager conv module + residual on CPU, weights in ``dtype`` (float32 or bfloat16)."""

    def __init__(self, params, dtype: torch.dtype = torch.float32, ln_eps: float = 1e-5, bn_eps: float = 1e-5):
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))  # noqa: E731
        self.dtype = dtype
        self.eps = ln_eps
        self.d_model = params.norm_weight.shape[0]
        self.inner = params.dw_weight.shape[0]
        self.ln_w = t(params.norm_weight).to(dtype)
        self.ln_b = t(params.norm_bias).to(dtype)
        self.w1 = t(params.up_weight)[:, :, None].to(dtype).contiguous()
        self.b1 = t(params.up_bias).to(dtype)
        self.w2 = t(params.down_weight)[:, :, None].to(dtype).contiguous()
        self.b2 = t(params.down_bias).to(dtype)
        # the fold, in fp32 from the weight as stored in `dtype`, then cast back
        w = t(params.dw_weight)[:, None, :].to(dtype).float()
        scale = t(params.bn_weight).to(dtype).float() * torch.rsqrt(t(params.bn_var).to(dtype).float() + bn_eps)
        self.dw_w = (w * scale.reshape(-1, 1, 1)).to(dtype).contiguous()
        self.dw_b = (t(params.bn_bias).to(dtype).float() - t(params.bn_mean).to(dtype).float() * scale).to(dtype)

    @torch.no_grad()
    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """x: (B, T, D) in the module's dtype -> conv(x) + x."""
        h = F.layer_norm(x, (self.d_model,), self.ln_w, self.ln_b, self.eps)
        h = F.conv1d(h.permute(0, 2, 1), self.w1, self.b1)
        h = F.glu(h, dim=1)
        h = F.conv1d(h, self.dw_w, self.dw_b, padding=K_DW // 2, groups=self.inner)
        h = F.silu(h)
        h = F.conv1d(h, self.w2, self.b2).permute(0, 2, 1)
        return h + x


@torch.no_grad()
def dwconv_silu(x_bct: torch.Tensor, weight_ck: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """The post-fold depthwise conv + SiLU of the reference's eager path on a (B, C, T) tensor: the computation the
    fused ``granite::dwconv_silu`` replaces (``conv_kernel.py:93``: ``F.silu(conv0(x))``)."""
    return F.silu(F.conv1d(x_bct, weight_ck[:, None, :], bias, padding=K_DW // 2, groups=x_bct.shape[1]))


@torch.no_grad()
def dwconv_silu_glu(x2_bct: torch.Tensor, weight_ck: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """``F.silu(conv0(F.glu(x2, dim=1)))`` (``conv_kernel.py:89``)."""
    return dwconv_silu(F.glu(x2_bct, dim=1), weight_ck, bias)
