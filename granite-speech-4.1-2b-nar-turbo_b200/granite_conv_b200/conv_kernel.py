"""Switch a model's Conformer conv modules onto the B200 kernels.

Mirrors ``enable_dwconv_silu`` (``script/models/granite_speech_nar/conv_kernel.py:62-116``): fold BN, require CUDA
+ bf16, test-fire the kernel on the (2, C, 37) shape against the module's own eager torch computation with the
magnitude-relative tolerance ``2e-2 * max(1, max|ref|)`` (``conv_kernel.py:88-104``), then switch every eligible
module.  Modes:

* ``"dwconv_silu"`` / ``"dwconv_silu_glu"`` — the reference's modes: set ``module._fused_conv`` so the reference
  ``ConformerConvModule.forward`` (``conformer.py:178-186``) calls ``torch.ops.granite.dwconv_silu[_glu]``, which
  this package registers on the sm_100a kernels;
* ``"conv_module"`` / ``"conv_module_i8w"`` — new: the whole module (LN, up_conv + GLU, depthwise + SiLU,
  down_conv) runs as ``torch.ops.granite.conv_module[_i8w]`` (the residual stays with the caller, as in
  ``ConformerBlock.forward``, ``conformer.py:207``).

Unlike the reference, a failure raises instead of returning 0 and leaving the torch path in place: there is no
silent fallback.  The environment switch is the reference's ``GRANITE_CONV_KERNEL`` (``attn_backends.py:71-75``).
"""
from __future__ import annotations

import os
import types

import torch
import torch.nn.functional as F
from torch import nn

from . import ops  # noqa: F401  (registers the granite:: ops)
from .weights import _is_conv_module, fold_conv_bn_, prepare_conv_module

MODES = ("dwconv_silu", "dwconv_silu_glu", "conv_module", "conv_module_i8w")


def conv_kernel_mode() -> str:
    """``GRANITE_CONV_KERNEL`` as the reference reads it (``attn_backends.py:71-75``)."""
    return os.environ.get("GRANITE_CONV_KERNEL", "").strip().lower()


def _fused_forward(self, x: torch.Tensor) -> torch.Tensor:
    return ops.run_conv_module(x, self._gsn_prepared, lengths=None, add_residual=False,
                               int8=self._fused_conv == "conv_module_i8w")


def _tol(ref: torch.Tensor) -> float:
    return 2e-2 * max(1.0, ref.float().abs().max().item())


@torch.no_grad()
def enable_dwconv_silu(model: nn.Module, mode: str = "dwconv_silu") -> int:
    """Fold BN and switch every eligible conv module to the B200 kernels; returns the number switched."""
    if mode not in MODES:
        raise ValueError(f"unknown GRANITE_CONV_KERNEL mode {mode!r}; expected one of {MODES}")
    mods = [m for m in model.modules() if _is_conv_module(m)]
    if not mods:
        return 0
    fold_conv_bn_(model)
    conv0 = mods[0].depth_conv.conv
    dev, dtype = conv0.weight.device, conv0.weight.dtype
    if dev.type != "cuda" or dtype != torch.bfloat16:
        raise RuntimeError(f"enable_dwconv_silu needs a CUDA bf16 model (got {dev.type}/{dtype})")

    # test-fire (conv_kernel.py:88-104): the kernel against the eager torch computation of the same module
    C = conv0.weight.shape[0]
    if mode == "dwconv_silu_glu":
        x2 = torch.randn(2, 2 * C, 37, device=dev, dtype=dtype)
        ref = F.silu(conv0(F.glu(x2, dim=1)))
        out = torch.ops.granite.dwconv_silu_glu(x2, conv0.weight, conv0.bias)
    elif mode == "dwconv_silu":
        x = torch.randn(2, C, 37, device=dev, dtype=dtype)
        ref = F.silu(conv0(x))
        out = torch.ops.granite.dwconv_silu(x, conv0.weight, conv0.bias)
    else:
        m0 = mods[0]
        D = m0.norm.weight.shape[0]
        x = torch.randn(2, 37, D, device=dev, dtype=dtype)
        h = m0.glu(m0.up_conv(m0.norm(x).permute(0, 2, 1)))
        ref = m0.down_conv(F.silu(m0.depth_conv(h))).permute(0, 2, 1)
        p0 = prepare_conv_module(m0, device=dev, int8=mode == "conv_module_i8w")
        out = ops.run_conv_module(x, p0, add_residual=False, int8=mode == "conv_module_i8w")
    err = (out.float() - ref.float()).abs().max().item()
    tol = _tol(ref) * (4.0 if mode == "conv_module_i8w" else 1.0)
    if not err <= tol:
        raise RuntimeError(f"enable_dwconv_silu({mode}): test-fire max|d|={err:.3e} > tol {tol:.3e}")

    n = 0
    for m in mods:
        conv = m.depth_conv.conv
        if not (isinstance(m.batch_norm, nn.Identity) and conv.bias is not None
                and getattr(m.depth_conv, "_symmetric", True)):
            continue
        m._fused_conv = mode
        if mode.startswith("conv_module"):
            m._gsn_prepared = prepare_conv_module(m, device=dev, int8=mode == "conv_module_i8w")
            m.forward = types.MethodType(_fused_forward, m)
        n += 1
    return n
