"""CPU oracle for the feed-forward halves of the Conformer block (test infrastructure only).

This file is the checker: only the tests import it.  The product path never calls it.

It restates, in numpy, the reference's eager algorithm:

* ``ConformerFeedForward.forward`` (``script/models/granite_speech_nar/conformer.py:33-40``): ``pre_norm``
  LayerNorm (``:27``), ``up_proj`` Linear D->4D with bias (``:28``), SiLU (``:29``), ``down_proj`` Linear 4D->D
  with bias (``:31``); dropout is the identity at inference;
* the half-step residual of ``ConformerBlock.forward``: ``x = 0.5 * ff(x) + x`` (``conformer.py:205``, ``:208``);
* the block's ``post_norm`` LayerNorm (``conformer.py:199``, ``:209``) is ``conv_module.layer_norm``.

Rounding modes for the bf16 block: ``"reference"`` rounds to bf16 wherever the reference's eager bf16 module
materialises a tensor (LayerNorm, up_proj, SiLU, down_proj, the scaled sum); ``"fp32"`` rounds nowhere.  With
``lengths`` the padded frames of the output are ``x + 0.5 * b_down`` (what a zero row after the SiLU gives), as the
B200 path writes them; valid frames do not depend on padding (no cross-frame arithmetic).
"""
from __future__ import annotations

import numpy as np

from .conv_module import _silu, bf16_round, layer_norm, pointwise


def prepare_ff_bf16(p):
    """Feed-forward parameters as a bf16 model load makes them (every tensor cast to bf16)."""
    r = bf16_round
    return dict(ln_w=r(p.norm_weight), ln_b=r(p.norm_bias), w_up=r(p.up_weight), b_up=r(p.up_bias),
                w_down=r(p.down_weight), b_down=r(p.down_bias), ln_eps=p.ln_eps)


def prepare_ff_fp32(p):
    return dict(ln_w=p.norm_weight, ln_b=p.norm_bias, w_up=p.up_weight, b_up=p.up_bias, w_down=p.down_weight,
                b_down=p.down_bias, ln_eps=p.ln_eps)


def feed_forward_half(x, prep, lengths=None, mode="reference", dtype=np.float64):
    """``x + 0.5 * ff(x)`` on channels-last ``x (B, T, D)``."""
    B, T, D = x.shape
    rnd = (lambda a: bf16_round(np.asarray(a, dtype=np.float32))) if mode == "reference" else (lambda a: a)
    xin = x.astype(np.float32)
    xn = rnd(layer_norm(xin, prep["ln_w"], prep["ln_b"], prep["ln_eps"], dtype=dtype)).reshape(B * T, D)
    h = rnd(pointwise(xn, prep["w_up"], prep["b_up"], dtype=dtype))
    a = rnd(_silu(np.asarray(h, dtype=dtype)))
    y = rnd(pointwise(a, prep["w_down"], prep["b_down"], dtype=dtype)).reshape(B, T, D)
    out = 0.5 * np.asarray(y, dtype=dtype) + xin.astype(dtype)
    if lengths is not None:
        pad = np.arange(T)[None, :] >= np.asarray(lengths)[:, None]
        half_b = 0.5 * np.asarray(prep["b_down"], dtype=dtype)
        out = np.where(pad[..., None], xin.astype(dtype) + half_b[None, None, :], out)
    return rnd(out) if mode == "reference" else out.astype(np.float32 if dtype == np.float32 else dtype)
