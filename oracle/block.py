"""CPU oracle for a whole Conformer block (test infrastructure only).

This file is the checker: only the tests import it.  The product path never calls it.

It composes the oracles of the block's steps in the order of ``ConformerBlock.forward``
(``script/models/granite_speech_nar/conformer.py:203-210``): ``x = 0.5 * ff1(x) + x`` (``oracle.feed_forward``),
``x = attn(x) + x`` (``oracle.attention``), ``x = conv(x) + x`` (``oracle.conv_module``), ``x = 0.5 * ff2(x) + x``,
``x = post_norm(x)`` (LayerNorm).  Rounding modes as in those files: ``"reference"`` rounds where the reference's
eager bf16 block materialises bf16 tensors, ``"fp32"`` nowhere.  With lengths, padded frames follow each step's
rule (x + bias of its last projection), then the post norm.
"""
from __future__ import annotations

import numpy as np

from . import attention as AT
from . import conv_module as O
from . import feed_forward as FF


def prepare_block(p, mode="reference"):
    if mode == "reference":
        return dict(ff1=FF.prepare_ff_bf16(p.ff1), attn=AT.prepare_attn_bf16(p.attn), conv=O.prepare_bf16(p.conv),
                    ff2=FF.prepare_ff_bf16(p.ff2), post_w=O.bf16_round(p.post_norm_weight),
                    post_b=O.bf16_round(p.post_norm_bias), eps=p.post_ln_eps)
    return dict(ff1=FF.prepare_ff_fp32(p.ff1), attn=AT.prepare_attn_fp32(p.attn), conv=O.prepare_fp32(p.conv),
                ff2=FF.prepare_ff_fp32(p.ff2), post_w=p.post_norm_weight, post_b=p.post_norm_bias,
                eps=p.post_ln_eps)


def conformer_block(x, prep, lengths=None, mode="reference", dtype=np.float64):
    conv_mode = "reference" if mode == "reference" else "fp32"
    x = FF.feed_forward_half(x, prep["ff1"], lengths=lengths, mode=mode, dtype=dtype)
    x = AT.attention_block(np.asarray(x, dtype=np.float32) if mode == "reference" else x, prep["attn"],
                           lengths=lengths, mode=mode, dtype=dtype)
    x = O.conv_module(np.asarray(x, dtype=np.float32) if mode == "reference" else x, prep["conv"], lengths=lengths,
                      mode=conv_mode, dtype=dtype)
    x = FF.feed_forward_half(x, prep["ff2"], lengths=lengths, mode=mode, dtype=dtype)
    y = O.layer_norm(np.asarray(x, dtype=dtype), prep["post_w"], prep["post_b"], prep["eps"], dtype=dtype)
    return O.bf16_round(np.asarray(y, dtype=np.float32)) if mode == "reference" else y
