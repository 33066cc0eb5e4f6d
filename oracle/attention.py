"""CPU oracle for the attention step of the Conformer block (test infrastructure only).

This file is the checker: only the tests and the benchmark's CPU-baseline leg import it.  The product path never
calls it.

It restates, in numpy, the reference's eager algorithm:

* ``ConformerAttention.forward`` (``script/models/granite_speech_nar/conformer.py:61-131``): ``pre_norm``
  LayerNorm (``:52``, ``:63``); zero-pad the frames to a multiple of ``context_size`` (``:70-73``); ``to_q`` and
  ``to_kv`` without bias, k = first half of ``to_kv`` (``:76-77``); split into blocks of ``context_size`` and
  heads of ``dim_head`` (``:79-81``); Shaw relative-position bias ``(q_i . rel[i - j + max_pos_emb]) * scale``
  computed from the bf16 query and rounded where the eager module materialises it (``:90-104``); queries and keys
  in the padding added to reach the block multiple are masked with ``-finfo.max`` (``:108-112``);
  ``scaled_dot_product_attention`` with that additive mask and ``scale = dim_head ** -0.5`` (``:114-127``);
  heads concatenated, padding dropped, ``to_out`` with bias (``:128-130``);
* the distances ``clamp(i - j, -context, context) + max_pos_emb`` of ``CTCEncoder`` (``conformer.py:254-262``);
* the residual of ``ConformerBlock.forward``: ``x = attn(x) + x`` (``conformer.py:206``).

Rounding modes: ``"reference"`` rounds to bf16 where the reference's eager bf16 module does -- LayerNorm output,
the q / k / v projections, the positional product and its scaled copy, the attention output (the bf16 MATH
backend of ``scaled_dot_product_attention`` computes in fp32 and rounds once: checked bit for bit against
torch's own output), ``to_out``, the residual sum; ``"fp32"`` rounds nowhere.

Lengths (no counterpart in the reference, which attends over every frame of the padded tensor): utterance ``b``
is computed as the reference computes ``x[b, :len_b]`` alone, and padded frames ``t >= len_b`` of the output are
``x + b_out`` (a zero attention context), as the B200 path writes them.
"""
from __future__ import annotations

import numpy as np

from .conv_module import bf16_round, layer_norm, pointwise

BF16_MAX = float(np.float32(3.3895313892515355e38))


def prepare_attn_bf16(p):
    """Attention parameters as a bf16 model load makes them (every tensor cast to bf16)."""
    r = bf16_round
    return dict(ln_w=r(p.norm_weight), ln_b=r(p.norm_bias), w_q=r(p.q_weight), w_kv=r(p.kv_weight),
                w_out=r(p.out_weight), b_out=r(p.out_bias), rel=r(p.rel_pos), heads=p.heads, context=p.context,
                max_pos=p.max_pos, ln_eps=p.ln_eps)


def prepare_attn_fp32(p):
    return dict(ln_w=p.norm_weight, ln_b=p.norm_bias, w_q=p.q_weight, w_kv=p.kv_weight, w_out=p.out_weight,
                b_out=p.out_bias, rel=p.rel_pos, heads=p.heads, context=p.context, max_pos=p.max_pos,
                ln_eps=p.ln_eps)


def attention_core(q, k, v, rel, heads, context, max_pos, mode="reference", dtype=np.float64):
    """Block-local attention of one utterance: q, k, v (T, heads * dh) -> context (T, heads * dh).

    Every one of the T frames is a real frame; the padding up to the block multiple is masked."""
    T, inner = q.shape
    dh = inner // heads
    cs = context
    rnd = (lambda a: bf16_round(np.asarray(a, dtype=np.float32))) if mode == "reference" else (lambda a: a)
    pad = (cs - T % cs) % cs
    P = T + pad
    nb = P // cs

    def blocks(a):   # (T, inner) -> (nb, heads, cs, dh)
        a = np.concatenate([np.asarray(a, dtype=dtype), np.zeros((pad, inner), dtype=dtype)], axis=0)
        return a.reshape(nb, cs, heads, dh).transpose(0, 2, 1, 3)

    qb, kb, vb = blocks(q), blocks(k), blocks(v)
    scale = dh ** -0.5
    seq = np.arange(cs)
    dists = np.clip(seq[:, None] - seq[None, :], -cs, cs) + max_pos          # (cs, cs)
    relg = np.asarray(rel, dtype=dtype)[dists]                              # (cs_i, cs_j, dh)
    # pos[m, h, i, j] = q[m, h, i] . relg[i, j]: batched over i
    qi = qb.transpose(2, 0, 1, 3).reshape(cs, nb * heads, dh)               # (i, m*h, d)
    pos = np.matmul(qi, relg.transpose(0, 2, 1))                             # (i, m*h, j)
    pos = pos.reshape(cs, nb, heads, cs).transpose(1, 2, 0, 3)               # (m, h, i, j)
    pos = rnd(rnd(pos) * np.float32(scale)) if mode == "reference" else pos * scale
    valid = (np.arange(P) < T).reshape(nb, cs)
    keep = valid[:, :, None] & valid[:, None, :]                            # (m, i, j)
    bias = np.where(keep[:, None], np.asarray(pos, dtype=dtype), -BF16_MAX)
    s = np.matmul(qb, kb.transpose(0, 1, 3, 2)) * scale + bias
    s = s - s.max(axis=-1, keepdims=True)
    e = np.exp(s)
    p = e / e.sum(axis=-1, keepdims=True)
    ctx = np.matmul(p, vb)                                                   # (m, h, cs, dh)
    ctx = ctx.transpose(0, 2, 1, 3).reshape(P, inner)[:T]
    return rnd(ctx)


def attention_block(x, prep, lengths=None, mode="reference", dtype=np.float64):
    """``x + ConformerAttention(x)`` on channels-last ``x (B, T, D)``."""
    B, T, D = x.shape
    rnd = (lambda a: bf16_round(np.asarray(a, dtype=np.float32))) if mode == "reference" else (lambda a: a)
    heads = prep["heads"]
    inner = prep["w_q"].shape[0]
    out = np.empty((B, T, D), dtype=np.float32 if mode == "reference" else dtype)
    xin = np.asarray(x, dtype=np.float32)
    for b in range(B):
        L = T if lengths is None else int(min(max(int(lengths[b]), 0), T))
        if L > 0:
            xb = xin[b, :L]
            xn = rnd(layer_norm(xb[None], prep["ln_w"], prep["ln_b"], prep["ln_eps"], dtype=dtype)[0])
            zero = np.zeros(3 * inner, dtype=np.float32)
            q = rnd(pointwise(np.asarray(xn), prep["w_q"], zero[:inner], dtype=dtype))
            kv = rnd(pointwise(np.asarray(xn), prep["w_kv"], zero[inner:], dtype=dtype))
            k, v = kv[:, :inner], kv[:, inner:]
            ctx = attention_core(q, k, v, prep["rel"], heads, prep["context"], prep["max_pos"], mode=mode,
                                 dtype=dtype)
            y = rnd(pointwise(np.asarray(ctx), prep["w_out"], prep["b_out"], dtype=dtype))
            out[b, :L] = rnd(np.asarray(y, dtype=dtype) + xb.astype(dtype))
        if L < T:
            out[b, L:] = rnd(xin[b, L:].astype(dtype) + np.asarray(prep["b_out"], dtype=dtype)[None, :])
    return out
