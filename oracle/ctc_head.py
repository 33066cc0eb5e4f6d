"""CPU oracle for the encoder's CTC heads and the CTC collapse (test infrastructure only).

This file is the checker: only the tests and the benchmark's CPU-baseline leg import it.  The product path never
calls it.

It restates, in numpy, the reference's eager algorithm:

* the middle layer's self-conditioning (``script/models/granite_speech_nar/conformer.py:320-324``):
  ``mid_logits = out(h)`` (bf16), ``mid_probs = softmax(float(mid_logits))``, ``blank = mid_probs[..., 0]``,
  ``h = h + out_mid(bf16(mid_probs))``;
* ``posterior_weighted_pool`` (``conformer.py:214-226``): frames padded to a multiple of the window with zero hidden
  state and zero importance, weights ``importance / (sum + 1e-8)`` per window, in fp32, then bf16
  (``conformer.py:338-341``), with ``importance = 1 - blank``;
* the BPE head ``out_bpe`` on each utterance's first ``ceil(len / window)`` pooled frames (``conformer.py:351-353``)
  and its argmax (``asr.py:123-134``, first index among equal values);
* ``_collapse_ids_flat`` (``asr.py:76-102``): keep an id where it starts the utterance or differs from its
  predecessor, and is not the blank.

Lengths (the reference pools over the padded tensor): utterance ``b`` is computed as the reference computes
``h[b, :len_b]`` alone; the self-conditioning writes ``h + b_mid`` and blank 1 on padded frames.
"""
from __future__ import annotations

import numpy as np

from .conv_module import bf16_round, pointwise


def prepare_ctc_bf16(p):
    r = bf16_round
    return dict(w_out=r(p.out_weight), b_out=r(p.out_bias), w_mid=r(p.mid_weight), b_mid=r(p.mid_bias),
                w_bpe=r(p.bpe_weight), b_bpe=r(p.bpe_bias), blank_id=p.blank_id, window=p.window)


def prepare_ctc_fp32(p):
    return dict(w_out=p.out_weight, b_out=p.out_bias, w_mid=p.mid_weight, b_mid=p.mid_bias, w_bpe=p.bpe_weight,
                b_bpe=p.bpe_bias, blank_id=p.blank_id, window=p.window)


def selfcond(h, prep, lengths=None, mode="reference", dtype=np.float64):
    """(h', blank) on channels-last ``h (B, T, D)``."""
    B, T, D = h.shape
    rnd = (lambda a: bf16_round(np.asarray(a, dtype=np.float32))) if mode == "reference" else (lambda a: a)
    hf = np.asarray(h, dtype=np.float32)
    logits = rnd(pointwise(hf.reshape(B * T, D), prep["w_out"], prep["b_out"], dtype=dtype))
    lg = np.asarray(logits, dtype=np.float32).astype(np.float64)
    e = np.exp(lg - lg.max(axis=-1, keepdims=True))
    probs = (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
    blank = probs[:, 0].reshape(B, T).copy()
    pin = rnd(probs) if mode == "reference" else probs
    if lengths is not None:
        pad = (np.arange(T)[None, :] >= np.asarray(lengths)[:, None]).reshape(-1)
        pin = np.where(pad[:, None], 0.0, pin)
        blank = np.where(pad.reshape(B, T), 1.0, blank).astype(np.float32)
    y = rnd(pointwise(np.asarray(pin), prep["w_mid"], prep["b_mid"], dtype=dtype)).reshape(B, T, D)
    out = rnd(np.asarray(y, dtype=dtype) + hf.astype(dtype))
    return out, blank


def pool(h, blank, lengths=None, window=4, mode="reference"):
    """(pooled list per utterance (P_b, D), pooled lengths)."""
    B, T, D = h.shape
    out, plen = [], []
    for b in range(B):
        L = T if lengths is None else int(min(max(int(lengths[b]), 0), T))
        P = -(-L // window)
        hb = np.zeros((P * window, D), dtype=np.float32)
        ib = np.zeros(P * window, dtype=np.float32)
        hb[:L] = np.asarray(h[b, :L], dtype=np.float32)
        ib[:L] = 1.0 - np.asarray(blank[b, :L], dtype=np.float32)
        hb = hb.reshape(P, window, D)
        ib = ib.reshape(P, window)
        w = ib / (ib.sum(axis=-1, keepdims=True) + np.float32(1e-8))
        pooled = (hb * w[..., None]).sum(axis=1)
        out.append(bf16_round(pooled) if mode == "reference" else pooled)
        plen.append(P)
    return out, np.array(plen, dtype=np.int32)


def head_logits(pooled_b, prep, mode="reference", dtype=np.float64):
    rnd = (lambda a: bf16_round(np.asarray(a, dtype=np.float32))) if mode == "reference" else (lambda a: a)
    return rnd(pointwise(np.asarray(pooled_b), prep["w_bpe"], prep["b_bpe"], dtype=dtype))


def collapse(ids, blank_id):
    ids = np.asarray(ids)
    if ids.size == 0:
        return ids.astype(np.int32)
    change = np.ones(ids.size, dtype=bool)
    change[1:] = ids[1:] != ids[:-1]
    return ids[change & (ids != blank_id)].astype(np.int32)


def decode(h, blank, prep, lengths=None, mode="reference"):
    """Per utterance: (argmax ids, logits, collapsed tokens)."""
    pooled, plen = pool(h, blank, lengths, prep["window"], mode=mode)
    res = []
    for pb in pooled:
        lg = head_logits(pb, prep, mode=mode)
        ids = np.argmax(np.asarray(lg), axis=-1).astype(np.int32)
        res.append((ids, lg, collapse(ids, prep["blank_id"])))
    return res, plen
