"""CPU oracle for the Conformer conv module (test infrastructure only).

This file is the checker: only the tests, the smoke check and the benchmark's CPU-baseline leg import it.  The
product path never calls it.

It restates, in numpy, the reference's eager algorithm for the path:

* ``ConformerConvModule.forward`` (``script/models/granite_speech_nar/conformer.py:175-189``): LayerNorm (``:164``),
  ``up_conv`` 1x1 Conv1d D->4D with bias (``:165``, ``:177``), ``GLU(dim=1)`` with value = first half and gate =
  second half (``:166``, ``:181``), depthwise Conv1d k=15 with symmetric zero padding 7 (``:134-155``),
  BatchNorm1d (``:169``) and SiLU (``:168``, ``:186``), ``down_conv`` 1x1 Conv1d 2D->D with bias (``:170``, ``:187``);
* the residual add of ``ConformerBlock.forward`` (``conformer.py:207``);
* the eval-mode BatchNorm fold (``script/models/granite_speech_nar/fold_bn.py:51-64``): fp32 ``scale = gamma *
  rsqrt(var + eps)``, ``W' = W * scale``, ``b' = beta - mean * scale``, cast to the weight dtype;
* the fused depthwise op ``dwconv1d_silu_bf16`` (``script/cuda_kernels/conv1d.py:21-42``):
  ``y = silu(bias + sum_j w[c, j] * x[t - 7 + j])`` with zeros outside [0, T), and its GLU variant
  (``conv1d.py:52-79``) which rounds ``a * sigmoid(g)`` to bf16 before the convolution.

Rounding modes for the bf16 module:

* ``"fused"`` rounds to bf16 where the B200 kernels do: LayerNorm output, GLU output, depthwise+SiLU output and
  the final sum (GEMM epilogues keep fp32 until the store).
* ``"reference"`` rounds at every point where the reference's eager bf16 module materialises a bf16 tensor:
  LayerNorm, up_conv, GLU, depthwise conv (+bias), SiLU, down_conv, residual sum.

Length masking (no counterpart in the reference module, which never reads ``attention_mask``): GLU rows with
``t >= len_b`` are zero before the depthwise conv and depthwise+SiLU rows with ``t >= len_b`` are zero, so the
valid rows equal the reference module run on the utterance trimmed to ``len_b`` frames; the padded rows of the
output are ``x + b2``.

Arithmetic is float64 unless a caller asks for float32 (the CPU baseline times the float32 form).
"""
from __future__ import annotations

import numpy as np

K_DW = 15
PAD_DW = K_DW // 2


# --------------------------------------------------------------------------------------------------------------
# bf16 helpers
def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); returns float32 holding bf16 values."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    r = (u + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)
    out = r.view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) of float32 values after round-to-nearest-even."""
    return (bf16_round(a).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << np.uint32(16)).view(np.float32)


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _silu(x):
    return x * _sigmoid(x)


# --------------------------------------------------------------------------------------------------------------
# pieces
def fold_bn(dw_weight, bn_weight, bn_bias, bn_mean, bn_var, eps, out_bf16: bool):
    """BatchNorm fold of ``fold_bn.py:51-64``: fp32 math, then a cast to the weight dtype (bf16 or fp32)."""
    f32 = np.float32
    scale = (bn_weight.astype(f32) * (f32(1.0) / np.sqrt(bn_var.astype(f32) + f32(eps)))).astype(f32)
    w = (dw_weight.astype(f32) * scale[:, None]).astype(f32)
    b = (bn_bias.astype(f32) - bn_mean.astype(f32) * scale).astype(f32)
    if out_bf16:
        return bf16_round(w), bf16_round(b)
    return w, b


def layer_norm(x, weight, bias, eps=1e-5, dtype=np.float64):
    """LayerNorm over the last axis with biased variance (``nn.LayerNorm``)."""
    xf = x.astype(dtype)
    mean = xf.mean(axis=-1, keepdims=True)
    var = ((xf - mean) ** 2).mean(axis=-1, keepdims=True)
    return (xf - mean) / np.sqrt(var + dtype(eps)) * weight.astype(dtype) + bias.astype(dtype)


def pointwise(x, weight, bias, dtype=np.float64):
    """1x1 Conv1d on channels-last rows: ``x @ W^T + b``."""
    return x.astype(dtype) @ weight.astype(dtype).T + bias.astype(dtype)


def glu(h, dtype=np.float64):
    """``nn.GLU(dim=channel)``: value = first half of the channels, gate = second half."""
    half = h.shape[-1] // 2
    a = h[..., :half].astype(dtype)
    g = h[..., half:].astype(dtype)
    return a * _sigmoid(g)


def depthwise(x, weight, bias, dtype=np.float64):
    """Depthwise k=15 conv along T on channels-last ``x (B, T, C)``, zero padding 7 on both sides, plus bias.
    ``weight`` is (C, K)."""
    B, T, C = x.shape
    K = weight.shape[1]
    pad = K // 2
    xp = np.zeros((B, T + 2 * pad, C), dtype=dtype)
    xp[:, pad:pad + T] = x
    w = weight.astype(dtype)
    acc = np.broadcast_to(bias.astype(dtype), (B, T, C)).copy()
    for j in range(K):
        acc += w[:, j] * xp[:, j:j + T]
    return acc


def _row_mask(B, T, lengths):
    if lengths is None:
        return None
    t = np.arange(T)[None, :]
    return t < np.asarray(lengths)[:, None]            # (B, T) True = valid


# --------------------------------------------------------------------------------------------------------------
# the reference's fused depthwise ops (``granite::dwconv_silu`` / ``granite::dwconv_silu_glu``)
def dwconv_silu(x_btc, weight_ck, bias, lengths=None, round_out=True):
    """``dwconv1d_silu_bf16`` semantics on channels-last input: fp32-or-better accumulate, SiLU, one bf16 round.
    With ``lengths``, input frames ``t >= len_b`` read as zero and output frames ``t >= len_b`` are zero."""
    B, T, C = x_btc.shape
    x = x_btc.astype(np.float64)
    m = _row_mask(B, T, lengths)
    if m is not None:
        x = x * m[..., None]
    y = _silu(depthwise(x, weight_ck, bias))
    if m is not None:
        y = y * m[..., None]
    return bf16_round(y.astype(np.float32)) if round_out else y


def dwconv_silu_glu(x2_btc, weight_ck, bias, lengths=None, round_out=True):
    """``dwconv1d_silu_glu_bf16`` semantics: GLU of the 2C input channels, rounded to bf16, then the fused
    depthwise conv + bias + SiLU."""
    g = bf16_round(glu(x2_btc).astype(np.float32))
    return dwconv_silu(g, weight_ck, bias, lengths=lengths, round_out=round_out)


# --------------------------------------------------------------------------------------------------------------
# whole module
def prepare_bf16(p):
    """bf16 module parameters: every parameter and BatchNorm buffer cast to bf16 (a bf16 model load), then the
    depthwise fold computed in fp32 from those bf16 values and cast back (``fold_bn.py:51-64``)."""
    r = bf16_round
    dw_w, dw_b = fold_bn(r(p.dw_weight), r(p.bn_weight), r(p.bn_bias), r(p.bn_mean), r(p.bn_var), p.bn_eps,
                         out_bf16=True)
    return dict(ln_w=r(p.norm_weight), ln_b=r(p.norm_bias), w1=r(p.up_weight), b1=r(p.up_bias),
                dw_w=dw_w, dw_b=dw_b, w2=r(p.down_weight), b2=r(p.down_bias), ln_eps=p.ln_eps)


def prepare_fp32(p):
    dw_w, dw_b = fold_bn(p.dw_weight, p.bn_weight, p.bn_bias, p.bn_mean, p.bn_var, p.bn_eps, out_bf16=False)
    return dict(ln_w=p.norm_weight, ln_b=p.norm_bias, w1=p.up_weight, b1=p.up_bias, dw_w=dw_w, dw_b=dw_b,
                w2=p.down_weight, b2=p.down_bias, ln_eps=p.ln_eps)


def quantize_per_channel(w):
    """Symmetric per-output-channel int8: ``s = absmax / 127``, ``q = round(w / s)`` clipped to [-127, 127].
    Returns (q int8, s float32)."""
    w = w.astype(np.float32)
    s = (np.abs(w).max(axis=1) / np.float32(127.0)).astype(np.float32)
    s = np.where(s == 0, np.float32(1.0), s).astype(np.float32)
    q = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s


def conv_module(x, prep, lengths=None, mode="fused", residual=True, dtype=np.float64):
    """The conv module plus the block's residual add on channels-last ``x (B, T, D)``.

    ``mode``: "fused" / "reference" (bf16 rounding points, see the module docstring) or "fp32" (no rounding).
    ``prep``: from :func:`prepare_bf16` / :func:`prepare_fp32`; ``w1``/``w2`` may be dequantised int8 weights.
    """
    B, T, D = x.shape
    rnd = (lambda a: bf16_round(np.asarray(a, dtype=np.float32))) if mode in ("fused", "reference") else (lambda a: a)
    ref_only = (lambda a: rnd(a)) if mode == "reference" else (lambda a: a)
    m = _row_mask(B, T, lengths)

    xin = x.astype(np.float32)
    xn = rnd(layer_norm(xin, prep["ln_w"], prep["ln_b"], prep["ln_eps"], dtype=dtype))
    h = ref_only(pointwise(xn.reshape(B * T, D), prep["w1"], prep["b1"], dtype=dtype))
    gl = rnd(glu(h, dtype=dtype)).reshape(B, T, -1)
    if m is not None:
        gl = gl * m[..., None]
    dconv = ref_only(depthwise(gl.astype(dtype), prep["dw_w"], prep["dw_b"], dtype=dtype))
    d = rnd(_silu(np.asarray(dconv, dtype=dtype)))
    if m is not None:
        d = d * m[..., None]
    y = ref_only(pointwise(np.asarray(d, dtype=dtype).reshape(B * T, -1), prep["w2"], prep["b2"], dtype=dtype))
    y = np.asarray(y, dtype=dtype).reshape(B, T, D)
    if residual:
        y = y + xin.astype(dtype)
    return rnd(y) if mode != "fp32" else y.astype(np.float32 if dtype == np.float32 else dtype)


# --------------------------------------------------------------------------------------------------------------
# W8A8: int8 weights and int8 activations (no reference code; torchao's W8A8 dynamic quantisation in
# ``script/bench_asr.py:92-105`` is the nearest analogue and is not vendored)
def quantize_rows(x):
    """Per-row symmetric int8 of activations: ``s = absmax / 127`` and ``q = rint(x / s)`` in fp32 (IEEE division,
    ties to even), clipped to [-127, 127]; ``q = 0`` and ``s = 0`` for an all-zero row.  Returns (q int8, s fp32)."""
    x = np.asarray(x, dtype=np.float32)
    s = (np.abs(x).max(axis=1) / np.float32(127.0)).astype(np.float32)
    safe = np.where(s == 0, np.float32(1.0), s).astype(np.float32)
    q = np.clip(np.rint(x / safe[:, None]), -127, 127)
    q = np.where(s[:, None] == 0, 0, q).astype(np.int8)
    return q, s


def conv_module_w8a8(x, prep, q1, s1, q2, s2, lengths=None, residual=True):
    """The conv module with int8 weights ``q1 [2I, D]``, ``q2 [D, I]`` (per-row scales ``s1``, ``s2``) and int8
    activations: the LayerNorm output and the depthwise output are quantised per row (:func:`quantize_rows`; rows
    of padding frames quantise to zero), each GEMM is an exact integer sum scaled by ``s_row * s_col``.  bf16
    rounding points as the B200 path: LayerNorm out, GLU out, depthwise + SiLU out, final sum."""
    B, T, D = x.shape
    m = _row_mask(B, T, lengths)
    mrow = None if m is None else m.reshape(-1, 1)
    xin = x.astype(np.float32)
    xn = bf16_round(layer_norm(xin, prep["ln_w"], prep["ln_b"], prep["ln_eps"]).astype(np.float32)).reshape(B * T, D)
    if mrow is not None:
        xn = xn * mrow
    qa, sa = quantize_rows(xn)
    acc = qa.astype(np.int64) @ q1.astype(np.int64).T
    h = acc.astype(np.float64) * sa.astype(np.float64)[:, None] * s1.astype(np.float64)[None, :] + prep["b1"]
    gl = bf16_round(glu(h).astype(np.float32)).reshape(B, T, -1)
    if m is not None:
        gl = gl * m[..., None]
    d = bf16_round(_silu(depthwise(gl.astype(np.float64), prep["dw_w"], prep["dw_b"])).astype(np.float32))
    d = d.reshape(B * T, -1)
    if mrow is not None:
        d = d * mrow
    qd, sd = quantize_rows(d)
    acc2 = qd.astype(np.int64) @ q2.astype(np.int64).T
    y = acc2.astype(np.float64) * sd.astype(np.float64)[:, None] * s2.astype(np.float64)[None, :] + prep["b2"]
    y = y.reshape(B, T, D)
    if residual:
        y = y + xin.astype(np.float64)
    return bf16_round(y.astype(np.float32))


# --------------------------------------------------------------------------------------------------------------
# parity metrics (``script/cuda_kernels/bench.py:31-44`` reports max-abs; rel-L2 is the second gate)
def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))
