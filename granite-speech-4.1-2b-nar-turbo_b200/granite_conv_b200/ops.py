"""``torch.library`` custom ops over libgsn_conv.so.

Same names and signatures as the reference's ops (``script/models/granite_speech_nar/conv_kernel.py:41-56``):

* ``granite::dwconv_silu(Tensor x, Tensor weight, Tensor bias) -> Tensor``
* ``granite::dwconv_silu_glu(Tensor x2, Tensor weight, Tensor bias) -> Tensor``

plus the ops of the whole module (new):

* ``granite::dwconv_silu_masked(x, weight, bias, lengths) -> Tensor``  (lengths int32 [B])
* ``granite::conv_module(x, ln_w, ln_b, w1_glu, b1_glu, dw_w, dw_b, w2, b2, lengths?, ln_eps, add_residual)``
* ``granite::conv_module_i8w(x, ln_w, ln_b, w1q_glu, s1_glu, b1_glu, dw_w, dw_b, w2q, s2, b2, lengths?, ln_eps,
  add_residual)``
* ``granite::conv_module_lnfold(x, w1g_glu, b1g_glu, c1_glu, dw_w, dw_b, w2, b2, lengths?, ln_eps, add_residual)``
  (the LayerNorm folded into the up_conv GEMM; T % 128 == 0)
* ``granite::feed_forward_half(x, ln_w, ln_b, w_up, b_up, w_down, b_down, lengths?, ln_eps)`` (x + 0.5 FF(x))
* ``granite::layer_norm(x, weight, bias, eps)`` (the block's post LayerNorm)
* ``granite::attention_block(x, ln_w, ln_b, w_qkv, b_qkv, w_out, b_out, rel, lengths?, heads, context, max_pos,
  ln_eps)`` (x + ConformerAttention(x), block-local with Shaw relative positions)
* ``granite::ctc_selfcond(x, w_out, b_out, w_mid, b_mid, lengths?, n_cls)`` -> (x', blank) (the middle CTC head)
* ``granite::bpe_ctc_decode(x, blank, lengths?, w, b, blank_id, window)`` -> (ids, tokens, counts) (BPE head)
* ``granite::linear(x, w, b)`` (nn.Linear; the encoder's input projection)

All are ``mutates_args=()``, CUDA-only, launch on ``torch.cuda.current_stream()`` (as ``jit.py:180-181``) and
have ``register_fake`` implementations whose strides equal the real outputs', so ``torch.compile(fullgraph=True)``
sees one opaque node per call.  Inputs in (B, C, T) may be channels-first contiguous (the reference layout) or a
channels-last view (``x.transpose(1, 2)`` of a contiguous [B, T, C]); the output keeps the input's layout.
There is no fallback: a CPU tensor or a failed launch raises.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

KERNEL_SIZE = 15


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(name: str, *ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{name}: every tensor must be on a CUDA device (got {t.device}); "
                               "the conv-module kernels have no CPU path")


def _is_channels_last_dense(x: torch.Tensor) -> bool:
    B, C, T = x.shape
    return x.stride(1) == 1 and x.stride(2) == C and (B == 1 or x.stride(0) == C * T)


def _dw_out(x: torch.Tensor, c_out: int) -> torch.Tensor:
    """Output of the depthwise ops: channels-last if the input is a dense channels-last view, else contiguous."""
    B, _, T = x.shape
    if _is_channels_last_dense(x) and x.shape[1] >= 1:
        return torch.empty_strided((B, c_out, T), (T * c_out, 1, c_out), dtype=x.dtype, device=x.device)
    return torch.empty((B, c_out, T), dtype=x.dtype, device=x.device)


def _prep_dw_input(x: torch.Tensor) -> torch.Tensor:
    if _is_channels_last_dense(x) or x.is_contiguous():
        return x
    return x.contiguous()


def _dw_call(name: str, entry: str, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, c_out: int,
             lengths: Optional[torch.Tensor]) -> torch.Tensor:
    _require_cuda(name, x, weight, bias, lengths)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or bias.dtype != torch.bfloat16:
        raise RuntimeError(f"{name}: bf16 tensors required (x {x.dtype}, weight {weight.dtype}, bias {bias.dtype})")
    if weight.shape[-1] != KERNEL_SIZE or weight.numel() != c_out * KERNEL_SIZE:
        raise RuntimeError(f"{name}: weight must be (C, 1, 15), got {tuple(weight.shape)}")
    x = _prep_dw_input(x)
    w = weight.contiguous()
    b = bias.contiguous()
    if lengths is not None:
        lengths = lengths.to(torch.int32).contiguous()
    y = _dw_out(x, c_out)
    B, _, T = x.shape
    _lib.call(entry, x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), B, c_out, T, KERNEL_SIZE,
              x.stride(0), x.stride(1), x.stride(2), y.stride(0), y.stride(1), y.stride(2), _ptr(lengths),
              _stream(x))
    return y


# ---------------------------------------------------------------------------------------------------------------
@torch.library.custom_op("granite::dwconv_silu", mutates_args=(), device_types="cuda")
def dwconv_silu(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """silu(depthwise_conv_k15(x) + bias), x (B, C, T) bf16, weight (C, 1, 15), bias (C,)."""
    return _dw_call("granite::dwconv_silu", "gsn_dwconv_silu_bf16", x, weight, bias, x.shape[1], None)


@dwconv_silu.register_fake
def _(x, weight, bias):
    return _dw_out(x, x.shape[1])


@torch.library.custom_op("granite::dwconv_silu_glu", mutates_args=(), device_types="cuda")
def dwconv_silu_glu(x2: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """silu(depthwise_conv_k15(glu(x2, dim=1)) + bias), x2 (B, 2C, T) -> (B, C, T)."""
    return _dw_call("granite::dwconv_silu_glu", "gsn_dwconv_silu_glu_bf16", x2, weight, bias, x2.shape[1] // 2,
                    None)


@dwconv_silu_glu.register_fake
def _(x2, weight, bias):
    return _dw_out(x2, x2.shape[1] // 2)


@torch.library.custom_op("granite::dwconv_silu_masked", mutates_args=(), device_types="cuda")
def dwconv_silu_masked(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                       lengths: torch.Tensor) -> torch.Tensor:
    """dwconv_silu with per-utterance lengths: frames t >= lengths[b] read as zero and are written as zero."""
    return _dw_call("granite::dwconv_silu_masked", "gsn_dwconv_silu_bf16", x, weight, bias, x.shape[1], lengths)


@dwconv_silu_masked.register_fake
def _(x, weight, bias, lengths):
    return _dw_out(x, x.shape[1])


# ---------------------------------------------------------------------------------------------------------------
def _module_common(name: str, x: torch.Tensor, ln_w: torch.Tensor, dw_w: torch.Tensor,
                   lengths: Optional[torch.Tensor], size_fn: str = "gsn_conv_module_workspace_bytes"):
    if x.dim() != 3 or x.dtype != torch.bfloat16:
        raise RuntimeError(f"{name}: x must be bf16 [B, T, D], got {x.dtype} {tuple(x.shape)}")
    B, T, D = x.shape
    if ln_w.shape[0] != D:
        raise RuntimeError(f"{name}: LayerNorm width {ln_w.shape[0]} != D {D}")
    inner = dw_w.shape[0]
    xc = x.contiguous()
    lens = None if lengths is None else lengths.to(device=x.device, dtype=torch.int32).contiguous()
    out = torch.empty_like(xc)
    nbytes = int(getattr(_lib.lib(), size_fn)(B, T, D, inner)) if B * T > 0 else 0
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    return xc, lens, out, ws, nbytes, B, T, D, inner


@torch.library.custom_op("granite::conv_module", mutates_args=(), device_types="cuda")
def conv_module(x: torch.Tensor, ln_w: torch.Tensor, ln_b: torch.Tensor, w1_glu: torch.Tensor,
                b1_glu: torch.Tensor, dw_w: torch.Tensor, dw_b: torch.Tensor, w2: torch.Tensor, b2: torch.Tensor,
                lengths: Optional[torch.Tensor], ln_eps: float, add_residual: bool) -> torch.Tensor:
    """ConformerConvModule.forward (+ the block's residual add when add_residual) on bf16 x [B, T, D]."""
    name = "granite::conv_module"
    _require_cuda(name, x, ln_w, ln_b, w1_glu, b1_glu, dw_w, dw_b, w2, b2, lengths)
    xc, lens, out, ws, nbytes, B, T, D, inner = _module_common(name, x, ln_w, dw_w, lengths)
    _lib.call("gsn_conv_module_bf16", xc.data_ptr(), ln_w.data_ptr(), ln_b.data_ptr(), w1_glu.data_ptr(),
              b1_glu.data_ptr(), dw_w.data_ptr(), dw_b.data_ptr(), w2.data_ptr(), b2.data_ptr(), _ptr(lens),
              1 if add_residual else 0, out.data_ptr(), B, T, D, inner, float(ln_eps), ws.data_ptr(), nbytes,
              _stream(xc))
    return out


@conv_module.register_fake
def _(x, ln_w, ln_b, w1_glu, b1_glu, dw_w, dw_b, w2, b2, lengths, ln_eps, add_residual):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("granite::conv_module_lnfold", mutates_args=(), device_types="cuda")
def conv_module_lnfold(x: torch.Tensor, w1g_glu: torch.Tensor, b1g_glu: torch.Tensor, c1_glu: torch.Tensor,
                       dw_w: torch.Tensor, dw_b: torch.Tensor, w2: torch.Tensor, b2: torch.Tensor,
                       lengths: Optional[torch.Tensor], ln_eps: float, add_residual: bool) -> torch.Tensor:
    """conv_module with the LayerNorm folded into the up_conv GEMM (weights from ``weights.fold_layernorm_``);
    T % 128 == 0."""
    name = "granite::conv_module_lnfold"
    _require_cuda(name, x, w1g_glu, b1g_glu, c1_glu, dw_w, dw_b, w2, b2, lengths)
    if x.dim() != 3 or x.dtype != torch.bfloat16:
        raise RuntimeError(f"{name}: x must be bf16 [B, T, D], got {x.dtype} {tuple(x.shape)}")
    B, T, D = x.shape
    inner = dw_w.shape[0]
    xc = x.contiguous()
    lens = None if lengths is None else lengths.to(device=x.device, dtype=torch.int32).contiguous()
    out = torch.empty_like(xc)
    nbytes = int(_lib.lib().gsn_conv_module_workspace_bytes(B, T, D, inner)) if B * T > 0 else 0
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    _lib.call("gsn_conv_module_lnfold_bf16", xc.data_ptr(), w1g_glu.data_ptr(), b1g_glu.data_ptr(), c1_glu.data_ptr(),
              dw_w.data_ptr(), dw_b.data_ptr(), w2.data_ptr(), b2.data_ptr(), _ptr(lens), 1 if add_residual else 0,
              out.data_ptr(), B, T, D, inner, float(ln_eps), ws.data_ptr(), nbytes, _stream(xc))
    return out


@conv_module_lnfold.register_fake
def _(x, w1g_glu, b1g_glu, c1_glu, dw_w, dw_b, w2, b2, lengths, ln_eps, add_residual):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("granite::conv_module_i8w", mutates_args=(), device_types="cuda")
def conv_module_i8w(x: torch.Tensor, ln_w: torch.Tensor, ln_b: torch.Tensor, w1q_glu: torch.Tensor,
                    s1_glu: torch.Tensor, b1_glu: torch.Tensor, dw_w: torch.Tensor, dw_b: torch.Tensor,
                    w2q: torch.Tensor, s2: torch.Tensor, b2: torch.Tensor, lengths: Optional[torch.Tensor],
                    ln_eps: float, add_residual: bool) -> torch.Tensor:
    """conv_module with int8 per-output-channel weights on both pointwise GEMMs (bf16 activations, fp32
    accumulate, the scale applied in the epilogue).  ``w1q_glu`` / ``w2q`` are the int8 weights, or their exact
    bf16 copies widened once beforehand (``PreparedConvModule.w1w_glu`` / ``w2w``), which skips the per-call
    widening."""
    name = "granite::conv_module_i8w"
    _require_cuda(name, x, ln_w, ln_b, w1q_glu, s1_glu, b1_glu, dw_w, dw_b, w2q, s2, b2, lengths)
    widened = w1q_glu.dtype == torch.bfloat16
    if widened != (w2q.dtype == torch.bfloat16) or (not widened and (w1q_glu.dtype != torch.int8 or
                                                                      w2q.dtype != torch.int8)):
        raise RuntimeError(f"{name}: weights must be both int8 or both their bf16 copies "
                           f"(got {w1q_glu.dtype}, {w2q.dtype})")
    # workspace with room for both weight matrices widened to bf16 (int8 weights): the GEMMs then run on bf16 tiles
    xc, lens, out, ws, nbytes, B, T, D, inner = _module_common(
        name, x, ln_w, dw_w, lengths,
        "gsn_conv_module_workspace_bytes" if widened else "gsn_conv_module_i8w_workspace_bytes")
    _lib.call("gsn_conv_module_i8w_widened" if widened else "gsn_conv_module_i8w", xc.data_ptr(), ln_w.data_ptr(), ln_b.data_ptr(), w1q_glu.data_ptr(),
              s1_glu.data_ptr(), b1_glu.data_ptr(), dw_w.data_ptr(), dw_b.data_ptr(), w2q.data_ptr(), s2.data_ptr(),
              b2.data_ptr(), _ptr(lens), 1 if add_residual else 0, out.data_ptr(), B, T, D, inner, float(ln_eps),
              ws.data_ptr(), nbytes, _stream(xc))
    return out


@conv_module_i8w.register_fake
def _(x, ln_w, ln_b, w1q_glu, s1_glu, b1_glu, dw_w, dw_b, w2q, s2, b2, lengths, ln_eps, add_residual):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("granite::conv_module_w8a8", mutates_args=(), device_types="cuda")
def conv_module_w8a8(x: torch.Tensor, ln_w: torch.Tensor, ln_b: torch.Tensor, w1q_glu: torch.Tensor,
                     s1_glu: torch.Tensor, b1_glu: torch.Tensor, dw_w: torch.Tensor, dw_b: torch.Tensor,
                     w2q: torch.Tensor, s2: torch.Tensor, b2: torch.Tensor, lengths: Optional[torch.Tensor],
                     ln_eps: float, add_residual: bool) -> torch.Tensor:
    """conv_module with int8 weights and int8 activations: the LayerNorm and depthwise outputs are quantised per
    row (symmetric, absmax / 127) and both pointwise GEMMs run int8 x int8 tensor-core MMAs with s32 accumulation,
    scaled by the row and column scales in the epilogue.  Same weights as ``conv_module_i8w``."""
    name = "granite::conv_module_w8a8"
    _require_cuda(name, x, ln_w, ln_b, w1q_glu, s1_glu, b1_glu, dw_w, dw_b, w2q, s2, b2, lengths)
    xc, lens, out, ws, nbytes, B, T, D, inner = _module_common(name, x, ln_w, dw_w, lengths,
                                                               "gsn_conv_module_w8a8_workspace_bytes")
    _lib.call("gsn_conv_module_w8a8", xc.data_ptr(), ln_w.data_ptr(), ln_b.data_ptr(), w1q_glu.data_ptr(),
              s1_glu.data_ptr(), b1_glu.data_ptr(), dw_w.data_ptr(), dw_b.data_ptr(), w2q.data_ptr(), s2.data_ptr(),
              b2.data_ptr(), _ptr(lens), 1 if add_residual else 0, out.data_ptr(), B, T, D, inner, float(ln_eps),
              ws.data_ptr(), nbytes, _stream(xc))
    return out


@conv_module_w8a8.register_fake
def _(x, ln_w, ln_b, w1q_glu, s1_glu, b1_glu, dw_w, dw_b, w2q, s2, b2, lengths, ln_eps, add_residual):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


# ---------------------------------------------------------------------------------------------------------------
# ---- the rest of the Conformer block: feed-forward halves and the post LayerNorm -------------------------------
@torch.library.custom_op("granite::feed_forward_half", mutates_args=(), device_types="cuda")
def feed_forward_half(x: torch.Tensor, ln_w: torch.Tensor, ln_b: torch.Tensor, w_up: torch.Tensor,
                      b_up: torch.Tensor, w_down: torch.Tensor, b_down: torch.Tensor,
                      lengths: Optional[torch.Tensor], ln_eps: float) -> torch.Tensor:
    """x + 0.5 * ConformerFeedForward(x) (conformer.py:23-40, :205, :208) on bf16 x [B, T, D]."""
    name = "granite::feed_forward_half"
    _require_cuda(name, x, ln_w, ln_b, w_up, b_up, w_down, b_down, lengths)
    if x.dim() != 3 or x.dtype != torch.bfloat16:
        raise RuntimeError(f"{name}: x must be bf16 [B, T, D], got {x.dtype} {tuple(x.shape)}")
    B, T, D = x.shape
    F = w_up.shape[0]
    xc = x.contiguous()
    lens = None if lengths is None else lengths.to(device=x.device, dtype=torch.int32).contiguous()
    out = torch.empty_like(xc)
    nbytes = int(_lib.lib().gsn_ff_half_workspace_bytes(B, T, D, F)) if B * T > 0 else 0
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    _lib.call("gsn_ff_half_bf16", xc.data_ptr(), ln_w.data_ptr(), ln_b.data_ptr(), w_up.data_ptr(), b_up.data_ptr(),
              w_down.data_ptr(), b_down.data_ptr(), _ptr(lens), out.data_ptr(), B, T, D, F, float(ln_eps),
              ws.data_ptr(), nbytes, _stream(xc))
    return out


@feed_forward_half.register_fake
def _(x, ln_w, ln_b, w_up, b_up, w_down, b_down, lengths, ln_eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("granite::layer_norm", mutates_args=(), device_types="cuda")
def layer_norm_op(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    """nn.LayerNorm over the last dim of bf16 x [..., D] (the block's post_norm, conformer.py:199, :209)."""
    _require_cuda("granite::layer_norm", x, weight, bias)
    D = x.shape[-1]
    x2 = x.contiguous().view(-1, D)
    return layernorm(x2, weight, bias, eps).view(x.shape)


@layer_norm_op.register_fake
def _(x, weight, bias, eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


# ---- block-local attention with Shaw relative positions -----------------------------------------------------------
@torch.library.custom_op("granite::attention_block", mutates_args=(), device_types="cuda")
def attention_block(x: torch.Tensor, ln_w: torch.Tensor, ln_b: torch.Tensor, w_qkv: torch.Tensor,
                    b_qkv: torch.Tensor, w_out: torch.Tensor, b_out: torch.Tensor, rel: torch.Tensor,
                    lengths: Optional[torch.Tensor], heads: int, context: int, max_pos: int,
                    ln_eps: float) -> torch.Tensor:
    """x + ConformerAttention(x) (conformer.py:61-131, :206) on bf16 x [B, T, D]."""
    name = "granite::attention_block"
    _require_cuda(name, x, ln_w, ln_b, w_qkv, b_qkv, w_out, b_out, rel, lengths)
    if x.dim() != 3 or x.dtype != torch.bfloat16:
        raise RuntimeError(f"{name}: x must be bf16 [B, T, D], got {x.dtype} {tuple(x.shape)}")
    B, T, D = x.shape
    dh = rel.shape[1]
    xc = x.contiguous()
    lens = None if lengths is None else lengths.to(device=x.device, dtype=torch.int32).contiguous()
    out = torch.empty_like(xc)
    nbytes = int(_lib.lib().gsn_attention_block_workspace_bytes(B, T, D, heads, dh)) if B * T > 0 else 0
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    _lib.call("gsn_attention_block_bf16", xc.data_ptr(), ln_w.data_ptr(), ln_b.data_ptr(), float(ln_eps),
              w_qkv.data_ptr(), b_qkv.data_ptr(), w_out.data_ptr(), b_out.data_ptr(), rel.data_ptr(), rel.shape[0],
              _ptr(lens), out.data_ptr(), B, T, D, heads, dh, context, max_pos, ws.data_ptr(), nbytes, _stream(xc))
    return out


@attention_block.register_fake
def _(x, ln_w, ln_b, w_qkv, b_qkv, w_out, b_out, rel, lengths, heads, context, max_pos, ln_eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


def run_attention_block(x: torch.Tensor, p, lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x + attention(x) with a :class:`~granite_conv_b200.weights.PreparedAttention`."""
    return torch.ops.granite.attention_block(x, p.ln_w, p.ln_b, p.w_qkv, p.b_qkv, p.w_out, p.b_out, p.rel, lengths,
                                             p.heads, p.context, p.max_pos, p.ln_eps)


def attention_core(qkv: torch.Tensor, rel: torch.Tensor, heads: int, lengths: Optional[torch.Tensor] = None,
                   context: int = 200, max_pos: int = 512, scale: Optional[float] = None) -> torch.Tensor:
    """The attention alone: qkv bf16 [B, T, 3 heads dh] (q | k | v) -> ctx bf16 [B, T, heads dh]."""
    _require_cuda("attention_core", qkv, rel, lengths)
    B, T, C = qkv.shape
    dh = rel.shape[1]
    inner = heads * dh
    q = qkv if qkv.stride(-1) == 1 else qkv.contiguous()
    ctx = torch.empty((B, T, inner), dtype=torch.bfloat16, device=qkv.device)
    lens = None if lengths is None else lengths.to(device=qkv.device, dtype=torch.int32).contiguous()
    if q.stride(0) != T * q.stride(1):
        q = q.contiguous()
    _lib.call("gsn_attention_core_bf16", q.data_ptr(), q.stride(1), rel.data_ptr(), rel.shape[0], ctx.data_ptr(),
              inner, _ptr(lens), B, T, heads, dh, context, max_pos, float(dh ** -0.5 if scale is None else scale),
              _stream(q))
    return ctx


# ---- CTC heads: self-conditioning, BPE pooling + head + argmax + collapse --------------------------------------------
@torch.library.custom_op("granite::ctc_selfcond", mutates_args=(), device_types="cuda")
def ctc_selfcond(x: torch.Tensor, w_out: torch.Tensor, b_out: torch.Tensor, w_mid: torch.Tensor,
                 b_mid: torch.Tensor, lengths: Optional[torch.Tensor], n_cls: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The middle layer's self-conditioning (conformer.py:320-324): returns (x + out_mid(softmax(out(x))), blank
    probability fp32 [B, T])."""
    name = "granite::ctc_selfcond"
    _require_cuda(name, x, w_out, b_out, w_mid, b_mid, lengths)
    B, T, D = x.shape
    xc = x.contiguous()
    lens = None if lengths is None else lengths.to(device=x.device, dtype=torch.int32).contiguous()
    out = torch.empty_like(xc)
    blank = torch.empty((B, T), dtype=torch.float32, device=x.device)
    nbytes = int(_lib.lib().gsn_ctc_selfcond_workspace_bytes(B, T, n_cls)) if B * T > 0 else 0
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    _lib.call("gsn_ctc_selfcond_bf16", xc.data_ptr(), w_out.data_ptr(), b_out.data_ptr(), n_cls, w_mid.data_ptr(),
              b_mid.data_ptr(), _ptr(lens), out.data_ptr(), blank.data_ptr(), B, T, D, ws.data_ptr(), nbytes,
              _stream(xc))
    return out, blank


@ctc_selfcond.register_fake
def _(x, w_out, b_out, w_mid, b_mid, lengths, n_cls):
    return torch.empty_like(x, memory_format=torch.contiguous_format), x.new_empty(x.shape[:2], dtype=torch.float32)


def pooled_frames(T: int, window: int = 4) -> int:
    """Rows per utterance of the pooled layout: ceil(T / window) rounded up to the 128-row tile."""
    p = (T + window - 1) // window
    return (p + 127) // 128 * 128


@torch.library.custom_op("granite::bpe_ctc_decode", mutates_args=(), device_types="cuda")
def bpe_ctc_decode(x: torch.Tensor, blank: torch.Tensor, lengths: Optional[torch.Tensor], w: torch.Tensor,
                   b: torch.Tensor, blank_id: int, window: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Posterior-weighted pooling (conformer.py:214-226, :336-341), the BPE head with its argmax (conformer.py:342-355,
    asr.py:123-134, the logits are never stored) and the CTC collapse (asr.py:76-102).  Returns (ids [B, Pp] int32,
    -1 past each utterance's pooled frames; tokens [B, Pp] int32, the first counts[b] valid; counts [B] int32)."""
    name = "granite::bpe_ctc_decode"
    _require_cuda(name, x, blank, lengths, w, b)
    B, T, D = x.shape
    Pp = pooled_frames(T, window)
    xc = x.contiguous()
    lens = None if lengths is None else lengths.to(device=x.device, dtype=torch.int32).contiguous()
    pooled = torch.empty((B, Pp, D), dtype=torch.bfloat16, device=x.device)
    plen = torch.empty((B,), dtype=torch.int32, device=x.device)
    ids = torch.empty((B, Pp), dtype=torch.int32, device=x.device)
    tokens = torch.empty((B, Pp), dtype=torch.int32, device=x.device)
    counts = torch.empty((B,), dtype=torch.int32, device=x.device)
    if B * T == 0:
        return ids, tokens, counts.zero_()
    st = _stream(xc)
    _lib.call("gsn_bpe_pool_bf16", xc.data_ptr(), blank.contiguous().data_ptr(), _ptr(lens), pooled.data_ptr(),
              plen.data_ptr(), B, T, D, Pp, window, st)
    nbytes = int(_lib.lib().gsn_bpe_head_workspace_bytes(B, Pp))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    _lib.call("gsn_bpe_head_ctc_bf16", pooled.data_ptr(), plen.data_ptr(), w.data_ptr(), b.data_ptr(), w.shape[0],
              blank_id, ids.data_ptr(), tokens.data_ptr(), counts.data_ptr(), B, Pp, D, ws.data_ptr(), nbytes, st)
    return ids, tokens, counts


@bpe_ctc_decode.register_fake
def _(x, blank, lengths, w, b, blank_id, window):
    B, T, _ = x.shape
    Pp = pooled_frames(T, window)
    i32 = torch.int32
    return x.new_empty((B, Pp), dtype=i32), x.new_empty((B, Pp), dtype=i32), x.new_empty((B,), dtype=i32)


def run_ctc_selfcond(x: torch.Tensor, p, lengths: Optional[torch.Tensor] = None):
    return torch.ops.granite.ctc_selfcond(x, p.w_out, p.b_out, p.w_mid, p.b_mid, lengths, p.n_cls)


def run_bpe_ctc_decode(x: torch.Tensor, blank: torch.Tensor, head, lengths: Optional[torch.Tensor] = None):
    return torch.ops.granite.bpe_ctc_decode(x, blank, lengths, head.w, head.b, head.blank_id, head.window)


@torch.library.custom_op("granite::linear", mutates_args=(), device_types="cuda")
def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """x W^T + b on bf16 x [..., K] (K % 8 == 0), W bf16 [N, K] (N % 256 == 0), b fp32 [N] (nn.Linear, e.g. the
    encoder's input projection, conformer.py:238, :289)."""
    _require_cuda("granite::linear", x, w, b)
    K = x.shape[-1]
    N = w.shape[0]
    x2 = x.contiguous().view(-1, K)
    out = torch.empty((x2.shape[0], N), dtype=torch.bfloat16, device=x.device)
    _lib.call("gsn_gemm_linear_bf16", x2.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr(), N, x2.shape[0], K, N,
              None, 0, _stream(x2))
    return out.view(*x.shape[:-1], N)


@linear.register_fake
def _(x, w, b):
    return x.new_empty((*x.shape[:-1], w.shape[0]))


def run_feed_forward_half(x: torch.Tensor, p, lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x + 0.5 * FF(x) with a :class:`~granite_conv_b200.weights.PreparedFeedForward`."""
    return torch.ops.granite.feed_forward_half(x, p.ln_w, p.ln_b, p.w_up, p.b_up, p.w_down, p.b_down, lengths,
                                               p.ln_eps)


def run_conv_module(x: torch.Tensor, p, lengths: Optional[torch.Tensor] = None, add_residual: bool = True,
                    int8: bool = False, ln_fold: Optional[bool] = None, w8a8: bool = False) -> torch.Tensor:
    """Call the fused module op with a :class:`~granite_conv_b200.weights.PreparedConvModule`.  ``ln_fold``: use
    the LayerNorm-folded op (default: when the weights carry the folded operands and T % 128 == 0).  ``w8a8``: the
    int8-weight, int8-activation op (needs weights prepared with int8)."""
    if w8a8:
        if not p.has_int8:
            raise RuntimeError("run_conv_module(w8a8=True): weights were prepared without int8")
        return torch.ops.granite.conv_module_w8a8(x, p.ln_w, p.ln_b, p.w1q_glu, p.s1_glu, p.b1_glu, p.dw_w, p.dw_b,
                                                  p.w2q, p.s2, p.b2, lengths, p.ln_eps, add_residual)
    if ln_fold is None:
        ln_fold = (not int8) and p.has_ln_fold and x.dim() == 3 and x.shape[1] % 128 == 0
    if ln_fold:
        if int8 or not p.has_ln_fold:
            raise RuntimeError("run_conv_module(ln_fold=True): needs bf16 weights prepared with ln_fold=True")
        return torch.ops.granite.conv_module_lnfold(x, p.w1g_glu, p.b1g_glu, p.c1_glu, p.dw_w, p.dw_b, p.w2, p.b2,
                                                    lengths, p.ln_eps, add_residual)
    if int8:
        if not p.has_int8:
            raise RuntimeError("run_conv_module(int8=True): weights were prepared without int8")
        w1, w2 = (p.w1w_glu, p.w2w) if p.w1w_glu is not None else (p.w1q_glu, p.w2q)
        return torch.ops.granite.conv_module_i8w(x, p.ln_w, p.ln_b, w1, p.s1_glu, p.b1_glu, p.dw_w, p.dw_b,
                                                 w2, p.s2, p.b2, lengths, p.ln_eps, add_residual)
    return torch.ops.granite.conv_module(x, p.ln_w, p.ln_b, p.w1_glu, p.b1_glu, p.dw_w, p.dw_b, p.w2, p.b2, lengths,
                                         p.ln_eps, add_residual)


# ---- single-kernel wrappers (tests, benchmarks) ---------------------------------------------------------------
def quant_rows(x2d: torch.Tensor, lengths: Optional[torch.Tensor] = None, T: int = 0):
    """Per-row symmetric int8 quantisation of bf16 rows: returns (q int8 [M, K], scale fp32 [M])."""
    _require_cuda("quant_rows", x2d, lengths)
    if x2d.dtype != torch.bfloat16 or x2d.dim() != 2 or x2d.stride(1) != 1:
        raise RuntimeError("quant_rows: expects a bf16 [M, K] tensor with unit column stride")
    M, K = x2d.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x2d.device)
    sc = torch.empty((M,), dtype=torch.float32, device=x2d.device)
    _lib.call("gsn_quant_rows_bf16", x2d.data_ptr(), x2d.stride(0), q.data_ptr(), sc.data_ptr(), M, K,
              _ptr(lengths), T, _stream(x2d))
    return q, sc

def layernorm(x2d: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-5,
              lengths: Optional[torch.Tensor] = None, T: int = 0) -> torch.Tensor:
    """LayerNorm of bf16 rows [M, D]; with lengths (int32 [M / T]) padding rows are left unwritten."""
    _require_cuda("layernorm", x2d, w, b, lengths)
    M, D = x2d.shape
    y = torch.empty_like(x2d)
    _lib.call("gsn_layernorm_bf16", x2d.data_ptr(), x2d.stride(0), w.data_ptr(), b.data_ptr(), y.data_ptr(),
              y.stride(0), M, D, float(eps), _ptr(lengths), T, _stream(x2d))
    return y


def gemm1_glu(a: torch.Tensor, w_glu: torch.Tensor, b_glu: torch.Tensor, scale_glu: Optional[torch.Tensor] = None,
              lengths: Optional[torch.Tensor] = None, T: int = 0) -> torch.Tensor:
    """h = GLU(a @ W1^T + b1) from GLU-interleaved weights; with lengths, tiles of pure padding are skipped."""
    _require_cuda("gemm1_glu", a, w_glu, b_glu, scale_glu, lengths)
    M, K = a.shape
    N = w_glu.shape[0]
    h = torch.empty((M, N // 2), dtype=torch.bfloat16, device=a.device)
    if scale_glu is None:
        _lib.call("gsn_gemm1_glu_bf16", a.data_ptr(), w_glu.data_ptr(), b_glu.data_ptr(), h.data_ptr(), M, K, N,
                  _ptr(lengths), T, _stream(a))
    else:
        _lib.call("gsn_gemm1_glu_i8w", a.data_ptr(), w_glu.data_ptr(), scale_glu.data_ptr(), b_glu.data_ptr(),
                  h.data_ptr(), M, K, N, _ptr(lengths), T, _stream(a))
    return h


def gemm1_glu_dwconv(a: torch.Tensor, w_glu: torch.Tensor, b_glu: torch.Tensor, dw_w: torch.Tensor,
                     dw_b: torch.Tensor, B: int, T: int, scale_glu: Optional[torch.Tensor] = None,
                     lengths: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """d = silu(depthwise(GLU(a @ W1^T + b1))) in one kernel, a = [B*T, K] frames (T % 128 == 0), bf16 weights
    (scale_glu: int8 weights already widened to bf16).  With lengths, d frames in [len, roundup128(len)) are zero
    and frames past that are left as they were in `out`."""
    _require_cuda("gemm1_glu_dwconv", a, w_glu, b_glu, dw_w, dw_b, scale_glu, lengths)
    M, K = a.shape
    N = w_glu.shape[0]
    d = torch.empty((M, N // 2), dtype=torch.bfloat16, device=a.device) if out is None else out
    _lib.call("gsn_gemm1_glu_dwconv_bf16", a.data_ptr(), w_glu.data_ptr(), _ptr(scale_glu), b_glu.data_ptr(),
              dw_w.data_ptr(), dw_b.data_ptr(), d.data_ptr(), B, T, K, N, _ptr(lengths), _stream(a))
    return d


def layernorm_stats(x2d: torch.Tensor, eps: float = 1e-5, lengths: Optional[torch.Tensor] = None,
                    T: int = 0) -> torch.Tensor:
    """Per-row (rstd, rstd * mean) of bf16 rows [M, D] as fp32 [M, 2]; padding rows (with lengths) unwritten."""
    _require_cuda("layernorm_stats", x2d, lengths)
    M, D = x2d.shape
    st = torch.empty((M, 2), dtype=torch.float32, device=x2d.device)
    _lib.call("gsn_layernorm_stats_bf16", x2d.data_ptr(), x2d.stride(0), st.data_ptr(), M, D, float(eps),
              _ptr(lengths), T, _stream(x2d))
    return st


def gemm2_residual(d: torch.Tensor, w: torch.Tensor, b: torch.Tensor, residual: Optional[torch.Tensor],
                   scale: Optional[torch.Tensor] = None, lengths: Optional[torch.Tensor] = None,
                   T: int = 0) -> torch.Tensor:
    """out = d @ W2^T + b2 (+ residual); with lengths, tiles of pure padding are written as residual + b2."""
    _require_cuda("gemm2_residual", d, w, b, residual, scale, lengths)
    M, K = d.shape
    N = w.shape[0]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=d.device)
    ld_res = residual.stride(0) if residual is not None else 0
    if scale is None:
        _lib.call("gsn_gemm2_residual_bf16", d.data_ptr(), w.data_ptr(), b.data_ptr(), _ptr(residual), ld_res,
                  out.data_ptr(), out.stride(0), M, K, N, _ptr(lengths), T, _stream(d))
    else:
        _lib.call("gsn_gemm2_residual_i8w", d.data_ptr(), w.data_ptr(), scale.data_ptr(), b.data_ptr(),
                  _ptr(residual), ld_res, out.data_ptr(), out.stride(0), M, K, N, _ptr(lengths), T, _stream(d))
    return out
