"""Weight preparation for the B200 conv-module kernels (load time, not the hot path).

* :func:`fold_conv_bn_` is the eval-mode BatchNorm fold of the reference (``fold_bn.py:33-68``): fp32
  ``scale = gamma * rsqrt(var + eps)``, ``W' = W * scale``, ``b' = beta - mean * scale``, cast back to the weight
  dtype, BatchNorm replaced by Identity; idempotent, requires eval mode.  It works on any module tree whose conv
  modules carry the reference attribute names (``depth_conv.conv``, ``batch_norm``).
* :func:`prepare_conv_module` lays the folded weights out for the kernels: up_conv rows interleaved per 256-row
  block as [128 value rows | 128 gate rows] so one GEMM tile holds both GLU halves, biases in fp32, and
  optionally int8 per-output-channel symmetric weights (``s = absmax / 127``) for the int8-weight GEMMs.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
from torch import nn

GLU_BLOCK = 128      # value (or gate) rows per 256-row GEMM tile


def _is_conv_module(m: nn.Module) -> bool:
    return all(hasattr(m, a) for a in ("norm", "up_conv", "depth_conv", "batch_norm", "down_conv"))


@torch.no_grad()
def fold_conv_bn_(model: nn.Module) -> int:
    """In-place fold of BatchNorm1d into the depthwise Conv1d of every conv module; returns how many were
    folded.  Mirrors ``fold_bn.fold_conv_bn_`` (``script/models/granite_speech_nar/fold_bn.py:33-68``)."""
    if model.training:
        raise RuntimeError("fold_conv_bn_: the model is in training mode; switch it with model.eval() so the "
                           "BatchNorm running statistics are what gets folded")
    folded = 0
    for m in model.modules():
        if not _is_conv_module(m) or isinstance(m.batch_norm, nn.Identity):
            continue
        conv = m.depth_conv.conv
        bn = m.batch_norm
        if bn.running_mean is None or bn.running_var is None:
            raise RuntimeError("fold_conv_bn_: this BatchNorm1d keeps no running mean/variance "
                               "(track_running_stats=False), so there is nothing to fold")
        w_dtype = conv.weight.dtype
        scale = bn.weight.detach().float() * torch.rsqrt(bn.running_var.detach().float() + float(bn.eps))
        new_w = conv.weight.detach().float() * scale.reshape(-1, 1, 1)
        new_b = bn.bias.detach().float() - bn.running_mean.detach().float() * scale
        if conv.bias is not None:               # a conv that already had a bias: BN(conv + b) = W'x + b*scale + b'
            new_b = new_b + conv.bias.detach().float() * scale
        conv.weight = nn.Parameter(new_w.to(w_dtype), requires_grad=False)
        conv.bias = nn.Parameter(new_b.to(w_dtype), requires_grad=False)
        m.batch_norm = nn.Identity()
        folded += 1
    return folded


def glu_interleave(t: torch.Tensor, block: int = GLU_BLOCK) -> torch.Tensor:
    """Reorder the 2C rows of an up_conv weight / bias / scale so that every 2*block rows hold ``block`` value
    rows followed by the matching ``block`` gate rows (GLU value = rows [0, C), gate = rows [C, 2C))."""
    rows = t.shape[0]
    if rows % (2 * block):
        raise ValueError(f"{rows} rows is not a multiple of {2 * block}")
    half = rows // 2
    rest = t.shape[1:]
    v = t[:half].reshape(half // block, block, *rest)
    g = t[half:].reshape(half // block, block, *rest)
    return torch.stack((v, g), dim=1).reshape(rows, *rest).contiguous()


def glu_deinterleave(t: torch.Tensor, block: int = GLU_BLOCK) -> torch.Tensor:
    rows = t.shape[0]
    rest = t.shape[1:]
    p = t.reshape(rows // (2 * block), 2, block, *rest)
    return torch.cat((p[:, 0].reshape(rows // 2, *rest), p[:, 1].reshape(rows // 2, *rest)), dim=0).contiguous()


def quantize_per_channel(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-row int8: ``s = absmax / 127`` (1 for an all-zero row), ``q = round(w / s)``."""
    wf = w.detach().float()
    s = wf.abs().amax(dim=1) / 127.0
    s = torch.where(s == 0, torch.ones_like(s), s)
    q = torch.clamp(torch.round(wf / s[:, None]), -127, 127).to(torch.int8)
    return q.contiguous(), s.contiguous()


@dataclass
class PreparedConvModule:
    """Device-resident operands of one conv module in the layouts the kernels take."""

    ln_w: torch.Tensor          # [D] bf16
    ln_b: torch.Tensor          # [D] bf16
    w1_glu: torch.Tensor        # [2I, D] bf16, GLU-interleaved rows
    b1_glu: torch.Tensor        # [2I] fp32, GLU-interleaved
    dw_w: torch.Tensor          # [I, 15] bf16, BN folded
    dw_b: torch.Tensor          # [I] bf16, BN folded
    w2: torch.Tensor            # [D, I] bf16
    b2: torch.Tensor            # [D] fp32
    ln_eps: float = 1e-5
    w1q_glu: Optional[torch.Tensor] = None   # [2I, D] int8, GLU-interleaved
    s1_glu: Optional[torch.Tensor] = None    # [2I] fp32
    w2q: Optional[torch.Tensor] = None       # [D, I] int8
    s2: Optional[torch.Tensor] = None        # [D] fp32
    # the int8 weights widened once to bf16 (exact: |q| <= 127), so the int8-weight module runs its GEMMs on bf16
    # tiles with the column scales without widening the constant weights on every call
    w1w_glu: Optional[torch.Tensor] = None   # [2I, D] bf16 = bf16(w1q_glu)
    w2w: Optional[torch.Tensor] = None       # [D, I] bf16 = bf16(w2q)
    # LayerNorm folded into the up_conv GEMM (gsn_fold_layernorm_bf16): W1 * gamma, b1 + W1 beta, column sums
    w1g_glu: Optional[torch.Tensor] = None   # [2I, D] bf16, GLU-interleaved
    b1g_glu: Optional[torch.Tensor] = None   # [2I] fp32
    c1_glu: Optional[torch.Tensor] = None    # [2I] fp32

    @property
    def d_model(self) -> int:
        return int(self.ln_w.shape[0])

    @property
    def d_inner(self) -> int:
        return int(self.dw_w.shape[0])

    @property
    def has_int8(self) -> bool:
        return self.w1q_glu is not None

    @property
    def has_ln_fold(self) -> bool:
        return self.w1g_glu is not None


@torch.no_grad()
def fold_layernorm_(p: PreparedConvModule) -> PreparedConvModule:
    """Add the LayerNorm-folded up_conv operands (on the GPU, by the library's fold kernel): W' = bf16(W1 * gamma),
    b' = b1 + W1 beta, c = column sums of W'.  Returns ``p``."""
    from . import _lib
    n, k = p.w1_glu.shape
    p.w1g_glu = torch.empty_like(p.w1_glu)
    p.b1g_glu = torch.empty(n, dtype=torch.float32, device=p.w1_glu.device)
    p.c1_glu = torch.empty(n, dtype=torch.float32, device=p.w1_glu.device)
    _lib.call("gsn_fold_layernorm_bf16", p.w1_glu.data_ptr(), p.b1_glu.data_ptr(), p.ln_w.data_ptr(),
              p.ln_b.data_ptr(), p.w1g_glu.data_ptr(), p.b1g_glu.data_ptr(), p.c1_glu.data_ptr(), n, k,
              torch.cuda.current_stream(p.w1_glu.device).cuda_stream)
    return p


@torch.no_grad()
def prepare_from_tensors(ln_w, ln_b, up_w, up_b, dw_w, dw_b, down_w, down_b, ln_eps=1e-5, device="cuda",
                         int8: bool = False, int8_source: Optional[tuple] = None,
                         ln_fold: bool = False) -> PreparedConvModule:
    """Build the kernel operands from folded module tensors (any dtype; up/down weights may keep the trailing
    Conv1d kernel dim of 1).  ``int8_source``, if given, is the (up_w, down_w) pair to quantise (e.g. the fp32
    originals); otherwise the given weights are quantised.  ``ln_fold`` adds the LayerNorm-folded up_conv
    operands (needs a GPU)."""
    bf = torch.bfloat16
    up_w = up_w.reshape(up_w.shape[0], -1)
    down_w = down_w.reshape(down_w.shape[0], -1)
    dw_w = dw_w.reshape(dw_w.shape[0], -1)
    dev = torch.device(device)
    p = PreparedConvModule(
        ln_w=ln_w.to(dev, bf).contiguous(), ln_b=ln_b.to(dev, bf).contiguous(),
        w1_glu=glu_interleave(up_w.to(dev, bf)), b1_glu=glu_interleave(up_b.to(dev, bf).float()),
        dw_w=dw_w.to(dev, bf).contiguous(), dw_b=dw_b.to(dev, bf).contiguous(),
        w2=down_w.to(dev, bf).contiguous(), b2=down_b.to(dev, bf).float().contiguous(),
        ln_eps=float(ln_eps))
    if int8:
        src_up, src_down = int8_source if int8_source is not None else (up_w, down_w)
        q1, s1 = quantize_per_channel(src_up.reshape(src_up.shape[0], -1))
        q2, s2 = quantize_per_channel(src_down.reshape(src_down.shape[0], -1))
        p.w1q_glu = glu_interleave(q1.to(dev))
        p.s1_glu = glu_interleave(s1.to(dev))
        p.w2q = q2.to(dev).contiguous()
        p.s2 = s2.to(dev).contiguous()
        p.w1w_glu = p.w1q_glu.to(bf).contiguous()
        p.w2w = p.w2q.to(bf).contiguous()
    if ln_fold:
        fold_layernorm_(p)
    return p


@torch.no_grad()
def prepare_conv_module(m: nn.Module, device="cuda", int8: bool = False) -> PreparedConvModule:
    """Operands of a (BN-folded) ConformerConvModule with the reference attribute names."""
    if not isinstance(m.batch_norm, nn.Identity):
        raise RuntimeError("prepare_conv_module needs a folded module (call fold_conv_bn_ first)")
    conv = m.depth_conv.conv
    return prepare_from_tensors(m.norm.weight, m.norm.bias, m.up_conv.weight, m.up_conv.bias, conv.weight,
                                conv.bias, m.down_conv.weight, m.down_conv.bias, ln_eps=m.norm.eps, device=device,
                                int8=int8)


def prepare_from_params(params, device="cuda", int8: bool = False, ln_fold: bool = False) -> PreparedConvModule:
    """Operands from unfolded float32 parameters (``synth.ConvModuleParams``) as a bf16 model load would make
    them: every tensor cast to bf16, then the BatchNorm fold in fp32 and a cast back to bf16
    (``fold_bn.py:51-64``).  int8 weights are quantised from the bf16 weights."""
    bf = torch.bfloat16
    t = lambda a: torch.from_numpy(a).to(bf)  # noqa: E731
    scale = t(params.bn_weight).float() * torch.rsqrt(t(params.bn_var).float() + float(params.bn_eps))
    dw_w = (t(params.dw_weight).float() * scale[:, None]).to(bf)
    dw_b = (t(params.bn_bias).float() - t(params.bn_mean).float() * scale).to(bf)
    return prepare_from_tensors(t(params.norm_weight), t(params.norm_bias), t(params.up_weight), t(params.up_bias),
                                dw_w, dw_b, t(params.down_weight), t(params.down_bias), ln_eps=params.ln_eps,
                                device=device, int8=int8, ln_fold=ln_fold)


@dataclass
class PreparedFeedForward:
    """Device operands of one ConformerFeedForward (``models/granite_speech_nar/conformer.py:23-40``)."""

    ln_w: torch.Tensor          # [D] bf16
    ln_b: torch.Tensor          # [D] bf16
    w_up: torch.Tensor          # [F, D] bf16 (up_proj.weight as stored)
    b_up: torch.Tensor          # [F] fp32
    w_down: torch.Tensor        # [D, F] bf16
    b_down: torch.Tensor        # [D] fp32
    ln_eps: float = 1e-5

    @property
    def d_model(self) -> int:
        return int(self.ln_w.shape[0])

    @property
    def d_ff(self) -> int:
        return int(self.w_up.shape[0])


@torch.no_grad()
def prepare_ff_from_tensors(ln_w, ln_b, up_w, up_b, down_w, down_b, ln_eps=1e-5, device="cuda") -> PreparedFeedForward:
    bf = torch.bfloat16
    dev = torch.device(device)
    return PreparedFeedForward(
        ln_w=ln_w.to(dev, bf).contiguous(), ln_b=ln_b.to(dev, bf).contiguous(),
        w_up=up_w.to(dev, bf).contiguous(), b_up=up_b.to(dev, bf).float().contiguous(),
        w_down=down_w.to(dev, bf).contiguous(), b_down=down_b.to(dev, bf).float().contiguous(), ln_eps=float(ln_eps))


@torch.no_grad()
def prepare_feed_forward(m: nn.Module, device="cuda") -> PreparedFeedForward:
    """Operands of a ConformerFeedForward with the reference attribute names (pre_norm, up_proj, down_proj)."""
    return prepare_ff_from_tensors(m.pre_norm.weight, m.pre_norm.bias, m.up_proj.weight, m.up_proj.bias,
                                   m.down_proj.weight, m.down_proj.bias, ln_eps=m.pre_norm.eps, device=device)


def prepare_ff_from_params(params, device="cuda") -> PreparedFeedForward:
    """Operands from float32 parameters (``synth.FeedForwardParams``) as a bf16 model load makes them."""
    t = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    return prepare_ff_from_tensors(t(params.norm_weight), t(params.norm_bias), t(params.up_weight),
                                   t(params.up_bias), t(params.down_weight), t(params.down_bias),
                                   ln_eps=params.ln_eps, device=device)


@dataclass
class PreparedAttention:
    """Device operands of one ConformerAttention (``models/granite_speech_nar/conformer.py:43-131``)."""

    ln_w: torch.Tensor          # [D] bf16
    ln_b: torch.Tensor          # [D] bf16
    w_qkv: torch.Tensor         # [3 inner, D] bf16: to_q.weight rows, then to_kv.weight rows (k, then v)
    b_qkv: torch.Tensor         # [3 inner] fp32 zeros (the projections have no bias)
    w_out: torch.Tensor         # [D, inner] bf16
    b_out: torch.Tensor         # [D] fp32
    rel: torch.Tensor           # [2 max_pos + 1, dim_head] bf16 (rel_pos_emb.weight)
    heads: int = 8
    context: int = 200
    max_pos: int = 512
    ln_eps: float = 1e-5

    @property
    def d_model(self) -> int:
        return int(self.ln_w.shape[0])

    @property
    def dim_head(self) -> int:
        return int(self.rel.shape[1])


@torch.no_grad()
def prepare_attn_from_tensors(ln_w, ln_b, q_w, kv_w, out_w, out_b, rel, heads=8, context=200, max_pos=512,
                              ln_eps=1e-5, device="cuda") -> PreparedAttention:
    bf = torch.bfloat16
    dev = torch.device(device)
    w_qkv = torch.cat([q_w.to(dev, bf), kv_w.to(dev, bf)], dim=0).contiguous()
    return PreparedAttention(
        ln_w=ln_w.to(dev, bf).contiguous(), ln_b=ln_b.to(dev, bf).contiguous(), w_qkv=w_qkv,
        b_qkv=torch.zeros(w_qkv.shape[0], dtype=torch.float32, device=dev), w_out=out_w.to(dev, bf).contiguous(),
        b_out=out_b.to(dev, bf).float().contiguous(), rel=rel.to(dev, bf).contiguous(), heads=int(heads),
        context=int(context), max_pos=int(max_pos), ln_eps=float(ln_eps))


@torch.no_grad()
def prepare_attention(m: nn.Module, device="cuda") -> PreparedAttention:
    """Operands of a ConformerAttention with the reference attribute names (pre_norm, to_q, to_kv, to_out,
    rel_pos_emb, num_heads, context_size, max_pos_emb)."""
    return prepare_attn_from_tensors(m.pre_norm.weight, m.pre_norm.bias, m.to_q.weight, m.to_kv.weight,
                                     m.to_out.weight, m.to_out.bias, m.rel_pos_emb.weight, heads=m.num_heads,
                                     context=m.context_size, max_pos=m.max_pos_emb, ln_eps=m.pre_norm.eps,
                                     device=device)


def prepare_attn_from_params(params, device="cuda") -> PreparedAttention:
    """Operands from float32 parameters (``synth.AttentionParams``) as a bf16 model load makes them."""
    t = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    return prepare_attn_from_tensors(t(params.norm_weight), t(params.norm_bias), t(params.q_weight),
                                     t(params.kv_weight), t(params.out_weight), t(params.out_bias),
                                     t(params.rel_pos), heads=params.heads, context=params.context,
                                     max_pos=params.max_pos, ln_eps=params.ln_eps, device=device)


# ---- CTC heads ------------------------------------------------------------------------------------------------
def _round_up(v: int, g: int) -> int:
    return (v + g - 1) // g * g


@dataclass
class PreparedSelfCond:
    """The middle layer's CTC head and its feedback (``conformer.py:240-241``, ``:320-324``), padded for the GEMMs:
    ``w_out`` [round_up(C, 256), D] (rows >= C zero), ``w_mid`` [D, round_up(C, 64)] (columns >= C zero)."""

    w_out: torch.Tensor         # bf16
    b_out: torch.Tensor         # fp32 [round_up(C, 256)]
    w_mid: torch.Tensor         # bf16
    b_mid: torch.Tensor         # fp32 [D]
    n_cls: int = 348


@dataclass
class PreparedBPEHead:
    """The BPE CTC head ``out_bpe`` (``conformer.py:251-252``, ``:338-355``): ``w`` [round_up(V, 256), D] bf16 (padded
    rows zero, their bias -inf so they never win the argmax), ``b`` fp32."""

    w: torch.Tensor
    b: torch.Tensor
    vocab: int
    blank_id: int
    window: int = 4


@torch.no_grad()
def prepare_selfcond_from_tensors(out_w, out_b, mid_w, mid_b, device="cuda") -> PreparedSelfCond:
    bf = torch.bfloat16
    dev = torch.device(device)
    C, D = out_w.shape
    w_out = torch.zeros((_round_up(C, 256), D), dtype=bf, device=dev)
    w_out[:C] = out_w.to(dev, bf)
    b_out = torch.zeros(_round_up(C, 256), dtype=torch.float32, device=dev)
    b_out[:C] = out_b.to(dev, bf).float()
    w_mid = torch.zeros((D, _round_up(C, 64)), dtype=bf, device=dev)
    w_mid[:, :C] = mid_w.to(dev, bf)
    return PreparedSelfCond(w_out=w_out, b_out=b_out, w_mid=w_mid.contiguous(),
                            b_mid=mid_b.to(dev, bf).float().contiguous(), n_cls=int(C))


@torch.no_grad()
def prepare_bpe_head_from_tensors(w, b, blank_id: int, window: int = 4, device="cuda") -> PreparedBPEHead:
    bf = torch.bfloat16
    dev = torch.device(device)
    V, D = w.shape
    Vp = _round_up(V, 256)
    wp = torch.zeros((Vp, D), dtype=bf, device=dev)
    wp[:V] = w.to(dev, bf)
    bp = torch.full((Vp,), float("-inf"), dtype=torch.float32, device=dev)
    bp[:V] = b.to(dev, bf).float()
    return PreparedBPEHead(w=wp, b=bp, vocab=int(V), blank_id=int(blank_id), window=int(window))


@torch.no_grad()
def prepare_ctc_heads(encoder: nn.Module, device="cuda") -> tuple:
    """(PreparedSelfCond, PreparedBPEHead) from a reference CTCEncoder (attributes out, out_mid, out_bpe, config)."""
    sc = prepare_selfcond_from_tensors(encoder.out.weight, encoder.out.bias, encoder.out_mid.weight,
                                       encoder.out_mid.bias, device=device)
    head = prepare_bpe_head_from_tensors(encoder.out_bpe.weight, encoder.out_bpe.bias,
                                         encoder.config.blank_token_id, encoder.config.bpe_pooling_window,
                                         device=device)
    return sc, head
