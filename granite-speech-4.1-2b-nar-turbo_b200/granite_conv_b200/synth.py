"""Seeded synthetic inputs for the Conformer conv module workloads.

There is no dataset or checkpoint on the build machines, so every workload is generated from a fixed seed with
numpy's PCG64 generator.  The shapes and distributions restate the workload definitions of the conv-module
benchmark:

* depthwise alone: bf16 ``[B=48, T=1024, C=2048]`` channels-last, folded weights ~N(0, 0.05), bias ~N(0, 0.02),
  x ~N(0, 1), every frame valid;
* one module: D=1024, inner 2048 (``EncoderConfig.hidden_dim`` x ``conv_expansion_factor``,
  ``models/granite_speech_nar/config.py:20,30``), depthwise k=15 (``config.py:29``); pointwise weights and biases
  ~N(0, 0.02), depthwise weight ~N(0, 0.02), BatchNorm running mean ~N(0, 0.1), var ~U(0.5, 1.5),
  gamma ~U(0.8, 1.2), beta ~N(0, 0.05), eps 1e-5; LayerNorm affine gamma ~N(1, 0.02), beta ~N(0, 0.02);
* utterance lengths: lognormal with median 600 frames and sigma 0.5, clipped to [64, 1536], the padded length
  rounded up to the 128-frame grid (``script/bench_asr.py:352-356``).

Seeds: workload ``n`` uses ``1000 + n``; layer ``l`` of a stack uses ``base + l``.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

D_MODEL = 1024          # EncoderConfig.hidden_dim
D_INNER = 2048          # hidden_dim * conv_expansion_factor
KERNEL = 15             # EncoderConfig.conv_kernel_size
FRAME_GRID = 128        # bench_asr.py FRAME_GRID used by the record run
EXEC_BATCH = 48         # bench_asr.py EXEC_BATCH used by the record run
LEN_MEDIAN = 600.0
LEN_SIGMA = 0.5
LEN_MIN, LEN_MAX = 64, 1536


@dataclass
class ConvModuleParams:
    """Raw (unfolded) parameters of one ConformerConvModule, named after the reference state_dict keys
    (``models/granite_speech_nar/conformer.py:164-170``).  All arrays are float32."""

    norm_weight: np.ndarray        # (D,)
    norm_bias: np.ndarray          # (D,)
    up_weight: np.ndarray          # (2I, D)   up_conv.weight[:, :, 0]
    up_bias: np.ndarray            # (2I,)
    dw_weight: np.ndarray          # (I, K)    depth_conv.conv.weight[:, 0, :]
    bn_mean: np.ndarray            # (I,)
    bn_var: np.ndarray             # (I,)
    bn_weight: np.ndarray          # (I,)
    bn_bias: np.ndarray            # (I,)
    down_weight: np.ndarray        # (D, I)    down_conv.weight[:, :, 0]
    down_bias: np.ndarray          # (D,)
    bn_eps: float = 1e-5
    ln_eps: float = 1e-5


def make_params(seed: int, d_model: int = D_MODEL, d_inner: int = D_INNER, kernel: int = KERNEL,
                w_std: float = 0.02) -> ConvModuleParams:
    """Random-init parameters of one conv module.  ``w_std`` scales the pointwise and depthwise weights; the
    benchmark value is 0.02, parity tests also use larger values so that the module output is not dwarfed by
    the residual."""
    g = np.random.default_rng(seed)
    f32 = np.float32
    return ConvModuleParams(
        norm_weight=(1.0 + g.normal(0.0, 0.02, d_model)).astype(f32),
        norm_bias=g.normal(0.0, 0.02, d_model).astype(f32),
        up_weight=g.normal(0.0, w_std, (2 * d_inner, d_model)).astype(f32),
        up_bias=g.normal(0.0, 0.02, 2 * d_inner).astype(f32),
        dw_weight=g.normal(0.0, w_std, (d_inner, kernel)).astype(f32),
        bn_mean=g.normal(0.0, 0.1, d_inner).astype(f32),
        bn_var=g.uniform(0.5, 1.5, d_inner).astype(f32),
        bn_weight=g.uniform(0.8, 1.2, d_inner).astype(f32),
        bn_bias=g.normal(0.0, 0.05, d_inner).astype(f32),
        down_weight=g.normal(0.0, w_std, (d_model, d_inner)).astype(f32),
        down_bias=g.normal(0.0, 0.02, d_model).astype(f32),
    )


FF_MULT = 4              # EncoderConfig.feedforward_mult


@dataclass
class FeedForwardParams:
    """Parameters of one ConformerFeedForward (``models/granite_speech_nar/conformer.py:23-40``), named after its
    state_dict keys (pre_norm, up_proj, down_proj).  All arrays are float32."""

    norm_weight: np.ndarray        # (D,)
    norm_bias: np.ndarray          # (D,)
    up_weight: np.ndarray          # (F, D)    up_proj.weight, F = 4 D
    up_bias: np.ndarray            # (F,)
    down_weight: np.ndarray        # (D, F)    down_proj.weight
    down_bias: np.ndarray          # (D,)
    ln_eps: float = 1e-5


def make_ff_params(seed: int, d_model: int = D_MODEL, mult: int = FF_MULT, w_std: float = 0.02) -> FeedForwardParams:
    """Random-init parameters of one feed-forward half, the same distributions as :func:`make_params`."""
    g = np.random.default_rng(seed)
    f32 = np.float32
    d_ff = mult * d_model
    return FeedForwardParams(
        norm_weight=(1.0 + g.normal(0.0, 0.02, d_model)).astype(f32),
        norm_bias=g.normal(0.0, 0.02, d_model).astype(f32),
        up_weight=g.normal(0.0, w_std, (d_ff, d_model)).astype(f32),
        up_bias=g.normal(0.0, 0.02, d_ff).astype(f32),
        down_weight=g.normal(0.0, w_std, (d_model, d_ff)).astype(f32),
        down_bias=g.normal(0.0, 0.02, d_model).astype(f32),
    )


NUM_HEADS = 8            # EncoderConfig.num_heads
DIM_HEAD = 128           # hidden_dim // num_heads
CONTEXT = 200            # EncoderConfig.context_size
MAX_POS_EMB = 512        # EncoderConfig.max_pos_emb


@dataclass
class AttentionParams:
    """Parameters of one ConformerAttention (``models/granite_speech_nar/conformer.py:43-59``), named after its
    state_dict keys (pre_norm, to_q, to_kv, to_out, rel_pos_emb).  All arrays are float32."""

    norm_weight: np.ndarray        # (D,)
    norm_bias: np.ndarray          # (D,)
    q_weight: np.ndarray           # (inner, D)      to_q.weight (no bias)
    kv_weight: np.ndarray          # (2 inner, D)    to_kv.weight (no bias): k rows, then v rows
    out_weight: np.ndarray         # (D, inner)      to_out.weight
    out_bias: np.ndarray           # (D,)
    rel_pos: np.ndarray            # (2 max_pos + 1, dim_head)   rel_pos_emb.weight
    heads: int = NUM_HEADS
    context: int = CONTEXT
    max_pos: int = MAX_POS_EMB
    ln_eps: float = 1e-5


def make_attn_params(seed: int, d_model: int = D_MODEL, heads: int = NUM_HEADS, w_std: float = 0.02,
                     rel_std: float = 1.0) -> AttentionParams:
    """Random-init parameters of one attention step: projections ~N(0, w_std), the relative-position table
    ~N(0, rel_std) (nn.Embedding's own initialisation is N(0, 1)), LayerNorm as in :func:`make_params`."""
    g = np.random.default_rng(seed)
    f32 = np.float32
    inner = heads * DIM_HEAD
    return AttentionParams(
        norm_weight=(1.0 + g.normal(0.0, 0.02, d_model)).astype(f32),
        norm_bias=g.normal(0.0, 0.02, d_model).astype(f32),
        q_weight=g.normal(0.0, w_std, (inner, d_model)).astype(f32),
        kv_weight=g.normal(0.0, w_std, (2 * inner, d_model)).astype(f32),
        out_weight=g.normal(0.0, w_std, (d_model, inner)).astype(f32),
        out_bias=g.normal(0.0, 0.02, d_model).astype(f32),
        rel_pos=g.normal(0.0, rel_std, (2 * MAX_POS_EMB + 1, DIM_HEAD)).astype(f32),
        heads=heads,
    )


@dataclass
class BlockParams:
    """Parameters of one ConformerBlock (``models/granite_speech_nar/conformer.py:190-199``)."""

    ff1: FeedForwardParams
    attn: AttentionParams
    conv: ConvModuleParams
    ff2: FeedForwardParams
    post_norm_weight: np.ndarray   # (D,)
    post_norm_bias: np.ndarray     # (D,)
    post_ln_eps: float = 1e-5


def make_block_params(seed: int, w_std: float = 0.02) -> BlockParams:
    """Random-init parameters of one Conformer block (each part from its own seed: seed * 10 + part)."""
    g = np.random.default_rng(seed)
    return BlockParams(
        ff1=make_ff_params(seed * 10 + 1, w_std=w_std), attn=make_attn_params(seed * 10 + 2, w_std=w_std),
        conv=make_params(seed * 10 + 3, w_std=w_std), ff2=make_ff_params(seed * 10 + 4, w_std=w_std),
        post_norm_weight=(1.0 + g.normal(0.0, 0.02, D_MODEL)).astype(np.float32),
        post_norm_bias=g.normal(0.0, 0.02, D_MODEL).astype(np.float32))


CTC_CLASSES = 348       # EncoderConfig.output_dim
BPE_VOCAB = 100352      # the BPE head's vocabulary: the LLM vocabulary (config.py:66), blank id 100257 inside it
BPE_BLANK = 100257      # GraniteSpeechNarConfig.blank_token_id (config.py:103)


@dataclass
class CTCHeadParams:
    """The encoder's CTC heads (``models/granite_speech_nar/conformer.py:240-252``): ``out`` (D -> C, the middle
    layer's head), ``out_mid`` (C -> D, its feedback), ``out_bpe`` (D -> V).  All arrays are float32."""

    out_weight: np.ndarray         # (C, D)
    out_bias: np.ndarray           # (C,)
    mid_weight: np.ndarray         # (D, C)
    mid_bias: np.ndarray           # (D,)
    bpe_weight: np.ndarray         # (V, D)
    bpe_bias: np.ndarray           # (V,)
    blank_id: int = BPE_BLANK
    window: int = 4


def make_ctc_params(seed: int, vocab: int = BPE_VOCAB, blank_id: int = BPE_BLANK, n_cls: int = CTC_CLASSES,
                    d_model: int = D_MODEL, w_std: float = 0.02) -> CTCHeadParams:
    """Random-init heads; the blank classes get a positive bias (blank is the most frequent CTC output)."""
    g = np.random.default_rng(seed)
    f32 = np.float32
    out_b = g.normal(0.0, 0.02, n_cls).astype(f32)
    out_b[0] += 1.0
    bpe_b = g.normal(0.0, 0.02, vocab).astype(f32)
    bpe_b[blank_id] += 3.5
    return CTCHeadParams(
        out_weight=g.normal(0.0, w_std * 3, (n_cls, d_model)).astype(f32), out_bias=out_b,
        mid_weight=g.normal(0.0, w_std, (d_model, n_cls)).astype(f32), mid_bias=g.normal(0.0, 0.02, d_model).astype(f32),
        bpe_weight=g.normal(0.0, w_std * 3, (vocab, d_model)).astype(f32), bpe_bias=bpe_b, blank_id=blank_id)


INPUT_DIM = 160         # EncoderConfig.input_dim


def make_input_params(seed: int, input_dim: int = INPUT_DIM, d_model: int = D_MODEL) -> tuple:
    """The encoder's input projection (``conformer.py:238``): weight ~N(0, 1/sqrt(input_dim)), bias ~N(0, 0.02)."""
    g = np.random.default_rng(seed)
    w = g.normal(0.0, input_dim ** -0.5, (d_model, input_dim)).astype(np.float32)
    return w, g.normal(0.0, 0.02, d_model).astype(np.float32)


def make_activations(seed: int, shape: tuple[int, ...]) -> np.ndarray:
    """x ~ N(0, 1), float32."""
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)


def make_dw_weights(seed: int, channels: int = D_INNER, kernel: int = KERNEL) -> tuple[np.ndarray, np.ndarray]:
    """Folded depthwise weight (C, K) ~N(0, 0.05) and bias (C,) ~N(0, 0.02) of the depthwise-alone workload."""
    g = np.random.default_rng(seed)
    w = g.normal(0.0, 0.05, (channels, kernel)).astype(np.float32)
    b = g.normal(0.0, 0.02, channels).astype(np.float32)
    return w, b


def sample_lengths(seed: int, n: int) -> np.ndarray:
    """Utterance lengths in encoder frames: round(exp(N(ln 600, 0.5))) clipped to [64, 1536]."""
    g = np.random.default_rng(seed)
    lens = np.rint(np.exp(g.normal(np.log(LEN_MEDIAN), LEN_SIGMA, n)))
    return np.clip(lens, LEN_MIN, LEN_MAX).astype(np.int32)


def round_up(v: int, grid: int) -> int:
    return ((int(v) + grid - 1) // grid) * grid
