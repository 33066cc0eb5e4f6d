"""The Conformer block of the Granite NAR encoder on the B200 ops (``models/granite_speech_nar/conformer.py:190-210``):

    x = 0.5 * ff1(x) + x          granite::feed_forward_half
    x = attn(x) + x               granite::attention_block  (block-local, Shaw relative positions)
    x = conv(x) + x               granite::conv_module_lnfold / conv_module (LayerNorm folded when T % 128 == 0)
    x = 0.5 * ff2(x) + x          granite::feed_forward_half
    x = post_norm(x)              granite::layer_norm

and a stack of such blocks (the encoder's 16 layers, ``config.py:19``).  With ``lengths`` each utterance's valid
frames equal the block run on the utterance alone; padded frames carry finite values (each step writes them as
its residual path plus bias, the post norm normalises them) and are never read by the valid ones.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch
from torch import nn

from . import ops
from .weights import (PreparedAttention, PreparedConvModule, PreparedFeedForward, prepare_attention,
                      prepare_attn_from_params, prepare_conv_module, prepare_feed_forward, prepare_ff_from_params,
                      prepare_from_params, fold_layernorm_)


@dataclass
class PreparedConformerBlock:
    ff1: PreparedFeedForward
    attn: PreparedAttention
    conv: PreparedConvModule
    ff2: PreparedFeedForward
    post_ln_w: torch.Tensor      # [D] bf16
    post_ln_b: torch.Tensor      # [D] bf16
    post_ln_eps: float = 1e-5


@torch.no_grad()
def prepare_conformer_block(block: nn.Module, device="cuda") -> PreparedConformerBlock:
    """Operands of a reference ConformerBlock (attributes ff1, attn, conv, ff2, post_norm) whose conv module's
    BatchNorm is already folded (``fold_conv_bn_``)."""
    conv = prepare_conv_module(block.conv, device=device)
    fold_layernorm_(conv)
    return PreparedConformerBlock(
        ff1=prepare_feed_forward(block.ff1, device=device), attn=prepare_attention(block.attn, device=device),
        conv=conv, ff2=prepare_feed_forward(block.ff2, device=device),
        post_ln_w=block.post_norm.weight.to(device, torch.bfloat16).contiguous(),
        post_ln_b=block.post_norm.bias.to(device, torch.bfloat16).contiguous(), post_ln_eps=block.post_norm.eps)


def prepare_block_from_params(params, device="cuda") -> PreparedConformerBlock:
    """Operands from float32 parameters (``synth.BlockParams``) as a bf16 model load makes them."""
    t = lambda a: torch.from_numpy(a).to(device=device, dtype=torch.bfloat16).contiguous()  # noqa: E731
    return PreparedConformerBlock(
        ff1=prepare_ff_from_params(params.ff1, device=device), attn=prepare_attn_from_params(params.attn, device=device),
        conv=prepare_from_params(params.conv, device=device, ln_fold=True),
        ff2=prepare_ff_from_params(params.ff2, device=device), post_ln_w=t(params.post_norm_weight),
        post_ln_b=t(params.post_norm_bias), post_ln_eps=params.post_ln_eps)


def run_conformer_block(x: torch.Tensor, p: PreparedConformerBlock,
                        lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One block on bf16 x [B, T, D] (GPU); lengths int32 [B] on the GPU or None."""
    x = ops.run_feed_forward_half(x, p.ff1, lengths)
    x = ops.run_attention_block(x, p.attn, lengths)
    x = ops.run_conv_module(x, p.conv, lengths=lengths)
    x = ops.run_feed_forward_half(x, p.ff2, lengths)
    return torch.ops.granite.layer_norm(x, p.post_ln_w, p.post_ln_b, p.post_ln_eps)


class ConformerEncoderStack:
    """Blocks applied in order (``CTCEncoder.forward``'s layer loop, ``conformer.py:317-318``; the input projection
    is outside).  With ``selfcond`` (a PreparedSelfCond) the middle CTC head feeds back after block
    ``selfcond_layer`` (1-based, ``conformer.py:320-324``); ``encode`` then also returns its blank probabilities."""

    def __init__(self, blocks: Sequence[PreparedConformerBlock], selfcond=None, selfcond_layer: Optional[int] = None):
        if not blocks:
            raise ValueError("empty stack")
        self.blocks = list(blocks)
        self.selfcond = selfcond
        self.selfcond_layer = selfcond_layer if selfcond_layer is not None else len(self.blocks) // 2

    def encode(self, x: torch.Tensor, lengths: Optional[torch.Tensor] = None):
        """(hidden, blank probabilities [B, T] fp32 or None)."""
        blank = None
        for i, p in enumerate(self.blocks, start=1):
            x = run_conformer_block(x, p, lengths)
            if self.selfcond is not None and i == self.selfcond_layer:
                x, blank = ops.run_ctc_selfcond(x, self.selfcond, lengths)
        return x, blank

    def __call__(self, x: torch.Tensor, lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.encode(x, lengths)[0]

    def transcribe(self, x: torch.Tensor, head, lengths: Optional[torch.Tensor] = None):
        """Encoder body, self-conditioning and the BPE CTC head: (ids, tokens, counts) as ``bpe_ctc_decode``."""
        if self.selfcond is None:
            raise ValueError("transcribe needs the self-conditioning head (its blank probabilities weight the pooling)")
        h, blank = self.encode(x, lengths)
        return ops.run_bpe_ctc_decode(h, blank, head, lengths)

    def run_chunks(self, chunks: Sequence[Tuple[torch.Tensor, Optional[torch.Tensor]]],
                   streams: Optional[Sequence[torch.cuda.Stream]] = None) -> List[torch.Tensor]:
        """Independent execution chunks through the stack, alternating between streams (two by default), as
        ``ConvModuleStack.run_chunks`` does."""
        from .stack import run_on_streams
        return run_on_streams(self, chunks, streams)
