"""The Granite NAR CTC encoder on the B200 ops (``models/granite_speech_nar/conformer.py:229-361``):

    h = input_linear(features)                                   granite::linear (160 -> 1024)
    for each of the Conformer blocks: h = block(h)               run_conformer_block
        after block `self_conditioning_layer`: h, blank = self-conditioning (granite::ctc_selfcond)
    ids, tokens, counts = BPE head on the pooled h (granite::bpe_ctc_decode), CTC-collapsed per utterance

With ``lengths`` each utterance's result equals the encoder run on that utterance alone (see the ops); without,
every frame of the padded tensor takes part, as in the reference's ``forward`` on a padded batch.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch
from torch import nn

from . import ops
from .block import ConformerEncoderStack, PreparedConformerBlock, prepare_block_from_params, prepare_conformer_block
from .weights import (PreparedBPEHead, PreparedSelfCond, fold_conv_bn_, prepare_bpe_head_from_tensors,
                      prepare_ctc_heads, prepare_selfcond_from_tensors)


class GraniteCTCEncoder:
    def __init__(self, w_in: torch.Tensor, b_in: torch.Tensor, blocks: Sequence[PreparedConformerBlock],
                 selfcond: PreparedSelfCond, head: PreparedBPEHead, selfcond_layer: Optional[int] = None):
        self.w_in = w_in            # [D, input_dim] bf16
        self.b_in = b_in            # [D] fp32
        self.stack = ConformerEncoderStack(blocks, selfcond=selfcond, selfcond_layer=selfcond_layer)
        self.head = head

    @classmethod
    @torch.no_grad()
    def from_reference(cls, encoder: nn.Module, device="cuda") -> "GraniteCTCEncoder":
        """From a reference CTCEncoder in eval mode (its conv modules' BatchNorm is folded in place)."""
        encoder.eval()
        fold_conv_bn_(encoder)
        selfcond, head = prepare_ctc_heads(encoder, device=device)
        blocks = [prepare_conformer_block(b, device=device) for b in encoder.layers]
        w_in = encoder.input_linear.weight.to(device, torch.bfloat16).contiguous()
        b_in = encoder.input_linear.bias.to(device, torch.bfloat16).float().contiguous()
        return cls(w_in, b_in, blocks, selfcond, head, selfcond_layer=encoder.config.self_conditioning_layer)

    @classmethod
    def from_params(cls, input_weight, input_bias, block_params, ctc_params, selfcond_layer=None,
                    device="cuda") -> "GraniteCTCEncoder":
        """From float32 parameters (``synth``) as a bf16 model load makes them."""
        bf = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
        blocks = [prepare_block_from_params(bp, device=device) for bp in block_params]
        cp = ctc_params
        sc = prepare_selfcond_from_tensors(bf(cp.out_weight), bf(cp.out_bias), bf(cp.mid_weight), bf(cp.mid_bias),
                                           device=device)
        head = prepare_bpe_head_from_tensors(bf(cp.bpe_weight), bf(cp.bpe_bias), cp.blank_id, cp.window,
                                             device=device)
        w_in = bf(input_weight).to(device).contiguous()
        b_in = bf(input_bias).to(device).float().contiguous()
        return cls(w_in, b_in, blocks, sc, head, selfcond_layer=selfcond_layer)

    def __call__(self, features: torch.Tensor, lengths: Optional[torch.Tensor] = None) -> dict:
        """features bf16 [B, T, input_dim] on the GPU -> dict(hidden [B, T, D] bf16, blank [B, T] fp32, ids, tokens,
        counts) with ids / tokens int32 [B, Pp] and counts int32 [B] as granite::bpe_ctc_decode returns them."""
        h = ops.linear(features, self.w_in, self.b_in)
        h, blank = self.stack.encode(h, lengths)
        ids, tokens, counts = ops.run_bpe_ctc_decode(h, blank, self.head, lengths)
        return dict(hidden=h, blank=blank, ids=ids, tokens=tokens, counts=counts)
