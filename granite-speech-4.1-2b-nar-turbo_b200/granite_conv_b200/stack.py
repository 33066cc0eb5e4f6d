"""A stack of Conformer conv modules (the encoder's 16 layers, ``models/granite_speech_nar/config.py:19``) run on
execution chunks, each layer followed by its residual add (``conformer.py:207``).  Only the conv modules are
stacked; the attention and feed-forward halves of each block are outside this package."""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import ops
from .weights import PreparedConvModule


class ConvModuleStack:
    def __init__(self, layers: Sequence[PreparedConvModule], int8: bool = False):
        if not layers:
            raise ValueError("empty stack")
        if int8 and not all(p.has_int8 for p in layers):
            raise ValueError("int8 stack needs weights prepared with int8=True")
        self.layers = list(layers)
        self.int8 = int8

    @property
    def d_model(self) -> int:
        return self.layers[0].d_model

    def __call__(self, x: torch.Tensor, lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x: bf16 [B, T, D] on the GPU; lengths: int32 [B] on the GPU or None.  Returns bf16 [B, T, D]."""
        for p in self.layers:
            x = ops.run_conv_module(x, p, lengths=lengths, add_residual=True, int8=self.int8)
        return x
