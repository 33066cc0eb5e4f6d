"""A stack of Conformer conv modules (the encoder's 16 layers, ``models/granite_speech_nar/config.py:19``) run on
execution chunks, each layer followed by its residual add (``conformer.py:207``).  Only the conv modules are
stacked; the attention and feed-forward halves of each block are outside this package."""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

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

    def run_chunks(self, chunks: Sequence[Tuple[torch.Tensor, Optional[torch.Tensor]]],
                   streams: Optional[Sequence[torch.cuda.Stream]] = None) -> List[torch.Tensor]:
        """Independent execution chunks (x, lengths) through the stack, chunk i on streams[i % len(streams)]
        (default: two streams).  The kernels are persistent grids of one CTA per SM, so a chunk's kernels start
        on the SMs another chunk's kernel has already released: the tail of each launch is filled.  Inputs must
        be ready on the current stream; the outputs are ready on it when this returns."""
        return run_on_streams(self, chunks, streams)


def run_on_streams(fn, chunks: Sequence[Tuple[torch.Tensor, Optional[torch.Tensor]]],
                   streams: Optional[Sequence[torch.cuda.Stream]] = None) -> List[torch.Tensor]:
    """fn(x, lengths) on each chunk, chunk i on streams[i % len(streams)] (default: the current stream and one
    more); inputs ready on the current stream, outputs ready on it on return."""
    if not chunks:
        return []
    cur = torch.cuda.current_stream(chunks[0][0].device)
    if streams is None:
        streams = [cur, torch.cuda.Stream(chunks[0][0].device)]
    ready = torch.cuda.Event()
    ready.record(cur)
    outs = []
    for i, (x, lengths) in enumerate(chunks):
        st = streams[i % len(streams)]
        st.wait_event(ready)
        with torch.cuda.stream(st):
            y = fn(x, lengths)
        if st is not cur:
            x.record_stream(st)
            if lengths is not None:
                lengths.record_stream(st)
            y.record_stream(cur)
        outs.append(y)
    for st in streams:
        if st is not cur:
            done = torch.cuda.Event()
            done.record(st)
            cur.wait_event(done)
    return outs
