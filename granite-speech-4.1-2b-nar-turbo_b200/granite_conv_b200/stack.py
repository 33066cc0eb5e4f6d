"""A stack of Conformer conv modules (the encoder's 16 layers, ``models/granite_speech_nar/config.py:19``) run on
execution chunks, each layer followed by its residual add (``conformer.py:207``).  Only the conv modules are
stacked; the attention and feed-forward halves of each block are outside this package."""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib, ops
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

    def chained(self, x: torch.Tensor) -> bool:
        """Whether the layers run chained: bf16 weights with the LayerNorm folded in and T % 128 == 0."""
        return (not self.int8 and all(p.has_ln_fold for p in self.layers) and x.dim() == 3
                and x.shape[1] % 128 == 0 and x.shape[2] % 256 == 0)

    def __call__(self, x: torch.Tensor, lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x: bf16 [B, T, D] on the GPU; lengths: int32 [B] on the GPU or None.  Returns bf16 [B, T, D].

        With LayerNorm-folded bf16 weights the layers are chained (gsn_conv_module_lnfold_chain_bf16): every
        layer's down_conv + residual also writes its output rows' statistics, which the next layer's folded
        LayerNorm reads, so only the first layer launches a statistics kernel."""
        if self.chained(x):
            return self._run_chained(x, lengths)
        for p in self.layers:
            x = ops.run_conv_module(x, p, lengths=lengths, add_residual=True, int8=self.int8)
        return x

    def _run_chained(self, x: torch.Tensor, lengths: Optional[torch.Tensor]) -> torch.Tensor:
        if x.dtype != torch.bfloat16 or not x.is_cuda:
            raise RuntimeError("ConvModuleStack: x must be a bf16 CUDA tensor")
        B, T, D = x.shape
        inner = self.layers[0].d_inner
        x = x.contiguous()
        lens = None if lengths is None else lengths.to(device=x.device, dtype=torch.int32).contiguous()
        if B * T == 0:
            return x.clone()
        L = _lib.lib()
        nbytes = int(L.gsn_conv_module_workspace_bytes(B, T, D, inner))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        stats = torch.empty((B * T, D // 256, 2), dtype=torch.float32, device=x.device)   # row partials, reused
        bufs = [torch.empty_like(x), torch.empty_like(x)]
        st = torch.cuda.current_stream(x.device).cuda_stream
        src = x
        for i, p in enumerate(self.layers):
            dst = bufs[i % 2]
            _lib.call("gsn_conv_module_lnfold_chain_bf16", src.data_ptr(), p.w1g_glu.data_ptr(), p.b1g_glu.data_ptr(),
                      p.c1_glu.data_ptr(), p.dw_w.data_ptr(), p.dw_b.data_ptr(), p.w2.data_ptr(), p.b2.data_ptr(),
                      None if lens is None else lens.data_ptr(), 1, dst.data_ptr(), B, T, D, inner, float(p.ln_eps),
                      None if i == 0 else stats.data_ptr(),
                      stats.data_ptr() if i + 1 < len(self.layers) else None, ws.data_ptr(), nbytes, st)
            src = dst
        return src

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
