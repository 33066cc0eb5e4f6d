"""Channels-first depthwise k=15 + bias + SiLU: the (B, C, T) layout with T innermost that ``granite::dwconv_silu``
and ``granite::dwconv_silu_glu`` receive at the reference's call site (``ConformerConvModule.forward``,
``script/models/granite_speech_nar/conformer.py:177-183``, the contiguous output of up_conv).  With T % 8 == 0 and
C % 16 == 0 both forms run on the tensor cores (the staged rows as Hankel A operands against per-channel Toeplitz
tables; in the GLU form converter warps first replace the staged value rows by the bf16 GLU, with the CUDA-core
kernels' arithmetic): the fp32 sums are formed in the tensor core's order, so both are held to the parity gate
against the channels-last kernel, the oracle and a torch fp32 convolution.  Lengths follow the reference's
zero-padding semantics."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from granite_conv_b200 import _lib, ops, synth  # noqa: F401
from oracle import conv_module as O
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _bf(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16)


def _weights(C, seed):
    w, b = synth.make_dw_weights(seed, channels=C)
    return _bf(w)[:, None, :].to(DEV), _bf(b).to(DEV)


def _pair(B, T, C, glu, seed):
    """The same frames as a contiguous (B, Cin, T) tensor and as a channels-last (B, Cin, T) view."""
    cin = 2 * C if glu else C
    g = torch.Generator(device=DEV).manual_seed(seed)
    x_btc = torch.randn((B, T, cin), generator=g, device=DEV).to(torch.bfloat16)
    return x_btc.transpose(1, 2).contiguous(), x_btc.transpose(1, 2)


@pytest.mark.parametrize("C", [48, 64, 256, 2048])
@pytest.mark.parametrize("T", [8, 64, 128, 136, 200, 256, 1024, 1032])
@pytest.mark.parametrize("glu", [False, True])
def test_cf_equals_channels_last(C, T, glu):
    B = 3
    w, b = _weights(C, 300 + C)
    x_cf, x_cl = _pair(B, T, C, glu, 17 * T + C)
    op = torch.ops.granite.dwconv_silu_glu if glu else torch.ops.granite.dwconv_silu
    y_cf = op(x_cf, w, b)
    y_cl = op(x_cl, w, b)
    assert y_cf.is_contiguous() and y_cf.shape == (B, C, T)
    form = "glu " if glu else ""
    s = assert_bf16_close(y_cf, y_cl.contiguous(), f"cf {form}(tensor cores) vs cl C={C} T={T}")
    assert s["rel_l2"] < 2e-3, s


@pytest.mark.parametrize("T", [64, 200, 1024])
@pytest.mark.parametrize("glu", [False, True])
def test_cf_vs_oracle(T, glu):
    B, C = 2, 256
    w, b = synth.make_dw_weights(77, channels=C)
    wb, bb = O.bf16_round(w), O.bf16_round(b)
    cin = 2 * C if glu else C
    x_btc = O.bf16_round(synth.make_activations(5000 + T, (B, T, cin)))
    ref = (O.dwconv_silu_glu if glu else O.dwconv_silu)(x_btc, wb, bb)
    op = torch.ops.granite.dwconv_silu_glu if glu else torch.ops.granite.dwconv_silu
    y = op(_bf(x_btc).to(DEV).transpose(1, 2).contiguous(), _bf(wb)[:, None, :].to(DEV), _bf(bb).to(DEV))
    s = assert_bf16_close(y.transpose(1, 2), ref, f"cf T={T} glu={glu}")
    print(f"cf T={T} glu={glu}: max|d| {s['max_abs']:.3e}, worst/gate {s['worst_ratio']:.3f}, rel-L2 {s['rel_l2']:.2e}")


@pytest.mark.parametrize("T", [128, 304, 1024, 1536, 2048])
@pytest.mark.parametrize("glu", [False, True])
def test_cf_lengths(T, glu):
    """Per-utterance lengths (frames past an utterance read as zero and are written as zero, ragged ends included):
    agreement with the channels-last kernel, padded frames exactly zero, and valid frames equal to the op on the
    trimmed utterance (the reference run on x[b, :, :len])."""
    C = 256
    lengths = np.array([T, 1, 0, T // 2 + 3, 64, 7, T - 9, min(T, 1031)], dtype=np.int32)
    B = lengths.size
    w, b = _weights(C, 91)
    x_cf, x_cl = _pair(B, T, C, glu, 7000 + T)
    lt = torch.from_numpy(lengths).to(DEV)
    if glu:
        # the GLU form has no masked op: mask through the C-ABI directly on both layouts
        y_cf = torch.empty((B, C, T), dtype=torch.bfloat16, device=DEV)
        y_cl = torch.empty_strided((B, C, T), (T * C, 1, C), dtype=torch.bfloat16, device=DEV)
        sp = torch.cuda.current_stream().cuda_stream
        for x, y in ((x_cf, y_cf), (x_cl, y_cl)):
            _lib.call("gsn_dwconv_silu_glu_bf16", x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), B, C, T,
                      15, *x.stride(), *y.stride(), lt.data_ptr(), sp)
    else:
        y_cf = torch.ops.granite.dwconv_silu_masked(x_cf, w, b, lt)
        y_cl = torch.ops.granite.dwconv_silu_masked(x_cl, w, b, lt)
    assert_bf16_close(y_cf, y_cl.contiguous(), f"masked cf {'glu ' if glu else ''}(tensor cores) vs cl T={T}")
    yc = y_cf.float().cpu()
    op = torch.ops.granite.dwconv_silu_glu if glu else torch.ops.granite.dwconv_silu
    for i, L in enumerate(lengths):
        assert not torch.any(yc[i, :, L:]), f"utterance {i}: padding frames not zero"
        if L == 0:
            continue
        # the reference op on the utterance trimmed to its length (zero padding = the same frames); with L % 8 == 0
        # the trimmed run takes the same kernel on the same frames, so the same bits
        yi = op(x_cf[i:i + 1, :, :L].contiguous(), w, b)
        if L % 8 == 0:
            assert torch.equal(yi[0].cpu(), y_cf[i, :, :L].cpu()), f"utterance {i} vs the trimmed run"
        else:
            assert_bf16_close(yi[0].float().cpu(), yc[i, :, :L], f"utterance {i} vs the trimmed run")


@pytest.mark.parametrize("T", [1024, 1028, 1001])
@pytest.mark.parametrize("glu", [False, True])
def test_cf_padded_rows_through_c_abi(T, glu):
    """Row strides larger than T (channel rows padded to 1040 frames, utterances padded by two rows) in and out:
    the kernel takes the strides as given and writes nothing outside the view.  T % 8 != 0 with 16-byte aligned
    strides must not take the tensor-core kernel (it moves whole 8-frame chunks) and must not touch the frames
    between T and the stride."""
    B, C, TP = 2, 128, 1040
    cin = 2 * C if glu else C
    w, b = _weights(C, 92)
    g = torch.Generator(device=DEV).manual_seed(93 + T)
    xbig = torch.randn((B, cin + 2, TP), generator=g, device=DEV).to(torch.bfloat16)
    x = xbig[:, :cin, :T]
    ybig = torch.full((B, C + 2, TP), 7.0, dtype=torch.bfloat16, device=DEV)
    y = ybig[:, :C, :T]
    entry = "gsn_dwconv_silu_glu_bf16" if glu else "gsn_dwconv_silu_bf16"
    _lib.call(entry, x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), B, C, T, 15,
              *x.stride(), *y.stride(), None, torch.cuda.current_stream().cuda_stream)
    op = torch.ops.granite.dwconv_silu_glu if glu else torch.ops.granite.dwconv_silu
    ref = op(x.contiguous(), w, b)
    if T % 8 == 0:
        assert torch.equal(y.contiguous(), ref)      # the same tensor-core kernel on the same frames
    else:
        assert_bf16_close(y.contiguous(), ref, f"padded rows T={T} glu={glu}")
    assert torch.all(ybig[:, :C, T:] == 7.0) and torch.all(ybig[:, C:] == 7.0), "wrote outside the view"


def test_cf_full_size():
    """The reference call site at the depthwise-alone size: (48, 2048, 1024) contiguous, all frames valid, against
    a torch fp32 convolution on the GPU and the channels-last kernel."""
    B, T, C = 48, 1024, 2048
    w, b = _weights(C, 1002)
    x_cf, x_cl = _pair(B, T, C, False, 1002)
    y = torch.ops.granite.dwconv_silu(x_cf, w, b)
    assert_bf16_close(y, torch.ops.granite.dwconv_silu(x_cl, w, b).contiguous(), "full-size cf vs cl")
    for i in range(0, B, 8):
        ref = F.silu(F.conv1d(x_cf[i:i + 8].float(), w.float(), b.float(), padding=7, groups=C))
        assert_bf16_close(y[i:i + 8].float(), ref, f"full-size cf batch {i}")


def test_cf_glu_full_size():
    """dwconv_silu_glu at the reference call site: (48, 4096, 1024) up_conv output -> (48, 2048, 1024), against the
    eager chain silu(conv1d(glu(x))) in fp32 (GLU rounded to bf16 as the reference kernel does) and the
    channels-last kernel."""
    B, T, C = 48, 1024, 2048
    w, b = _weights(C, 1003)
    x_cf, x_cl = _pair(B, T, C, True, 1003)
    y = torch.ops.granite.dwconv_silu_glu(x_cf, w, b)
    assert_bf16_close(y, torch.ops.granite.dwconv_silu_glu(x_cl, w, b).contiguous(), "full-size cf glu vs cl")
    for i in range(0, B, 8):
        xs = x_cf[i:i + 8].float()
        gl = F.glu(xs, dim=1).to(torch.bfloat16).float()
        ref = F.silu(F.conv1d(gl, w.float(), b.float(), padding=7, groups=C))
        assert_bf16_close(y[i:i + 8].float(), ref, f"full-size cf glu batch {i}")
