"""Depthwise k=15 + bias + SiLU kernels (``granite::dwconv_silu`` and ``granite::dwconv_silu_glu``) against the
oracle, the committed reference goldens and, at full size, a torch fp32 convolution on the same device."""
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from granite_conv_b200 import ops, synth  # noqa: F401
from oracle import conv_module as O
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def _bf(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16)


def _dw_params(C, seed=1002):
    w, b = synth.make_dw_weights(seed, channels=C)
    return O.bf16_round(w), O.bf16_round(b)


def _oracle_btc(x_btc, w, b, lengths=None, glu=False):
    f = O.dwconv_silu_glu if glu else O.dwconv_silu
    return f(x_btc, w, b, lengths=lengths)


def test_reference_testfire_golden():
    """(1, 2048, 37) channels-first, as the reference's test-fire and self-test feed it (conv_kernel.py:95,
    conv1d.py:132-138): compare with the fp64 golden and the eager bf16 chain stored from the reference."""
    g = np.load(os.path.join(GOLDEN, "dwconv_silu_b1c2048t37.npz"))
    w, b = _dw_params(2048)
    x = O.bf16_round(synth.make_activations(1502, (1, 2048, 37)))
    y = torch.ops.granite.dwconv_silu(_bf(x).to(DEV), _bf(w)[:, None, :].to(DEV), _bf(b).to(DEV))
    assert y.shape == (1, 2048, 37) and y.is_contiguous()
    assert_bf16_close(y, O.from_bf16_bits(g["golden_fp64"]), "dwconv vs fp64 golden")
    assert_bf16_close(y, O.from_bf16_bits(g["eager"]), "dwconv vs eager bf16")
    x2 = O.bf16_round(synth.make_activations(1602, (1, 4096, 37)))
    y2 = torch.ops.granite.dwconv_silu_glu(_bf(x2).to(DEV), _bf(w)[:, None, :].to(DEV), _bf(b).to(DEV))
    assert y2.shape == (1, 2048, 37)
    assert_bf16_close(y2, O.from_bf16_bits(g["eager_glu"]), "dwconv_glu vs eager bf16")


def test_reference_selftest_stats_t261():
    g = np.load(os.path.join(GOLDEN, "dwconv_silu_stats_c2048t261.npz"))
    w, b = _dw_params(2048)
    x = O.bf16_round(synth.make_activations(1702, (1, 2048, 261)))
    y = torch.ops.granite.dwconv_silu(_bf(x).to(DEV), _bf(w)[:, None, :].to(DEV), _bf(b).to(DEV)).float().cpu()
    ys = y.double().numpy()
    cs, cq = ys.sum(axis=-1).reshape(-1), (ys * ys).sum(axis=-1).reshape(-1)
    assert np.all(np.abs(cs - g["chan_sum"]) <= 0.05 + 1e-3 * np.abs(g["chan_sum"]))
    assert np.all(np.abs(cq - g["chan_sumsq"]) <= 1e-2 + 1e-2 * np.abs(g["chan_sumsq"]))


@pytest.mark.parametrize("B,T", [(1, 1), (2, 5), (2, 37), (3, 64), (2, 65), (1, 200), (2, 261), (1, 843)])
@pytest.mark.parametrize("layout", ["channels_last", "channels_first"])
@pytest.mark.parametrize("glu", [False, True])
def test_dwconv_vs_oracle(B, T, layout, glu):
    C = 256
    w, b = _dw_params(C, seed=77)
    cin = 2 * C if glu else C
    x_btc = O.bf16_round(synth.make_activations(900 + T, (B, T, cin)))
    ref = _oracle_btc(x_btc, w, b, glu=glu)
    xt = _bf(x_btc).to(DEV)                                   # [B, T, Cin]
    xin = xt.transpose(1, 2) if layout == "channels_last" else xt.transpose(1, 2).contiguous()
    op = torch.ops.granite.dwconv_silu_glu if glu else torch.ops.granite.dwconv_silu
    y = op(xin, _bf(w)[:, None, :].to(DEV), _bf(b).to(DEV))
    assert y.shape == (B, C, T)
    if layout == "channels_last":
        assert y.stride() == (T * C, 1, C)
    else:
        assert y.is_contiguous()
    assert_bf16_close(y.transpose(1, 2), ref, f"dw {layout} glu={glu} B={B} T={T}")


@pytest.mark.parametrize("layout", ["channels_last", "channels_first"])
def test_dwconv_lengths(layout):
    C, T = 256, 300
    lengths = np.array([300, 1, 0, 129, 64, 7], dtype=np.int32)
    B = lengths.size
    w, b = _dw_params(C, seed=78)
    x_btc = O.bf16_round(synth.make_activations(4242, (B, T, C)))
    ref = O.dwconv_silu(x_btc, w, b, lengths=lengths)
    xt = _bf(x_btc).to(DEV)
    xin = xt.transpose(1, 2) if layout == "channels_last" else xt.transpose(1, 2).contiguous()
    y = torch.ops.granite.dwconv_silu_masked(xin, _bf(w)[:, None, :].to(DEV), _bf(b).to(DEV),
                                             torch.from_numpy(lengths).to(DEV))
    yb = y.transpose(1, 2).float().cpu().numpy()
    assert_bf16_close(yb, ref, f"masked dw {layout}")
    for i, L in enumerate(lengths):          # padded frames are exactly zero
        assert not np.any(yb[i, L:])
    # valid frames equal the op on the trimmed utterance
    for i, L in enumerate(lengths):
        if L == 0:
            continue
        yi = torch.ops.granite.dwconv_silu(xt[i:i + 1, :L].transpose(1, 2).contiguous(),
                                           _bf(w)[:, None, :].to(DEV), _bf(b).to(DEV))
        np.testing.assert_array_equal(yi.transpose(1, 2)[0].float().cpu().numpy(), yb[i, :L])


@pytest.mark.parametrize("C,T", [(2048, 1024), (192, 261), (64, 37)])
def test_dwconv_tile_shapes_agree(C, T):
    """Without lengths the channels-last kernel runs 64-channel x 64-frame tiles; with lengths (all frames valid here)
    128-channel x 32-frame tiles.  Both accumulate in the same order: equal bit for bit.  C = 192 and 64 reach the
    first shape only (not a multiple of 128 channels); they are checked against the oracle."""
    B = 3
    w, b = _dw_params(C, seed=80)
    x_btc = O.bf16_round(synth.make_activations(6161 + C, (B, T, C)))
    xt = _bf(x_btc).to(DEV)
    wt, bt = _bf(w)[:, None, :].to(DEV), _bf(b).to(DEV)
    y = torch.ops.granite.dwconv_silu(xt.transpose(1, 2), wt, bt)
    assert y.stride() == (T * C, 1, C)
    if C % 128 == 0:
        full = torch.full((B,), T, dtype=torch.int32, device=DEV)
        ym = torch.ops.granite.dwconv_silu_masked(xt.transpose(1, 2), wt, bt, full)
        assert torch.equal(y, ym)
    else:
        assert_bf16_close(y.transpose(1, 2), O.dwconv_silu(x_btc, w, b), f"dw C={C} T={T}")


def test_dwconv_generic_strides_and_odd_channels():
    """C not a multiple of the channels-last tile and a non-dense view take the generic path."""
    C, T, B = 96, 50, 2
    w, b = _dw_params(C, seed=79)
    x_btc = O.bf16_round(synth.make_activations(5151, (B, T, 2 * C)))[:, :, ::2]       # stride-2 channels
    ref = O.dwconv_silu(np.ascontiguousarray(x_btc), w, b)
    xt = torch.from_numpy(O.bf16_round(synth.make_activations(5151, (B, T, 2 * C)))).to(torch.bfloat16).to(DEV)
    xin = xt[:, :, ::2].transpose(1, 2)
    y = torch.ops.granite.dwconv_silu(xin, _bf(w)[:, None, :].to(DEV), _bf(b).to(DEV))
    assert_bf16_close(y.transpose(1, 2), ref, "generic strides")


def test_dwconv_full_size_channels_last():
    """The depthwise-alone workload [48, 1024, 2048] channels-last: torch fp32 conv on the GPU as the reference,
    plus the oracle on two utterances."""
    B, T, C = 48, 1024, 2048
    w, b = synth.make_dw_weights(1002)
    wt = _bf(w).to(DEV)
    bt = _bf(b).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(1002)
    x = torch.randn((B, T, C), generator=g, device=DEV).to(torch.bfloat16)
    y = torch.ops.granite.dwconv_silu(x.transpose(1, 2), wt[:, None, :], bt)
    assert y.stride() == (T * C, 1, C)
    ref = F.silu(F.conv1d(x.transpose(1, 2).float(), wt[:, None, :].float(), bt.float(), padding=7, groups=C))
    for i in range(0, B, 8):
        assert_bf16_close(y[i:i + 8].float(), ref[i:i + 8], f"full-size dw batch {i}")
    for i in (0, B - 1):
        xo = x[i:i + 1].float().cpu().numpy()
        assert_bf16_close(y[i:i + 1].transpose(1, 2), O.dwconv_silu(xo, O.bf16_round(w), O.bf16_round(b)),
                          f"oracle utt {i}")


def test_dwconv_errors():
    w = torch.zeros(8, 1, 14, dtype=torch.bfloat16, device=DEV)
    b = torch.zeros(8, dtype=torch.bfloat16, device=DEV)
    x = torch.zeros(1, 8, 10, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError):
        torch.ops.granite.dwconv_silu(x, w, b)                          # kernel size 14
    with pytest.raises(RuntimeError):
        torch.ops.granite.dwconv_silu(x.float(), w[..., :1].expand(8, 1, 15).contiguous(), b)   # fp32 input
    empty = torch.ops.granite.dwconv_silu(torch.zeros(0, 8, 10, dtype=torch.bfloat16, device=DEV),
                                          torch.zeros(8, 1, 15, dtype=torch.bfloat16, device=DEV), b)
    assert empty.shape == (0, 8, 10)
