"""A whole Conformer block (feed-forward halves, block-local attention, conv module, post norm) on the B200 ops
against the reference block's golden and the block oracle."""
import os

import numpy as np
import pytest
import torch

from granite_conv_b200 import ConformerEncoderStack, _lib, prepare_block_from_params, run_conformer_block, synth
from oracle import block as BK
from oracle import conv_module as O
from parity import assert_bf16_close, stats

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).to(DEV)


def test_block_vs_reference_golden():
    """Against the reference block's bf16 output: rel-L2 <= 5e-3 and 1.5x the element gate.  The block chains four
    bf16 residual steps and a LayerNorm: the reference's own bf16 output is already at 0.88x the element gate (rel-L2
    3.9e-3) from exact arithmetic on the same bf16 weights, so the full gate is applied against that exact form."""
    g = np.load(os.path.join(GOLDEN, "block_b2_t237_w002.npz"))
    params = synth.make_block_params(1301, w_std=0.02)
    p = prepare_block_from_params(params, device=DEV)
    x = O.bf16_round(synth.make_activations(1801, (2, 237, synth.D_MODEL)))
    y = run_conformer_block(_t(x), p)
    lens = g["lengths"]
    yl = run_conformer_block(_t(x), p, torch.from_numpy(lens).to(DEV)).float().cpu().numpy()
    valid = np.concatenate([yl[b, :L] for b, L in enumerate(lens)], axis=0)
    for out, ref, what in ((y, O.from_bf16_bits(g["bf16"]), "whole"), (valid, O.from_bf16_bits(g["trimmed"]), "trimmed")):
        s = stats(out, ref)
        assert s["rel_l2"] <= 5e-3 and s["worst_ratio"] <= 1.5, f"block {what} vs reference: {s}"
    exact = BK.conformer_block(x, BK.prepare_block(params), mode="fp32")
    assert_bf16_close(y, exact, "block vs exact arithmetic on the bf16 weights")
    exact_l = BK.conformer_block(x, BK.prepare_block(params), lengths=lens, mode="fp32")
    for b, L in enumerate(lens):
        assert_bf16_close(yl[b, :L], exact_l[b, :L], f"block trimmed b={b}")
    assert np.isfinite(yl).all()


@pytest.mark.parametrize("B,T", [(3, 256), (2, 640)])
def test_block_vs_oracle_masked(B, T):
    params = synth.make_block_params(900 + T, w_std=0.02)
    p = prepare_block_from_params(params, device=DEV)
    x = O.bf16_round(synth.make_activations(901 + T, (B, T, synth.D_MODEL)))
    lens = np.maximum(1, (np.arange(B) * 157 + T // 3) % (T + 1)).astype(np.int32)
    lens[0] = T
    y = run_conformer_block(_t(x), p, torch.from_numpy(lens).to(DEV)).float().cpu().numpy()
    ref = BK.conformer_block(x, BK.prepare_block(params), lengths=lens, mode="fp32")   # bf16 weights, exact math
    for b, L in enumerate(lens):
        assert_bf16_close(y[b, :L], ref[b, :L], f"block B={B} T={T} b={b}")
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0


def test_encoder_stack_chunks_match_single_calls():
    blocks = [prepare_block_from_params(synth.make_block_params(950 + i), device=DEV) for i in range(2)]
    enc = ConformerEncoderStack(blocks)
    chunks = []
    for i, (B, T) in enumerate([(2, 256), (3, 128)]):
        x = torch.randn((B, T, synth.D_MODEL), device=DEV).bfloat16()
        lens = torch.tensor([T] + [T // 2] * (B - 1), dtype=torch.int32, device=DEV)
        chunks.append((x, lens))
    outs = enc.run_chunks(chunks)
    for (x, lens), y in zip(chunks, outs):
        assert torch.equal(y, enc(x, lens))
