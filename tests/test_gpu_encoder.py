"""The whole CTC encoder on the B200 ops (``GraniteCTCEncoder``: input projection, Conformer blocks,
self-conditioning, BPE head with the fused argmax, CTC collapse) against the reference's own ``CTCEncoder.forward``
(two blocks), and the input projection's GEMM with K = 160."""
import os

import numpy as np
import pytest
import torch

from granite_conv_b200 import GraniteCTCEncoder, ops, synth
from oracle import conv_module as O
from parity import assert_bf16_close, stats

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


@pytest.mark.parametrize("M,K", [(300, 160), (128, 8), (5, 72)])
def test_linear_with_k_off_the_64_grid(M, K):
    g = torch.Generator(device=DEV).manual_seed(K)
    x = torch.randn((M, K), generator=g, device=DEV).bfloat16()
    w = (torch.randn((1024, K), generator=g, device=DEV) * K ** -0.5).bfloat16()
    b = torch.randn((1024,), generator=g, device=DEV) * 0.1
    y = ops.linear(x, w, b)
    assert_bf16_close(y, (x.float() @ w.float().t() + b).cpu().numpy(), f"linear K={K}")


def _encoder():
    w_in, b_in = synth.make_input_params(1501)
    blocks = [synth.make_block_params(1503 + i, w_std=0.02) for i in range(2)]
    cp = synth.make_ctc_params(1502, vocab=2048, blank_id=7)
    return GraniteCTCEncoder.from_params(w_in, b_in, blocks, cp, selfcond_layer=1, device=DEV)


def _edit_distance(a, b):
    d = np.arange(len(b) + 1)
    for i, x in enumerate(a, 1):
        prev, d[0] = d[0], i
        for j, y in enumerate(b, 1):
            prev, d[j] = d[j], min(d[j] + 1, d[j - 1] + 1, prev + (x != y))
    return int(d[-1])


@pytest.mark.parametrize("tag", ["whole", "trimmed"])
def test_encoder_vs_reference_forward(tag):
    """Hidden state within rel-L2 1e-2 of the reference's bf16 CTCEncoder (two blocks and the self-conditioning chain
    bf16 roundings; the element gate is checked per block elsewhere); BPE argmax ids equal wherever the reference's
    best logit leads by more than 2 %, and at >= 97 % of the pooled frames; transcripts within as many edits as
    there are differing ids."""
    g = np.load(os.path.join(GOLDEN, "encoder_l2_b2_t237_v2048.npz"))
    enc = _encoder()
    feats = O.bf16_round(synth.make_activations(1601, (2, 237, synth.INPUT_DIM)))
    lens = None if tag == "whole" else torch.from_numpy(g["lengths"]).to(DEV)
    out = enc(torch.from_numpy(feats).to(torch.bfloat16).to(DEV), lens)
    L = [237, 237] if lens is None else list(g["lengths"])
    h = out["hidden"].float().cpu().numpy()
    hv = np.concatenate([h[b, :n] for b, n in enumerate(L)])
    s = stats(hv, O.from_bf16_bits(g[f"{tag}_hidden"]))
    assert s["rel_l2"] <= 1e-2, s
    seg = g[f"{tag}_segments"]
    ids = out["ids"].cpu().numpy()
    got = np.concatenate([ids[b, :n] for b, n in enumerate(seg)])
    ref = g[f"{tag}_ids"]
    lg = O.from_bf16_bits(g[f"{tag}_logits"])
    top2 = np.sort(lg, axis=-1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 0.02 * np.abs(top2[:, 1])
    assert (got[clear] == ref[clear]).all()
    assert (got == ref).mean() >= 0.97, (got == ref).mean()
    tokens, counts = out["tokens"].cpu().numpy(), out["counts"].cpu().numpy()
    ref_tok = np.split(g[f"{tag}_tokens"], np.cumsum(g[f"{tag}_counts"])[:-1])
    off = np.concatenate([[0], np.cumsum(seg)])
    for b in range(2):
        n_diff = int((got[off[b]:off[b + 1]] != ref[off[b]:off[b + 1]]).sum())
        assert _edit_distance(list(tokens[b, :counts[b]]), list(ref_tok[b])) <= n_diff
