"""The encoder's CTC heads on the B200 (``granite::ctc_selfcond``, ``granite::bpe_ctc_decode``): self-conditioning,
posterior-weighted pooling, the BPE head with its argmax fused into the GEMM epilogue, and the CTC collapse, against
the reference encoder's golden and the oracle."""
import os

import numpy as np
import pytest
import torch

from granite_conv_b200 import _lib, ops, synth
from granite_conv_b200.weights import prepare_bpe_head_from_tensors, prepare_selfcond_from_tensors
from oracle import conv_module as O
from oracle import ctc_head as CH
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def _t(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).to(DEV)


def _heads(p):
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    sc = prepare_selfcond_from_tensors(bf(p.out_weight), bf(p.out_bias), bf(p.mid_weight), bf(p.mid_bias), device=DEV)
    hd = prepare_bpe_head_from_tensors(bf(p.bpe_weight), bf(p.bpe_bias), p.blank_id, p.window, device=DEV)
    return sc, hd


def _tie_or_equal(logits_ref, ids_out, ids_ref):
    top2 = np.sort(logits_ref, axis=-1)[:, -2:]
    tie = (top2[:, 1] - top2[:, 0]) <= np.maximum(np.abs(top2[:, 1]), 1e-30) * 2.0 ** -7
    return (ids_out == ids_ref) | tie


@pytest.mark.parametrize("tag", ["whole", "trimmed"])
def test_ctc_heads_vs_reference_golden(tag):
    g = np.load(os.path.join(GOLDEN, "ctc_heads_b2_t37_v2048.npz"))
    p = synth.make_ctc_params(1401, vocab=2048, blank_id=7)
    sc, hd = _heads(p)
    x = O.bf16_round(synth.make_activations(1901, (2, 37, synth.D_MODEL)))
    lens = None if tag == "whole" else torch.from_numpy(g["lengths"]).to(DEV)
    h, blank = ops.run_ctc_selfcond(_t(x), sc, lens)
    L = [37, 37] if lens is None else list(g["lengths"])
    hn = h.float().cpu().numpy()
    assert_bf16_close(np.concatenate([hn[b, :n] for b, n in enumerate(L)]), O.from_bf16_bits(g[f"{tag}_hidden"]),
                      f"selfcond {tag}")
    ids, tokens, counts = ops.run_bpe_ctc_decode(h, blank, hd, lens)
    ids, tokens, counts = ids.cpu().numpy(), tokens.cpu().numpy(), counts.cpu().numpy()
    seg = g[f"{tag}_segments"]
    got = np.concatenate([ids[b, :n] for b, n in enumerate(seg)])
    assert (ids[0, seg[0]:] == -1).all() and (ids[1, seg[1]:] == -1).all()
    ok = _tie_or_equal(O.from_bf16_bits(g[f"{tag}_logits"]), got, g[f"{tag}_ids"])
    assert ok.all(), f"argmax differs away from a near-tie: {got} vs {g[f'{tag}_ids']}"
    if (got == g[f"{tag}_ids"]).all():
        np.testing.assert_array_equal(counts, g[f"{tag}_counts"])
        np.testing.assert_array_equal(np.concatenate([tokens[b, :c] for b, c in enumerate(counts)]),
                                      g[f"{tag}_tokens"])


@pytest.mark.parametrize("B,T,V", [(3, 640, 4096), (2, 128, synth.BPE_VOCAB)])
def test_ctc_heads_vs_oracle(B, T, V):
    p = synth.make_ctc_params(1500 + T, vocab=V, blank_id=min(V - 1, synth.BPE_BLANK))
    sc, hd = _heads(p)
    x = O.bf16_round(synth.make_activations(1501 + T, (B, T, synth.D_MODEL)))
    lens = np.maximum(1, (np.arange(B) * 97 + T // 2) % (T + 1)).astype(np.int32)
    lens[0] = T
    ld = torch.from_numpy(lens).to(DEV)
    h, blank = ops.run_ctc_selfcond(_t(x), sc, ld)
    prep = CH.prepare_ctc_bf16(p)
    h_ref, blank_ref = CH.selfcond(x, prep, lengths=lens)
    hn, bn = h.float().cpu().numpy(), blank.cpu().numpy()
    for b, L in enumerate(lens):
        assert_bf16_close(hn[b, :L], h_ref[b, :L], f"selfcond b={b}")
        np.testing.assert_allclose(bn[b, :L], blank_ref[b, :L], atol=2e-3, rtol=2e-2)
        assert (bn[b, L:] == 1.0).all()
    # the head on the GPU's own hidden state and blank probabilities, checked against the oracle's head on them
    ids, tokens, counts = ops.run_bpe_ctc_decode(h, blank, hd, ld)
    ids, tokens, counts = ids.cpu().numpy(), tokens.cpu().numpy(), counts.cpu().numpy()
    res, plen = CH.decode(hn, bn, prep, lengths=lens)
    for b in range(B):
        ref_ids, ref_lg, ref_tok = res[b]
        n = int(plen[b])
        assert (ids[b, n:] == -1).all()
        ok = _tie_or_equal(np.asarray(ref_lg), ids[b, :n], ref_ids)
        assert ok.mean() == 1.0, f"b={b}: {np.flatnonzero(~ok)}"
        if (ids[b, :n] == ref_ids).all():
            np.testing.assert_array_equal(tokens[b, :counts[b]], ref_tok)
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0


def test_argmax_ties_pick_the_lowest_index():
    """Several vocabulary rows give the same (largest) logit: the lowest index wins, as torch.argmax does."""
    B, T, D, V = 1, 16, synth.D_MODEL, 1024
    g = np.random.default_rng(4)
    w = O.bf16_round(g.normal(0, 0.05, (V, D)).astype(np.float32))
    for dup in (900, 300, 301):
        w[dup] = w[517]
    b = np.zeros(V, dtype=np.float32)
    hd = prepare_bpe_head_from_tensors(_t(w), _t(b), blank_id=V - 1, window=4, device=DEV)
    x = O.bf16_round(g.normal(0, 1, (B, T, D)).astype(np.float32))
    x[0] = O.bf16_round(np.tile(w[517], (T, 1)) * 4)      # every frame aligned with row 517 (and its copies)
    blank = torch.zeros((B, T), dtype=torch.float32, device=DEV)
    ids, tokens, counts = ops.run_bpe_ctc_decode(_t(x), blank, hd, None)
    assert (ids.cpu().numpy()[0, :4] == 300).all()          # 300 < 301 < 517 < 900
    assert counts.item() == 1 and tokens[0, 0].item() == 300


def test_ctc_compile_fullgraph():
    p = synth.make_ctc_params(3, vocab=1024, blank_id=5)
    sc, hd = _heads(p)
    x = torch.randn((2, 256, synth.D_MODEL), device=DEV).bfloat16()
    lens = torch.tensor([256, 100], dtype=torch.int32, device=DEV)

    def f(x):
        h, blank = ops.run_ctc_selfcond(x, sc, lens)
        return ops.run_bpe_ctc_decode(h, blank, hd, lens)

    a = torch.compile(f, fullgraph=True)(x)
    b = f(x)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
