"""Block-local Shaw attention (``granite::attention_block``, ``gsn_attention_core_bf16``) against the reference
goldens and the oracle."""
import os

import numpy as np
import pytest
import torch

from granite_conv_b200 import _lib, ops, synth
from granite_conv_b200.weights import prepare_attn_from_params
from oracle import attention as AT
from oracle import conv_module as O
from parity import assert_bf16_close, stats

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"
H, DH = synth.NUM_HEADS, synth.DIM_HEAD
INNER = H * DH


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).to(DEV)


def _qkv(seed, B, T, q_std=1.0):
    """q | k | v rows with moderate logits: q, k ~ N(0, q_std^2), v ~ N(0, 1), rounded to bf16."""
    g = np.random.default_rng(seed)
    q = g.normal(0.0, q_std, (B, T, INNER))
    k = g.normal(0.0, q_std, (B, T, INNER))
    v = g.normal(0.0, 1.0, (B, T, INNER))
    return O.bf16_round(np.concatenate([q, k, v], axis=-1).astype(np.float32))


def _rel(seed, std=0.1):
    g = np.random.default_rng(seed)
    return O.bf16_round(g.normal(0.0, std, (2 * synth.MAX_POS_EMB + 1, DH)).astype(np.float32))


def _core_ref(qkv, rel, lens):
    B, T, _ = qkv.shape
    out = np.zeros((B, T, INNER), dtype=np.float32)
    for b in range(B):
        L = int(lens[b])
        if L > 0:
            q, k, v = qkv[b, :L, :INNER], qkv[b, :L, INNER:2 * INNER], qkv[b, :L, 2 * INNER:]
            out[b, :L] = AT.attention_core(q, k, v, rel, H, synth.CONTEXT, synth.MAX_POS_EMB, mode="fp32")
    return out


@pytest.mark.parametrize("B,T,lens", [
    (1, 1, None), (1, 37, None), (2, 99, None), (2, 100, None), (1, 101, None), (2, 200, None), (2, 237, None),
    (3, 300, [300, 150, 101]), (4, 400, [399, 200, 100, 1]), (2, 1536, [1536, 777]), (3, 256, [0, 256, 13]),
])
def test_attention_core_vs_oracle(B, T, lens):
    qkv = _qkv(100 + T + B, B, T, q_std=0.3)
    rel = _rel(7 + T)
    lens_np = np.full(B, T, dtype=np.int32) if lens is None else np.array(lens, dtype=np.int32)
    ctx = ops.attention_core(_t(qkv), _t(rel), H, None if lens is None else torch.from_numpy(lens_np).to(DEV))
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0
    ref = _core_ref(qkv, rel, lens_np)
    got = ctx.float().cpu().numpy()
    for b, L in enumerate(lens_np):
        if L > 0:
            assert_bf16_close(got[b, :L], ref[b, :L], f"attention core B={B} T={T} b={b} L={L}")
        assert not got[b, L:].any(), "frames past the length carry a zero context"


def test_attention_core_peaky_logits():
    """Large logits (softmax close to one-hot) and a large positional table."""
    B, T = 2, 400
    qkv = _qkv(11, B, T, q_std=1.0)
    rel = _rel(12, std=1.0)
    ctx = ops.attention_core(_t(qkv), _t(rel), H)
    ref = _core_ref(qkv, rel, np.full(B, T))
    s = stats(ctx, ref)
    assert s["rel_l2"] <= 1e-2, s


def test_attention_core_skew_pins_each_distance():
    """q, k = 0 and one distance's table row set: each query then sees a bias on exactly one key (i - j = delta),
    so the softmax picks that key's v.  Checks the relative-position skew for every query row and both tiles."""
    B, T = 1, 200
    qkv = np.zeros((B, T, 3 * INNER), dtype=np.float32)
    qkv[..., :INNER] = 1.0                            # q = 1: q . rel[row] = sum(rel[row])
    v = np.random.default_rng(3).normal(0, 1, (T, INNER)).astype(np.float32)
    qkv[0, :, 2 * INNER:] = O.bf16_round(v)
    for delta in (-150, -37, -1, 0, 1, 99, 100, 199):
        rel = np.zeros((2 * synth.MAX_POS_EMB + 1, DH), dtype=np.float32)
        rel[synth.MAX_POS_EMB + delta] = 1.0          # bias sqrt(128) * 128 ** -0.5 * ... large for that distance
        ctx = ops.attention_core(_t(qkv), _t(rel), H).float().cpu().numpy()[0]
        ref = _core_ref(qkv, rel, np.array([T]))[0]
        assert_bf16_close(ctx, ref, f"skew delta={delta}")


@pytest.mark.parametrize("tag,seed,w_std,T", [("w002_t237", 1201, 0.02, 237), ("w006_t37", 1202, 0.06, 37),
                                              ("w006_t237", 1203, 0.06, 237)])
def test_attention_block_vs_reference_golden(tag, seed, w_std, T):
    """x + ConformerAttention(x) against the reference module's bf16 output (whole and trimmed).  At w_std 0.06
    the reference's own bf16 and fp32 outputs differ by 7.4x the element gate (the logits amplify one rounding of
    q), so there the gate is rel-L2 <= 1e-2 and the element gate against the fp32 golden is not applied."""
    g = np.load(os.path.join(GOLDEN, f"attn_b2_{tag}.npz"))
    p = prepare_attn_from_params(synth.make_attn_params(seed, w_std=w_std), device=DEV)
    x = O.bf16_round(synth.make_activations(seed + 500, (2, T, synth.D_MODEL)))
    y = ops.run_attention_block(_t(x), p)
    lens = g["lengths"]
    yl = ops.run_attention_block(_t(x), p, torch.from_numpy(lens).to(DEV)).float().cpu().numpy()
    valid = np.concatenate([yl[b, :L] for b, L in enumerate(lens)], axis=0)
    for out, ref, what in ((y, O.from_bf16_bits(g["bf16"]), "whole"), (valid, O.from_bf16_bits(g["trimmed"]), "trimmed")):
        if w_std <= 0.02:
            assert_bf16_close(out, ref, f"attention block {tag} {what} vs reference")
        else:
            s = stats(out, ref)
            assert s["rel_l2"] <= 1e-2, f"attention block {tag} {what}: {s}"
    bo = O.bf16_round(synth.make_attn_params(seed, w_std=w_std).out_bias)
    for b, L in enumerate(lens):
        np.testing.assert_array_equal(yl[b, L:], O.bf16_round(x[b, L:] + bo))


@pytest.mark.parametrize("B,T,masked", [(2, 256, False), (3, 640, True), (2, 1536, True)])
def test_attention_block_vs_oracle(B, T, masked):
    params = synth.make_attn_params(700 + T, w_std=0.02)
    p = prepare_attn_from_params(params, device=DEV)
    x = O.bf16_round(synth.make_activations(701 + T, (B, T, synth.D_MODEL)))
    lens = None
    if masked:
        lens = np.maximum(1, (np.arange(B) * 211 + T // 3) % (T + 1)).astype(np.int32)
        lens[0] = T
    y = ops.run_attention_block(_t(x), p, None if lens is None else torch.from_numpy(lens).to(DEV))
    ref = AT.attention_block(x, AT.prepare_attn_bf16(params), lengths=lens, mode="reference")
    assert_bf16_close(y, ref, f"attention block B={B} T={T} masked={masked}")
    assert _lib.device_status(torch.cuda.current_stream().cuda_stream) == 0


def test_attention_block_compile_fullgraph():
    p = prepare_attn_from_params(synth.make_attn_params(5), device=DEV)
    x = torch.randn((2, 256, synth.D_MODEL), device=DEV).bfloat16()
    f = lambda x: ops.run_attention_block(x, p)  # noqa: E731
    assert torch.equal(torch.compile(f, fullgraph=True)(x), f(x))


def test_gemm_linear_skips_padding_tiles():
    """out = a W^T + b; with lengths the 128-row tiles of pure padding are left untouched."""
    B, T, K, N = 3, 256, 1024, 3072
    M = B * T
    g = torch.Generator(device=DEV).manual_seed(9)
    a = torch.randn((M, K), generator=g, device=DEV).bfloat16()
    w = (torch.randn((N, K), generator=g, device=DEV) * 0.03).bfloat16()
    b = torch.randn((N,), generator=g, device=DEV) * 0.1
    out = torch.full((M, N), 7.0, dtype=torch.bfloat16, device=DEV)
    lens = torch.tensor([256, 100, 0], dtype=torch.int32, device=DEV)
    _lib.call("gsn_gemm_linear_bf16", a.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr(), N, M, K, N,
              lens.data_ptr(), T, torch.cuda.current_stream().cuda_stream)
    ref = (a.float() @ w.float().t() + b).cpu().numpy()
    o = out.float().cpu().numpy()
    active = np.concatenate([np.arange(0, 256), np.arange(256, 384)])      # tiles holding valid frames
    assert_bf16_close(o[active], ref[active], "linear gemm")
    assert (o[384:] == 7.0).all(), "tiles of pure padding are not written"


def test_attention_core_ignores_padding_rows():
    """q|k|v rows of frames past the length hold NaN / Inf: masked keys never reach a valid output (their logits
    are replaced, their V rows zeroed before P V), and padded frames get a zero context."""
    B, T = 3, 512
    qkv = _qkv(21, B, T, q_std=0.3)
    lens = np.array([512, 201, 77], dtype=np.int32)
    ref = _core_ref(qkv, _rel(22), lens)
    bad = qkv.copy()
    for b, L in enumerate(lens):
        bad[b, L:, 0::2] = np.nan
        bad[b, L:, 1::2] = np.inf
    ctx = ops.attention_core(_t(bad), _t(_rel(22)), H, torch.from_numpy(lens).to(DEV)).float().cpu().numpy()
    for b, L in enumerate(lens):
        assert_bf16_close(ctx[b, :L], ref[b, :L], f"b={b} L={L}")
        assert not ctx[b, L:].any()


@pytest.mark.parametrize("heads", [2, 4])
def test_attention_core_other_head_counts(heads):
    """The kernel walks (query tile, utterance, block, head) units for any head count: 2 and 4 heads of 128."""
    B, T = 2, 437
    inner = heads * DH
    g = np.random.default_rng(40 + heads)
    qkv = O.bf16_round(np.concatenate([g.normal(0, 0.3, (B, T, inner)), g.normal(0, 0.3, (B, T, inner)),
                                       g.normal(0, 1.0, (B, T, inner))], axis=-1).astype(np.float32))
    rel = _rel(41)
    lens = np.array([T, 250], dtype=np.int32)
    ctx = ops.attention_core(_t(qkv), _t(rel), heads, torch.from_numpy(lens).to(DEV)).float().cpu().numpy()
    for b, L in enumerate(lens):
        q, k, v = qkv[b, :L, :inner], qkv[b, :L, inner:2 * inner], qkv[b, :L, 2 * inner:]
        ref = AT.attention_core(q, k, v, rel, heads, synth.CONTEXT, synth.MAX_POS_EMB, mode="fp32")
        assert_bf16_close(ctx[b, :L], ref, f"heads={heads} b={b}")
        assert not ctx[b, L:].any()


def test_attention_block_d512_four_heads():
    """The attention step at D = 512 with 4 heads of 128 (the LayerNorm and both GEMMs at that width)."""
    params = synth.make_attn_params(77, d_model=512, heads=4, w_std=0.03)
    p = prepare_attn_from_params(params, device=DEV)
    x = O.bf16_round(synth.make_activations(78, (2, 384, 512)))
    lens = np.array([384, 190], dtype=np.int32)
    y = ops.run_attention_block(_t(x), p, torch.from_numpy(lens).to(DEV))
    ref = AT.attention_block(x, AT.prepare_attn_bf16(params), lengths=lens, mode="reference")
    assert_bf16_close(y, ref, "attention block D=512 heads=4")
