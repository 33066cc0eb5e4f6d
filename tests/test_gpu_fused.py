"""up_conv + GLU + depthwise + SiLU in one kernel (``gsn_gemm1_glu_dwconv_bf16``) against the two-kernel path it
replaces (GLU GEMM writing the GLU tensor, then the depthwise kernel): identical bits on every frame the fused
kernel writes, zeros on [len, roundup128(len)), untouched frames past that."""
import numpy as np
import pytest
import torch

from granite_conv_b200 import ops, synth
from granite_conv_b200.weights import prepare_from_params
from oracle import conv_module as O
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
SENTINEL = 0x7F7F  # bf16 bit pattern of a large finite value, left in frames the kernel must not write


def _prep(seed, int8=False):
    return prepare_from_params(synth.make_params(seed, w_std=0.05), device=DEV, int8=int8)


def _two_kernel(a, p, B, T, lengths, scale=None, w=None):
    w = p.w1_glu if w is None else w
    h = ops.gemm1_glu(a, w, p.b1_glu, None, None, T) if scale is None else _gemm1_scaled(a, w, scale, p.b1_glu)
    hv = h.view(B, T, -1).transpose(1, 2)           # (B, C, T) channels-last view
    if lengths is None:
        y = torch.ops.granite.dwconv_silu(hv, p.dw_w.view(-1, 1, 15), p.dw_b)
    else:
        y = torch.ops.granite.dwconv_silu_masked(hv, p.dw_w.view(-1, 1, 15), p.dw_b, lengths)
    return y.transpose(1, 2).reshape(B * T, -1)


def _gemm1_scaled(a, w_bf16, scale, b):
    from granite_conv_b200 import _lib
    M, K = a.shape
    N = w_bf16.shape[0]
    h = torch.empty((M, N // 2), dtype=torch.bfloat16, device=a.device)
    _lib.call("gsn_gemm1_glu_bf16s", a.data_ptr(), w_bf16.data_ptr(), scale.data_ptr(), b.data_ptr(), h.data_ptr(),
              M, K, N, None, 0, torch.cuda.current_stream().cuda_stream)
    return h


def _check(d, ref, B, T, lens):
    d = d.view(B, T, -1)
    ref = ref.view(B, T, -1)
    for b in range(B):
        L = T if lens is None else int(lens[b])
        end = T if lens is None else min(T, -(-L // 128) * 128)
        assert torch.equal(d[b, :L], ref[b, :L]), f"utterance {b}: frames [0, {L})"
        assert torch.count_nonzero(d[b, L:end]) == 0, f"utterance {b}: frames [{L}, {end}) must be zero"
        assert bool((d[b, end:].view(torch.int16) == SENTINEL).all()), f"utterance {b}: frames >= {end} written"


@pytest.mark.parametrize("B,T,lens", [
    (4, 128, None),
    (3, 256, [256, 130, 7]),
    (2, 384, [384, 128]),
    (5, 512, [0, 1, 127, 129, 512]),
    (3, 896, None),
    (6, 1536, [1536, 641, 640, 639, 64, 1500]),
    (7, 1152, [1152, 1025, 1024, 769, 768, 385, 384]),
    (10, 384, None),                                     # 160 units on 148 SMs: the last 12 split in halves
    (12, 640, [640, 639, 600, 513, 512, 300, 257, 256, 129, 128, 1, 0]),
])
def test_fused_equals_two_kernels(B, T, lens):
    p = _prep(40 + T)
    a = torch.from_numpy(O.bf16_round(synth.make_activations(41 + T, (B * T, synth.D_MODEL)))).to(DEV)
    a = a.to(torch.bfloat16)
    lt = None if lens is None else torch.tensor(lens, dtype=torch.int32, device=DEV)
    d = torch.full((B * T, p.d_inner), 0, dtype=torch.int16, device=DEV).fill_(SENTINEL).view(torch.bfloat16)
    ops.gemm1_glu_dwconv(a, p.w1_glu, p.b1_glu, p.dw_w, p.dw_b, B, T, lengths=lt, out=d)
    ref = _two_kernel(a, p, B, T, lt)
    torch.cuda.synchronize()
    _check(d, ref, B, T, lens)


def test_fused_scaled_weights():
    """int8 weights widened to bf16 with the column scale in the epilogue (the int8 module's path)."""
    from granite_conv_b200 import _lib
    B, T, lens = 3, 256, [256, 200, 33]
    p = _prep(77, int8=True)
    w1b = torch.empty(p.w1q_glu.shape, dtype=torch.bfloat16, device=DEV)
    _lib.call("gsn_widen_i8_bf16", p.w1q_glu.data_ptr(), w1b.data_ptr(), p.w1q_glu.numel(), None, None, 0,
              torch.cuda.current_stream().cuda_stream)
    a = torch.from_numpy(O.bf16_round(synth.make_activations(78, (B * T, synth.D_MODEL)))).to(DEV)
    a = a.to(torch.bfloat16)
    lt = torch.tensor(lens, dtype=torch.int32, device=DEV)
    d = torch.full((B * T, p.d_inner), 0, dtype=torch.int16, device=DEV).fill_(SENTINEL).view(torch.bfloat16)
    ops.gemm1_glu_dwconv(a, w1b, p.b1_glu, p.dw_w, p.dw_b, B, T, scale_glu=p.s1_glu, lengths=lt, out=d)
    ref = _two_kernel(a, p, B, T, lt, scale=p.s1_glu, w=w1b)
    torch.cuda.synchronize()
    _check(d, ref, B, T, lens)


def test_fused_large_batch_natural_order():
    """More utterances than the kernel orders by length (512): units in natural order."""
    B, T = 520, 128
    rng = np.random.default_rng(5)
    lens = rng.integers(0, T + 1, size=B).astype(np.int32)
    p = _prep(91)
    a = torch.randn((B * T, synth.D_MODEL), generator=torch.Generator(device=DEV).manual_seed(3),
                    device=DEV).to(torch.bfloat16)
    lt = torch.from_numpy(lens).to(DEV)
    d = torch.full((B * T, p.d_inner), 0, dtype=torch.int16, device=DEV).fill_(SENTINEL).view(torch.bfloat16)
    ops.gemm1_glu_dwconv(a, p.w1_glu, p.b1_glu, p.dw_w, p.dw_b, B, T, lengths=lt, out=d)
    ref = _two_kernel(a, p, B, T, lt)
    torch.cuda.synchronize()
    _check(d, ref, B, T, lens)


def test_fused_vs_oracle():
    """Independent of the two-kernel path: the fused output against the numpy oracle's depthwise output."""
    B, T, lens = 2, 256, np.array([256, 150], dtype=np.int32)
    params = synth.make_params(123, w_std=0.05)
    p = prepare_from_params(params, device=DEV)
    x = O.bf16_round(synth.make_activations(124, (B, T, synth.D_MODEL)))
    prep = O.prepare_bf16(params)
    t = O.bf16_round(O.layer_norm(x, prep["ln_w"], prep["ln_b"], 1e-5).astype(np.float32))
    a = torch.from_numpy(np.ascontiguousarray(t.reshape(B * T, -1))).to(torch.bfloat16).to(DEV)
    d = ops.gemm1_glu_dwconv(a, p.w1_glu, p.b1_glu, p.dw_w, p.dw_b, B, T,
                             lengths=torch.from_numpy(lens).to(DEV)).view(B, T, -1).float().cpu().numpy()
    h = O.bf16_round(O.glu(O.pointwise(t.reshape(B * T, -1), prep["w1"], prep["b1"])).astype(np.float32))
    ref = O.dwconv_silu(h.reshape(B, T, -1), prep["dw_w"], prep["dw_b"], lengths=lens)
    for b, L in enumerate(lens):
        assert_bf16_close(d[b, :L], ref[b, :L], f"fused utterance {b}")

