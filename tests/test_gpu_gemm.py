"""tcgen05 GEMMs (up_conv + GLU epilogue, down_conv + residual epilogue; bf16 and int8 weights) and the LayerNorm
kernel against the oracle's pieces on bf16-valued inputs."""
import numpy as np
import pytest
import torch

from granite_conv_b200 import ops
from granite_conv_b200.weights import glu_interleave, quantize_per_channel
from oracle import conv_module as O
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand(seed, shape, std=1.0):
    return O.bf16_round(np.random.default_rng(seed).normal(0.0, std, shape).astype(np.float32))


def _t(a, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).to(DEV)


@pytest.mark.parametrize("M,K,N", [(128, 1024, 4096), (200, 1024, 4096), (1, 1024, 4096), (37 * 2, 1024, 4096),
                                   (128, 64, 256), (300, 192, 512), (1024, 1024, 4096)])
def test_gemm1_glu(M, K, N):
    a = _rand(M * 7 + K, (M, K))
    w = _rand(11 + N, (N, K), std=0.05)
    b = _rand(12 + N, (N,), std=0.02)
    h = ops.gemm1_glu(_t(a), glu_interleave(_t(w)), glu_interleave(_t(b, torch.float32)))
    ref = O.bf16_round(O.glu(O.pointwise(a, w, b)).astype(np.float32))
    assert_bf16_close(h, ref, f"gemm1 M={M} K={K} N={N}")


@pytest.mark.parametrize("M,K,N", [(128, 2048, 1024), (200, 2048, 1024), (1, 2048, 1024), (129, 64, 256),
                                   (1024, 2048, 1024)])
@pytest.mark.parametrize("with_residual", [True, False])
def test_gemm2_residual(M, K, N, with_residual):
    d = _rand(M + K, (M, K), std=0.5)
    w = _rand(21 + N, (N, K), std=0.05)
    b = _rand(22 + N, (N,), std=0.02)
    r = _rand(23 + M, (M, N))
    out = ops.gemm2_residual(_t(d), _t(w), _t(b, torch.float32), _t(r) if with_residual else None)
    ref = O.pointwise(d, w, b) + (r if with_residual else 0.0)
    assert_bf16_close(out, O.bf16_round(ref.astype(np.float32)), f"gemm2 M={M} res={with_residual}")


def test_gemm2_strided_rows():
    """Residual and output given as column slices of wider rows (row stride > N)."""
    M, K, N = 160, 256, 256
    d = _rand(1, (M, K), std=0.5)
    w = _rand(2, (N, K), std=0.05)
    b = _rand(3, (N,), std=0.02)
    rw = _rand(4, (M, 2 * N))
    res = _t(rw)[:, N:]
    out = torch.empty((M, 2 * N), dtype=torch.bfloat16, device=DEV)[:, :N]
    from granite_conv_b200 import _lib
    dt, wt, bt = _t(d), _t(w), _t(b, torch.float32)
    _lib.call("gsn_gemm2_residual_bf16", dt.data_ptr(), wt.data_ptr(), bt.data_ptr(), res.data_ptr(), res.stride(0),
              out.data_ptr(), out.stride(0), M, K, N, None, 0, torch.cuda.current_stream().cuda_stream)
    ref = O.bf16_round((O.pointwise(d, w, b) + rw[:, N:]).astype(np.float32))
    assert_bf16_close(out, ref, "gemm2 strided")


@pytest.mark.parametrize("epilogue,extra_rows", [("residual", 0), ("residual", 50), ("silu", 0), ("silu", 77)])
def test_gemm_result_independent_of_grid(epilogue, extra_rows):
    """A grid with more tiles than SMs (a partial last wave) gives, bit for bit, the same rows as calls small
    enough to run one tile per CTA: a tile's result does not depend on which CTA computes it or when."""
    from granite_conv_b200 import _lib
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    K, N = (2048, 1024) if epilogue == "residual" else (1024, 4096)
    per_m = N // 256
    m_blocks = sms // per_m + max(1, 12 // per_m)
    M = m_blocks * 128 - (128 - extra_rows if extra_rows else 0)
    assert 0 < (-(-M // 128)) * per_m - sms <= sms // 2
    g = torch.Generator(device=DEV).manual_seed(31 + extra_rows)
    a = torch.randn((M, K), generator=g, device=DEV).bfloat16()
    w = (torch.randn((N, K), generator=g, device=DEV) * 0.03).bfloat16()
    b = torch.randn((N,), generator=g, device=DEV) * 0.1
    r = torch.randn((M, N), generator=g, device=DEV).bfloat16()
    stream = torch.cuda.current_stream().cuda_stream

    def run(rows):
        a_, r_ = a[rows], r[rows]
        m = a_.shape[0]
        out = torch.empty((m, N), dtype=torch.bfloat16, device=DEV)
        if epilogue == "residual":
            _lib.call("gsn_gemm2_residual_bf16", a_.data_ptr(), w.data_ptr(), b.data_ptr(), r_.data_ptr(), N,
                      out.data_ptr(), N, m, K, N, None, 0, stream)
        else:
            _lib.call("gsn_gemm_silu_bf16", a_.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr(), m, K, N,
                      None, 0, stream)
        return out

    whole = run(slice(0, M))
    step = 8 * 128
    parts = torch.cat([run(slice(i, min(M, i + step))) for i in range(0, M, step)])
    torch.cuda.synchronize()
    assert torch.equal(whole, parts)
    assert _lib.device_status(stream) == 0


@pytest.mark.parametrize("M", [128, 333])
def test_gemm_int8_weights(M):
    K1, N1 = 1024, 4096
    a = _rand(5 + M, (M, K1))
    w1 = np.random.default_rng(6).normal(0, 0.02, (N1, K1)).astype(np.float32)
    b1 = _rand(7, (N1,), std=0.02)
    q1, s1 = quantize_per_channel(torch.from_numpy(w1))
    h = ops.gemm1_glu(_t(a), glu_interleave(q1.to(DEV)), glu_interleave(_t(b1, torch.float32)),
                      glu_interleave(s1.to(DEV)))
    w1_deq = q1.float().numpy() * s1.numpy()[:, None]
    ref1 = O.bf16_round(O.glu(O.pointwise(a, w1_deq, b1)).astype(np.float32))
    assert_bf16_close(h, ref1, "gemm1 int8")

    K2, N2 = 2048, 1024
    d = _rand(8 + M, (M, K2), std=0.5)
    w2 = np.random.default_rng(9).normal(0, 0.02, (N2, K2)).astype(np.float32)
    b2 = _rand(10, (N2,), std=0.02)
    r = _rand(11, (M, N2))
    q2, s2 = quantize_per_channel(torch.from_numpy(w2))
    out = ops.gemm2_residual(_t(d), q2.to(DEV), _t(b2, torch.float32), _t(r), s2.to(DEV))
    w2_deq = q2.float().numpy() * s2.numpy()[:, None]
    assert_bf16_close(out, O.bf16_round((O.pointwise(d, w2_deq, b2) + r).astype(np.float32)), "gemm2 int8")


def test_gemm_shape_errors():
    a = torch.zeros((128, 100), dtype=torch.bfloat16, device=DEV)      # K not a multiple of 8
    w = torch.zeros((256, 100), dtype=torch.bfloat16, device=DEV)
    b = torch.zeros((256,), dtype=torch.float32, device=DEV)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        ops.gemm1_glu(a, w, b)
    a = torch.zeros((128, 64), dtype=torch.bfloat16, device=DEV)
    w = torch.zeros((200, 64), dtype=torch.bfloat16, device=DEV)      # N not a multiple of 256
    with pytest.raises(RuntimeError, match="multiple of 256"):
        ops.gemm2_residual(a, w, torch.zeros((200,), dtype=torch.float32, device=DEV), None)
    h = ops.gemm1_glu(torch.zeros((0, 64), dtype=torch.bfloat16, device=DEV),
                      torch.zeros((256, 64), dtype=torch.bfloat16, device=DEV),
                      torch.zeros((256,), dtype=torch.float32, device=DEV))
    assert h.shape == (0, 128)


def test_gemms_skip_padding_tiles():
    """With lengths (T on the 128 grid): rows of tiles that hold valid frames match the dense result, GEMM2 tiles of
    pure padding are residual + bias, and LayerNorm leaves padding rows untouched."""
    T, lens = 384, np.array([384, 1, 129, 0, 256], dtype=np.int32)
    B = lens.size
    M, K1, N1, K2, N2 = B * T, 1024, 4096, 2048, 1024
    a = _rand(1, (M, K1))
    w1 = _rand(2, (N1, K1), std=0.05)
    b1 = _rand(3, (N1,), std=0.02)
    lt = torch.from_numpy(lens).to(DEV)
    h_dense = ops.gemm1_glu(_t(a), glu_interleave(_t(w1)), glu_interleave(_t(b1, torch.float32)))
    h_skip = ops.gemm1_glu(_t(a), glu_interleave(_t(w1)), glu_interleave(_t(b1, torch.float32)), lengths=lt, T=T)
    d = _rand(4, (M, K2), std=0.5)
    w2 = _rand(5, (N2, K2), std=0.05)
    b2 = _rand(6, (N2,), std=0.02)
    r = _rand(7, (M, N2))
    o_dense = ops.gemm2_residual(_t(d), _t(w2), _t(b2, torch.float32), _t(r))
    o_skip = ops.gemm2_residual(_t(d), _t(w2), _t(b2, torch.float32), _t(r), lengths=lt, T=T)
    x = _rand(8, (M, 1024))
    g, bt = _rand(9, (1024,), std=0.02) + 1.0, _rand(10, (1024,), std=0.02)
    y_dense = ops.layernorm(_t(x), _t(O.bf16_round(g)), _t(bt))
    y_skip = ops.layernorm(_t(x), _t(O.bf16_round(g)), _t(bt), lengths=lt, T=T)
    for b, L in enumerate(lens):
        rows = slice(b * T, b * T + ((int(L) + 127) // 128) * 128)
        assert torch.equal(h_skip[rows], h_dense[rows]), f"gemm1 utt {b}"
        assert torch.equal(o_skip[rows], o_dense[rows]), f"gemm2 utt {b}"
        assert torch.equal(y_skip[b * T:b * T + int(L)], y_dense[b * T:b * T + int(L)]), f"layernorm utt {b}"
        pad = slice(rows.stop, (b + 1) * T)
        ref = O.bf16_round((r[pad] + b2[None, :]).astype(np.float32))
        np.testing.assert_array_equal(o_skip[pad].float().cpu().numpy(), ref)


@pytest.mark.parametrize("M,D", [(1, 1024), (37, 1024), (1000, 1024), (64, 256), (64, 512), (33, 2048),
                                 (20001, 1024), (5003, 2048), (9999, 512)])
def test_layernorm(M, D):
    x = _rand(M + D, (M, D)) * 3.0 + 0.5
    x = O.bf16_round(x.astype(np.float32))
    w = O.bf16_round((1.0 + np.random.default_rng(1).normal(0, 0.02, D)).astype(np.float32))
    b = _rand(2, (D,), std=0.02)
    y = ops.layernorm(_t(x), _t(w), _t(b))
    ref = O.bf16_round(O.layer_norm(x, w, b).astype(np.float32))
    assert_bf16_close(y, ref, f"layernorm M={M} D={D}")
