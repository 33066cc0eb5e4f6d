// LayerNorm over the channel dim of channels-last frames (ConformerConvModule.norm,
// models/granite_speech_nar/conformer.py:164,176): y = (x - mean) * rsqrt(var + eps) * gamma + beta with the biased
// variance, statistics in fp32, output rounded to bf16 (the operand of the up_conv GEMM).
//
// One warp per frame: D = 32 lanes x 8 channels x (D / 256) 16-byte vectors, two-pass statistics from registers,
// so the row is read from HBM exactly once and written once.
#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

namespace gsn {

namespace ln_impl {

constexpr int LN_WARPS = 8;

template <int V>  // V = D / 256 16-byte vectors per lane
__global__ void __launch_bounds__(LN_WARPS * 32)
    layernorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, const __nv_bfloat16* __restrict__ gamma,
                     const __nv_bfloat16* __restrict__ beta, __nv_bfloat16* __restrict__ y, int64_t ld_y, int M,
                     float eps, const int* __restrict__ lengths, int T) {
  constexpr int D = V * 256;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * LN_WARPS + (threadIdx.x >> 5);
  if (row >= M) return;
  if (lengths != nullptr) {               // padding frames: their LayerNorm output is never consumed
    const int b = row / T;
    if (row - b * T >= __ldg(lengths + b)) return;
  }
  const __nv_bfloat16* xr = x + (int64_t)row * ld_x;
  float v[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(xr + i * 256 + lane * 8));
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[i][2 * k] = bf16lo_to_f32(w[k]);
      v[i][2 * k + 1] = bf16hi_to_f32(w[k]);
    }
  }
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) sum += v[i][k];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum * (1.0f / D);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float d = v[i][k] - mean;
      sq = fmaf(d, d, sq);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq * (1.0f / D) + eps);

  __nv_bfloat16* yr = y + (int64_t)row * ld_y;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const uint4 g = __ldg(reinterpret_cast<const uint4*>(gamma + i * 256 + lane * 8));
    const uint4 bb = __ldg(reinterpret_cast<const uint4*>(beta + i * 256 + lane * 8));
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
    const uint32_t bw[4] = {bb.x, bb.y, bb.z, bb.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float y0 = fmaf((v[i][2 * k] - mean) * rstd, bf16lo_to_f32(gw[k]), bf16lo_to_f32(bw[k]));
      const float y1 = fmaf((v[i][2 * k + 1] - mean) * rstd, bf16hi_to_f32(gw[k]), bf16hi_to_f32(bw[k]));
      o[k] = pack_bf16x2(y0, y1);
    }
    *reinterpret_cast<uint4*>(yr + i * 256 + lane * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Row statistics only, for the LayerNorm folded into the up_conv GEMM: stats[row] = (rstd, rstd * mean), the
// same two-pass fp32 statistics as layernorm_kernel; padding frames are left unwritten.
template <int V>
__global__ void __launch_bounds__(LN_WARPS * 32)
    ln_stats_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, float2* __restrict__ stats, int M, float eps,
                    const int* __restrict__ lengths, int T) {
  constexpr int D = V * 256;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * LN_WARPS + (threadIdx.x >> 5);
  if (row >= M) return;
  if (lengths != nullptr) {
    const int b = row / T;
    if (row - b * T >= __ldg(lengths + b)) return;
  }
  const __nv_bfloat16* xr = x + (int64_t)row * ld_x;
  float v[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(xr + i * 256 + lane * 8));
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[i][2 * k] = bf16lo_to_f32(w[k]);
      v[i][2 * k + 1] = bf16hi_to_f32(w[k]);
    }
  }
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) sum += v[i][k];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum * (1.0f / D);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float d = v[i][k] - mean;
      sq = fmaf(d, d, sq);
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq * (1.0f / D) + eps);
  if (lane == 0) stats[row] = make_float2(rstd, rstd * mean);
}

// LayerNorm folded into the following pointwise conv: W' = bf16(W * gamma) (per input channel k), b' = b + W beta,
// c = sum_k W'[n, k] in fp32, so that LN(x) W^T + b = rstd * (x W'^T) - (rstd * mean) * c + b'.  One warp per
// output row n of W [N, K] (bf16), K % 256 == 0.
__global__ void __launch_bounds__(LN_WARPS * 32)
    fold_ln_kernel(const __nv_bfloat16* __restrict__ w, const float* __restrict__ bias,
                   const __nv_bfloat16* __restrict__ gamma, const __nv_bfloat16* __restrict__ beta,
                   __nv_bfloat16* __restrict__ w_out, float* __restrict__ bias_out, float* __restrict__ colsum,
                   int N, int K) {
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * LN_WARPS + (threadIdx.x >> 5);
  if (n >= N) return;
  float bsum = 0.f, csum = 0.f;
  for (int k0 = lane * 8; k0 < K; k0 += 256) {
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + (int64_t)n * K + k0));
    const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gamma + k0));
    const uint4 bv = __ldg(reinterpret_cast<const uint4*>(beta + k0));
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float w0 = bf16lo_to_f32(ww[k]), w1 = bf16hi_to_f32(ww[k]);
      const uint32_t p = pack_bf16x2(w0 * bf16lo_to_f32(gw[k]), w1 * bf16hi_to_f32(gw[k]));
      o[k] = p;
      bsum = fmaf(w0, bf16lo_to_f32(bw[k]), bsum);
      bsum = fmaf(w1, bf16hi_to_f32(bw[k]), bsum);
      csum += bf16lo_to_f32(p) + bf16hi_to_f32(p);
    }
    *reinterpret_cast<uint4*>(w_out + (int64_t)n * K + k0) = make_uint4(o[0], o[1], o[2], o[3]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    bsum += __shfl_xor_sync(0xffffffffu, bsum, o);
    csum += __shfl_xor_sync(0xffffffffu, csum, o);
  }
  if (lane == 0) {
    bias_out[n] = bias[n] + bsum;
    colsum[n] = csum;
  }
}

}  // namespace ln_impl
using namespace ln_impl;

int launch_ln_stats(const __nv_bfloat16* x, int64_t ld_x, float2* stats, int M, int D, float eps, const int* lengths,
                    int T, cudaStream_t stream) {
  if (M == 0) return 0;
  const int grid = (M + LN_WARPS - 1) / LN_WARPS;
  switch (D) {
    case 256: ln_stats_kernel<1><<<grid, LN_WARPS * 32, 0, stream>>>(x, ld_x, stats, M, eps, lengths, T); break;
    case 512: ln_stats_kernel<2><<<grid, LN_WARPS * 32, 0, stream>>>(x, ld_x, stats, M, eps, lengths, T); break;
    case 1024: ln_stats_kernel<4><<<grid, LN_WARPS * 32, 0, stream>>>(x, ld_x, stats, M, eps, lengths, T); break;
    case 2048: ln_stats_kernel<8><<<grid, LN_WARPS * 32, 0, stream>>>(x, ld_x, stats, M, eps, lengths, T); break;
    default: return (int)cudaErrorInvalidValue;
  }
  return (int)cudaGetLastError();
}

int launch_fold_ln(const __nv_bfloat16* w, const float* bias, const __nv_bfloat16* gamma, const __nv_bfloat16* beta,
                   __nv_bfloat16* w_out, float* bias_out, float* colsum, int N, int K, cudaStream_t stream) {
  if (N == 0) return 0;
  if (K % 256) return (int)cudaErrorInvalidValue;
  fold_ln_kernel<<<(N + LN_WARPS - 1) / LN_WARPS, LN_WARPS * 32, 0, stream>>>(w, bias, gamma, beta, w_out, bias_out,
                                                                               colsum, N, K);
  return (int)cudaGetLastError();
}

int launch_layernorm(const __nv_bfloat16* x, int64_t ld_x, const __nv_bfloat16* gamma, const __nv_bfloat16* beta,
                     __nv_bfloat16* y, int64_t ld_y, int M, int D, float eps, const int* lengths, int T,
                     cudaStream_t stream) {
  if (M == 0) return 0;
  const int grid = (M + LN_WARPS - 1) / LN_WARPS;
  switch (D) {
    case 256: layernorm_kernel<1><<<grid, LN_WARPS * 32, 0, stream>>>(x, ld_x, gamma, beta, y, ld_y, M, eps, lengths, T); break;
    case 512: layernorm_kernel<2><<<grid, LN_WARPS * 32, 0, stream>>>(x, ld_x, gamma, beta, y, ld_y, M, eps, lengths, T); break;
    case 1024: layernorm_kernel<4><<<grid, LN_WARPS * 32, 0, stream>>>(x, ld_x, gamma, beta, y, ld_y, M, eps, lengths, T); break;
    case 2048: layernorm_kernel<8><<<grid, LN_WARPS * 32, 0, stream>>>(x, ld_x, gamma, beta, y, ld_y, M, eps, lengths, T); break;
    default: return (int)cudaErrorInvalidValue;
  }
  return (int)cudaGetLastError();
}

}  // namespace gsn
