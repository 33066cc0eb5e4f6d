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

}  // namespace ln_impl
using namespace ln_impl;

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
