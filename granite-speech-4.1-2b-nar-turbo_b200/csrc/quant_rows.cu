// Per-row symmetric int8 quantisation of bf16 activations, the activation side of the W8A8 conv module (int8
// weights and int8 activations on the kind::i8 tensor-core path).  No counterpart in the reference, whose nearest
// analogue is torchao's W8A8 dynamic quantisation (script/bench_asr.py:92-105, not vendored):
//   scale[m] = max_k |x[m, k]| / 127        (fp32, IEEE division)
//   q[m, k]  = rint(x[m, k] / scale[m])     (round half to even, IEEE division; 0 where scale[m] == 0)
// One warp per row: 16-byte loads of 8 bf16, a shuffle max, then the same loads again for the quantisation (the row
// is 2-4 KB and sits in L1 / L2 between the two passes).  Rows of padding frames (lengths) get scale = 0, and q = 0
// when `zero_padding` is set; inside the W8A8 module they keep whatever q they held, since every GEMM that reads
// them either multiplies the row's s32 sum by its zero scale or masks the row (any int8 values give a finite sum:
// at most 127^2 x K < 2^31), which saves writing a K-byte row of zeros per padding frame.
#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

namespace gsn {

namespace quant_impl {

__global__ void __launch_bounds__(256)
    quant_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int8_t* __restrict__ q,
                      float* __restrict__ scale, int M, int K, const int* lengths, int T, int zero_padding) {
  const int row = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  int8_t* qr = q + (int64_t)row * K;
  if (lengths) {
    const int b = row / T;
    if (row - b * T >= __ldg(lengths + b)) {           // a padding frame
      if (lane == 0) scale[row] = 0.f;
      if (zero_padding)
        for (int d = lane * 8; d < K; d += 256) *reinterpret_cast<uint2*>(qr + d) = make_uint2(0u, 0u);
      return;
    }
  }
  const __nv_bfloat16* xr = x + (int64_t)row * ldx;
  float amax = 0.f;
  for (int d = lane * 8; d < K; d += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + d);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) amax = fmaxf(amax, fmaxf(fabsf(bf16lo_to_f32(w[i])), fabsf(bf16hi_to_f32(w[i]))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = __fdiv_rn(amax, 127.0f);
  if (lane == 0) scale[row] = s;
  for (int d = lane * 8; d < K; d += 256) {
    uint32_t packed[2] = {0u, 0u};
    if (s > 0.f) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + d);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xv = (i & 1) ? bf16hi_to_f32(w[i >> 1]) : bf16lo_to_f32(w[i >> 1]);
        const int qi = max(-127, min(127, __float2int_rn(__fdiv_rn(xv, s))));
        packed[i >> 2] |= ((uint32_t)qi & 0xFFu) << (8 * (i & 3));
      }
    }
    *reinterpret_cast<uint2*>(qr + d) = make_uint2(packed[0], packed[1]);
  }
}

// LayerNorm + per-row quantisation in one pass (the W8A8 module's first GEMM operand): the LayerNorm of
// layernorm.cu (two-pass fp32 statistics from registers, y = (x - mean) * rstd * gamma + beta) rounded to bf16 as
// that kernel stores it, then scale = max |y| / 127 and q = rint(y / scale) as quant_rows_kernel computes them, so
// the result is bit-identical to the two kernels in sequence without the bf16 LayerNorm tensor.  One warp per row.
template <int V>  // V = D / 256 16-byte vectors per lane
__global__ void __launch_bounds__(256)
    layernorm_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, const __nv_bfloat16* __restrict__ gamma,
                           const __nv_bfloat16* __restrict__ beta, int8_t* __restrict__ q, float* __restrict__ scale,
                           int M, float eps, const int* __restrict__ lengths, int T, int zero_padding) {
  constexpr int D = V * 256;
  const int lane = threadIdx.x & 31;
  const int row = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (row >= M) return;
  int8_t* qr = q + (int64_t)row * D;
  if (lengths != nullptr) {               // padding frames: scale = 0 (and q = 0 with zero_padding)
    const int b = row / T;
    if (row - b * T >= __ldg(lengths + b)) {
      if (zero_padding) {
#pragma unroll
        for (int i = 0; i < V; ++i) *reinterpret_cast<uint2*>(qr + i * 256 + lane * 8) = make_uint2(0u, 0u);
      }
      if (lane == 0) scale[row] = 0.f;
      return;
    }
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
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const uint4 g = __ldg(reinterpret_cast<const uint4*>(gamma + i * 256 + lane * 8));
    const uint4 bb = __ldg(reinterpret_cast<const uint4*>(beta + i * 256 + lane * 8));
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
    const uint32_t bw[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float y0 = fmaf((v[i][2 * k] - mean) * rstd, bf16lo_to_f32(gw[k]), bf16lo_to_f32(bw[k]));
      const float y1 = fmaf((v[i][2 * k + 1] - mean) * rstd, bf16hi_to_f32(gw[k]), bf16hi_to_f32(bw[k]));
      const uint32_t yb = pack_bf16x2(y0, y1);          // the bf16 LayerNorm output
      v[i][2 * k] = bf16lo_to_f32(yb);
      v[i][2 * k + 1] = bf16hi_to_f32(yb);
      amax = fmaxf(amax, fmaxf(fabsf(v[i][2 * k]), fabsf(v[i][2 * k + 1])));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = __fdiv_rn(amax, 127.0f);
  if (lane == 0) scale[row] = s;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    uint32_t packed[2] = {0u, 0u};
    if (s > 0.f) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int qi = max(-127, min(127, __float2int_rn(__fdiv_rn(v[i][k], s))));
        packed[k >> 2] |= ((uint32_t)qi & 0xFFu) << (8 * (k & 3));
      }
    }
    *reinterpret_cast<uint2*>(qr + i * 256 + lane * 8) = make_uint2(packed[0], packed[1]);
  }
}

}  // namespace quant_impl

int launch_layernorm_quant(const __nv_bfloat16* x, int64_t ld_x, const __nv_bfloat16* gamma,
                           const __nv_bfloat16* beta, int8_t* q, float* scale, int M, int D, float eps,
                           const int* lengths, int T, int zero_padding, cudaStream_t stream) {
  if (M <= 0) return 0;
  if (lengths && T <= 0) return (int)cudaErrorInvalidValue;
  const int grid = (int)(((int64_t)M * 32 + 255) / 256);
  const int zp = zero_padding;
  switch (D) {
    case 256: quant_impl::layernorm_quant_kernel<1><<<grid, 256, 0, stream>>>(x, ld_x, gamma, beta, q, scale, M, eps, lengths, T, zp); break;
    case 512: quant_impl::layernorm_quant_kernel<2><<<grid, 256, 0, stream>>>(x, ld_x, gamma, beta, q, scale, M, eps, lengths, T, zp); break;
    case 1024: quant_impl::layernorm_quant_kernel<4><<<grid, 256, 0, stream>>>(x, ld_x, gamma, beta, q, scale, M, eps, lengths, T, zp); break;
    case 2048: quant_impl::layernorm_quant_kernel<8><<<grid, 256, 0, stream>>>(x, ld_x, gamma, beta, q, scale, M, eps, lengths, T, zp); break;
    default: return (int)cudaErrorInvalidValue;
  }
  return (int)cudaGetLastError();
}

int launch_quant_rows(const __nv_bfloat16* x, int64_t ldx, int8_t* q, float* scale, int M, int K,
                      const int* lengths, int T, int zero_padding, cudaStream_t stream) {
  if (M <= 0) return 0;
  if (K <= 0 || K % 8 || ldx % 8 || (lengths && T <= 0)) return (int)cudaErrorInvalidValue;
  const int blocks = (int)(((int64_t)M * 32 + 255) / 256);
  quant_impl::quant_rows_kernel<<<blocks, 256, 0, stream>>>(x, ldx, q, scale, M, K, lengths, T, zero_padding);
  return (int)cudaGetLastError();
}

}  // namespace gsn
