// Per-row symmetric int8 quantisation of bf16 activations, the activation side of the W8A8 conv module (int8
// weights and int8 activations on the kind::i8 tensor-core path).  No counterpart in the reference, whose nearest
// analogue is torchao's W8A8 dynamic quantisation (script/bench_asr.py:92-105, not vendored):
//   scale[m] = max_k |x[m, k]| / 127        (fp32, IEEE division)
//   q[m, k]  = rint(x[m, k] / scale[m])     (round half to even, IEEE division; 0 where scale[m] == 0)
// One warp per row: 16-byte loads of 8 bf16, a shuffle max, then the same loads again for the quantisation (the row
// is 2-4 KB and sits in L1 / L2 between the two passes).  Rows of padding frames (lengths) get q = 0, scale = 0.
#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

namespace gsn {

namespace quant_impl {

__global__ void __launch_bounds__(256)
    quant_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int8_t* __restrict__ q,
                      float* __restrict__ scale, int M, int K, const int* lengths, int T) {
  const int row = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  bool valid = true;
  if (lengths) {
    const int b = row / T;
    valid = row - b * T < __ldg(lengths + b);
  }
  const __nv_bfloat16* xr = x + (int64_t)row * ldx;
  int8_t* qr = q + (int64_t)row * K;
  float amax = 0.f;
  if (valid) {
    for (int d = lane * 8; d < K; d += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + d);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) amax = fmaxf(amax, fmaxf(fabsf(bf16lo_to_f32(w[i])), fabsf(bf16hi_to_f32(w[i]))));
    }
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

}  // namespace quant_impl

int launch_quant_rows(const __nv_bfloat16* x, int64_t ldx, int8_t* q, float* scale, int M, int K,
                      const int* lengths, int T, cudaStream_t stream) {
  if (M <= 0) return 0;
  if (K <= 0 || K % 8 || ldx % 8 || (lengths && T <= 0)) return (int)cudaErrorInvalidValue;
  const int blocks = (int)(((int64_t)M * 32 + 255) / 256);
  quant_impl::quant_rows_kernel<<<blocks, 256, 0, stream>>>(x, ldx, q, scale, M, K, lengths, T);
  return (int)cudaGetLastError();
}

}  // namespace gsn
