// The encoder's CTC heads around the Conformer stack (models/granite_speech_nar/conformer.py:320-355) and the CTC
// collapse of the transcript (models/granite_speech_nar/asr.py:76-102), on sm_100a:
//
//   self-conditioning at the middle layer (conformer.py:320-324):
//     mid_logits = h W_out^T + b_out      (gemm_kernel<LINEAR>, 348 classes padded to 512 rows of W_out)
//     mid_probs  = softmax(float(mid_logits)), blank = mid_probs[:, 0]          -> ctc_softmax_kernel
//     h          = h + (bf16(mid_probs) W_mid^T + b_mid)   (gemm_kernel<RESIDUAL>, K = 348 padded to 384)
//   BPE head (conformer.py:336-355):
//     pooled     = posterior_weighted_pool(h, 1 - blank, window 4)              -> bpe_pool_kernel
//     logits     = pooled W_bpe^T + b_bpe, ids = argmax(logits)     (gemm_kernel<ARGMAX>: logits never stored)
//   collapse (asr.py:76-102): keep id[p] when p starts the utterance or id[p] != id[p-1], and id[p] != blank
//                                                                               -> ctc_collapse_kernel
#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

namespace gsn {

namespace ctc_impl {

// One warp per frame: softmax over the C class logits (bf16 in, fp32 math), bf16 probabilities out (columns
// [C, ld_p) zero), the blank probability (class 0) in fp32.  Padding frames (t >= len[b]): probabilities zero,
// blank probability 1 (so their pooling weight 1 - blank is zero).
__global__ void __launch_bounds__(256)
    ctc_softmax_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld_l, __nv_bfloat16* __restrict__ probs,
                       int64_t ld_p, float* __restrict__ blank, int M, int C, int kpad, const int* lengths, int T) {
  const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (warp >= M) return;
  const int row = warp;
  bool valid = true;
  if (lengths) {
    const int b = row / T;
    valid = row - b * T < __ldg(lengths + b);
  }
  const __nv_bfloat16* lr = logits + (int64_t)row * ld_l;
  __nv_bfloat16* pr = probs + (int64_t)row * ld_p;
  if (!valid) {
    for (int c = lane; c < kpad; c += 32) pr[c] = __float2bfloat16_rn(0.f);
    if (lane == 0) blank[row] = 1.0f;
    return;
  }
  constexpr int MAXV = 16;                 // up to 512 classes per row in registers
  float v[MAXV];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < C ? __bfloat162float(lr[c]) : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    v[i] = lane + 32 * i < C ? expf(v[i] - mx) : 0.f;
    sum += v[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.0f / sum;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = lane + 32 * i;
    const float pv = v[i] * inv;
    if (c < kpad) pr[c] = __float2bfloat16_rn(c < C ? pv : 0.f);
    if (c == 0) blank[row] = pv;
  }
}

// One warp per pooled frame (b, p): frames t = 4p .. 4p+3 below the utterance length, weights
// (1 - blank_t) / (sum + 1e-8) (posterior_weighted_pool, conformer.py:214-226, fp32), bf16 out.  Pooled frames past
// ceil(len / 4) are written as zero; plen[b] = ceil(len / 4).
__global__ void __launch_bounds__(256)
    bpe_pool_kernel(const __nv_bfloat16* __restrict__ h, const float* __restrict__ blank,
                    __nv_bfloat16* __restrict__ pooled, int* __restrict__ plen, const int* lengths, int B, int T,
                    int D, int Pp, int window) {
  const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (warp >= B * Pp) return;
  const int b = warp / Pp, pp = warp - b * Pp;
  const int L = lengths ? min(max(__ldg(lengths + b), 0), T) : T;
  const int np = (L + window - 1) / window;
  if (pp == 0 && lane == 0) plen[b] = np;
  __nv_bfloat16* out = pooled + ((int64_t)b * Pp + pp) * D;
  if (pp >= np) {
    for (int d = lane * 8; d < D; d += 256) *reinterpret_cast<uint4*>(out + d) = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  float w[8];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int t = pp * window + k;
    w[k] = k < window && t < L ? 1.0f - __ldg(blank + (int64_t)b * T + t) : 0.f;
    s += w[k];
  }
  const float den = s + 1e-8f;
#pragma unroll
  for (int k = 0; k < 8; ++k) w[k] = w[k] / den;
  for (int d = lane * 8; d < D; d += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int t = pp * window + k;
      if (k >= window || t >= L) continue;
      const uint4 x = *reinterpret_cast<const uint4*>(h + ((int64_t)b * T + t) * D + d);
      const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = fmaf(bf16lo_to_f32(xw[i]), w[k], acc[2 * i]);
        acc[2 * i + 1] = fmaf(bf16hi_to_f32(xw[i]), w[k], acc[2 * i + 1]);
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + d) = o;
  }
}

// One CTA per utterance: argmax ids from the keys (-1 past plen), then the CTC collapse into tokens[b, 0:count)
// (-1 after it).
__global__ void __launch_bounds__(256)
    ctc_collapse_kernel(const unsigned long long* __restrict__ keys, const int* __restrict__ plen,
                        int* __restrict__ ids, int* __restrict__ tokens, int* __restrict__ counts, int Pp,
                        int blank_id) {
  __shared__ int warp_sums[8];
  __shared__ int carry;
  const int b = blockIdx.x;
  const int n = min(max(plen[b], 0), Pp);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const unsigned long long* kb = keys + (int64_t)b * Pp;
  int* ib = ids + (int64_t)b * Pp;
  int* tb = tokens + (int64_t)b * Pp;
  for (int base = 0; base < Pp; base += blockDim.x) {
    const int p = base + (int)threadIdx.x;
    int id = -1, prev = -1;
    if (p < n) {
      id = (int)(0xFFFFFFFFu - (uint32_t)(kb[p] & 0xFFFFFFFFull));
      if (p > 0) prev = (int)(0xFFFFFFFFu - (uint32_t)(kb[p - 1] & 0xFFFFFFFFull));
    }
    if (p < Pp) ib[p] = id;
    const bool keep = p < n && (p == 0 || id != prev) && id != blank_id;
    const unsigned ball = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) warp_sums[wid] = __popc(ball);
    __syncthreads();
    int before = carry;
    for (int w = 0; w < wid; ++w) before += warp_sums[w];
    const int pos = before + __popc(ball & ((1u << lane) - 1u));
    if (keep) tb[pos] = id;
    __syncthreads();
    if (threadIdx.x == 0) {
      int tot = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += warp_sums[w];
      carry += tot;
    }
    __syncthreads();
  }
  const int total = carry;
  for (int p = total + (int)threadIdx.x; p < Pp; p += blockDim.x) tb[p] = -1;   // defined past the transcript
  if (threadIdx.x == 0) counts[b] = total;
}

}  // namespace ctc_impl

int launch_ctc_softmax(const __nv_bfloat16* logits, int64_t ld_l, __nv_bfloat16* probs, int64_t ld_p, float* blank,
                       int M, int C, int kpad, const int* lengths, int T, cudaStream_t stream) {
  if (M <= 0) return 0;
  if (C > 512 || kpad > 512) return (int)cudaErrorInvalidValue;
  const int blocks = (int)(((int64_t)M * 32 + 255) / 256);
  ctc_impl::ctc_softmax_kernel<<<blocks, 256, 0, stream>>>(logits, ld_l, probs, ld_p, blank, M, C, kpad, lengths, T);
  return (int)cudaGetLastError();
}

int launch_bpe_pool(const __nv_bfloat16* h, const float* blank, __nv_bfloat16* pooled, int* plen, const int* lengths,
                    int B, int T, int D, int Pp, int window, cudaStream_t stream) {
  if (B <= 0 || Pp <= 0) return 0;
  if (window < 1 || window > 8 || D % 256) return (int)cudaErrorInvalidValue;
  const int blocks = (int)(((int64_t)B * Pp * 32 + 255) / 256);
  ctc_impl::bpe_pool_kernel<<<blocks, 256, 0, stream>>>(h, blank, pooled, plen, lengths, B, T, D, Pp, window);
  return (int)cudaGetLastError();
}

int launch_ctc_collapse(const unsigned long long* keys, const int* plen, int* ids, int* tokens, int* counts, int B,
                        int Pp, int blank_id, cudaStream_t stream) {
  if (B <= 0) return 0;
  ctc_impl::ctc_collapse_kernel<<<B, 256, 0, stream>>>(keys, plen, ids, tokens, counts, Pp, blank_id);
  return (int)cudaGetLastError();
}

}  // namespace gsn
