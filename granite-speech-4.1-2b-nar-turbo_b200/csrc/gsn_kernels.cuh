// Host-side launchers of the conv-module kernels (implemented in gemm_sm100.cu, dwconv.cu, layernorm.cu).
// All return a cudaError_t-style status from the launch; argument validation happens in capi.cu.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gsn {

// ---- tensor maps (capi.cu) --------------------------------------------------------------------------------
// Encodes a tiled TMA descriptor.  dims/strides follow cuTensorMapEncodeTiled: dims[0] is the innermost
// (contiguous) extent, strides[i] is the byte stride of dims[i + 1].
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

int device_sm_count();

// ---- GEMMs (gemm_sm100.cu) --------------------------------------------------------------------------------
// out = epilogue(A[M,K] (bf16, row-major) x W[N,K]^T)
//   GLU:      W rows are interleaved per 256-row block as [128 value rows | 128 gate rows]; out is [M, N/2]:
//             out[m, 128*j + c] = (acc[m, 256*j + c] * s + b) * sigmoid(acc[m, 256*j + 128 + c] * s + b)
//   RESIDUAL: out[m, n] = acc[m, n] * s + b[n] (+ residual[m, n] when residual is not null)
// `col_scale` (per W row) is null for bf16 weights; with int8 weights W is int8 and dequantised in shared memory.
struct GemmArgs {
  const __nv_bfloat16* a;
  const void* w;                 // bf16 [N, K] or int8 [N, K]
  const float* bias;             // [N], same row order as W
  const float* col_scale;        // [N] or null
  const __nv_bfloat16* residual; // RESIDUAL only: [M, N], row stride ld_res, or null
  __nv_bfloat16* out;
  int64_t ld_out, ld_res;
  int M, N, K;
  int w_int8;
  const int* lengths;            // null, or per-utterance valid frames: 128-row tiles of pure padding are
  int T;                         //   skipped (GLU, SILU) or written as residual + bias (RESIDUAL); T % 128 == 0
  float out_scale = 1.0f;        // RESIDUAL: out = out_scale * (acc * col_scale + bias) + residual
  unsigned long long* argmax_keys = nullptr;   // ARGMAX: [M] keys, zeroed by the caller
  int n_major = 0;               // walk the tiles column block by column block (each W tile read once)
  int a_int8 = 0;                // W8A8: a is int8 [M, K] and w int8 [N, K] (kind::i8 MMAs, s32 accumulate);
  const float* row_scale = nullptr;   //   acc is scaled by row_scale[m] * col_scale[n] (GLU and RESIDUAL only)
  int withhold_load = -1;        // test only (>= 0): every CTA's producer arms the barrier of its operand load #k
                                 //   without issuing the copies, so the MMA warp's bounded wait runs out
  float2* row_partials = nullptr;  // RESIDUAL only: [M][N / 256] (mean, M2) of each output row's 256-column blocks
};

// LINEAR: out = acc + b, 128-row tiles of pure padding skipped (nothing written there)
// ARGMAX: no output tensor; per row m, atomicMax(keys[m], (ordered bits of bf16(acc + b[n])) << 32 | ~n) over n
enum GemmEpilogue { kEpiGlu = 0, kEpiResidual = 1, kEpiSilu = 2, kEpiLinear = 3, kEpiArgmax = 4 };

int launch_gemm(const GemmArgs& args, int epilogue, cudaStream_t stream);
// Per-row symmetric int8 quantisation: scale[m] = max_k |x[m, k]| / 127, q[m, k] = rint(x[m, k] / scale[m]) (q = 0
// and scale = 0 for an all-zero row; with lengths, rows of padding frames get scale = 0, and q = 0 only with
// zero_padding).  x bf16 [M, K] (row stride ldx), q int8 [M, K] dense.  K % 8 == 0, 16-byte aligned rows.
int launch_quant_rows(const __nv_bfloat16* x, int64_t ldx, int8_t* q, float* scale, int M, int K,
                      const int* lengths, int T, int zero_padding, cudaStream_t stream);
// LayerNorm (launch_layernorm's arithmetic, rounded to bf16) and launch_quant_rows' quantisation in one pass: q int8
// [M, D] dense, scale[M]; D in {256, 512, 1024, 2048}.
int launch_layernorm_quant(const __nv_bfloat16* x, int64_t ld_x, const __nv_bfloat16* gamma,
                           const __nv_bfloat16* beta, int8_t* q, float* scale, int M, int D, float eps,
                           const int* lengths, int T, int zero_padding, cudaStream_t stream);
// int8 -> bf16 widening of two weight arrays (n0, n1 bytes, multiples of 16; 16-byte aligned pointers).
int launch_widen_i8(const void* q0, void* o0, int64_t n0, const void* q1, void* o1, int64_t n1, cudaStream_t stream);

// ---- up_conv + GLU + depthwise + SiLU in one kernel (gemm_glu_dw_sm100.cu) ------------------------------------
// a: [B*T, K] bf16; w: [N, K] bf16 GLU-interleaved (N = 2 * inner); d: [B*T, inner] bf16.  T % 128 == 0.
struct GemmDwArgs {
  const __nv_bfloat16* a;
  const __nv_bfloat16* w;
  const float* bias;             // [N] GLU-interleaved
  const float* col_scale;        // [N] or null
  const __nv_bfloat16* dw_w;     // [inner, 15]
  const __nv_bfloat16* dw_b;     // [inner]
  __nv_bfloat16* d;
  const int* lengths;            // [B] or null
  int B, T, K, N;
  const float2* row_stats;       // LayerNorm folded in: a = raw frames, per-row (rstd, rstd * mean) [B*T]; or null
  const float* colsum;           // with row_stats: [N] column sums of w
  int a_int8 = 0;                // W8A8: a int8 [B*T, K], w int8 [N, K] (kind::i8), needs col_scale and row_scale
  const float* row_scale = nullptr;
  const float2* row_partials = nullptr;   // LayerNorm folded in, instead of row_stats: [B*T][K / 256] (mean, M2) of
  float ln_eps = 0.f;                     //   each row's 256-column blocks, merged here into (rstd, rstd * mean)
};
int launch_gemm_glu_dw(const GemmDwArgs& args, cudaStream_t stream);

// ---- depthwise conv k=15 + bias + SiLU (dwconv.cu) -------------------------------------------------------
// x: (B, C, T) logical, element strides sxB, sxC, sxT; y likewise.  GLU: x holds 2C channels (value | gate).
struct DwArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* w;        // (C, K) contiguous, K = 15
  const __nv_bfloat16* bias;     // (C,)
  __nv_bfloat16* y;
  const int* lengths;            // (B,) or null
  int64_t sxB, sxC, sxT, syB, syC, syT;
  int B, C, T;
  int glu;
  int withhold_tile = -1;        // test only (>= 0): every CTA arms the barrier of its tile #k without the copy
};

int launch_dwconv(const DwArgs& args, cudaStream_t stream);
// the channels-first form on the tensor cores (dwconv_mma_sm100.cu), plain or GLU: T innermost in x and y,
// C % 16 == 0, T % 8 == 0, 16-byte aligned rows (element strides of C and B multiples of 8)
int launch_dwconv_cf_mma(const DwArgs& args, cudaStream_t stream);

// ---- LayerNorm over the last dim (layernorm.cu) -------------------------------------------------------------
// lengths (optional): rows r with r % T >= lengths[r / T] are padding and are skipped.
int launch_layernorm(const __nv_bfloat16* x, int64_t ld_x, const __nv_bfloat16* gamma, const __nv_bfloat16* beta,
                     __nv_bfloat16* y, int64_t ld_y, int M, int D, float eps, const int* lengths, int T,
                     cudaStream_t stream);
// Row statistics (rstd, rstd * mean) of the LayerNorm, for the LayerNorm folded into the up_conv GEMM.
int launch_ln_stats(const __nv_bfloat16* x, int64_t ld_x, float2* stats, int M, int D, float eps, const int* lengths,
                    int T, cudaStream_t stream);
// W' = bf16(W * gamma), b' = b + W beta, colsum = sum_k W'[n, k] (fp32) for W [N, K] bf16.
int launch_fold_ln(const __nv_bfloat16* w, const float* bias, const __nv_bfloat16* gamma, const __nv_bfloat16* beta,
                   __nv_bfloat16* w_out, float* bias_out, float* colsum, int N, int K, cudaStream_t stream);

// ---- block-local Shaw attention core (attention_sm100.cu) ----------------------------------------------------
// qkv: [B, T, ld_qkv] bf16 rows holding q | k | v (each H * 128 columns); rel: [n_rel, 128] bf16 (row
// max_pos + i - j is the relative embedding of query i and key j); ctx: [B, T, ld_ctx] bf16, columns h * 128 + d.
// Blocks of 200 frames, dim_head 128 (fixed by the kernel); ld_qkv and ld_ctx multiples of 8.
struct AttnArgs {
  const __nv_bfloat16* qkv;
  int64_t ld_qkv;
  const __nv_bfloat16* rel;
  int n_rel;
  __nv_bfloat16* ctx;
  int64_t ld_ctx;
  const int* lengths;            // [B] or null
  int B, T, H;
  int max_pos;
  float scale;
};
int launch_attention(const AttnArgs& args, cudaStream_t stream);

// ---- CTC heads (ctc_head.cu) ----------------------------------------------------------------------------------
int launch_ctc_softmax(const __nv_bfloat16* logits, int64_t ld_l, __nv_bfloat16* probs, int64_t ld_p, float* blank,
                       int M, int C, int kpad, const int* lengths, int T, cudaStream_t stream);
int launch_bpe_pool(const __nv_bfloat16* h, const float* blank, __nv_bfloat16* pooled, int* plen, const int* lengths,
                    int B, int T, int D, int Pp, int window, cudaStream_t stream);
int launch_ctc_collapse(const unsigned long long* keys, const int* plen, int* ids, int* tokens, int* counts, int B,
                        int Pp, int blank_id, cudaStream_t stream);

// ---- self-test of the bounded wait (capi.cu) ----------------------------------------------------------------
int launch_wait_selftest(uint64_t limit_ns, cudaStream_t stream);

}  // namespace gsn
