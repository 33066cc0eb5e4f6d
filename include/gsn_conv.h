/* C ABI of the B200 (sm_100a) Conformer conv-module kernels: libgsn_conv.so.
 *
 * Every entry point is `extern "C"`, takes plain device pointers, sizes and element strides, launches on the
 * given CUDA stream (a cudaStream_t; NULL = legacy default stream) and returns a status code: GSN_OK (0) or one
 * of the GSN_ERR_* values, with a message in gsn_last_error_string() (per calling thread).  Nothing here
 * allocates device memory; the caller owns every buffer.  Calls are asynchronous with respect to the host, as
 * kernel launches are.
 *
 * bf16 tensors are passed as `const void*` to IEEE bfloat16 data; fp32 vectors as `const float*`; lengths as
 * int32.  The reference interface each entry point replaces is cited beside it (paths inside the reference
 * project ccyrene/granite-speech-4.1-2b-nar-turbo).
 */
#ifndef GSN_CONV_H_
#define GSN_CONV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* gsn_stream_t; /* same type as cudaStream_t / CUstream */

enum {
  GSN_OK = 0,
  GSN_ERR_INVALID_ARG = 1,   /* null pointer, negative size, wrong kernel size */
  GSN_ERR_UNSUPPORTED = 2,   /* shape / stride / alignment outside what the kernels handle */
  GSN_ERR_CUDA = 3,          /* a CUDA runtime error at launch */
  GSN_ERR_DRIVER = 4,        /* cuTensorMapEncodeTiled unavailable or it rejected a descriptor */
  GSN_ERR_WORKSPACE = 5,     /* workspace smaller than gsn_conv_module_workspace_bytes() */
  GSN_ERR_DEVICE_STATUS = 6  /* a kernel recorded a timeout in the device status word */
};

/* Library version: major * 10000 + minor * 100 + patch. */
int gsn_version(void);

/* Message of the last failed call on this thread ("" after a successful call). */
const char* gsn_last_error_string(void);

/* ---- depthwise conv k=15 + bias + SiLU -------------------------------------------------------------------
 * Replaces granite::dwconv_silu (script/models/granite_speech_nar/conv_kernel.py:41-43), i.e. dwconv1d_silu
 * (script/cuda_kernels/conv1d.py:102-114) and its kernel dwconv1d_silu_bf16 (conv1d.py:21-42):
 *   y[b,c,t] = silu(bias[c] + sum_{j<K} weight[c,j] * x[b,c,t-K/2+j]), zero padding outside [0,T).
 * x, y: logical (B, C, T) bf16 with element strides (sxB, sxC, sxT) / (syB, syC, syT); channels-last
 * (sxC == 1) and channels-first (sxT == 1) both work.  Channels-first with 16-byte aligned rows (strides of C and
 * B multiples of 8), T % 8 == 0 and C % 16 == 0 runs on the tensor cores (the reference call site's contiguous
 * (B, C, T) at T on the 8-frame grid); other strides and a ragged T take a slower generic path.  weight:
 * (C, 1, K) bf16 contiguous, K must be 15; bias: (C,) bf16.  lengths: NULL or int32[B]; frames t >= lengths[b]
 * read as zero and are written as zero (the reference op has no lengths). */
int gsn_dwconv_silu_bf16(const void* x, const void* weight, const void* bias, void* y, int B, int C, int T, int K,
                         int64_t sxB, int64_t sxC, int64_t sxT, int64_t syB, int64_t syC, int64_t syT,
                         const int32_t* lengths, gsn_stream_t stream);

/* Replaces granite::dwconv_silu_glu (conv_kernel.py:49-56) = dwconv1d_silu_glu (conv1d.py:85-99): x2 holds 2C
 * channels, value = [0, C), gate = [C, 2C); the GLU product is rounded to bf16 before the convolution
 * (conv1d.py:70-73).  C is the OUTPUT channel count; strides are those of x2 (B, 2C, T) and y (B, C, T). */
int gsn_dwconv_silu_glu_bf16(const void* x2, const void* weight, const void* bias, void* y, int B, int C, int T,
                             int K, int64_t sxB, int64_t sxC, int64_t sxT, int64_t syB, int64_t syC, int64_t syT,
                             const int32_t* lengths, gsn_stream_t stream);

/* ---- LayerNorm over the channel dim of channels-last rows ------------------------------------------------
 * Replaces ConformerConvModule.norm (script/models/granite_speech_nar/conformer.py:164, :176).  x, y: [M, D]
 * bf16 with row strides ld_x, ld_y (elements, multiples of 8); gamma, beta: [D] bf16; D in {256,512,1024,2048}.
 * lengths: NULL, or int32[M / T]: rows r with r % T >= lengths[r / T] are padding and are left unwritten. */
int gsn_layernorm_bf16(const void* x, int64_t ld_x, const void* gamma, const void* beta, void* y, int64_t ld_y,
                       int M, int D, float eps, const int32_t* lengths, int T, gsn_stream_t stream);

/* ---- pointwise_conv1 + GLU ------------------------------------------------------------------------------
 * Replaces up_conv + GLU (conformer.py:165-166, :177, :181): h[m, c] = v * sigmoid(g) with
 * v = (a[m,:] . W1[c,:]) + b1[c], g = (a[m,:] . W1[C+c,:]) + b1[C+c], C = N/2.
 * a: [M, K] bf16 contiguous; h: [M, N/2] bf16 contiguous.  w1_glu / b1_glu hold W1 and b1 with their rows
 * interleaved per 256-row block as [128 value rows | the matching 128 gate rows] (gsn_interleave_glu_rows).
 * K % 8 == 0, N % 256 == 0, pointers 16-byte aligned.  b1_glu is fp32.
 * lengths: NULL, or int32[M / T] with T % 128 == 0: the rows are M / T utterances of T frames and 128-row tiles
 * made only of padding frames (t >= lengths[b]) are skipped, their rows of h left unwritten. */
int gsn_gemm1_glu_bf16(const void* a, const void* w1_glu, const float* b1_glu, void* h, int M, int K, int N,
                       const int32_t* lengths, int T, gsn_stream_t stream);

/* int8-weight form: w1q_glu int8 [N, K] (interleaved), s1_glu fp32 [N] per-row scale (W1 ~= w1q * s1). */
int gsn_gemm1_glu_i8w(const void* a, const void* w1q_glu, const float* s1_glu, const float* b1_glu, void* h, int M,
                      int K, int N, const int32_t* lengths, int T, gsn_stream_t stream);

/* ---- pointwise_conv2 + residual -------------------------------------------------------------------------
 * Replaces down_conv (conformer.py:170, :187) plus the block's residual add (conformer.py:207):
 * out[m, n] = (d[m,:] . W2[n,:]) + b2[n] + residual[m, n].  d: [M, K] bf16; residual, out: [M, N] bf16 with
 * row strides ld_res, ld_out (multiples of 8); residual may be NULL (no add).  K % 8 == 0, N % 256 == 0.
 * b2 is fp32.  lengths / T as for gsn_gemm1_glu_bf16: 128-row tiles of pure padding skip the MMA and are written
 * as residual + b2 (what a zero row of d gives). */
int gsn_gemm2_residual_bf16(const void* d, const void* w2, const float* b2, const void* residual, int64_t ld_res,
                            void* out, int64_t ld_out, int M, int K, int N, const int32_t* lengths, int T,
                            gsn_stream_t stream);

int gsn_gemm2_residual_i8w(const void* d, const void* w2q, const float* s2, const float* b2, const void* residual,
                           int64_t ld_res, void* out, int64_t ld_out, int M, int K, int N, const int32_t* lengths,
                           int T, gsn_stream_t stream);

/* ---- up_conv + GLU + depthwise + SiLU in one kernel ---------------------------------------------------------
 * No single counterpart in the reference: the composition up_conv (conformer.py:165,177) -> GLU (:166,:181) ->
 * granite::dwconv_silu (conv_kernel.py:41-43, i.e. dwconv1d_silu_bf16 of cuda_kernels/conv1d.py:21-42).  The GLU
 * tensor stays in shared memory: each CTA walks one utterance's frames for one block of 128 channels.
 * a: [B*T, K] bf16 (the LayerNorm output); w1_glu / b1_glu / s1_glu (NULL for bf16 weights) as for
 * gsn_gemm1_glu_bf16 / gsn_gemm1_glu_bf16s; dw_w [N/2, 15] bf16, dw_b [N/2] bf16 (BN folded); d: [B*T, N/2] bf16
 * = silu(depthwise(glu(a W1^T + b1))).  T % 128 == 0, K % 64 == 0, N % 256 == 0.  lengths: NULL or int32[B]:
 * GLU frames t >= lengths[b] are zero, d frames in [len, roundup128(len)) are written as zero and frames past
 * that are not written (the residual GEMM with the same lengths skips those tiles).  d equals
 * gsn_gemm1_glu_bf16 followed by gsn_dwconv_silu_bf16 bit for bit on every frame it writes. */
int gsn_gemm1_glu_dwconv_bf16(const void* a, const void* w1_glu, const float* s1_glu, const float* b1_glu,
                              const void* dw_w, const void* dw_b, void* d, int B, int T, int K, int N,
                              const int32_t* lengths, gsn_stream_t stream);

/* ---- LayerNorm folded into the up_conv GEMM -----------------------------------------------------------------
 * No single counterpart in the reference: ConformerConvModule.norm (conformer.py:164,176) followed by up_conv
 * (:165,177).  LN(x) W^T + b = rstd * (x W'^T) - (rstd * mean) * c + b' with W' = bf16(W * gamma) (per input
 * channel), b' = b + W beta and c = sum_k W'[n, k]: the GEMM runs on the raw frames and the LayerNorm output is
 * never written.  Unlike the two-step path it does not round the LayerNorm output to bf16 (the weights carry gamma
 * instead); results agree with the reference module within the same tolerances.
 *
 * gsn_fold_layernorm_bf16: once per weight set.  w1_glu [N, K] bf16 (GLU-interleaved), b1_glu [N] fp32, ln_w /
 * ln_b [K] bf16 -> w1g_glu [N, K] bf16, b1g_glu [N] fp32, c1_glu [N] fp32.  K % 256 == 0.
 * gsn_layernorm_stats_bf16: stats [M][2] fp32 = (rstd, rstd * mean) per frame, the statistics of
 * gsn_layernorm_bf16; frames t >= lengths[b] are left unwritten.
 * gsn_gemm1_lnfold_glu_dwconv_bf16: gsn_gemm1_glu_dwconv_bf16 on the raw frames x [B*T, K] with the folded
 * weights and the row statistics.
 * gsn_conv_module_lnfold_bf16: gsn_conv_module_bf16 with the folded weights (T % 128 == 0), three launches:
 * statistics, fused up_conv + GLU + depthwise + SiLU, down_conv + residual.  Workspace as for
 * gsn_conv_module_bf16. */
int gsn_fold_layernorm_bf16(const void* w1_glu, const float* b1_glu, const void* ln_w, const void* ln_b,
                            void* w1g_glu, float* b1g_glu, float* c1_glu, int N, int K, gsn_stream_t stream);

int gsn_layernorm_stats_bf16(const void* x, int64_t ld_x, float* stats, int M, int D, float eps,
                             const int32_t* lengths, int T, gsn_stream_t stream);

int gsn_gemm1_lnfold_glu_dwconv_bf16(const void* x, const void* w1g_glu, const float* b1g_glu, const float* c1_glu,
                                     const float* row_stats, const void* dw_w, const void* dw_b, void* d, int B,
                                     int T, int K, int N, const int32_t* lengths, gsn_stream_t stream);

int gsn_conv_module_lnfold_bf16(const void* x, const void* w1g_glu, const float* b1g_glu, const float* c1_glu,
                                const void* dw_w, const void* dw_b, const void* w2, const float* b2,
                                const int32_t* lengths, int add_residual, void* out, int B, int T, int D, int inner,
                                float ln_eps, void* workspace, size_t workspace_bytes, gsn_stream_t stream);

/* ---- a stack of LayerNorm-folded modules: each layer's row statistics from the previous layer's down_conv -------
 * No counterpart in the reference, which runs every layer's LayerNorm (conformer.py:164,176) on its own.  In a stack
 * (the encoder's conv modules back to back, conformer.py:207 feeding the next block) the down_conv + residual
 * epilogue already holds each output row, so it also writes the row's statistics for the next layer's folded
 * LayerNorm: per row and 256-column block, (mean, M2) = (the block's mean, its sum of squared deviations) of the
 * bf16 outputs, "row partials" [M][N / 256] fp32 pairs.  The next up_conv kernel merges a row's blocks into
 * (rstd, rstd * mean) with the equal-count update of Chan et al.; no statistics launch and no extra read of x.
 * The merged statistics equal the two-pass ones up to fp32 rounding.
 *
 * gsn_gemm2_residual_stats_bf16: gsn_gemm2_residual_bf16 that also writes row_partials [M][N / 256] (every row of
 * the M range, padding rows included).  N % 256 == 0.
 * gsn_gemm1_lnfold_partials_glu_dwconv_bf16: gsn_gemm1_lnfold_glu_dwconv_bf16 with the row statistics formed from
 * row_partials [B*T][K / 256] (K % 256 == 0, K <= 2048) and ln_eps instead of read from row_stats.
 * gsn_conv_module_lnfold_chain_bf16: gsn_conv_module_lnfold_bf16 for one layer of such a stack.  stats_in: the row
 * partials of x written by the previous layer's call, or NULL (the first layer: a statistics launch as in
 * gsn_conv_module_lnfold_bf16); stats_out: where to write the row partials of out, or NULL.  Both [B*T][D / 256]
 * fp32 pairs, 8-byte aligned; they may be the same buffer (the up_conv kernel has read stats_in before the
 * down_conv kernel writes stats_out, on the same stream).  Workspace as for gsn_conv_module_bf16. */
int gsn_gemm2_residual_stats_bf16(const void* d, const void* w2, const float* b2, const void* residual,
                                  int64_t ld_res, void* out, int64_t ld_out, int M, int K, int N,
                                  const int32_t* lengths, int T, float* row_partials, gsn_stream_t stream);

int gsn_gemm1_lnfold_partials_glu_dwconv_bf16(const void* x, const void* w1g_glu, const float* b1g_glu,
                                              const float* c1_glu, const float* row_partials, float ln_eps,
                                              const void* dw_w, const void* dw_b, void* d, int B, int T, int K,
                                              int N, const int32_t* lengths, gsn_stream_t stream);

int gsn_conv_module_lnfold_chain_bf16(const void* x, const void* w1g_glu, const float* b1g_glu, const float* c1_glu,
                                      const void* dw_w, const void* dw_b, const void* w2, const float* b2,
                                      const int32_t* lengths, int add_residual, void* out, int B, int T, int D,
                                      int inner, float ln_eps, const float* stats_in, float* stats_out,
                                      void* workspace, size_t workspace_bytes, gsn_stream_t stream);

/* ---- int8 weights widened once per call -------------------------------------------------------------------
 * No counterpart in the reference (its int8 analogue is torchao W8A8, bench_asr.py:92-105).  For large M the
 * weight bytes are negligible next to the activations, so the int8 module widens both weight matrices to bf16
 * (exact integers) once per call and runs the GEMMs on bf16 tiles, keeping the per-column scale in the epilogue.
 * gsn_widen_i8_bf16 widens two int8 arrays (n0, n1 bytes, multiples of 16, 16-byte aligned; either may be 0) into
 * bf16 arrays of 2 * n bytes.  gsn_gemm1_glu_bf16s / gsn_gemm2_residual_bf16s are gsn_gemm1_glu_i8w /
 * gsn_gemm2_residual_i8w with those widened bf16 weights; results are bit-identical to the int8-staged forms. */
int gsn_widen_i8_bf16(const void* q0, void* out0, int64_t n0, const void* q1, void* out1, int64_t n1,
                      gsn_stream_t stream);

int gsn_gemm1_glu_bf16s(const void* a, const void* w1_glu, const float* s1_glu, const float* b1_glu, void* h, int M,
                        int K, int N, const int32_t* lengths, int T, gsn_stream_t stream);

int gsn_gemm2_residual_bf16s(const void* d, const void* w2, const float* s2, const float* b2, const void* residual,
                             int64_t ld_res, void* out, int64_t ld_out, int M, int K, int N, const int32_t* lengths,
                             int T, gsn_stream_t stream);

/* ---- whole conv module + residual -------------------------------------------------------------------------
 * Replaces ConformerConvModule.forward (conformer.py:175-189) followed by the residual add of
 * ConformerBlock.forward (conformer.py:207), with BatchNorm folded (fold_bn.py:33-68):
 *   out = x + down_conv(silu(dwconv(glu(up_conv(layernorm(x))))))
 * (add_residual = 0 returns the module output alone, for callers that add the residual themselves as
 * ConformerBlock.forward does.)
 * x, out: [B, T, D] bf16 contiguous (channels-last frames), D = 1024 and inner 2048 in the Granite encoder but
 * any D in {256,512,1024,2048} with 2*inner % 256 == 0 works.  lengths: NULL or int32[B]: GLU frames
 * t >= lengths[b] are zeroed before the depthwise conv and its output there is zero, so valid frames equal the
 * module run on the trimmed utterance and padded frames of `out` equal x + b2.
 * workspace: device buffer of at least gsn_conv_module_workspace_bytes(B, T, D, inner) bytes, 256-byte aligned. */
size_t gsn_conv_module_workspace_bytes(int B, int T, int D, int inner);

int gsn_conv_module_bf16(const void* x, const void* ln_w, const void* ln_b, const void* w1_glu,
                         const float* b1_glu, const void* dw_w, const void* dw_b, const void* w2, const float* b2,
                         const int32_t* lengths, int add_residual, void* out, int B, int T, int D, int inner,
                         float ln_eps, void* workspace, size_t workspace_bytes, gsn_stream_t stream);

/* int8-weight module (w1q_glu [2*inner, D], w2q [D, inner] int8 with fp32 per-output-channel scales s1_glu, s2;
 * no reference code: the nearest is torchao W8A8 in bench_asr.py:92-105).  With workspace_bytes >=
 * gsn_conv_module_i8w_workspace_bytes(B, T, D, inner) both weight matrices are first widened to bf16 (exact
 * integers) inside the workspace and the GEMMs run on bf16 tiles at the bf16 tensor rate; with at least
 * gsn_conv_module_workspace_bytes(B, T, D, inner) the GEMMs widen each staged int8 W tile in shared memory
 * instead.  Both give bit-identical results. */
size_t gsn_conv_module_i8w_workspace_bytes(int B, int T, int D, int inner);

int gsn_conv_module_i8w(const void* x, const void* ln_w, const void* ln_b, const void* w1q_glu,
                        const float* s1_glu, const float* b1_glu, const void* dw_w, const void* dw_b,
                        const void* w2q, const float* s2, const float* b2, const int32_t* lengths,
                        int add_residual, void* out, int B, int T, int D, int inner, float ln_eps, void* workspace,
                        size_t workspace_bytes, gsn_stream_t stream);

/* The int8-weight module with the weights already widened to bf16 by the caller, once (w1w_glu, w2w: bf16 copies of
 * w1q_glu, w2q, exact since |q| <= 127); the GEMMs run on bf16 tiles with the per-output-channel scales, and the
 * constant weights are not widened again on every call.  Workspace: gsn_conv_module_workspace_bytes(B, T, D,
 * inner).  Bit-identical to gsn_conv_module_i8w.  No reference counterpart (see gsn_conv_module_i8w). */
int gsn_conv_module_i8w_widened(const void* x, const void* ln_w, const void* ln_b, const void* w1w_glu,
                                const float* s1_glu, const float* b1_glu, const void* dw_w, const void* dw_b,
                                const void* w2w, const float* s2, const float* b2, const int32_t* lengths,
                                int add_residual, void* out, int B, int T, int D, int inner, float ln_eps,
                                void* workspace, size_t workspace_bytes, gsn_stream_t stream);

/* W8A8 module: int8 weights (as for gsn_conv_module_i8w: w1q_glu [2*inner, D] GLU-interleaved, w2q [D, inner],
 * fp32 per-output-channel scales s1_glu, s2) and int8 activations: the LayerNorm output and the depthwise output
 * are quantised per row (gsn_quant_rows_bf16) and both pointwise GEMMs run kind::i8 tensor-core MMAs with s32
 * accumulation, scaled by row_scale[m] * col_scale[n] in the epilogue.  No reference code: the nearest is torchao's
 * W8A8 dynamic quantisation in bench_asr.py:92-105 (not vendored).  Workspace: at least
 * gsn_conv_module_w8a8_workspace_bytes(B, T, D, inner), 256-byte aligned. */
size_t gsn_conv_module_w8a8_workspace_bytes(int B, int T, int D, int inner);

int gsn_conv_module_w8a8(const void* x, const void* ln_w, const void* ln_b, const void* w1q_glu,
                         const float* s1_glu, const float* b1_glu, const void* dw_w, const void* dw_b,
                         const void* w2q, const float* s2, const float* b2, const int32_t* lengths, int add_residual,
                         void* out, int B, int T, int D, int inner, float ln_eps, void* workspace,
                         size_t workspace_bytes, gsn_stream_t stream);

/* Per-row symmetric int8 quantisation used by gsn_conv_module_w8a8 (no reference counterpart): for each row m of
 * x (bf16 [M, K], row stride ldx), scale[m] = max_k |x[m, k]| / 127 and q[m, k] = rint(x[m, k] / scale[m]) (IEEE
 * fp32 division, ties to even; q = 0 and scale = 0 for an all-zero row).  With lengths (M = B * T), rows of
 * padding frames get q = 0 and scale = 0.  q is int8 [M, K] dense.  K % 8 == 0, x rows 16-byte aligned. */
int gsn_quant_rows_bf16(const void* x, int64_t ldx, void* q, float* scale, int M, int K, const int32_t* lengths,
                        int T, gsn_stream_t stream);

/* ---- feed-forward halves of the Conformer block ---------------------------------------------------------------
 * Replace ConformerFeedForward (conformer.py:23-40: pre_norm -> up_proj -> SiLU -> down_proj) together with the
 * block's half-step residual x + 0.5 * ff(x) (conformer.py:205, :208).  Dropout is the identity (inference).
 * gsn_gemm_silu_bf16: h = silu(a W^T + b), a [M, K], W [N, K] bf16 (the Linear weight as stored), b [N] fp32;
 * lengths / T as for gsn_gemm1_glu_bf16: rows of pure-padding tiles are left unwritten, other padding rows are
 * written as zero (what a masked input gives).  K % 8, N % 256 == 0.
 * gsn_gemm_residual_scaled_bf16: out = out_scale * (d W^T + b) + residual (residual may be NULL), otherwise as
 * gsn_gemm2_residual_bf16.
 * gsn_ff_half_bf16: out = x + 0.5 * down(silu(up(layernorm(x)))) on x [B, T, D] bf16, w_up [F, D], w_down [D, F]
 * bf16, b_up [F], b_down [D] fp32, LayerNorm gamma / beta bf16; with lengths and T % 128 == 0, padded frames of
 * out are x + 0.5 * b_down.  Workspace: gsn_ff_half_workspace_bytes(B, T, D, F) bytes, 256-byte aligned. */
int gsn_gemm_silu_bf16(const void* a, const void* w, const float* b, void* h, int M, int K, int N,
                       const int32_t* lengths, int T, gsn_stream_t stream);

int gsn_gemm_residual_scaled_bf16(const void* d, const void* w, const float* b, const void* residual, int64_t ld_res,
                                  void* out, int64_t ld_out, int M, int K, int N, float out_scale,
                                  const int32_t* lengths, int T, gsn_stream_t stream);

size_t gsn_ff_half_workspace_bytes(int B, int T, int D, int F);

int gsn_ff_half_bf16(const void* x, const void* ln_w, const void* ln_b, const void* w_up, const float* b_up,
                     const void* w_down, const float* b_down, const int32_t* lengths, void* out, int B, int T, int D,
                     int F, float ln_eps, void* workspace, size_t workspace_bytes, gsn_stream_t stream);

/* ---- block-local attention with Shaw relative positions (ConformerAttention) --------------------------------
 * Replaces ConformerAttention.forward (models/granite_speech_nar/conformer.py:61-131) and, with the residual, the
 * attention step of ConformerBlock.forward (conformer.py:206): frames are cut into blocks of `context` frames; in
 * a block, head h of query i attends to the block's keys j with logits
 *   scale * (q_i . k_j) + scale * (q_i . rel[i - j + max_pos_emb])            (conformer.py:90-104, :114-128)
 * where rel is the rel_pos_emb table [n_rel = 2 max_pos_emb + 1, dim_head] (the reference's attention_dists,
 * conformer.py:254-262, index the same rows).  Keys past the frames are masked (conformer.py:108-112).  With
 * lengths, frames t >= lengths[b] are masked as keys too and get a zero context, so each utterance's result
 * equals the module run on the utterance alone; without lengths every one of the T frames takes part, as in the
 * reference.  Supported: dim_head 128, context 200 (the model's EncoderConfig), any even number of heads.
 * gsn_attention_core_bf16: the attention itself.  qkv [B, T, ld_qkv] bf16 rows hold q | k | v (each heads *
 * dim_head columns: to_q, then to_kv's two halves, conformer.py:81-82); ctx [B, T, ld_ctx] bf16 receives the
 * heads' outputs side by side (conformer.py:129).  ld_qkv, ld_ctx multiples of 8; 16-byte aligned pointers.
 * gsn_attention_block_bf16: out = x + to_out(attention(LayerNorm(x))) on x [B, T, D] bf16; w_qkv [3 inner, D] bf16
 * = [to_q.weight; to_kv.weight], b_qkv [3 inner] fp32 (zeros for the reference's bias-free projections), w_out
 * [D, inner] bf16, b_out [D] fp32, LayerNorm gamma / beta bf16.  With lengths and T % 128 == 0, padded frames of
 * out are x + b_out.  Without lengths every frame of x must be finite.
 * Workspace: gsn_attention_block_workspace_bytes(B, T, D, heads, dim_head) bytes, 256-byte aligned. */
int gsn_attention_core_bf16(const void* qkv, int64_t ld_qkv, const void* rel_table, int n_rel, void* ctx,
                            int64_t ld_ctx, const int32_t* lengths, int B, int T, int heads, int dim_head,
                            int context, int max_pos_emb, float scale, gsn_stream_t stream);

size_t gsn_attention_block_workspace_bytes(int B, int T, int D, int heads, int dim_head);

/* gsn_gemm_linear_bf16: out = a W^T + b (a [M, K] bf16, W [N, K] bf16, b [N] fp32, out rows of stride ld_out); with
 * lengths (T % 128 == 0, M a multiple of T) the 128-row tiles made only of padding frames are skipped and left
 * unwritten.  The q|k|v projection of the attention step, the encoder's input projection (K = 160).  K % 8,
 * N % 256 == 0. */
int gsn_gemm_linear_bf16(const void* a, const void* w, const float* b, void* out, int64_t ld_out, int M, int K, int N,
                         const int32_t* lengths, int T, gsn_stream_t stream);

int gsn_attention_block_bf16(const void* x, const void* ln_w, const void* ln_b, float ln_eps, const void* w_qkv,
                             const float* b_qkv, const void* w_out, const float* b_out, const void* rel_table,
                             int n_rel, const int32_t* lengths, void* out, int B, int T, int D, int heads,
                             int dim_head, int context, int max_pos_emb, void* workspace, size_t workspace_bytes,
                             gsn_stream_t stream);

/* ---- CTC heads ----------------------------------------------------------------------------------------------
 * The encoder's heads around the Conformer stack (models/granite_speech_nar/conformer.py:320-355) and the CTC
 * collapse of asr.py:76-102.  Frames are rows of [B, T, D] bf16; lengths (device int32 [B]) as elsewhere.
 * gsn_ctc_selfcond_bf16: the self-conditioning of the middle layer (conformer.py:320-324): logits = h W_out^T + b_out
 * over n_cls classes (bf16), p = softmax(float(logits)), blank[m] = p[m, 0] (fp32 [B*T]), h_out = h + bf16(p) W_mid^T
 * + b_mid.  w_out [round_up(n_cls, 256), D] bf16 with rows >= n_cls zero, b_out [round_up(n_cls, 256)] fp32; w_mid
 * [D, round_up(n_cls, 64)] bf16 with columns >= n_cls zero, b_mid [D] fp32; n_cls <= 512, D % 256 == 0.  Padding
 * frames (t >= lengths[b]) get blank = 1.  Workspace: gsn_ctc_selfcond_workspace_bytes(B, T, n_cls), 256-aligned.
 * gsn_bpe_pool_bf16: posterior_weighted_pool (conformer.py:214-226) with importance 1 - blank over windows of
 * `window` frames, frames t >= lengths[b] left out; pooled [B, Pp, D] bf16 (Pp >= ceil(T / window); pooled frames
 * past ceil(len / window) are zero), pooled_lengths[b] = ceil(len / window) (device int32 [B]).
 * gsn_bpe_head_ctc_bf16: the BPE head out_bpe (conformer.py:338-355) and its argmax + collapse (asr.py:123-134):
 * ids[b, p] = argmax_v bf16(pooled W_bpe^T + b_bpe) (lowest v among equal values; -1 past pooled_lengths[b]),
 * tokens[b, 0:counts[b]] = the collapsed ids (a new id or the utterance's first, and not blank_id), -1 after.  The logits
 * are never stored: the GEMM's epilogue keeps each row's best value.  w_bpe [V, D] bf16 (pad V to a multiple of
 * 256 with rows of zeros and b_bpe = -inf), b_bpe [V] fp32; Pp % 128 == 0; ids, tokens [B, Pp] int32, counts [B].
 * Workspace: gsn_bpe_head_workspace_bytes(B, Pp) bytes (one 64-bit key per pooled frame), 256-aligned. */
size_t gsn_ctc_selfcond_workspace_bytes(int B, int T, int n_cls);

int gsn_ctc_selfcond_bf16(const void* h, const void* w_out, const float* b_out, int n_cls, const void* w_mid,
                          const float* b_mid, const int32_t* lengths, void* h_out, float* blank, int B, int T, int D,
                          void* workspace, size_t workspace_bytes, gsn_stream_t stream);

int gsn_bpe_pool_bf16(const void* h, const float* blank, const int32_t* lengths, void* pooled, int32_t* pooled_lengths,
                      int B, int T, int D, int Pp, int window, gsn_stream_t stream);

size_t gsn_bpe_head_workspace_bytes(int B, int Pp);

int gsn_bpe_head_ctc_bf16(const void* pooled, const int32_t* pooled_lengths, const void* w_bpe, const float* b_bpe,
                          int V, int blank_id, int32_t* ids, int32_t* tokens, int32_t* counts, int B, int Pp, int D,
                          void* workspace, size_t workspace_bytes, gsn_stream_t stream);

/* ---- whole module without any allocation ------------------------------------------------------------------
 * No counterpart in the reference.  For callers that cannot allocate device memory where they run the module —
 * a plugin inside a host application that owns the GPU memory budget and its allocator, or a latency-critical
 * path where cudaMalloc / cudaFree would synchronise the device.  Same contract as gsn_conv_module_bf16 without
 * the workspace arguments: the scratch is a fixed array of GSN_NOALLOC_SCRATCH_BYTES (32 MiB) inside the
 * library's device image, held by every GPU that loads the library until the process exits, so a call needs
 * gsn_conv_module_workspace_bytes(B, T, D, inner) <= 32 MiB (at D = 1024, inner = 2048: B * T <= 4096 frames)
 * and larger problems are rejected with GSN_ERR_WORKSPACE.  Nothing is allocated, neither here nor per call.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) with that device
 * current, so make the first call on each device before any stream capture; that address is kept for the life of
 * the process, so resetting a device (cudaDeviceReset) after its first call is not supported.  Every call shares the one array:
 * calls that may overlap on the GPU (other streams, other host threads) race on it and must be serialised by the
 * caller.  The array keeps the previous call's contents; the module writes every scratch byte it reads, so
 * nothing needs clearing between calls. */
#define GSN_NOALLOC_SCRATCH_BYTES 33554432
int gsn_conv_module_bf16_noalloc(const void* x, const void* ln_w, const void* ln_b, const void* w1_glu,
                                 const float* b1_glu, const void* dw_w, const void* dw_b, const void* w2,
                                 const float* b2, const int32_t* lengths, int add_residual, void* out, int B, int T,
                                 int D, int inner, float ln_eps, gsn_stream_t stream);

/* ---- weight preparation --------------------------------------------------------------------------------
 * Device-to-device copy of `rows` x `row_bytes` with the GLU row interleave used by gsn_gemm1_*: output block j
 * (256 rows) = input rows [128 j, 128 j + 128) followed by rows [rows/2 + 128 j, rows/2 + 128 j + 128).
 * rows % 256 == 0.  Works for weights (row_bytes = K * elem), biases and scales (row_bytes = elem). */
int gsn_interleave_glu_rows(const void* src, void* dst, int rows, int64_t row_bytes, gsn_stream_t stream);

/* ---- failure detection ---------------------------------------------------------------------------------
 * Every spin-wait in these kernels is bounded (2 s); one that runs out records a code in a per-device status
 * word and the kernel unwinds.  gsn_device_status synchronises `stream`, returns the word in *status and
 * clears it when `clear` is non-zero.  gsn_selftest_bounded_wait launches one CTA that waits on an mbarrier
 * nothing will complete, with a limit of limit_ns (<= 2e9); the status word then reads 0x1FF. */
int gsn_device_status(int* status, int clear, gsn_stream_t stream);
int gsn_selftest_bounded_wait(uint64_t limit_ns, gsn_stream_t stream);

/* Test entry points for the unwind path of the production kernels (no reference counterpart).  Each launches the
 * kernel on the caller's operands with one TMA copy per CTA armed on its barrier but never issued, so a bounded
 * wait runs out (after 2 s) as it would if a copy never arrived:
 *   gsn_selftest_gemm_withheld_bf16: the down_conv + residual GEMM (operands as gsn_gemm2_residual_bf16, dense
 *     row strides, K >= 128), withholding each CTA's second operand load, so one K-block of MMAs has run into the
 *     TMEM accumulator when the MMA warp gives up;
 *   gsn_selftest_dwconv_withheld_bf16: the depthwise kernel (operands as gsn_dwconv_silu_bf16, without lengths),
 *     withholding each CTA's first tile; the layouts the TMA kernels take (channels-last rows, or T innermost with
 *     16-byte aligned rows and C % 64 == 0) exercise it.
 * Every role then unwinds: copies in flight land, TMEM is freed, the kernel returns, and gsn_device_status reads a
 * timeout code (0x101-0x104).  The output is left partly written; the context stays usable. */
int gsn_selftest_gemm_withheld_bf16(const void* d, const void* w, const float* b, const void* residual, void* out,
                                    int M, int K, int N, gsn_stream_t stream);
int gsn_selftest_dwconv_withheld_bf16(const void* x, const void* w, const void* b, void* y, int B, int C, int T,
                                      int64_t sxB, int64_t sxC, int64_t sxT, int64_t syB, int64_t syC, int64_t syT,
                                      gsn_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GSN_CONV_H_ */
