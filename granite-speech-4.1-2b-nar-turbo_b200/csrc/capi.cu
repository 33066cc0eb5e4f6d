// extern "C" entry points of libgsn_conv.so (declared in include/gsn_conv.h): argument checks, TMA descriptor
// encoding through the driver entry point, and the composite conv-module launch sequence.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "gsn_conv.h"
#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

#define GSN_VERSION 10000

namespace gsn {

namespace capi_impl {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = '\0';
  return GSN_OK;
}

int cuda_fail(int rc, const char* what) {
  return fail(GSN_ERR_CUDA, "%s: CUDA error %d (%s)", what, rc, cudaGetErrorString((cudaError_t)rc));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];

__global__ void wait_selftest_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // nothing ever arrives on `bar`: the bounded wait must give up, record the status and return
  mbar_wait_bounded(&bar, 0, &abort_flag, kStatusTimeoutSelftest, limit_ns);
  __syncthreads();
}

}  // namespace capi_impl
using namespace capi_impl;

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(GSN_ERR_DRIVER, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GSN_ERR_DRIVER, "cuTensorMapEncodeTiled failed with CUresult %d", (int)r);
  return 0;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  if (dev < kMaxDevices) {
    int c = g_sm_count[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int c = 0;
  if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
  if (dev < kMaxDevices) g_sm_count[dev].store(c, std::memory_order_relaxed);
  return c;
}

int launch_wait_selftest(uint64_t limit_ns, cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns);
  return (int)cudaGetLastError();
}

}  // namespace gsn

using namespace gsn;

namespace {

// a launcher status is either a GSN_* code already described in g_err, or a raw cudaError_t
int finish(int rc, const char* what) {
  if (rc == 0) return ok();
  if (rc == GSN_ERR_DRIVER) return rc;
  return cuda_fail(rc, what);
}

// returns -1 for a valid empty problem (nothing to launch), 0 to launch, or a GSN_ERR_* code
int check_dw(const void* x, const void* w, const void* b, const void* y, int B, int C, int T, int K) {
  if (B < 0 || C < 0 || T < 0) return fail(GSN_ERR_INVALID_ARG, "dwconv: negative size B=%d C=%d T=%d", B, C, T);
  if (K != 15) return fail(GSN_ERR_UNSUPPORTED, "dwconv: kernel size %d, only 15 is supported", K);
  if ((int64_t)B * C * T == 0) return -1;
  if (!x || !w || !b || !y) return fail(GSN_ERR_INVALID_ARG, "dwconv: null pointer");
  if (!aligned(x, 2) || !aligned(y, 2) || !aligned(w, 2) || !aligned(b, 2))
    return fail(GSN_ERR_UNSUPPORTED, "dwconv: bf16 pointers must be 2-byte aligned");
  return 0;
}

// returns -1 for a valid empty problem (M == 0), 0 to launch, or a GSN_ERR_* code
int check_gemm(const char* name, const void* a, const void* w, const float* bias, const void* out, int M, int K,
               int N) {
  if (M < 0 || K <= 0 || N <= 0) return fail(GSN_ERR_INVALID_ARG, "%s: bad sizes M=%d K=%d N=%d", name, M, K, N);
  if (K % 8 != 0) return fail(GSN_ERR_UNSUPPORTED, "%s: K=%d must be a multiple of 8 (16-byte rows)", name, K);
  if (N % 256 != 0) return fail(GSN_ERR_UNSUPPORTED, "%s: N=%d must be a multiple of 256", name, N);
  if (M == 0) return -1;
  if (!a || !w || !bias || !out) return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (!aligned(a, 16) || !aligned(w, 16) || !aligned(out, 16) || !aligned(bias, 16))
    return fail(GSN_ERR_UNSUPPORTED, "%s: pointers must be 16-byte aligned", name);
  return 0;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

bool ln_dim_ok(int D) { return D == 256 || D == 512 || D == 1024 || D == 2048; }

}  // namespace

extern "C" {

int gsn_version(void) { return GSN_VERSION; }

const char* gsn_last_error_string(void) { return g_err; }

int gsn_dwconv_silu_bf16(const void* x, const void* weight, const void* bias, void* y, int B, int C, int T, int K,
                         int64_t sxB, int64_t sxC, int64_t sxT, int64_t syB, int64_t syC, int64_t syT,
                         const int32_t* lengths, gsn_stream_t stream) {
  if (int rc = check_dw(x, weight, bias, y, B, C, T, K)) return rc < 0 ? ok() : rc;
  DwArgs a{(const __nv_bfloat16*)x, (const __nv_bfloat16*)weight, (const __nv_bfloat16*)bias, (__nv_bfloat16*)y,
           lengths, sxB, sxC, sxT, syB, syC, syT, B, C, T, 0};
  return finish(launch_dwconv(a, (cudaStream_t)stream), "gsn_dwconv_silu_bf16");
}

int gsn_dwconv_silu_glu_bf16(const void* x2, const void* weight, const void* bias, void* y, int B, int C, int T,
                             int K, int64_t sxB, int64_t sxC, int64_t sxT, int64_t syB, int64_t syC, int64_t syT,
                             const int32_t* lengths, gsn_stream_t stream) {
  if (int rc = check_dw(x2, weight, bias, y, B, C, T, K)) return rc < 0 ? ok() : rc;
  DwArgs a{(const __nv_bfloat16*)x2, (const __nv_bfloat16*)weight, (const __nv_bfloat16*)bias, (__nv_bfloat16*)y,
           lengths, sxB, sxC, sxT, syB, syC, syT, B, C, T, 1};
  return finish(launch_dwconv(a, (cudaStream_t)stream), "gsn_dwconv_silu_glu_bf16");
}

int gsn_layernorm_bf16(const void* x, int64_t ld_x, const void* gamma, const void* beta, void* y, int64_t ld_y,
                       int M, int D, float eps, const int32_t* lengths, int T, gsn_stream_t stream) {
  if (M < 0) return fail(GSN_ERR_INVALID_ARG, "layernorm: M=%d", M);
  if (!ln_dim_ok(D)) return fail(GSN_ERR_UNSUPPORTED, "layernorm: D=%d not in {256,512,1024,2048}", D);
  if (M == 0) return ok();
  if (!x || !gamma || !beta || !y) return fail(GSN_ERR_INVALID_ARG, "layernorm: null pointer");
  if (ld_x % 8 || ld_y % 8 || ld_x < D || ld_y < D || !aligned(x, 16) || !aligned(y, 16) || !aligned(gamma, 16) ||
      !aligned(beta, 16))
    return fail(GSN_ERR_UNSUPPORTED, "layernorm: rows must be 16-byte aligned (ld %% 8 == 0)");
  if (lengths && (T <= 0 || M % T != 0))
    return fail(GSN_ERR_UNSUPPORTED, "layernorm: with lengths, T=%d must divide M=%d", T, M);
  return finish(launch_layernorm((const __nv_bfloat16*)x, ld_x, (const __nv_bfloat16*)gamma,
                                 (const __nv_bfloat16*)beta, (__nv_bfloat16*)y, ld_y, M, D, eps, lengths, T,
                                 (cudaStream_t)stream),
                "gsn_layernorm_bf16");
}

// lengths != NULL: rows are M / T utterances of T frames (T % 128 == 0) and tiles of pure padding are skipped
static int check_lengths(const char* name, const int32_t* lengths, int T, int M) {
  if (!lengths) return 0;
  if (T <= 0 || T % 128 != 0 || M % T != 0)
    return fail(GSN_ERR_UNSUPPORTED, "%s: with lengths, T=%d must be a positive multiple of 128 dividing M=%d", name,
                T, M);
  return 0;
}

// i8: W is int8; scaled: the accumulator is multiplied by a per-column scale (int8 weights, staged as int8 or
// already widened to bf16)
static int gemm1(const void* a, const void* w, const float* scale, const float* b, void* h, int M, int K, int N,
                 const int32_t* lengths, int T, int i8, int scaled, gsn_stream_t stream, const char* name) {
  if (int rc = check_gemm(name, a, w, b, h, M, K, N)) return rc < 0 ? ok() : rc;
  if (scaled && (!scale || !aligned(scale, 16))) return fail(GSN_ERR_INVALID_ARG, "%s: scale pointer", name);
  if (int rc = check_lengths(name, lengths, T, M)) return rc;
  GemmArgs g{(const __nv_bfloat16*)a, w, b, scaled ? scale : nullptr, nullptr, (__nv_bfloat16*)h, (int64_t)(N / 2),
             0, M, N, K, i8, lengths, T};
  return finish(launch_gemm(g, kEpiGlu, (cudaStream_t)stream), name);
}

static int gemm2(const void* d, const void* w, const float* scale, const float* b, const void* res, int64_t ld_res,
                 void* out, int64_t ld_out, int M, int K, int N, const int32_t* lengths, int T, int i8,
                 int scaled, gsn_stream_t stream, const char* name, float* row_partials = nullptr) {
  if (int rc = check_gemm(name, d, w, b, out, M, K, N)) return rc < 0 ? ok() : rc;
  if (res && !aligned(res, 16)) return fail(GSN_ERR_UNSUPPORTED, "%s: residual must be 16-byte aligned", name);
  if (scaled && (!scale || !aligned(scale, 16))) return fail(GSN_ERR_INVALID_ARG, "%s: scale pointer", name);
  if (ld_out % 8 || ld_out < N || (res && (ld_res % 8 || ld_res < N)))
    return fail(GSN_ERR_UNSUPPORTED, "%s: row strides must be >= N and multiples of 8", name);
  if (int rc = check_lengths(name, lengths, T, M)) return rc;
  if (row_partials && (N % 256 || !aligned(row_partials, 8)))
    return fail(GSN_ERR_UNSUPPORTED, "%s: row partials need N %% 256 == 0 and 8-byte alignment", name);
  GemmArgs g{(const __nv_bfloat16*)d, w, b, scaled ? scale : nullptr, (const __nv_bfloat16*)res,
             (__nv_bfloat16*)out, ld_out, ld_res, M, N, K, i8, lengths, T};
  g.row_partials = (float2*)row_partials;
  return finish(launch_gemm(g, kEpiResidual, (cudaStream_t)stream), name);
}

int gsn_gemm1_glu_bf16(const void* a, const void* w1_glu, const float* b1_glu, void* h, int M, int K, int N,
                       const int32_t* lengths, int T, gsn_stream_t stream) {
  return gemm1(a, w1_glu, nullptr, b1_glu, h, M, K, N, lengths, T, 0, 0, stream, "gsn_gemm1_glu_bf16");
}

int gsn_gemm1_glu_i8w(const void* a, const void* w1q_glu, const float* s1_glu, const float* b1_glu, void* h, int M,
                      int K, int N, const int32_t* lengths, int T, gsn_stream_t stream) {
  return gemm1(a, w1q_glu, s1_glu, b1_glu, h, M, K, N, lengths, T, 1, 1, stream, "gsn_gemm1_glu_i8w");
}

int gsn_gemm1_glu_bf16s(const void* a, const void* w1_glu, const float* s1_glu, const float* b1_glu, void* h, int M,
                        int K, int N, const int32_t* lengths, int T, gsn_stream_t stream) {
  return gemm1(a, w1_glu, s1_glu, b1_glu, h, M, K, N, lengths, T, 0, 1, stream, "gsn_gemm1_glu_bf16s");
}

int gsn_gemm2_residual_bf16(const void* d, const void* w2, const float* b2, const void* residual, int64_t ld_res,
                            void* out, int64_t ld_out, int M, int K, int N, const int32_t* lengths, int T,
                            gsn_stream_t stream) {
  return gemm2(d, w2, nullptr, b2, residual, ld_res, out, ld_out, M, K, N, lengths, T, 0, 0, stream,
               "gsn_gemm2_residual_bf16");
}

int gsn_gemm2_residual_stats_bf16(const void* d, const void* w2, const float* b2, const void* residual,
                                  int64_t ld_res, void* out, int64_t ld_out, int M, int K, int N,
                                  const int32_t* lengths, int T, float* row_partials, gsn_stream_t stream) {
  if (!row_partials && M > 0) return fail(GSN_ERR_INVALID_ARG, "gsn_gemm2_residual_stats_bf16: null row_partials");
  return gemm2(d, w2, nullptr, b2, residual, ld_res, out, ld_out, M, K, N, lengths, T, 0, 0, stream,
               "gsn_gemm2_residual_stats_bf16", row_partials);
}

int gsn_gemm2_residual_i8w(const void* d, const void* w2q, const float* s2, const float* b2, const void* residual,
                           int64_t ld_res, void* out, int64_t ld_out, int M, int K, int N, const int32_t* lengths,
                           int T, gsn_stream_t stream) {
  return gemm2(d, w2q, s2, b2, residual, ld_res, out, ld_out, M, K, N, lengths, T, 1, 1, stream,
               "gsn_gemm2_residual_i8w");
}

int gsn_gemm2_residual_bf16s(const void* d, const void* w2, const float* s2, const float* b2, const void* residual,
                             int64_t ld_res, void* out, int64_t ld_out, int M, int K, int N, const int32_t* lengths,
                             int T, gsn_stream_t stream) {
  return gemm2(d, w2, s2, b2, residual, ld_res, out, ld_out, M, K, N, lengths, T, 0, 1, stream,
               "gsn_gemm2_residual_bf16s");
}

int gsn_gemm1_glu_dwconv_bf16(const void* a, const void* w1_glu, const float* s1_glu, const float* b1_glu,
                              const void* dw_w, const void* dw_b, void* d, int B, int T, int K, int N,
                              const int32_t* lengths, gsn_stream_t stream) {
  const char* name = "gsn_gemm1_glu_dwconv_bf16";
  if (B < 0 || T < 0 || K <= 0 || N <= 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d K=%d N=%d", name, B, T, K, N);
  if ((int64_t)B * T == 0) return ok();
  if ((int64_t)B * T > (int64_t)0x7fffffff) return fail(GSN_ERR_UNSUPPORTED, "%s: B*T too large", name);
  if (!a || !w1_glu || !b1_glu || !dw_w || !dw_b || !d) return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (T % 128 || K % 64 || N % 256)
    return fail(GSN_ERR_UNSUPPORTED, "%s: needs T %% 128 == 0, K %% 64 == 0, N %% 256 == 0 (T=%d K=%d N=%d)", name, T,
                K, N);
  if (!aligned(a, 16) || !aligned(w1_glu, 16) || !aligned(d, 16) || !aligned(b1_glu, 16) ||
      (s1_glu && !aligned(s1_glu, 16)) || !aligned(dw_w, 2) || !aligned(dw_b, 2))
    return fail(GSN_ERR_UNSUPPORTED, "%s: a, w1, d, b1, s1 must be 16-byte aligned", name);
  GemmDwArgs g{(const __nv_bfloat16*)a, (const __nv_bfloat16*)w1_glu, b1_glu, s1_glu, (const __nv_bfloat16*)dw_w,
               (const __nv_bfloat16*)dw_b, (__nv_bfloat16*)d, lengths, B, T, K, N};
  return finish(launch_gemm_glu_dw(g, (cudaStream_t)stream), name);
}

int gsn_gemm1_lnfold_glu_dwconv_bf16(const void* x, const void* w1g_glu, const float* b1g_glu, const float* c1_glu,
                                     const float* row_stats, const void* dw_w, const void* dw_b, void* d, int B,
                                     int T, int K, int N, const int32_t* lengths, gsn_stream_t stream) {
  const char* name = "gsn_gemm1_lnfold_glu_dwconv_bf16";
  if (B < 0 || T < 0 || K <= 0 || N <= 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d K=%d N=%d", name, B, T, K, N);
  if ((int64_t)B * T == 0) return ok();
  if ((int64_t)B * T > (int64_t)0x7fffffff) return fail(GSN_ERR_UNSUPPORTED, "%s: B*T too large", name);
  if (!x || !w1g_glu || !b1g_glu || !c1_glu || !row_stats || !dw_w || !dw_b || !d)
    return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (T % 128 || K % 64 || N % 256)
    return fail(GSN_ERR_UNSUPPORTED, "%s: needs T %% 128 == 0, K %% 64 == 0, N %% 256 == 0 (T=%d K=%d N=%d)", name, T,
                K, N);
  if (!aligned(x, 16) || !aligned(w1g_glu, 16) || !aligned(d, 16) || !aligned(b1g_glu, 16) || !aligned(c1_glu, 16) ||
      !aligned(row_stats, 8) || !aligned(dw_w, 2) || !aligned(dw_b, 2))
    return fail(GSN_ERR_UNSUPPORTED, "%s: x, w1g, d, b1g, c1 must be 16-byte aligned, row_stats 8-byte", name);
  GemmDwArgs g{(const __nv_bfloat16*)x, (const __nv_bfloat16*)w1g_glu, b1g_glu, nullptr, (const __nv_bfloat16*)dw_w,
               (const __nv_bfloat16*)dw_b, (__nv_bfloat16*)d, lengths, B, T, K, N, (const float2*)row_stats, c1_glu};
  return finish(launch_gemm_glu_dw(g, (cudaStream_t)stream), name);
}

int gsn_gemm1_lnfold_partials_glu_dwconv_bf16(const void* x, const void* w1g_glu, const float* b1g_glu,
                                              const float* c1_glu, const float* row_partials, float ln_eps,
                                              const void* dw_w, const void* dw_b, void* d, int B, int T, int K,
                                              int N, const int32_t* lengths, gsn_stream_t stream) {
  const char* name = "gsn_gemm1_lnfold_partials_glu_dwconv_bf16";
  if (B < 0 || T < 0 || K <= 0 || N <= 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d K=%d N=%d", name, B, T, K, N);
  if ((int64_t)B * T == 0) return ok();
  if ((int64_t)B * T > (int64_t)0x7fffffff) return fail(GSN_ERR_UNSUPPORTED, "%s: B*T too large", name);
  if (!x || !w1g_glu || !b1g_glu || !c1_glu || !row_partials || !dw_w || !dw_b || !d)
    return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (T % 128 || K % 256 || K > 2048 || N % 256)
    return fail(GSN_ERR_UNSUPPORTED, "%s: needs T %% 128 == 0, K %% 256 == 0, K <= 2048, N %% 256 == 0 (T=%d K=%d N=%d)",
                name, T, K, N);
  if (!aligned(x, 16) || !aligned(w1g_glu, 16) || !aligned(d, 16) || !aligned(b1g_glu, 16) || !aligned(c1_glu, 16) ||
      !aligned(row_partials, 8) || !aligned(dw_w, 2) || !aligned(dw_b, 2))
    return fail(GSN_ERR_UNSUPPORTED, "%s: x, w1g, d, b1g, c1 must be 16-byte aligned, row_partials 8-byte", name);
  GemmDwArgs g{(const __nv_bfloat16*)x, (const __nv_bfloat16*)w1g_glu, b1g_glu, nullptr, (const __nv_bfloat16*)dw_w,
               (const __nv_bfloat16*)dw_b, (__nv_bfloat16*)d, lengths, B, T, K, N, nullptr, c1_glu};
  g.row_partials = (const float2*)row_partials;
  g.ln_eps = ln_eps;
  return finish(launch_gemm_glu_dw(g, (cudaStream_t)stream), name);
}

int gsn_layernorm_stats_bf16(const void* x, int64_t ld_x, float* stats, int M, int D, float eps,
                             const int32_t* lengths, int T, gsn_stream_t stream) {
  const char* name = "gsn_layernorm_stats_bf16";
  if (M < 0) return fail(GSN_ERR_INVALID_ARG, "%s: M=%d", name, M);
  if (!ln_dim_ok(D)) return fail(GSN_ERR_UNSUPPORTED, "%s: D=%d not in {256,512,1024,2048}", name, D);
  if (M == 0) return ok();
  if (!x || !stats) return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (ld_x % 8 || ld_x < D || !aligned(x, 16) || !aligned(stats, 8))
    return fail(GSN_ERR_UNSUPPORTED, "%s: rows must be 16-byte aligned (ld %% 8 == 0), stats 8-byte", name);
  if (lengths && (T <= 0 || M % T != 0))
    return fail(GSN_ERR_UNSUPPORTED, "%s: with lengths, T=%d must divide M=%d", name, T, M);
  return finish(launch_ln_stats((const __nv_bfloat16*)x, ld_x, (float2*)stats, M, D, eps, lengths, T,
                                (cudaStream_t)stream),
                name);
}

int gsn_fold_layernorm_bf16(const void* w1_glu, const float* b1_glu, const void* ln_w, const void* ln_b,
                            void* w1g_glu, float* b1g_glu, float* c1_glu, int N, int K, gsn_stream_t stream) {
  const char* name = "gsn_fold_layernorm_bf16";
  if (N < 0 || K <= 0) return fail(GSN_ERR_INVALID_ARG, "%s: N=%d K=%d", name, N, K);
  if (N == 0) return ok();
  if (K % 256) return fail(GSN_ERR_UNSUPPORTED, "%s: K=%d must be a multiple of 256", name, K);
  if (!w1_glu || !b1_glu || !ln_w || !ln_b || !w1g_glu || !b1g_glu || !c1_glu)
    return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (!aligned(w1_glu, 16) || !aligned(ln_w, 16) || !aligned(ln_b, 16) || !aligned(w1g_glu, 16))
    return fail(GSN_ERR_UNSUPPORTED, "%s: weights and LayerNorm vectors must be 16-byte aligned", name);
  return finish(launch_fold_ln((const __nv_bfloat16*)w1_glu, b1_glu, (const __nv_bfloat16*)ln_w,
                               (const __nv_bfloat16*)ln_b, (__nv_bfloat16*)w1g_glu, b1g_glu, c1_glu, N, K,
                               (cudaStream_t)stream),
                name);
}

int gsn_widen_i8_bf16(const void* q0, void* out0, int64_t n0, const void* q1, void* out1, int64_t n1,
                      gsn_stream_t stream) {
  const char* name = "gsn_widen_i8_bf16";
  if (n0 < 0 || n1 < 0 || n0 % 16 || n1 % 16)
    return fail(GSN_ERR_INVALID_ARG, "%s: sizes %lld, %lld must be non-negative multiples of 16", name,
                (long long)n0, (long long)n1);
  if ((n0 && (!q0 || !out0)) || (n1 && (!q1 || !out1))) return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if ((n0 && (!aligned(q0, 16) || !aligned(out0, 16))) || (n1 && (!aligned(q1, 16) || !aligned(out1, 16))))
    return fail(GSN_ERR_UNSUPPORTED, "%s: pointers must be 16-byte aligned", name);
  return finish(launch_widen_i8(q0, out0, n0, q1, out1, n1, (cudaStream_t)stream), name);
}

int gsn_gemm_silu_bf16(const void* a, const void* w, const float* b, void* h, int M, int K, int N,
                       const int32_t* lengths, int T, gsn_stream_t stream) {
  const char* name = "gsn_gemm_silu_bf16";
  if (int rc = check_gemm(name, a, w, b, h, M, K, N)) return rc < 0 ? ok() : rc;
  if (int rc = check_lengths(name, lengths, T, M)) return rc;
  GemmArgs g{(const __nv_bfloat16*)a, w, b, nullptr, nullptr, (__nv_bfloat16*)h, (int64_t)N, 0, M, N, K, 0,
             lengths, T};
  return finish(launch_gemm(g, kEpiSilu, (cudaStream_t)stream), name);
}

int gsn_gemm_linear_bf16(const void* a, const void* w, const float* b, void* out, int64_t ld_out, int M, int K, int N,
                         const int32_t* lengths, int T, gsn_stream_t stream) {
  const char* name = "gsn_gemm_linear_bf16";
  if (int rc = check_gemm(name, a, w, b, out, M, K, N)) return rc < 0 ? ok() : rc;
  if (ld_out % 8 || ld_out < N) return fail(GSN_ERR_UNSUPPORTED, "%s: ld_out must be >= N and a multiple of 8", name);
  if (int rc = check_lengths(name, lengths, T, M)) return rc;
  GemmArgs g{(const __nv_bfloat16*)a, w, b, nullptr, nullptr, (__nv_bfloat16*)out, ld_out, 0, M, N, K, 0, lengths, T};
  return finish(launch_gemm(g, kEpiLinear, (cudaStream_t)stream), name);
}

int gsn_gemm_residual_scaled_bf16(const void* d, const void* w, const float* b, const void* residual, int64_t ld_res,
                                  void* out, int64_t ld_out, int M, int K, int N, float out_scale,
                                  const int32_t* lengths, int T, gsn_stream_t stream) {
  const char* name = "gsn_gemm_residual_scaled_bf16";
  if (int rc = check_gemm(name, d, w, b, out, M, K, N)) return rc < 0 ? ok() : rc;
  if (residual && !aligned(residual, 16)) return fail(GSN_ERR_UNSUPPORTED, "%s: residual must be 16-byte aligned", name);
  if (ld_out % 8 || ld_out < N || (residual && (ld_res % 8 || ld_res < N)))
    return fail(GSN_ERR_UNSUPPORTED, "%s: row strides must be >= N and multiples of 8", name);
  if (int rc = check_lengths(name, lengths, T, M)) return rc;
  GemmArgs g{(const __nv_bfloat16*)d, w, b, nullptr, (const __nv_bfloat16*)residual, (__nv_bfloat16*)out, ld_out,
             ld_res, M, N, K, 0, lengths, T, out_scale};
  return finish(launch_gemm(g, kEpiResidual, (cudaStream_t)stream), name);
}

size_t gsn_ff_half_workspace_bytes(int B, int T, int D, int F) {
  if (B <= 0 || T <= 0 || D <= 0 || F <= 0) return 0;
  const size_t M = (size_t)B * (size_t)T;
  return align256(M * (size_t)D * 2) + align256(M * (size_t)F * 2);
}

int gsn_ff_half_bf16(const void* x, const void* ln_w, const void* ln_b, const void* w_up, const float* b_up,
                     const void* w_down, const float* b_down, const int32_t* lengths, void* out, int B, int T, int D,
                     int F, float ln_eps, void* workspace, size_t workspace_bytes, gsn_stream_t stream) {
  const char* name = "gsn_ff_half_bf16";
  if (B < 0 || T < 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d", name, B, T);
  if ((int64_t)B * T == 0) return ok();
  if (!x || !ln_w || !ln_b || !w_up || !b_up || !w_down || !b_down || !out)
    return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (!ln_dim_ok(D) || F % 256 != 0)
    return fail(GSN_ERR_UNSUPPORTED, "%s: D=%d F=%d (D in {256..2048}, F %% 256 == 0)", name, D, F);
  if ((int64_t)B * T > (int64_t)0x7fffffff) return fail(GSN_ERR_UNSUPPORTED, "%s: B*T too large", name);
  const int M = B * T;
  const size_t need = gsn_ff_half_workspace_bytes(B, T, D, F);
  if (!workspace || workspace_bytes < need)
    return fail(GSN_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu required", name, workspace_bytes, need);
  if (!aligned(workspace, 256)) return fail(GSN_ERR_UNSUPPORTED, "%s: workspace must be 256-byte aligned", name);
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(w_up, 16) || !aligned(w_down, 16) || !aligned(b_up, 16) ||
      !aligned(b_down, 16))
    return fail(GSN_ERR_UNSUPPORTED, "%s: x, out, weights and biases must be 16-byte aligned", name);
  // workspace: t = LayerNorm output [M, D], then h = silu(t W_up^T + b_up) [M, F]
  __nv_bfloat16* t = (__nv_bfloat16*)workspace;
  __nv_bfloat16* h = (__nv_bfloat16*)((char*)workspace + align256((size_t)M * D * 2));
  const cudaStream_t st = (cudaStream_t)stream;
  const int32_t* skip = (lengths && T % 128 == 0) ? lengths : nullptr;
  int rc = launch_layernorm((const __nv_bfloat16*)x, D, (const __nv_bfloat16*)ln_w, (const __nv_bfloat16*)ln_b, t, D,
                            M, D, ln_eps, skip, T, st);
  if (rc) return finish(rc, name);
  GemmArgs g1{t, w_up, b_up, nullptr, nullptr, h, (int64_t)F, 0, M, F, D, 0, skip, T};
  rc = launch_gemm(g1, kEpiSilu, st);
  if (rc) return finish(rc, name);
  // the half-step residual of ConformerBlock.forward: out = x + 0.5 * (h W_down^T + b_down)
  GemmArgs g2{h, w_down, b_down, nullptr, (const __nv_bfloat16*)x, (__nv_bfloat16*)out, D, D, M, D, F, 0, skip, T,
              0.5f};
  return finish(launch_gemm(g2, kEpiResidual, st), name);
}

// ---- block-local Shaw attention ------------------------------------------------------------------------------
static int check_attention(const char* name, int heads, int dim_head, int context, int max_pos_emb, int n_rel) {
  if (dim_head != 128 || context != 200)
    return fail(GSN_ERR_UNSUPPORTED, "%s: dim_head=%d context=%d (only 128 and 200 are supported)", name, dim_head,
                context);
  if (heads <= 0) return fail(GSN_ERR_INVALID_ARG, "%s: heads=%d", name, heads);
  if (max_pos_emb < context || n_rel < max_pos_emb + context)
    return fail(GSN_ERR_INVALID_ARG, "%s: max_pos_emb=%d n_rel=%d (need max_pos_emb >= %d, n_rel >= max_pos_emb + %d)",
                name, max_pos_emb, n_rel, context, context);
  return 0;
}

int gsn_attention_core_bf16(const void* qkv, int64_t ld_qkv, const void* rel_table, int n_rel, void* ctx,
                            int64_t ld_ctx, const int32_t* lengths, int B, int T, int heads, int dim_head,
                            int context, int max_pos_emb, float scale, gsn_stream_t stream) {
  const char* name = "gsn_attention_core_bf16";
  if (B < 0 || T < 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d", name, B, T);
  if (int rc = check_attention(name, heads, dim_head, context, max_pos_emb, n_rel)) return rc;
  if ((int64_t)B * T == 0) return ok();
  if (!qkv || !rel_table || !ctx) return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  const int64_t inner = (int64_t)heads * dim_head;
  if (ld_qkv < 3 * inner || ld_qkv % 8 || ld_ctx < inner || ld_ctx % 8)
    return fail(GSN_ERR_UNSUPPORTED, "%s: ld_qkv=%lld (>= %lld) and ld_ctx=%lld (>= %lld) must be multiples of 8", name,
                (long long)ld_qkv, (long long)(3 * inner), (long long)ld_ctx, (long long)inner);
  if (!aligned(qkv, 16) || !aligned(ctx, 16) || !aligned(rel_table, 16))
    return fail(GSN_ERR_UNSUPPORTED, "%s: pointers must be 16-byte aligned", name);
  AttnArgs a{(const __nv_bfloat16*)qkv, ld_qkv, (const __nv_bfloat16*)rel_table, n_rel, (__nv_bfloat16*)ctx,
             ld_ctx, lengths, B, T, heads, max_pos_emb, scale};
  return finish(launch_attention(a, (cudaStream_t)stream), name);
}

size_t gsn_attention_block_workspace_bytes(int B, int T, int D, int heads, int dim_head) {
  if (B <= 0 || T <= 0 || D <= 0 || heads <= 0 || dim_head <= 0) return 0;
  const size_t M = (size_t)B * (size_t)T, inner = (size_t)heads * (size_t)dim_head;
  return align256(M * (size_t)D * 2) + align256(M * 3 * inner * 2) + align256(M * inner * 2);
}

int gsn_attention_block_bf16(const void* x, const void* ln_w, const void* ln_b, float ln_eps, const void* w_qkv,
                             const float* b_qkv, const void* w_out, const float* b_out, const void* rel_table,
                             int n_rel, const int32_t* lengths, void* out, int B, int T, int D, int heads,
                             int dim_head, int context, int max_pos_emb, void* workspace, size_t workspace_bytes,
                             gsn_stream_t stream) {
  const char* name = "gsn_attention_block_bf16";
  if (B < 0 || T < 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d", name, B, T);
  if (int rc = check_attention(name, heads, dim_head, context, max_pos_emb, n_rel)) return rc;
  if ((int64_t)B * T == 0) return ok();
  if (!x || !ln_w || !ln_b || !w_qkv || !b_qkv || !w_out || !b_out || !rel_table || !out)
    return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  const int inner = heads * dim_head;
  if (!ln_dim_ok(D) || (3 * inner) % 256 != 0)
    return fail(GSN_ERR_UNSUPPORTED, "%s: D=%d heads=%d (D in {256..2048}, heads even)", name, D, heads);
  if ((int64_t)B * T > (int64_t)0x7fffffff) return fail(GSN_ERR_UNSUPPORTED, "%s: B*T too large", name);
  const int M = B * T;
  const size_t need = gsn_attention_block_workspace_bytes(B, T, D, heads, dim_head);
  if (!workspace || workspace_bytes < need)
    return fail(GSN_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu required", name, workspace_bytes, need);
  if (!aligned(workspace, 256)) return fail(GSN_ERR_UNSUPPORTED, "%s: workspace must be 256-byte aligned", name);
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(w_qkv, 16) || !aligned(w_out, 16) || !aligned(b_qkv, 16) ||
      !aligned(b_out, 16) || !aligned(rel_table, 16) || !aligned(ln_w, 16) || !aligned(ln_b, 16))
    return fail(GSN_ERR_UNSUPPORTED, "%s: tensors must be 16-byte aligned", name);
  // workspace: t = LayerNorm output [M, D], qkv = t [Wq; Wkv]^T [M, 3 inner], ctx [M, inner]
  __nv_bfloat16* t = (__nv_bfloat16*)workspace;
  __nv_bfloat16* qkv = (__nv_bfloat16*)((char*)workspace + align256((size_t)M * D * 2));
  __nv_bfloat16* ctx = (__nv_bfloat16*)((char*)qkv + align256((size_t)M * 3 * inner * 2));
  const cudaStream_t st = (cudaStream_t)stream;
  const int32_t* skip = (lengths && T % 128 == 0) ? lengths : nullptr;
  // with lengths, padding frames are neither normalised nor projected (128-row tiles of pure padding are skipped):
  // the attention masks those keys and zeroes their V rows before use, and writes a zero context for them
  int rc = launch_layernorm((const __nv_bfloat16*)x, D, (const __nv_bfloat16*)ln_w, (const __nv_bfloat16*)ln_b, t, D,
                            M, D, ln_eps, skip, T, st);
  if (rc) return finish(rc, name);
  GemmArgs g1{t, w_qkv, b_qkv, nullptr, nullptr, qkv, (int64_t)3 * inner, 0, M, 3 * inner, D, 0, skip, T};
  rc = launch_gemm(g1, kEpiLinear, st);
  if (rc) return finish(rc, name);
  AttnArgs a{qkv, (int64_t)3 * inner, (const __nv_bfloat16*)rel_table, n_rel, ctx, (int64_t)inner, lengths, B, T,
             heads, max_pos_emb, 1.0f / sqrtf((float)dim_head)};
  rc = launch_attention(a, st);
  if (rc) return finish(rc, name);
  // to_out + the block's residual: out = x + ctx W_out^T + b_out
  GemmArgs g2{ctx, w_out, b_out, nullptr, (const __nv_bfloat16*)x, (__nv_bfloat16*)out, D, D, M, D, inner, 0, skip,
              T};
  return finish(launch_gemm(g2, kEpiResidual, st), name);
}

// ---- CTC heads ----------------------------------------------------------------------------------------------
static int round_up_i(int v, int g) { return (v + g - 1) / g * g; }

size_t gsn_ctc_selfcond_workspace_bytes(int B, int T, int n_cls) {
  if (B <= 0 || T <= 0 || n_cls <= 0) return 0;
  const size_t M = (size_t)B * (size_t)T;
  return align256(M * (size_t)round_up_i(n_cls, 256) * 2) + align256(M * (size_t)round_up_i(n_cls, 64) * 2);
}

int gsn_ctc_selfcond_bf16(const void* h, const void* w_out, const float* b_out, int n_cls, const void* w_mid,
                          const float* b_mid, const int32_t* lengths, void* h_out, float* blank, int B, int T, int D,
                          void* workspace, size_t workspace_bytes, gsn_stream_t stream) {
  const char* name = "gsn_ctc_selfcond_bf16";
  if (B < 0 || T < 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d", name, B, T);
  if (n_cls <= 0 || n_cls > 512) return fail(GSN_ERR_UNSUPPORTED, "%s: n_cls=%d (1..512)", name, n_cls);
  if (D <= 0 || D % 256) return fail(GSN_ERR_UNSUPPORTED, "%s: D=%d must be a multiple of 256", name, D);
  if ((int64_t)B * T == 0) return ok();
  if (!h || !w_out || !b_out || !w_mid || !b_mid || !h_out || !blank)
    return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if ((int64_t)B * T > (int64_t)0x7fffffff) return fail(GSN_ERR_UNSUPPORTED, "%s: B*T too large", name);
  const int M = B * T, n_pad = round_up_i(n_cls, 256), k_pad = round_up_i(n_cls, 64);
  const size_t need = gsn_ctc_selfcond_workspace_bytes(B, T, n_cls);
  if (!workspace || workspace_bytes < need)
    return fail(GSN_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu required", name, workspace_bytes, need);
  if (!aligned(workspace, 256) || !aligned(h, 16) || !aligned(h_out, 16) || !aligned(w_out, 16) ||
      !aligned(w_mid, 16) || !aligned(b_out, 16) || !aligned(b_mid, 16))
    return fail(GSN_ERR_UNSUPPORTED, "%s: tensors must be 16-byte aligned (workspace 256)", name);
  __nv_bfloat16* logits = (__nv_bfloat16*)workspace;
  __nv_bfloat16* probs = (__nv_bfloat16*)((char*)workspace + align256((size_t)M * n_pad * 2));
  const cudaStream_t st = (cudaStream_t)stream;
  const int32_t* skip = (lengths && T % 128 == 0) ? lengths : nullptr;
  GemmArgs g1{(const __nv_bfloat16*)h, w_out, b_out, nullptr, nullptr, logits, (int64_t)n_pad, 0, M, n_pad, D, 0, skip,
              T};
  int rc = launch_gemm(g1, kEpiLinear, st);
  if (rc) return finish(rc, name);
  rc = launch_ctc_softmax(logits, n_pad, probs, k_pad, blank, M, n_cls, k_pad, lengths, T, st);
  if (rc) return finish(rc, name);
  // h_out = h + probs W_mid^T + b_mid (conformer.py:324)
  GemmArgs g2{probs, w_mid, b_mid, nullptr, (const __nv_bfloat16*)h, (__nv_bfloat16*)h_out, D, D, M, D, k_pad, 0, skip,
              T};
  return finish(launch_gemm(g2, kEpiResidual, st), name);
}

int gsn_bpe_pool_bf16(const void* h, const float* blank, const int32_t* lengths, void* pooled, int32_t* pooled_lengths,
                      int B, int T, int D, int Pp, int window, gsn_stream_t stream) {
  const char* name = "gsn_bpe_pool_bf16";
  if (B < 0 || T < 0 || window < 1 || window > 8)
    return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d window=%d", name, B, T, window);
  if (D <= 0 || D % 256) return fail(GSN_ERR_UNSUPPORTED, "%s: D=%d must be a multiple of 256", name, D);
  if ((int64_t)B * T == 0) return ok();
  if (Pp < (T + window - 1) / window) return fail(GSN_ERR_INVALID_ARG, "%s: Pp=%d < ceil(T / window)", name, Pp);
  if (!h || !blank || !pooled || !pooled_lengths) return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (!aligned(h, 16) || !aligned(pooled, 16)) return fail(GSN_ERR_UNSUPPORTED, "%s: 16-byte alignment", name);
  return finish(launch_bpe_pool((const __nv_bfloat16*)h, blank, (__nv_bfloat16*)pooled, pooled_lengths, lengths, B, T,
                                D, Pp, window, (cudaStream_t)stream),
                name);
}

size_t gsn_bpe_head_workspace_bytes(int B, int Pp) {
  if (B <= 0 || Pp <= 0) return 0;
  return align256((size_t)B * (size_t)Pp * 8);
}

int gsn_bpe_head_ctc_bf16(const void* pooled, const int32_t* pooled_lengths, const void* w_bpe, const float* b_bpe,
                          int V, int blank_id, int32_t* ids, int32_t* tokens, int32_t* counts, int B, int Pp, int D,
                          void* workspace, size_t workspace_bytes, gsn_stream_t stream) {
  const char* name = "gsn_bpe_head_ctc_bf16";
  if (B < 0 || Pp < 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d Pp=%d", name, B, Pp);
  if (V <= 0 || V % 256 || D <= 0 || D % 64)
    return fail(GSN_ERR_UNSUPPORTED, "%s: V=%d (multiple of 256) D=%d (multiple of 64)", name, V, D);
  if ((int64_t)B * Pp == 0) return ok();
  if (Pp % 128) return fail(GSN_ERR_UNSUPPORTED, "%s: Pp=%d must be a multiple of 128", name, Pp);
  if (!pooled || !pooled_lengths || !w_bpe || !b_bpe || !ids || !tokens || !counts)
    return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if ((int64_t)B * Pp > (int64_t)0x7fffffff) return fail(GSN_ERR_UNSUPPORTED, "%s: B*Pp too large", name);
  const size_t need = gsn_bpe_head_workspace_bytes(B, Pp);
  if (!workspace || workspace_bytes < need)
    return fail(GSN_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu required", name, workspace_bytes, need);
  if (!aligned(workspace, 256) || !aligned(pooled, 16) || !aligned(w_bpe, 16) || !aligned(b_bpe, 16))
    return fail(GSN_ERR_UNSUPPORTED, "%s: tensors must be 16-byte aligned (workspace 256)", name);
  const cudaStream_t st = (cudaStream_t)stream;
  unsigned long long* keys = (unsigned long long*)workspace;
  cudaError_t e = cudaMemsetAsync(keys, 0, (size_t)B * Pp * 8, st);
  if (e != cudaSuccess) return cuda_fail((int)e, name);
  const int M = B * Pp;
  GemmArgs g{(const __nv_bfloat16*)pooled, w_bpe, b_bpe, nullptr, nullptr, nullptr, 0, 0, M, V, D, 0,
             pooled_lengths, Pp};
  g.argmax_keys = keys;
  g.n_major = 1;
  int rc = launch_gemm(g, kEpiArgmax, st);
  if (rc) return finish(rc, name);
  return finish(launch_ctc_collapse(keys, pooled_lengths, ids, tokens, counts, B, Pp, blank_id, st), name);
}

size_t gsn_conv_module_workspace_bytes(int B, int T, int D, int inner) {
  if (B <= 0 || T <= 0 || D <= 0 || inner <= 0) return 0;
  const size_t M = (size_t)B * (size_t)T;
  const size_t wide = (size_t)(inner > D ? inner : D);
  return align256(M * (size_t)inner * 2) + align256(M * wide * 2);
}

size_t gsn_conv_module_i8w_workspace_bytes(int B, int T, int D, int inner) {
  const size_t base = gsn_conv_module_workspace_bytes(B, T, D, inner);
  if (base == 0) return 0;
  return base + align256((size_t)2 * inner * D * 2) + align256((size_t)D * inner * 2);
}

static int conv_module(const void* x, const void* ln_w, const void* ln_b, const void* w1, const float* s1,
                       const float* b1, const void* dw_w, const void* dw_b, const void* w2, const float* s2,
                       const float* b2, const int32_t* lengths, int add_residual, void* out, int B, int T, int D,
                       int inner, float eps, void* ws, size_t ws_bytes, int i8, gsn_stream_t stream,
                       const char* name) {
  if (B < 0 || T < 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d", name, B, T);
  if ((int64_t)B * T == 0) return ok();
  if (!x || !ln_w || !ln_b || !w1 || !b1 || !dw_w || !dw_b || !w2 || !b2 || !out)
    return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (i8 && (!s1 || !s2)) return fail(GSN_ERR_INVALID_ARG, "%s: null scale pointer", name);
  if (!ln_dim_ok(D) || (2 * inner) % 256 != 0 || inner % 128 != 0)
    return fail(GSN_ERR_UNSUPPORTED, "%s: D=%d inner=%d (D in {256..2048}, inner %% 128 == 0)", name, D, inner);
  if ((int64_t)B * T > (int64_t)0x7fffffff) return fail(GSN_ERR_UNSUPPORTED, "%s: B*T too large", name);
  const int M = B * T;
  if (M == 0) return ok();
  const size_t need = gsn_conv_module_workspace_bytes(B, T, D, inner);
  if (!ws || ws_bytes < need)
    return fail(GSN_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu required", name, ws_bytes, need);
  if (!aligned(ws, 256)) return fail(GSN_ERR_UNSUPPORTED, "%s: workspace must be 256-byte aligned", name);
  if (!aligned(x, 16) || !aligned(out, 16)) return fail(GSN_ERR_UNSUPPORTED, "%s: x/out must be 16-byte aligned", name);

  // workspace: h = GLU output [M, inner]; t = LayerNorm output [M, D], later reused for the depthwise output
  // (with T on the 128 grid the GLU tensor is never materialised and the depthwise output takes h's place);
  // int8 weights with room for them: w1 and w2 widened to bf16 after that
  __nv_bfloat16* h = (__nv_bfloat16*)ws;
  __nv_bfloat16* t = (__nv_bfloat16*)((char*)ws + align256((size_t)M * inner * 2));
  const cudaStream_t st = (cudaStream_t)stream;
  // i8: 0 bf16 weights, 1 int8 weights, 2 int8 weights widened to bf16 once by the caller (scales still apply)
  int w_i8 = i8 == 1;
  if (i8 == 1 && ws_bytes >= gsn_conv_module_i8w_workspace_bytes(B, T, D, inner)) {
    if (!aligned(w1, 16) || !aligned(w2, 16))
      return fail(GSN_ERR_UNSUPPORTED, "%s: int8 weights must be 16-byte aligned", name);
    void* w1b = (char*)ws + need;
    void* w2b = (char*)w1b + align256((size_t)2 * inner * D * 2);
    int rc = launch_widen_i8(w1, w1b, (int64_t)2 * inner * D, w2, w2b, (int64_t)D * inner, st);
    if (rc) return finish(rc, name);
    w1 = w1b;
    w2 = w2b;
    w_i8 = 0;   // bf16 tiles from here on; the column scales stay
  }

  // with lengths and T on the 128-frame grid, 128-row tiles of pure padding skip the LayerNorm and GEMM work
  const int32_t* skip = (lengths && T % 128 == 0) ? lengths : nullptr;
  int rc = launch_layernorm((const __nv_bfloat16*)x, D, (const __nv_bfloat16*)ln_w, (const __nv_bfloat16*)ln_b, t, D,
                            M, D, eps, skip, T, st);
  if (rc) return finish(rc, name);
  // the depthwise input: d = the depthwise output, [M, inner]
  const __nv_bfloat16* dsrc = t;
  if (T % 128 == 0 && !w_i8) {
    // frames on the 128 grid: GLU and depthwise run inside the up_conv GEMM; d goes to h's place
    GemmDwArgs gd{t, (const __nv_bfloat16*)w1, b1, i8 ? s1 : nullptr, (const __nv_bfloat16*)dw_w,
                  (const __nv_bfloat16*)dw_b, h, lengths, B, T, D, 2 * inner};
    rc = launch_gemm_glu_dw(gd, st);
    if (rc) return finish(rc, name);
    dsrc = h;
  } else {
    GemmArgs g1{t, w1, b1, i8 ? s1 : nullptr, nullptr, h, (int64_t)inner, 0, M, 2 * inner, D, w_i8, skip, T};
    rc = launch_gemm(g1, kEpiGlu, st);
    if (rc) return finish(rc, name);
    DwArgs dw{h, (const __nv_bfloat16*)dw_w, (const __nv_bfloat16*)dw_b, t, lengths,
              (int64_t)T * inner, 1, inner, (int64_t)T * inner, 1, inner, B, inner, T, 0};
    rc = launch_dwconv(dw, st);
    if (rc) return finish(rc, name);
  }
  GemmArgs g2{dsrc, w2, b2, i8 ? s2 : nullptr, add_residual ? (const __nv_bfloat16*)x : nullptr,
              (__nv_bfloat16*)out, D, D, M, D, inner, w_i8, skip, T};
  rc = launch_gemm(g2, kEpiResidual, st);
  return finish(rc, name);
}

// The LayerNorm-folded module: row statistics (a launch, or the previous layer's row partials), the fused up_conv
// kernel, down_conv + residual (writing the next layer's row partials when stats_out is given).
static int lnfold_module(const void* x, const void* w1g_glu, const float* b1g_glu, const float* c1_glu,
                         const void* dw_w, const void* dw_b, const void* w2, const float* b2, const int32_t* lengths,
                         int add_residual, void* out, int B, int T, int D, int inner, float ln_eps,
                         const float* stats_in, float* stats_out, void* workspace, size_t workspace_bytes,
                         gsn_stream_t stream, const char* name) {
  if (B < 0 || T < 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d", name, B, T);
  if ((int64_t)B * T == 0) return ok();
  if (!x || !w1g_glu || !b1g_glu || !c1_glu || !dw_w || !dw_b || !w2 || !b2 || !out)
    return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (!ln_dim_ok(D) || (2 * inner) % 256 != 0 || inner % 128 != 0)
    return fail(GSN_ERR_UNSUPPORTED, "%s: D=%d inner=%d (D in {256..2048}, inner %% 128 == 0)", name, D, inner);
  if (T % 128) return fail(GSN_ERR_UNSUPPORTED, "%s: T=%d must be a multiple of 128", name, T);
  if ((int64_t)B * T > (int64_t)0x7fffffff) return fail(GSN_ERR_UNSUPPORTED, "%s: B*T too large", name);
  const int M = B * T;
  const size_t need = gsn_conv_module_workspace_bytes(B, T, D, inner);
  if (!workspace || workspace_bytes < need)
    return fail(GSN_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu required", name, workspace_bytes, need);
  if (!aligned(workspace, 256)) return fail(GSN_ERR_UNSUPPORTED, "%s: workspace must be 256-byte aligned", name);
  if (!aligned(x, 16) || !aligned(out, 16)) return fail(GSN_ERR_UNSUPPORTED, "%s: x/out must be 16-byte aligned", name);
  if ((stats_in && !aligned(stats_in, 8)) || (stats_out && !aligned(stats_out, 8)))
    return fail(GSN_ERR_UNSUPPORTED, "%s: row partials must be 8-byte aligned", name);
  // workspace: d = the depthwise output [M, inner], then the row statistics [M] x (rstd, rstd * mean)
  __nv_bfloat16* d = (__nv_bfloat16*)workspace;
  float2* stats = (float2*)((char*)workspace + align256((size_t)M * inner * 2));
  const cudaStream_t st = (cudaStream_t)stream;
  int rc = 0;
  if (!stats_in) {
    rc = launch_ln_stats((const __nv_bfloat16*)x, D, stats, M, D, ln_eps, lengths, T, st);
    if (rc) return finish(rc, name);
  }
  GemmDwArgs gd{(const __nv_bfloat16*)x, (const __nv_bfloat16*)w1g_glu, b1g_glu, nullptr, (const __nv_bfloat16*)dw_w,
                (const __nv_bfloat16*)dw_b, d, lengths, B, T, D, 2 * inner, stats_in ? nullptr : stats, c1_glu};
  gd.row_partials = (const float2*)stats_in;
  gd.ln_eps = ln_eps;
  rc = launch_gemm_glu_dw(gd, st);
  if (rc) return finish(rc, name);
  GemmArgs g2{d, w2, b2, nullptr, add_residual ? (const __nv_bfloat16*)x : nullptr, (__nv_bfloat16*)out, D, D, M, D,
              inner, 0, lengths, T};
  g2.row_partials = (float2*)stats_out;
  return finish(launch_gemm(g2, kEpiResidual, st), name);
}

int gsn_conv_module_lnfold_bf16(const void* x, const void* w1g_glu, const float* b1g_glu, const float* c1_glu,
                                const void* dw_w, const void* dw_b, const void* w2, const float* b2,
                                const int32_t* lengths, int add_residual, void* out, int B, int T, int D, int inner,
                                float ln_eps, void* workspace, size_t workspace_bytes, gsn_stream_t stream) {
  return lnfold_module(x, w1g_glu, b1g_glu, c1_glu, dw_w, dw_b, w2, b2, lengths, add_residual, out, B, T, D, inner,
                       ln_eps, nullptr, nullptr, workspace, workspace_bytes, stream, "gsn_conv_module_lnfold_bf16");
}

int gsn_conv_module_lnfold_chain_bf16(const void* x, const void* w1g_glu, const float* b1g_glu, const float* c1_glu,
                                      const void* dw_w, const void* dw_b, const void* w2, const float* b2,
                                      const int32_t* lengths, int add_residual, void* out, int B, int T, int D,
                                      int inner, float ln_eps, const float* stats_in, float* stats_out,
                                      void* workspace, size_t workspace_bytes, gsn_stream_t stream) {
  return lnfold_module(x, w1g_glu, b1g_glu, c1_glu, dw_w, dw_b, w2, b2, lengths, add_residual, out, B, T, D, inner,
                       ln_eps, stats_in, stats_out, workspace, workspace_bytes, stream,
                       "gsn_conv_module_lnfold_chain_bf16");
}

int gsn_conv_module_bf16(const void* x, const void* ln_w, const void* ln_b, const void* w1_glu,
                         const float* b1_glu, const void* dw_w, const void* dw_b, const void* w2, const float* b2,
                         const int32_t* lengths, int add_residual, void* out, int B, int T, int D, int inner,
                         float ln_eps, void* workspace, size_t workspace_bytes, gsn_stream_t stream) {
  return conv_module(x, ln_w, ln_b, w1_glu, nullptr, b1_glu, dw_w, dw_b, w2, nullptr, b2, lengths, add_residual, out,
                     B, T, D, inner, ln_eps, workspace, workspace_bytes, 0, stream, "gsn_conv_module_bf16");
}

int gsn_conv_module_i8w(const void* x, const void* ln_w, const void* ln_b, const void* w1q_glu,
                        const float* s1_glu, const float* b1_glu, const void* dw_w, const void* dw_b,
                        const void* w2q, const float* s2, const float* b2, const int32_t* lengths,
                        int add_residual, void* out, int B, int T, int D, int inner, float ln_eps, void* workspace,
                        size_t workspace_bytes, gsn_stream_t stream) {
  return conv_module(x, ln_w, ln_b, w1q_glu, s1_glu, b1_glu, dw_w, dw_b, w2q, s2, b2, lengths, add_residual, out, B,
                     T, D, inner, ln_eps, workspace, workspace_bytes, 1, stream, "gsn_conv_module_i8w");
}

int gsn_conv_module_i8w_widened(const void* x, const void* ln_w, const void* ln_b, const void* w1w_glu,
                                const float* s1_glu, const float* b1_glu, const void* dw_w, const void* dw_b,
                                const void* w2w, const float* s2, const float* b2, const int32_t* lengths,
                                int add_residual, void* out, int B, int T, int D, int inner, float ln_eps,
                                void* workspace, size_t workspace_bytes, gsn_stream_t stream) {
  return conv_module(x, ln_w, ln_b, w1w_glu, s1_glu, b1_glu, dw_w, dw_b, w2w, s2, b2, lengths, add_residual, out, B,
                     T, D, inner, ln_eps, workspace, workspace_bytes, 2, stream, "gsn_conv_module_i8w_widened");
}

int gsn_quant_rows_bf16(const void* x, int64_t ldx, void* q, float* scale, int M, int K, const int32_t* lengths,
                        int T, gsn_stream_t stream) {
  const char* name = "gsn_quant_rows_bf16";
  if (M < 0 || K <= 0) return fail(GSN_ERR_INVALID_ARG, "%s: M=%d K=%d", name, M, K);
  if (M == 0) return ok();
  if (!x || !q || !scale) return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (K % 8 || ldx < K || ldx % 8 || !aligned(x, 16) || !aligned(q, 8))
    return fail(GSN_ERR_UNSUPPORTED, "%s: K=%d ldx=%lld (K %% 8 == 0, 16-byte aligned rows)", name, K, (long long)ldx);
  if (lengths && (T <= 0 || M % T)) return fail(GSN_ERR_INVALID_ARG, "%s: lengths need M %% T == 0 (T=%d)", name, T);
  return finish(launch_quant_rows((const __nv_bfloat16*)x, ldx, (int8_t*)q, scale, M, K, lengths, T, 1,
                                  (cudaStream_t)stream), name);
}

size_t gsn_conv_module_w8a8_workspace_bytes(int B, int T, int D, int inner) {
  const size_t base = gsn_conv_module_workspace_bytes(B, T, D, inner);
  if (base == 0) return 0;
  const size_t M = (size_t)B * (size_t)T;
  const size_t wide = (size_t)(inner > D ? inner : D);
  return base + align256(M * wide) + align256(M * 4);
}

int gsn_conv_module_w8a8(const void* x, const void* ln_w, const void* ln_b, const void* w1q_glu,
                         const float* s1_glu, const float* b1_glu, const void* dw_w, const void* dw_b,
                         const void* w2q, const float* s2, const float* b2, const int32_t* lengths, int add_residual,
                         void* out, int B, int T, int D, int inner, float ln_eps, void* workspace,
                         size_t workspace_bytes, gsn_stream_t stream) {
  const char* name = "gsn_conv_module_w8a8";
  if (B < 0 || T < 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d", name, B, T);
  if ((int64_t)B * T == 0) return ok();
  if (!x || !ln_w || !ln_b || !w1q_glu || !s1_glu || !b1_glu || !dw_w || !dw_b || !w2q || !s2 || !b2 || !out)
    return fail(GSN_ERR_INVALID_ARG, "%s: null pointer", name);
  if (!ln_dim_ok(D) || (2 * inner) % 256 != 0 || inner % 128 != 0)
    return fail(GSN_ERR_UNSUPPORTED, "%s: D=%d inner=%d (D in {256..2048}, inner %% 128 == 0)", name, D, inner);
  if ((int64_t)B * T > (int64_t)0x7fffffff) return fail(GSN_ERR_UNSUPPORTED, "%s: B*T too large", name);
  const int M = B * T;
  const size_t need = gsn_conv_module_w8a8_workspace_bytes(B, T, D, inner);
  if (!workspace || workspace_bytes < need)
    return fail(GSN_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu required", name, workspace_bytes, need);
  if (!aligned(workspace, 256)) return fail(GSN_ERR_UNSUPPORTED, "%s: workspace must be 256-byte aligned", name);
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(w1q_glu, 16) || !aligned(w2q, 16))
    return fail(GSN_ERR_UNSUPPORTED, "%s: x, out and the int8 weights must be 16-byte aligned", name);

  // workspace: h = GLU output [M, inner] bf16; t = the depthwise output [M, inner] bf16; q = int8 activations
  // [M, max(D, inner)] (the LayerNorm output quantised in the LayerNorm pass, then the depthwise output); rs = their
  // per-row scales [M]
  const size_t wide = (size_t)(inner > D ? inner : D);
  __nv_bfloat16* h = (__nv_bfloat16*)workspace;
  __nv_bfloat16* t = (__nv_bfloat16*)((char*)workspace + align256((size_t)M * inner * 2));
  int8_t* q = (int8_t*)((char*)t + align256((size_t)M * wide * 2));
  float* rs = (float*)((char*)q + align256((size_t)M * wide));
  const cudaStream_t st = (cudaStream_t)stream;
  const int32_t* skip = (lengths && T % 128 == 0) ? lengths : nullptr;

  int rc = launch_layernorm_quant((const __nv_bfloat16*)x, D, (const __nv_bfloat16*)ln_w, (const __nv_bfloat16*)ln_b,
                                  q, rs, M, D, ln_eps, lengths, T, 0, st);
  if (rc) return finish(rc, name);
  if (T % 128 == 0 && D % 128 == 0) {
    // frames on the 128 grid: GLU, depthwise and SiLU run inside the kind::i8 up_conv GEMM (the GLU tensor is never
    // written); t receives the depthwise output
    GemmDwArgs gd{(const __nv_bfloat16*)q, (const __nv_bfloat16*)w1q_glu, b1_glu, s1_glu, (const __nv_bfloat16*)dw_w,
                  (const __nv_bfloat16*)dw_b, t, lengths, B, T, D, 2 * inner};
    gd.a_int8 = 1;
    gd.row_scale = rs;
    rc = launch_gemm_glu_dw(gd, st);
    if (rc) return finish(rc, name);
  } else {
    GemmArgs g1{(const __nv_bfloat16*)q, w1q_glu, b1_glu, s1_glu, nullptr, h, (int64_t)inner, 0, M, 2 * inner, D, 1,
                skip, T};
    g1.a_int8 = 1;
    g1.row_scale = rs;
    rc = launch_gemm(g1, kEpiGlu, st);
    if (rc) return finish(rc, name);
    DwArgs dw{h, (const __nv_bfloat16*)dw_w, (const __nv_bfloat16*)dw_b, t, lengths,
              (int64_t)T * inner, 1, inner, (int64_t)T * inner, 1, inner, B, inner, T, 0};
    rc = launch_dwconv(dw, st);
    if (rc) return finish(rc, name);
  }
  // padding rows: only their zero scale (the GEMMs multiply those rows' sums by it or mask them)
  rc = launch_quant_rows(t, inner, q, rs, M, inner, lengths, T, 0, st);
  if (rc) return finish(rc, name);
  GemmArgs g2{(const __nv_bfloat16*)q, w2q, b2, s2, add_residual ? (const __nv_bfloat16*)x : nullptr,
              (__nv_bfloat16*)out, D, D, M, D, inner, 1, skip, T};
  g2.a_int8 = 1;
  g2.row_scale = rs;
  rc = launch_gemm(g2, kEpiResidual, st);
  return finish(rc, name);
}

}  // extern "C"

// ---- whole module with library-owned scratch -------------------------------------------------------------------
// Some callers cannot allocate device memory at the point where they run the module: a plugin inside a host
// application that owns the GPU memory budget and its allocator, or a latency-critical path where cudaMalloc /
// cudaFree would synchronise the device.  For them the workspace of the module lives in this fixed array, part of
// the library's device image: every GPU that loads the library holds it until the process exits, and nothing is
// allocated per call.  Host code must not pass the array's name to a kernel (it is a host-side stand-in, not a
// device address); the device address is fetched once per device with cudaGetSymbolAddress.
namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[GSN_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (set-up on the first call per device).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail((int)e, "gsn_conv_module_bf16_noalloc (cudaGetDevice)");
  if (dev < 0 || dev >= kMaxDevices) return fail(GSN_ERR_UNSUPPORTED, "noalloc: device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return cuda_fail((int)(e != cudaSuccess ? e : cudaErrorInvalidSymbol),
                       "gsn_conv_module_bf16_noalloc (cudaGetSymbolAddress of the static scratch)");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace

extern "C" {

int gsn_conv_module_bf16_noalloc(const void* x, const void* ln_w, const void* ln_b, const void* w1_glu,
                                 const float* b1_glu, const void* dw_w, const void* dw_b, const void* w2,
                                 const float* b2, const int32_t* lengths, int add_residual, void* out, int B, int T,
                                 int D, int inner, float ln_eps, gsn_stream_t stream) {
  const char* name = "gsn_conv_module_bf16_noalloc";
  if (B < 0 || T < 0) return fail(GSN_ERR_INVALID_ARG, "%s: B=%d T=%d", name, B, T);
  if ((int64_t)B * T == 0) return ok();
  // the same shape rule as the workspace entry point, checked first so an unsupported D or inner is reported as
  // such rather than as a scratch-size problem
  if (!ln_dim_ok(D) || (2 * inner) % 256 != 0 || inner % 128 != 0)
    return fail(GSN_ERR_UNSUPPORTED, "%s: D=%d inner=%d (D in {256..2048}, inner %% 128 == 0)", name, D, inner);
  const size_t need = gsn_conv_module_workspace_bytes(B, T, D, inner);
  if (need > (size_t)GSN_NOALLOC_SCRATCH_BYTES)
    return fail(GSN_ERR_WORKSPACE,
                "%s: B=%d T=%d D=%d inner=%d needs %zu bytes of scratch, above the library's static %d bytes "
                "(at D=1024, inner=2048 at most %d frames per call); use gsn_conv_module_bf16 with a caller "
                "workspace",
                name, B, T, D, inner, need, GSN_NOALLOC_SCRATCH_BYTES, GSN_NOALLOC_SCRATCH_BYTES / 8192);
  void* ws = nullptr;
  if (int rc = noalloc_scratch(&ws)) return rc;
  return conv_module(x, ln_w, ln_b, w1_glu, nullptr, b1_glu, dw_w, dw_b, w2, nullptr, b2, lengths, add_residual, out,
                     B, T, D, inner, ln_eps, ws, (size_t)GSN_NOALLOC_SCRATCH_BYTES, 0, stream, name);
}

int gsn_interleave_glu_rows(const void* src, void* dst, int rows, int64_t row_bytes, gsn_stream_t stream) {
  if (!src || !dst) return fail(GSN_ERR_INVALID_ARG, "interleave: null pointer");
  if (rows <= 0 || rows % 256 != 0 || row_bytes <= 0)
    return fail(GSN_ERR_UNSUPPORTED, "interleave: rows=%d must be a positive multiple of 256", rows);
  const int half = rows / 2;
  const size_t blk = (size_t)128 * (size_t)row_bytes;
  for (int j = 0; j < rows / 256; ++j) {
    const char* s = (const char*)src;
    char* d = (char*)dst + (size_t)j * 2 * blk;
    cudaError_t e = cudaMemcpyAsync(d, s + (size_t)j * blk, blk, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(d + blk, s + ((size_t)half + (size_t)j * 128) * (size_t)row_bytes, blk,
                          cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail((int)e, "gsn_interleave_glu_rows");
  }
  return ok();
}

int gsn_device_status(int* status, int clear, gsn_stream_t stream) {
  if (!status) return fail(GSN_ERR_INVALID_ARG, "device_status: null pointer");
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail((int)e, "gsn_device_status (stream sync)");
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, gsn::g_device_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail((int)e, "gsn_device_status (read)");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(gsn::g_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail((int)e, "gsn_device_status (clear)");
  }
  *status = v;
  return ok();
}

int gsn_selftest_bounded_wait(uint64_t limit_ns, gsn_stream_t stream) {
  if (limit_ns == 0 || limit_ns > 2000000000ull)
    return fail(GSN_ERR_INVALID_ARG, "selftest: limit_ns must be in (0, 2e9]");
  return finish(launch_wait_selftest(limit_ns, (cudaStream_t)stream), "gsn_selftest_bounded_wait");
}

int gsn_selftest_gemm_withheld_bf16(const void* d, const void* w, const float* b, const void* residual, void* out,
                                    int M, int K, int N, gsn_stream_t stream) {
  const char* name = "gsn_selftest_gemm_withheld_bf16";
  if (int rc = check_gemm(name, d, w, b, out, M, K, N)) return rc < 0 ? ok() : rc;
  if (residual && !aligned(residual, 16)) return fail(GSN_ERR_UNSUPPORTED, "%s: residual must be 16-byte aligned", name);
  if (K < 128) return fail(GSN_ERR_UNSUPPORTED, "%s: K=%d must span at least two 64-wide K-blocks", name, K);
  GemmArgs g{(const __nv_bfloat16*)d, w, b, nullptr, (const __nv_bfloat16*)residual, (__nv_bfloat16*)out,
             (int64_t)N, (int64_t)N, M, N, K, 0, nullptr, 0};
  g.withhold_load = 1;    // every CTA's second operand load: one K-block of MMAs has run when the wait runs out
  return finish(launch_gemm(g, kEpiResidual, (cudaStream_t)stream), name);
}

int gsn_selftest_dwconv_withheld_bf16(const void* x, const void* w, const void* b, void* y, int B, int C, int T,
                                      int64_t sxB, int64_t sxC, int64_t sxT, int64_t syB, int64_t syC, int64_t syT,
                                      gsn_stream_t stream) {
  const char* name = "gsn_selftest_dwconv_withheld_bf16";
  if (int rc = check_dw(x, w, b, y, B, C, T, 15)) return rc < 0 ? ok() : rc;
  DwArgs a{(const __nv_bfloat16*)x, (const __nv_bfloat16*)w, (const __nv_bfloat16*)b, (__nv_bfloat16*)y, nullptr,
           sxB, sxC, sxT, syB, syC, syT, B, C, T, 0};
  a.withhold_tile = 0;    // every CTA's first tile
  return finish(launch_dwconv(a, (cudaStream_t)stream), name);
}

}  // extern "C"
