// Depthwise Conv1d k=15 (+ folded BatchNorm bias) + SiLU on sm_100a, optionally with the GLU in front.
//
// Semantics (script/cuda_kernels/conv1d.py:21-42, and the GLU form conv1d.py:52-79):
//   y[b, c, t] = silu(bias[c] + sum_{j<15} w[c, j] * x[b, c, t - 7 + j]),   x = 0 outside [0, T)
//   GLU form:   x[b, c, t] = bf16(a[b, c, t] * sigmoid(g[b, c, t])), a = channels [0, C), g = channels [C, 2C)
// plus per-utterance lengths (not in the reference op): frames t >= len[b] read as zero and are written as zero.
// Accumulation is fp32 and the output is rounded to bf16 once, as in the reference kernel.
//
// Two layouts:
//  * channels-last (element stride of C is 1; the conv-module layout [B, T, C]): a CTA owns 128 channels of one
//    utterance and walks 4 time tiles of 64 frames.  Each tile plus its 7-frame halo on both sides (78 rows x 256
//    bytes) is staged in shared memory by a 3-D TMA load; out-of-range frames (t < 0, t >= T) arrive zero-filled.
//    Two stages: the TMA for tile i+2 is issued as soon as tile i has been consumed.  A warp owns 16 output
//    frames, a lane 4 channels (8-byte shared-memory rows, conflict-free), with the 60 weights in registers and
//    packed fp32x2 FMAs.
//  * channels-first (element stride of T is 1; the layout the reference op receives from up_conv): a CTA owns 32
//    channels x 128 frames, stages the rows (plus halo) in shared memory as fp32 with plain coalesced loads
//    (row strides need not be 16-byte multiples there, e.g. T = 37), and transposes the result through shared
//    memory for coalesced stores.
#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

namespace gsn {

namespace dw_impl {

constexpr int KW = 15;
constexpr int HALO = 7;

// ----------------------------------------------------------------------------------------------------------------
// channels-last
constexpr int CL_CC = 128;                // channels per CTA
constexpr int CL_TT = 64;                 // output frames per tile
constexpr int CL_ROWS = CL_TT + 2 * HALO; // 78 staged rows
constexpr int CL_THREADS = 128;           // 4 warps x 16 frames
constexpr int CL_FPW = CL_TT / 4;         // frames per warp
constexpr int CL_TILES = 4;               // tiles per CTA
constexpr int CL_ROW_BYTES = CL_CC * 2;
constexpr int CL_TILE_BYTES = CL_ROWS * CL_ROW_BYTES;  // 19968

template <bool GLU>
struct __align__(128) ClSmem {
  uint8_t x[2][GLU ? 2 : 1][CL_TILE_BYTES];
  uint64_t full[2];
  int abort_flag;
};

struct ClParams {
  const __nv_bfloat16* w;
  const __nv_bfloat16* bias;
  __nv_bfloat16* y;
  const int* lengths;
  int64_t syB, syT;
  int T, C;
};

__device__ __forceinline__ float2 bf16x2_to_f2(uint32_t v) { return make_float2(bf16lo_to_f32(v), bf16hi_to_f32(v)); }

// GLU of one packed bf16 pair, rounded to bf16 and widened back (conv1d.py:70-73 rounds the product to bf16)
__device__ __forceinline__ float2 glu_pair(uint32_t a, uint32_t g) {
  const float a0 = bf16lo_to_f32(a), a1 = bf16hi_to_f32(a);
  const float g0 = bf16lo_to_f32(g), g1 = bf16hi_to_f32(g);
  const uint32_t r = pack_bf16x2(a0 * sigmoid_fast(g0), a1 * sigmoid_fast(g1));
  return bf16x2_to_f2(r);
}

template <bool GLU>
__global__ void __launch_bounds__(CL_THREADS, 3)
    dwconv_cl_kernel(const __grid_constant__ CUtensorMap tmX, ClParams p) {
  extern __shared__ uint8_t smem_raw[];
  ClSmem<GLU>& s = *reinterpret_cast<ClSmem<GLU>*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int c0 = blockIdx.x * CL_CC;
  const int b = blockIdx.z;
  const int t_begin = blockIdx.y * (CL_TT * CL_TILES);
  const int T = p.T;
  int n_tiles = (T - t_begin + CL_TT - 1) / CL_TT;
  if (n_tiles > CL_TILES) n_tiles = CL_TILES;
  const int len = p.lengths ? min(max(__ldg(p.lengths + b), 0), T) : T;
  constexpr uint32_t kTxBytes = (GLU ? 2 : 1) * CL_TILE_BYTES;

  if (tid == 0) {
    mbar_init(&s.full[0], 1);
    mbar_init(&s.full[1], 1);
    s.abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
  }
  __syncthreads();

  auto issue = [&](int i) {
    const int st = i & 1;
    const int t_in = t_begin + i * CL_TT - HALO;
    mbar_arrive_expect_tx(&s.full[st], kTxBytes);
    tma_load_3d(s.x[st][0], &tmX, &s.full[st], c0, t_in, b);
    if (GLU) tma_load_3d(s.x[st][GLU ? 1 : 0], &tmX, &s.full[st], c0 + p.C, t_in, b);
  };
  if (tid == 0) {
    if (n_tiles > 0) issue(0);
    if (n_tiles > 1) issue(1);
  }

  // weights of this lane's 4 channels, as fp32 pairs: wr[j][0] = (c, c+1), wr[j][1] = (c+2, c+3)
  const int cl = c0 + lane * 4;
  float2 wr[KW][2];
  {
    const __nv_bfloat16* wp = p.w + (int64_t)cl * KW;
#pragma unroll
    for (int j = 0; j < KW; ++j) {
      wr[j][0] = make_float2(__bfloat162float(wp[j]), __bfloat162float(wp[KW + j]));
      wr[j][1] = make_float2(__bfloat162float(wp[2 * KW + j]), __bfloat162float(wp[3 * KW + j]));
    }
  }
  const float2 bias01 = make_float2(__bfloat162float(p.bias[cl]), __bfloat162float(p.bias[cl + 1]));
  const float2 bias23 = make_float2(__bfloat162float(p.bias[cl + 2]), __bfloat162float(p.bias[cl + 3]));

  bool alive = true;
  for (int i = 0; i < n_tiles; ++i) {
    const int st = i & 1;
    if (alive) alive = mbar_wait_bounded(&s.full[st], (uint32_t)((i >> 1) & 1), &s.abort_flag, kStatusTimeoutDw);
    const int t0 = t_begin + i * CL_TT;
    if (alive) {
      float2 acc[CL_FPW][2];
#pragma unroll
      for (int f = 0; f < CL_FPW; ++f) {
        acc[f][0] = bias01;
        acc[f][1] = bias23;
      }
      const int row0 = warp * CL_FPW;                // first staged row read by this warp
      const int t_row0 = t0 - HALO + row0;           // its frame index
      const uint8_t* xa = s.x[st][0] + row0 * CL_ROW_BYTES + lane * 8;
      const uint8_t* xg = s.x[st][GLU ? 1 : 0] + row0 * CL_ROW_BYTES + lane * 8;
#pragma unroll
      for (int r = 0; r < CL_FPW + 2 * HALO; ++r) {
        float2 x01, x23;
        const uint2 va = *reinterpret_cast<const uint2*>(xa + r * CL_ROW_BYTES);
        if (GLU) {
          const uint2 vg = *reinterpret_cast<const uint2*>(xg + r * CL_ROW_BYTES);
          x01 = glu_pair(va.x, vg.x);
          x23 = glu_pair(va.y, vg.y);
        } else {
          x01 = bf16x2_to_f2(va.x);
          x23 = bf16x2_to_f2(va.y);
        }
        if (t_row0 + r >= len) {  // frames past the utterance read as zero (t >= T is zero-filled by TMA)
          x01 = make_float2(0.f, 0.f);
          x23 = make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int f = 0; f < CL_FPW; ++f) {
          const int j = r - f;
          if (j >= 0 && j < KW) {
            acc[f][0] = ffma2(wr[j][0], x01, acc[f][0]);
            acc[f][1] = ffma2(wr[j][1], x23, acc[f][1]);
          }
        }
      }
      __nv_bfloat16* yb = p.y + (int64_t)b * p.syB + cl;
#pragma unroll
      for (int f = 0; f < CL_FPW; ++f) {
        const int t = t0 + row0 + f;
        if (t < T) {
          uint2 o;
          if (t < len) {
            o.x = pack_bf16x2(silu_fast(acc[f][0].x), silu_fast(acc[f][0].y));
            o.y = pack_bf16x2(silu_fast(acc[f][1].x), silu_fast(acc[f][1].y));
          } else {
            o.x = 0u;
            o.y = 0u;
          }
          *reinterpret_cast<uint2*>(yb + (int64_t)t * p.syT) = o;
        }
      }
    }
    __syncthreads();  // stage st fully consumed by every warp
    if (tid == 0 && alive && !s.abort_flag && i + 2 < n_tiles) {
      fence_proxy_async_smem();
      issue(i + 2);
    }
  }
  if (tid == 0 && s.abort_flag) {
    // unwinding after a timeout: let outstanding copies land before the shared memory is released
    for (int i = n_tiles - 2; i < n_tiles; ++i)
      if (i >= 0) mbar_wait_bounded(&s.full[i & 1], (uint32_t)((i >> 1) & 1), nullptr, kStatusTimeoutDw, 100000000ull);
  }
}

// ----------------------------------------------------------------------------------------------------------------
// channels-first
constexpr int CF_CC = 32;                   // channels per CTA
constexpr int CF_TT = 128;                  // output frames per CTA
constexpr int CF_W = CF_TT + 2 * HALO;      // 142 staged frames per channel
constexpr int CF_PITCH = CF_W + 1;          // odd pitch: conflict-free column reads
constexpr int CF_THREADS = 128;             // 4 warps x 32 frames, lane = channel
constexpr int CF_FPT = 32;                  // frames per thread

struct CfParams {
  const __nv_bfloat16* x;
  const __nv_bfloat16* w;
  const __nv_bfloat16* bias;
  __nv_bfloat16* y;
  const int* lengths;
  int64_t sxB, sxC, sxT, syB, syC, syT;
  int C, T;
};

template <bool GLU>
__global__ void __launch_bounds__(CF_THREADS)
    dwconv_cf_kernel(CfParams p) {
  __shared__ float xs[CF_CC * CF_PITCH];
  const int tid = threadIdx.x;
  const int t0 = blockIdx.x * CF_TT;
  const int c0 = blockIdx.y * CF_CC;
  const int b = blockIdx.z;
  const int T = p.T;
  const int len = p.lengths ? min(max(__ldg(p.lengths + b), 0), T) : T;
  const __nv_bfloat16* xb = p.x + (int64_t)b * p.sxB;

  // stage x[c0 .. c0+32) x [t0-7, t0+135) as fp32, zero outside [0, len)
  for (int e = tid; e < CF_CC * CF_W; e += CF_THREADS) {
    const int cc = e / CF_W;
    const int tt = e - cc * CF_W;
    const int t = t0 - HALO + tt;
    const int c = c0 + cc;
    float v = 0.f;
    if (t >= 0 && t < len && c < p.C) {
      const float a = __bfloat162float(xb[(int64_t)c * p.sxC + (int64_t)t * p.sxT]);
      if (GLU) {
        const float g = __bfloat162float(xb[(int64_t)(c + p.C) * p.sxC + (int64_t)t * p.sxT]);
        v = __bfloat162float(__float2bfloat16_rn(a * sigmoid_fast(g)));
      } else {
        v = a;
      }
    }
    xs[cc * CF_PITCH + tt] = v;
  }
  __syncthreads();

  const int lane = tid & 31;
  const int q = tid >> 5;
  const int c = c0 + lane;
  float acc[CF_FPT];
  float wr[KW];
  const bool c_ok = c < p.C;
  const float bv = c_ok ? __bfloat162float(p.bias[c]) : 0.f;
#pragma unroll
  for (int j = 0; j < KW; ++j) wr[j] = c_ok ? __bfloat162float(p.w[(int64_t)c * KW + j]) : 0.f;
#pragma unroll
  for (int f = 0; f < CF_FPT; ++f) acc[f] = bv;
  const float* xr = xs + lane * CF_PITCH + q * CF_FPT;
#pragma unroll
  for (int r = 0; r < CF_FPT + 2 * HALO; ++r) {
    const float xv = xr[r];
#pragma unroll
    for (int f = 0; f < CF_FPT; ++f) {
      const int j = r - f;
      if (j >= 0 && j < KW) acc[f] = fmaf(wr[j], xv, acc[f]);
    }
  }
  __syncthreads();  // xs is reused as the output transpose buffer
  __nv_bfloat16* ys = reinterpret_cast<__nv_bfloat16*>(xs);   // [32 channels][128 + 2 frames]
  constexpr int OP = CF_TT + 2;
#pragma unroll
  for (int f = 0; f < CF_FPT; ++f) {
    const int t = t0 + q * CF_FPT + f;
    ys[lane * OP + q * CF_FPT + f] = __float2bfloat16_rn(t < len ? silu_fast(acc[f]) : 0.f);
  }
  __syncthreads();
  __nv_bfloat16* yb = p.y + (int64_t)b * p.syB;
  for (int e = tid; e < CF_CC * CF_TT; e += CF_THREADS) {
    const int cc = e / CF_TT;
    const int tt = e - cc * CF_TT;
    const int t = t0 + tt;
    if (t < T && c0 + cc < p.C) yb[(int64_t)(c0 + cc) * p.syC + (int64_t)t * p.syT] = ys[cc * OP + tt];
  }
}

}  // namespace dw_impl
using namespace dw_impl;

int launch_dwconv(const DwArgs& a, cudaStream_t stream) {
  if (a.B == 0 || a.T == 0 || a.C == 0) return 0;
  const bool cl = (a.sxC == 1 && a.syC == 1 && (a.C % CL_CC) == 0 && (a.sxT % 8) == 0 && (a.sxB % 8) == 0 &&
                   (a.syT % 4) == 0 && (a.syB % 4) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.y) & 7) == 0);
  if (cl) {
    // x viewed as [B][T][Cx] with Cx = C (or 2C for GLU) channels contiguous
    CUtensorMap tm;
    const uint64_t cx = (uint64_t)a.C * (a.glu ? 2 : 1);
    const uint64_t dims[3] = {cx, (uint64_t)a.T, (uint64_t)a.B};
    const uint64_t strides[2] = {(uint64_t)a.sxT * 2, (uint64_t)a.sxB * 2};
    const uint32_t box[3] = {CL_CC, CL_ROWS, 1};
    int rc = encode_tmap(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a.x, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    ClParams p{a.w, a.bias, a.y, a.lengths, a.syB, a.syT, a.T, a.C};
    dim3 grid(a.C / CL_CC, (a.T + CL_TT * CL_TILES - 1) / (CL_TT * CL_TILES), a.B);
    if (a.glu) {
      const int smem = (int)sizeof(ClSmem<true>) + 128;
      cudaError_t e = cudaFuncSetAttribute(dwconv_cl_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return (int)e;
      dwconv_cl_kernel<true><<<grid, CL_THREADS, smem, stream>>>(tm, p);
    } else {
      const int smem = (int)sizeof(ClSmem<false>) + 128;
      cudaError_t e = cudaFuncSetAttribute(dwconv_cl_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return (int)e;
      dwconv_cl_kernel<false><<<grid, CL_THREADS, smem, stream>>>(tm, p);
    }
    return (int)cudaGetLastError();
  }
  CfParams p{a.x, a.w, a.bias, a.y, a.lengths, a.sxB, a.sxC, a.sxT, a.syB, a.syC, a.syT, a.C, a.T};
  dim3 grid((a.T + CF_TT - 1) / CF_TT, (a.C + CF_CC - 1) / CF_CC, a.B);
  if (a.glu)
    dwconv_cf_kernel<true><<<grid, CF_THREADS, 0, stream>>>(p);
  else
    dwconv_cf_kernel<false><<<grid, CF_THREADS, 0, stream>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace gsn
