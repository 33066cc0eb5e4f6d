// Depthwise Conv1d k=15 (+ folded BatchNorm bias) + SiLU on sm_100a, optionally with the GLU in front.
//
// Semantics (script/cuda_kernels/conv1d.py:21-42, and the GLU form conv1d.py:52-79):
//   y[b, c, t] = silu(bias[c] + sum_{j<15} w[c, j] * x[b, c, t - 7 + j]),   x = 0 outside [0, T)
//   GLU form:   x[b, c, t] = bf16(a[b, c, t] * sigmoid(g[b, c, t])), a = channels [0, C), g = channels [C, 2C)
// plus per-utterance lengths (not in the reference op): frames t >= len[b] read as zero and are written as zero.
// Accumulation is fp32 and the output is rounded to bf16 once, as in the reference kernel.
//
// Two layouts:
//  * channels-last (element stride of C is 1; the conv-module layout [B, T, C]): a CTA owns CC channels of one
//    utterance over TILES consecutive time tiles of TT frames (channel tile fastest in blockIdx.x, so the CTAs
//    running together read whole frame rows).  Each tile plus its 7-frame halo on both sides ((TT + 14) rows of
//    CC * 2 bytes) is staged in shared memory by a 3-D TMA load, out-of-range frames (t < 0, t >= T) arriving
//    zero-filled, through a 3-stage ring: the load of tile i + 3 is issued as soon as tile i has been consumed.  A
//    warp owns FPW output frames, a lane CPT channels (conflict-free shared-memory rows), with the 15 x CPT weights
//    in registers and packed fp32x2 FMAs.  Tiles entirely inside the utterance take an unmasked path, tiles past
//    its end skip their load, and a CTA whose frames are all padding only writes zeros.  Two tile shapes: without
//    lengths a lane owns 2 channels x 32 frames (46 staged rows feed 32 outputs, so fewer bf16 unpacks and shared
//    loads per output); with lengths, and in the GLU form, 4 channels x 8 frames (short tiles waste less work past
//    an utterance's end).  Both accumulate every output in the same order, so they agree bit for bit.
//  * channels-first (element stride of T is 1; the layout the reference op receives from up_conv): with 16-byte
//    aligned rows, T % 8 == 0 and C % 16 == 0 the taps run on the tensor cores (dwconv_mma_sm100.cu).  Otherwise
//    (a ragged T such as 37, unaligned rows, any other stride pattern) a CTA owns 32 channels x 128 frames, stages
//    the rows (plus halo) in shared memory as fp32 with plain coalesced loads, and transposes the result through
//    shared memory for coalesced stores of exactly the frames below T.
#include <algorithm>
#include <type_traits>

#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

namespace gsn {

namespace dw_impl {

constexpr int KW = 15;
constexpr int HALO = 7;

// ----------------------------------------------------------------------------------------------------------------
// channels-last

// Tile shape: channels per lane, frames per warp, warps per CTA, time tiles per CTA, and the resident CTAs per SM
// the register allocation must allow.
template <int CPT_, int FPW_, int WARPS_, int SEG_, int MINB_>
struct ClShape {
  static constexpr int CPT = CPT_, FPW = FPW_, WARPS = WARPS_, SEG = SEG_, MINB = MINB_;
};
using ShapeDense = ClShape<2, 32, 2, 4, 8>;    // no lengths: 64 channels x 64 frames per tile, 128 registers
using ShapeMasked = ClShape<4, 8, 4, 8, 4>;    // lengths or GLU: 128 channels x 32 frames per tile

template <class S, bool GLU>
struct ClCfg {
  static constexpr int CPT = S::CPT;
  static constexpr int FPW = S::FPW;
  static constexpr int WARPS = S::WARPS;
  static constexpr int NP = CPT / 2;               // fp32 pairs per lane
  static constexpr int CC = 32 * CPT;              // channels per tile
  static constexpr int TT = FPW * WARPS;           // output frames per tile
  static constexpr int ROWS = TT + 2 * HALO;       // staged rows
  static constexpr int ROW_BYTES = CC * 2;
  static constexpr int TILE_BYTES = ROWS * ROW_BYTES;
  static constexpr int STAGES = 3;
  static constexpr int THREADS = 32 * WARPS;
  static constexpr int TILES = S::SEG;             // consecutive time tiles per CTA
  static constexpr int MIN_CTAS = GLU ? 3 : S::MINB;
};

template <class S, bool GLU>
struct __align__(128) ClSmem {
  using C = ClCfg<S, GLU>;
  uint8_t x[C::STAGES][GLU ? 2 : 1][C::TILE_BYTES];
  uint64_t full[C::STAGES];
  int abort_flag;
};

struct ClParams {
  const __nv_bfloat16* w;
  const __nv_bfloat16* bias;
  __nv_bfloat16* y;
  const int* lengths;
  int64_t syB, syT;
  int T, C;
  int withhold;        // test only: tile #k of every CTA armed but never loaded (-1: none)
};

__device__ __forceinline__ float2 bf16x2_to_f2(uint32_t v) { return make_float2(bf16lo_to_f32(v), bf16hi_to_f32(v)); }

// Packed fp32 pairs kept as 64-bit registers from the unpack through the FMAs, so the pair operands of
// fma.rn.f32x2 never have to be assembled from separately allocated halves.
typedef uint64_t pk2;
__device__ __forceinline__ pk2 pk_from_bf16x2(uint32_t v) {
  pk2 d;
  asm("{\n\t.reg .b32 lo, hi;\n\tshl.b32 lo, %1, 16;\n\tand.b32 hi, %1, 0xFFFF0000;\n\tmov.b64 %0, {lo, hi};\n\t}"
      : "=l"(d) : "r"(v));
  return d;
}
__device__ __forceinline__ pk2 pk_make(float lo, float hi) {
  pk2 d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ float2 pk_split(pk2 v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return make_float2(lo, hi);
}
__device__ __forceinline__ pk2 pk_fma(pk2 a, pk2 b, pk2 c) {
  pk2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// GLU of one packed bf16 pair, rounded to bf16 and widened back (conv1d.py:70-73 rounds the product to bf16)
__device__ __forceinline__ float2 glu_pair(uint32_t a, uint32_t g) {
  const float a0 = bf16lo_to_f32(a), a1 = bf16hi_to_f32(a);
  const float g0 = bf16lo_to_f32(g), g1 = bf16hi_to_f32(g);
  const uint32_t r = pack_bf16x2(a0 * sigmoid_fast(g0), a1 * sigmoid_fast(g1));
  return bf16x2_to_f2(r);
}

template <int NP>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t (&w)[NP]) {
  if constexpr (NP == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (NP == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}

template <int NP>
__device__ __forceinline__ void stg_words(__nv_bfloat16* p, const uint32_t (&w)[NP]) {
  if constexpr (NP == 4) {
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  } else if constexpr (NP == 2) {
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  } else {
    *reinterpret_cast<uint32_t*>(p) = w[0];
  }
}

template <class S, bool GLU>
__global__ void __launch_bounds__(ClCfg<S, GLU>::THREADS, ClCfg<S, GLU>::MIN_CTAS)
    dwconv_cl_kernel(const __grid_constant__ CUtensorMap tmX, ClParams p) {
  using Cfg = ClCfg<S, GLU>;
  constexpr int CPT = Cfg::CPT;
  constexpr int FPW = Cfg::FPW;
  constexpr int WARPS = Cfg::WARPS;
  constexpr int NP = Cfg::NP;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int TT = Cfg::TT;
  extern __shared__ uint8_t smem_raw[];
  auto& s = *reinterpret_cast<ClSmem<S, GLU>*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int T = p.T;
  const int c0 = blockIdx.x * Cfg::CC;
  const int b = blockIdx.z;
  const int t_begin = blockIdx.y * (TT * Cfg::TILES);
  const int t_end = min(T, t_begin + TT * Cfg::TILES);
  const int len = p.lengths ? min(max(__ldg(p.lengths + b), 0), T) : T;
  __nv_bfloat16* yb = p.y + (int64_t)b * p.syB + c0 + lane * CPT;

  if (t_begin >= len) {
    // every frame of this CTA is padding: zeros, no loads
    uint32_t z[NP];
#pragma unroll
    for (int q = 0; q < NP; ++q) z[q] = 0u;
    for (int t = t_begin + warp; t < t_end; t += WARPS) stg_words<NP>(yb + (int64_t)t * p.syT, z);
    return;
  }
  const int n_tiles = (t_end - t_begin + TT - 1) / TT;
  constexpr uint32_t kTxBytes = (GLU ? 2 : 1) * Cfg::TILE_BYTES;

  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) mbar_init(&s.full[i], 1);
    s.abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
  }
  __syncthreads();

  // producer side (thread 0): load tile i into stage i % STAGES, or, if every output frame of it is padding,
  // complete the stage's phase without a copy
  auto issue = [&](int i) {
    const int st = i % STAGES;
    const int t0 = t_begin + i * TT;
    if (t0 >= len) {
      mbar_arrive(&s.full[st]);
      return;
    }
    mbar_arrive_expect_tx(&s.full[st], kTxBytes);
    if (i == p.withhold) return;                     // test only: armed, no copy, so the bounded wait runs out
    tma_load_3d(s.x[st][0], &tmX, &s.full[st], c0, t0 - HALO, b);
    if (GLU) tma_load_3d(s.x[st][GLU ? 1 : 0], &tmX, &s.full[st], c0 + p.C, t0 - HALO, b);
  };
  int issued = 0;                                    // tiles handed to stages so far (thread 0)
  if (tid == 0) {
    for (; issued < STAGES && issued < n_tiles; ++issued) issue(issued);
  }

  // weights of this lane's channels, as fp32 pairs: wr[j][q] = (channel 2q, channel 2q + 1).  Weights and bias are
  // held halved (exact), so the accumulator is h = x / 2 and silu(x) = h + h * tanh(h) needs no extra multiply.
  pk2 wr[KW][NP];
  pk2 bias[NP];
  {
    const __nv_bfloat16* wp = p.w + (int64_t)(c0 + lane * CPT) * KW;
#pragma unroll
    for (int j = 0; j < KW; ++j)
#pragma unroll
      for (int q = 0; q < NP; ++q)
        wr[j][q] = pk_make(0.5f * __bfloat162float(wp[(2 * q) * KW + j]),
                           0.5f * __bfloat162float(wp[(2 * q + 1) * KW + j]));
#pragma unroll
    for (int q = 0; q < NP; ++q)
      bias[q] = pk_make(0.5f * __bfloat162float(p.bias[c0 + lane * CPT + 2 * q]),
                        0.5f * __bfloat162float(p.bias[c0 + lane * CPT + 2 * q + 1]));
  }

  bool alive = true;
  const int row0 = warp * FPW;                       // first output frame (and staged row) of this warp
  for (int i = 0; i < n_tiles; ++i) {
    const int st = i % STAGES;
    const int t0 = t_begin + i * TT;
    if (alive)
      alive = mbar_wait_bounded(&s.full[st], (uint32_t)((i / STAGES) & 1), &s.abort_flag, kStatusTimeoutDw);
    if (alive && t0 >= len) {
      // every output frame of the tile is padding
      uint32_t z[NP];
#pragma unroll
      for (int q = 0; q < NP; ++q) z[q] = 0u;
#pragma unroll
      for (int f = 0; f < FPW; ++f) {
        const int t = t0 + row0 + f;
        if (t < T) stg_words<NP>(yb + (int64_t)t * p.syT, z);
      }
    } else if (alive) {
      // MASKED: some staged row or output frame lies past the utterance's end.  The unmasked body is a separate
      // instantiation, so the common case carries no per-row or per-frame selects.
      auto tile = [&](auto masked_tag) {
        constexpr bool MASKED = decltype(masked_tag)::value;
        pk2 acc[FPW][NP];  // frame f starts from the bias at its first tap (row r = f), as bias + w0 x0 + w1 x1 ...
        uint32_t o[FPW][NP];                           // the packed outputs
        auto silu_frame = [&](int f) {
          const bool valid = !MASKED || t0 + row0 + f < len;
#pragma unroll
          for (int q = 0; q < NP; ++q) {
            const float2 h = pk_split(acc[f][q]);
            const float2 s2 = pk_split(pk_fma(acc[f][q], pk_make(tanh_approx(h.x), tanh_approx(h.y)), acc[f][q]));
            o[f][q] = valid ? pack_bf16x2(s2.x, s2.y) : 0u;
          }
        };
        const int t_row0 = t0 - HALO + row0;
        const uint8_t* xa = s.x[st][0] + row0 * Cfg::ROW_BYTES + lane * (CPT * 2);
        const uint8_t* xg = s.x[st][GLU ? 1 : 0] + row0 * Cfg::ROW_BYTES + lane * (CPT * 2);
#pragma unroll
        for (int r = 0; r < FPW + 2 * HALO; ++r) {
          uint32_t va[NP];
          lds_words<NP>(xa + r * Cfg::ROW_BYTES, va);
          pk2 xv[NP];
          if (GLU) {
            uint32_t vg[NP];
            lds_words<NP>(xg + r * Cfg::ROW_BYTES, vg);
#pragma unroll
            for (int q = 0; q < NP; ++q) {
              const float2 g2 = glu_pair(va[q], vg[q]);
              xv[q] = pk_make(g2.x, g2.y);
            }
          } else {
#pragma unroll
            for (int q = 0; q < NP; ++q) xv[q] = pk_from_bf16x2(va[q]);
          }
          if (MASKED && t_row0 + r >= len) {  // frames past the utterance read as zero (t >= T is zero-filled)
#pragma unroll
            for (int q = 0; q < NP; ++q) xv[q] = 0ull;
          }
#pragma unroll
          for (int f = 0; f < FPW; ++f) {
            const int j = r - f;
            if (j >= 0 && j < KW) {
#pragma unroll
              for (int q = 0; q < NP; ++q) acc[f][q] = pk_fma(wr[j][q], xv[q], j == 0 ? bias[q] : acc[f][q]);
            }
          }
        }
#pragma unroll
        for (int f = 0; f < FPW; ++f) silu_frame(f);
        __nv_bfloat16* yt = yb + (int64_t)(t0 + row0) * p.syT;
#pragma unroll
        for (int f = 0; f < FPW; ++f, yt += p.syT) {
          if (!MASKED || t0 + row0 + f < T) stg_words<NP>(yt, o[f]);
        }
      };
      if (t0 + TT + HALO <= len)
        tile(std::false_type{});
      else
        tile(std::true_type{});
    }
    __syncthreads();  // stage st fully consumed by every warp
    if (tid == 0 && alive && !s.abort_flag && issued < n_tiles) {
      fence_proxy_async_smem();
      issue(issued);
      ++issued;
    }
  }
  if (tid == 0 && s.abort_flag) {
    // unwinding after a timeout: let the copies still in flight (the last STAGES issued) land before the shared
    // memory is released
    for (int k = issued > STAGES ? issued - STAGES : 0; k < issued; ++k)
      mbar_wait_bounded(&s.full[k % STAGES], (uint32_t)((k / STAGES) & 1), nullptr, kStatusTimeoutDw, 100000000ull);
  }
}

template <class S, bool GLU>
int launch_cl(const DwArgs& a, cudaStream_t stream) {
  using Cfg = ClCfg<S, GLU>;
  CUtensorMap tm;
  const uint64_t cx = (uint64_t)a.C * (GLU ? 2 : 1);
  const uint64_t dims[3] = {cx, (uint64_t)a.T, (uint64_t)a.B};
  const uint64_t strides[2] = {(uint64_t)a.sxT * 2, (uint64_t)a.sxB * 2};
  const uint32_t box[3] = {(uint32_t)Cfg::CC, (uint32_t)Cfg::ROWS, 1};
  int rc = encode_tmap(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a.x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  ClParams p;
  p.w = a.w;
  p.bias = a.bias;
  p.y = a.y;
  p.lengths = a.lengths;
  p.syB = a.syB;
  p.syT = a.syT;
  p.T = a.T;
  p.C = a.C;
  p.withhold = a.withhold_tile;
  const int64_t t_chunks = ((int64_t)a.T + Cfg::TT * Cfg::TILES - 1) / (Cfg::TT * Cfg::TILES);
  if (t_chunks > 65535 || a.B > 65535) return (int)cudaErrorInvalidValue;
  auto kern = dwconv_cl_kernel<S, GLU>;
  const int smem = (int)sizeof(ClSmem<S, GLU>) + 128;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return (int)e;
  dim3 grid(a.C / Cfg::CC, (unsigned)t_chunks, a.B);
  kern<<<grid, Cfg::THREADS, smem, stream>>>(tm, p);
  return (int)cudaGetLastError();
}

// ----------------------------------------------------------------------------------------------------------------
// GLU of bf16 words (used by the tensor-core depthwise kernel's converters, dwconv_mma_sm100.cu)
__device__ __forceinline__ pk2 pk_mul(pk2 a, pk2 b) {
  pk2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// GLU of one word of value frames and the matching word of gate frames, rounded to bf16: the same arithmetic as
// glu_pair (a * (0.5 + 0.5 * tanh(g / 2)), one rounding), on the frame pair packed.
__device__ __forceinline__ uint32_t glu_word(uint32_t a, uint32_t g) {
  const pk2 av = pk_from_bf16x2(a);
  const float2 gh = pk_split(pk_mul(pk_from_bf16x2(g), pk_make(0.5f, 0.5f)));
  const pk2 sg = pk_fma(pk_make(0.5f, 0.5f), pk_make(tanh_approx(gh.x), tanh_approx(gh.y)), pk_make(0.5f, 0.5f));
  const float2 r = pk_split(pk_mul(av, sg));
  return pack_bf16x2(r.x, r.y);
}

// ----------------------------------------------------------------------------------------------------------------
// channels-first, any strides (row strides that are not 16-byte multiples, e.g. T = 37, or C not a multiple of 64)
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
  // the channels-last kernel of shape S applies when both tensors are channels-last with 16-byte aligned frame rows
  // in x, C a multiple of the tile's channels and y's lane stores (CPT bf16) aligned
  auto cl_ok = [&](auto shape) {
    using Cfg = ClCfg<decltype(shape), false>;
    return a.sxC == 1 && a.syC == 1 && (a.C % Cfg::CC) == 0 && (a.sxT % 8) == 0 && (a.sxB % 8) == 0 &&
           (a.syT % Cfg::CPT) == 0 && (a.syB % Cfg::CPT) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.y) & (2 * Cfg::CPT - 1)) == 0;
  };
  if (!a.glu && !a.lengths && cl_ok(ShapeDense{})) return launch_cl<ShapeDense, false>(a, stream);
  if (cl_ok(ShapeMasked{}))
    return a.glu ? launch_cl<ShapeMasked, true>(a, stream) : launch_cl<ShapeMasked, false>(a, stream);
  // both forms on the tensor cores (dwconv_mma_sm100.cu) when rows are 16-byte aligned, C % 16 == 0 and T % 8 == 0
  // (the kernel moves whole 8-frame chunks: a ragged row end would be read and written past T)
  const bool mma_ok = a.sxT == 1 && a.syT == 1 && (a.C % 16) == 0 && (a.T % 8) == 0 && (a.sxC % 8) == 0 &&
                      (a.sxB % 8) == 0 && (a.syC % 8) == 0 && (a.syB % 8) == 0 && a.sxC >= a.T && a.syC >= a.T &&
                      (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0;
  if (mma_ok) return launch_dwconv_cf_mma(a, stream);
  // anything else (a ragged T, unaligned rows, C % 16 != 0) takes the generic kernel, which stores frame by frame
  CfParams p{a.x, a.w, a.bias, a.y, a.lengths, a.sxB, a.sxC, a.sxT, a.syB, a.syC, a.syT, a.C, a.T};
  dim3 grid((a.T + CF_TT - 1) / CF_TT, (a.C + CF_CC - 1) / CF_CC, a.B);
  if (a.glu)
    dwconv_cf_kernel<true><<<grid, CF_THREADS, 0, stream>>>(p);
  else
    dwconv_cf_kernel<false><<<grid, CF_THREADS, 0, stream>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace gsn
