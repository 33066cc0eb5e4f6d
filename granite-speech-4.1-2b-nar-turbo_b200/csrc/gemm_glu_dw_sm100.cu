// up_conv + GLU with the depthwise conv k=15 (+ folded BatchNorm bias) + SiLU fused into the GEMM epilogue, on
// sm_100a: the GLU tensor [M, inner] never leaves the SM.
//
//   up_conv (models/granite_speech_nar/conformer.py:165,177) + GLU (:166,:181) + depthwise (:134-155,:168-169)
//   + SiLU (:186): d[b, t, c] = silu(bdw[c] + sum_{j<15} wdw[c, j] * glu(a W1^T + b1)[b, t - 7 + j, c])
//
// Work unit: one utterance b and one block of 128 GLU channels (256 GEMM columns: [128 value | 128 gate] rows of
// the GLU-interleaved W1).  A CTA walks the unit's 128-frame tiles in time order, so each tile's depthwise
// outputs need only the last 14 GLU rows of the previous tile, which stay in shared memory: nothing is
// recomputed and the GLU rows are never written to global memory.  Units are ordered longest utterance first
// (channel block fastest, so the 16 CTAs sharing an utterance's A tiles run together and read them from L2) and
// dealt to the persistent CTAs in a snake order.
//
// Roles (320 threads, one CTA per SM):
//   warp 0      TMA producer: A 128x64 (frames of the tile) + W 256x64 per stage, 128-byte swizzle, 3 stages
//   warp 1      TMEM allocator (2 x 256 columns) and single-thread UMMA issuer, M=128 N=256 K=16
//   warps 2-9   epilogue.  Per tile: (1) TMEM -> GLU -> bf16 rows 14..141 of the staging window (warp w reads
//               its TMEM lane quarter w % 4, warps 2-5 the first 64 channels, 6-9 the last 64); the accumulator
//               buffer is released right after; (2) depthwise + SiLU over the window: lane = 4 channels, warp =
//               16 output frames, weights (halved) in registers, fp32x2 FMAs in the order of the standalone
//               depthwise kernel, so the result is bit-identical to GEMM -> GLU tensor -> depthwise kernel; the
//               warp's 16 x 128 outputs leave through a staging box in shared memory and one TMA store (boxes
//               that would start before frame 0 or reach past the written range use plain stores);
//               (3) the first epilogue warp moves window rows 128..141 to rows 0..13 for the next tile.  After
//               the last tile a flush pass computes the final 7 frames with zero GLU rows on the right.
// Lengths: GLU rows of frames t >= len[b] are zero, depthwise frames in [len, roundup128(len)) are written as
// zero (the residual GEMM reads whole 128-row tiles), frames beyond are never touched.
#include <type_traits>

#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

namespace gsn {

namespace gdw_impl {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGES = 3;
constexpr int EPI_WARPS = 8;
constexpr int EPI_THREADS = 32 * EPI_WARPS;
constexpr int THREADS = 64 + EPI_THREADS;
constexpr int CH = BN / 2;                 // GLU channels per unit
constexpr int KW = 15, HALO = 7;
constexpr int WROWS = BM + 2 * HALO;       // staging window: 14 rows of the previous tile + the tile's 128
constexpr int WPITCH = CH * 2 + 16;        // 272 bytes: 16-byte row stores of consecutive lanes hit distinct banks
constexpr int MAX_SORT_B = 512;            // utterances ordered by length up to this batch size
constexpr uint32_t TMEM_COLS = 512;
constexpr int kEpiBar = 1;                 // named barrier of the epilogue warps
constexpr int FPW = 16;                    // output frames per epilogue warp and tile
constexpr int OUT_BOX_BYTES = FPW * CH * 2;   // a warp's 16 x 128 bf16 output box: 4 KB

struct Params {
  const float* bias;          // [N] GLU-interleaved, fp32
  const float* col_scale;     // [N] or null
  const __nv_bfloat16* dw_w;  // [inner, 15]
  const __nv_bfloat16* dw_b;  // [inner]
  __nv_bfloat16* d;           // [B * T, inner]
  const int* lengths;         // [B] or null
  const float2* row_stats;    // LayerNorm folded in: per-row (rstd, rstd * mean), rows b * T + t
  const float* colsum;        // LayerNorm folded in: [N] column sums of W'
  const float* row_scale;     // A8: per-row scale of the int8 activations, rows b * T + t
  const float2* row_partials; // LayerNorm folded in, instead of row_stats: per row K / 256 blocks of (mean, M2)
  float ln_eps;
  int B, T, K, N;
};

struct __align__(1024) Smem {
  uint8_t a[STAGES][A_BYTES];
  uint8_t b[STAGES][B_BYTES];
  uint8_t out[EPI_WARPS][OUT_BOX_BYTES];   // per-warp output box for the TMA store
  uint8_t win[WROWS * WPITCH];
  float vb[BN];               // the unit's GLU bias columns, halved
  float vs[BN];               // the unit's column scales, halved (0.5 without scales)
  float vc[BN];               // LayerNorm folded in: the unit's column sums times the halved scales
  int lens[MAX_SORT_B];       // clamped lengths
  short order[MAX_SORT_B];    // utterances, most tiles first
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(offsetof(Smem, b) % 1024 == 0 && offsetof(Smem, win) % 16 == 0 && offsetof(Smem, out) % 128 == 0,
              "alignment");
static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory size");

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

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync %0, %1;" ::"n"(kEpiBar), "n"(EPI_THREADS) : "memory"); }

// The unit sequence, identical in every role: utterance rank r (most tiles first) x channel block, dealt to the
// CTAs in snake order over the passes of gridDim.x units.  When the last pass holds at most half a grid of units,
// each of them is split into two halves of 64 channels (N=128 MMAs) on two CTAs, so that pass ends in half the
// time: whole units make the busiest CTA take one unit more than most others.
struct Unit {
  int b, n_blk, len, half;    // half: -1 for the whole 128-channel block, else 0 / 1 (channels 64 * half + [0, 64))
};
struct Units {
  const Smem* s;
  const int* lengths;
  int B, T, nb, total;
  bool sorted;
  __device__ int len_of(int b) const {
    if (sorted) return s->lens[b];
    return lengths ? min(max(__ldg(lengths + b), 0), T) : T;
  }
  // step-th unit of this CTA: false when there is none
  __device__ bool get(int step, Unit& u) const {
    const int G = gridDim.x, j = blockIdx.x;
    const int passes = total / G, rem = total - passes * G;
    const bool split = rem > 0 && 2 * rem <= G;
    const int pos = (step & 1) ? (G - 1 - j) : j;
    int i;
    u.half = -1;
    if (step < passes || !split) {
      i = step * G + pos;
      if (i >= total) return false;
    } else {
      if (step > passes || pos >= 2 * rem) return false;
      i = passes * G + (pos >> 1);
      u.half = pos & 1;
    }
    const int r = i / nb;
    u.n_blk = i - r * nb;
    u.b = sorted ? s->order[r] : r;
    u.len = len_of(u.b);
    return true;
  }
};

// SCALED: per-column scale on the accumulator (int8 weights widened to bf16).  LNF: LayerNorm folded in -- A holds
// the raw frames, W the weights times gamma, and the accumulator becomes rstd * (acc - mean * colsum) + bias; with
// LNF = 1 the row statistics come as (rstd, rstd * mean), with LNF = 2 as the previous residual GEMM's per-block
// (mean, M2), merged here.
// A8 (W8A8): A and W are int8 (128 per K-block, the same bytes per stage as 64 bf16), kind::i8 MMAs with s32
// accumulators; the epilogue takes fp32(acc) * row_scale * col_scale + bias, as the standalone int8 GEMM does.
template <bool SCALED, int LNF, bool A8 = false>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_glu_dw_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmW64, const __grid_constant__ CUtensorMap tmD, Params p) {
  static_assert(!(A8 && (LNF || !SCALED)), "W8A8 takes per-column scales and no folded LayerNorm");
  constexpr uint32_t IDESC = A8 ? make_idesc_s8_s32(BM, BN) : make_idesc_bf16_f32(BM, BN);
  constexpr uint32_t IDESC_HALF = A8 ? make_idesc_s8_s32(BM, BN / 2) : make_idesc_bf16_f32(BM, BN / 2);
  constexpr int KBE = A8 ? 2 * BK : BK;       // elements per K-block
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  const int num_kb = p.K / KBE;
  const int inner = p.N / 2;
  const bool sorted = p.B <= MAX_SORT_B;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], EPI_WARPS);
    }
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmW64);
    tma_prefetch_desc(&tmD);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  // lengths, then the longest-first order (rank = utterances with more tiles, ties by index)
  if (sorted) {
    for (int b = threadIdx.x; b < p.B; b += THREADS)
      s.lens[b] = p.lengths ? min(max(__ldg(p.lengths + b), 0), p.T) : p.T;
  }
  tc_fence_before();
  __syncthreads();
  if (sorted) {
    for (int b = threadIdx.x; b < p.B; b += THREADS) {
      const int nt = (s.lens[b] + BM - 1) / BM;
      int rank = 0;
      for (int o = 0; o < p.B; ++o) {
        const int no = (s.lens[o] + BM - 1) / BM;
        rank += (no > nt) || (no == nt && o < b);
      }
      s.order[rank] = (short)b;
    }
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;
  const Units units{&s, p.lengths, p.B, p.T, p.N / BN, p.B * (p.N / BN), sorted};

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    const uint64_t pol_w = l2_policy_evict_last();
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    Unit u;
    for (int step = 0; ok && units.get(step, u); ++step) {
      const int nt = (u.len + BM - 1) / BM;
      for (int k = 0; k < nt && ok; ++k) {
        const int row0 = u.b * p.T + k * BM;
        for (int kb = 0; kb < num_kb; ++kb) {
          bool got = mbar_wait_bounded(&s.empty[stage], phase ^ 1u, abort_flag, kStatusTimeoutProducer);
          got = __shfl_sync(0xffffffffu, got, 0);
          if (!got) {
            ok = false;
            break;
          }
          if (lane == 0) {
            if (u.half < 0) {
              mbar_arrive_expect_tx(&s.full[stage], A_BYTES + B_BYTES);
              tma_load_2d(s.a[stage], &tmA, &s.full[stage], kb * KBE, row0);
              tma_load_2d_hint(s.b[stage], &tmW, &s.full[stage], kb * KBE, u.n_blk * BN, pol_w);
            } else {
              // half unit: W rows of its 64 value channels, then of their 64 gate channels (8-row swizzle atoms,
              // so the two 64-row boxes form one 128-row tile)
              const int w0 = u.n_blk * BN + 64 * u.half;
              mbar_arrive_expect_tx(&s.full[stage], A_BYTES + B_BYTES / 2);
              tma_load_2d(s.a[stage], &tmA, &s.full[stage], kb * KBE, row0);
              tma_load_2d_hint(s.b[stage], &tmW64, &s.full[stage], kb * KBE, w0, pol_w);
              tma_load_2d_hint(s.b[stage] + B_BYTES / 4, &tmW64, &s.full[stage], kb * KBE, w0 + CH, pol_w);
            }
          }
          __syncwarp();
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    if (!ok && lane == 0) {
      // unwinding after a timeout: the last STAGES loads may still be in flight
      for (int back = 1; back <= STAGES && back <= issued; ++back) {
        const int idx = issued - back;
        mbar_wait_bounded(&s.full[idx % STAGES], (uint32_t)((idx / STAGES) & 1), nullptr, kStatusTimeoutProducer,
                          100000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- UMMA issuer
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int local = 0;
    Unit u;
    for (int step = 0; ok && units.get(step, u); ++step) {
      const int nt = (u.len + BM - 1) / BM;
      const uint32_t idesc = u.half < 0 ? IDESC : IDESC_HALF;
      for (int k = 0; k < nt && ok; ++k) {
        const int acc = local & 1;
        const uint32_t use_par = (uint32_t)((local >> 1) & 1);
        ++local;
        bool got = mbar_wait_bounded(&s.tempty[acc], use_par ^ 1u, abort_flag, kStatusTimeoutMma);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          bool ready = mbar_wait_bounded(&s.full[stage], phase, abort_flag, kStatusTimeoutMma);
          ready = __shfl_sync(0xffffffffu, ready, 0);
          if (!ready) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint64_t adesc = make_sw128_kmajor_desc(smem_u32(s.a[stage]));
            const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(s.b[stage]));
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              if constexpr (A8)
                umma_i8(d_tmem, adesc + (uint64_t)(2 * kk), bdesc + (uint64_t)(2 * kk), idesc,
                        (kb | kk) != 0 ? 1u : 0u);
              else
                umma_f16(d_tmem, adesc + (uint64_t)(2 * kk), bdesc + (uint64_t)(2 * kk), idesc,
                         (kb | kk) != 0 ? 1u : 0u);
            }
            umma_commit(&s.empty[stage]);
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (lane == 0) umma_commit(&s.tfull[acc]);
        __syncwarp();
      }
    }
    if (lane == 0) umma_commit(&s.mma_done);
    __syncwarp();
    mbar_wait_bounded(&s.mma_done, 0, nullptr, kStatusTimeoutMma, 100000000ull);
  } else {
    // ---------------------------------------------------------------- epilogue: GLU -> window -> depthwise
    // Every epilogue warp runs the same unit / tile sequence and meets every named barrier, also after a wait
    // ran out (ok == false: the work is skipped, the barriers are not), so the barrier counts always match.
    const int e = warp - 2;             // 0..7
    const int et = threadIdx.x - 64;    // 0..255
    const int q = warp & 3;             // TMEM lane quarter of this warp
    const int grp = e >> 2;             // whole unit: GLU channels [64 grp, 64 grp + 64); half unit: [32 grp, +32)
    bool ok = true;
    int local = 0;
    Unit u;
    for (int step = 0; units.get(step, u); ++step) {
      const int b = u.b, len = u.len;
      const int nt = (len + BM - 1) / BM;
      if (nt == 0) continue;
      const bool whole = u.half < 0;
      const int nch = whole ? CH : CH / 2;               // channels of the unit
      const int gate_col = whole ? CH : CH / 2;          // accumulator column of the first gate channel
      const int c0 = u.n_blk * CH + (whole ? 0 : (CH / 2) * u.half);   // first GLU / depthwise channel
      // depthwise lanes: a whole unit gives each lane 4 of its 128 channels; a half unit gives lanes l and l + 16
      // the same 4 of its 64 channels, for the first and the second 8 of the warp's 16 frames
      const int lch = whole ? lane : (lane & 15);
      const int store_end = min(nt * BM, p.T);           // frames written: [0, len) values, [len, store_end) zero
      __nv_bfloat16* drow = p.d + (int64_t)b * p.T * inner + c0 + lch * 4;

      // unit setup: bias / scale columns (value columns, then gate columns, as in the accumulator), zero left
      // halo (frames -14..-1), this lane's depthwise weights
      epi_bar();
      if (et < 2 * nch) {
        const int col = u.n_blk * BN + (whole ? et : (et < nch ? nch * u.half + et : CH + nch * u.half + et - nch));
        s.vb[et] = 0.5f * __ldg(p.bias + col);
        s.vs[et] = SCALED ? 0.5f * __ldg(p.col_scale + col) : 0.5f;
        if (LNF) s.vc[et] = s.vs[et] * __ldg(p.colsum + col);
      }
      if (et < 2 * HALO * 16) {
        const int r = et >> 4, c = et & 15;
        *reinterpret_cast<uint4*>(s.win + r * WPITCH + c * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
      pk2 wr[KW][2];
      pk2 wb[2];
      {
        const __nv_bfloat16* wp = p.dw_w + (int64_t)(c0 + lch * 4) * KW;
#pragma unroll
        for (int j = 0; j < KW; ++j)
#pragma unroll
          for (int qq = 0; qq < 2; ++qq)
            wr[j][qq] = pk_make(0.5f * __bfloat162float(wp[(2 * qq) * KW + j]),
                                0.5f * __bfloat162float(wp[(2 * qq + 1) * KW + j]));
#pragma unroll
        for (int qq = 0; qq < 2; ++qq)
          wb[qq] = pk_make(0.5f * __bfloat162float(p.dw_b[c0 + lch * 4 + 2 * qq]),
                           0.5f * __bfloat162float(p.dw_b[c0 + lch * 4 + 2 * qq + 1]));
      }
      epi_bar();

      for (int k = 0; k <= nt; ++k) {
        const int t0 = k * BM;                           // frame of window row 14
        const bool flush = k == nt;
        if (!flush) {
          // (1) accumulator -> GLU -> window rows 14 + r, r = this lane's row of the tile
          const int acc = local & 1;
          const uint32_t use_par = (uint32_t)((local >> 1) & 1);
          ++local;
          const int r = q * 32 + lane;
          const bool valid = t0 + r < len;
          // this row's LayerNorm statistics / activation scale, loaded ahead of the accumulator wait so that their
          // latency is not on the GLU step's path (padding rows have none; their GLU row is zero anyway)
          float rs = 1.f, rsm = 0.f;
          if (LNF && valid) {
            if constexpr (LNF == 2) {
              // merge the row's 256-column blocks of equal counts one by one (Chan et al.): block j moves the mean
              // by delta / (j + 1) and adds its M2 plus delta^2 * 256 j / (j + 1); rstd as the statistics kernel
              // forms it
              const float2* pp = p.row_partials + ((int64_t)b * p.T + t0 + r) * (p.K / 256);
              const int np = p.K / 256;
              const float2 p0 = __ldg(pp);
              float mean = p0.x, m2 = p0.y;
#pragma unroll
              for (int j = 1; j < 8; ++j) {
                if (j < np) {
                  const float2 v = __ldg(pp + j);
                  const float delta = v.x - mean;
                  mean = fmaf(delta, 1.0f / (float)(j + 1), mean);
                  m2 += fmaf(delta * delta, 256.0f * (float)j / (float)(j + 1), v.y);
                }
              }
              rs = rsqrtf(m2 * (1.0f / (float)p.K) + p.ln_eps);
              rsm = rs * mean;
            } else {
              const float2 st = __ldg(p.row_stats + (int64_t)b * p.T + t0 + r);
              rs = st.x;
              rsm = st.y;
            }
          }
          if (A8 && valid) rs = __ldg(p.row_scale + (int64_t)b * p.T + t0 + r);
          if (ok) {
            bool got = mbar_wait_bounded(&s.tfull[acc], use_par, abort_flag, kStatusTimeoutEpilogue);
            ok = __shfl_sync(0xffffffffu, got, 0);
          }
          if (ok) {
            tc_fence_after();
            const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
            uint8_t* wrow = s.win + (2 * HALO + r) * WPITCH;
            const float rsh = 0.5f * rs;                 // bf16 weights: the halved column scale is 0.5
            const int nsub = whole ? 2 : 1;              // 32-channel sub-tiles of this warp
            for (int uu = 0; uu < nsub; ++uu) {
              const int cb = whole ? grp * 64 + uu * 32 : grp * 32;   // first of the sub-tile's 32 GLU channels
              uint32_t va[2][16], vg[2][16];
              tmem_ld16(t_row + (uint32_t)cb, va[0]);
              tmem_ld16(t_row + (uint32_t)(cb + 16), va[1]);
              tmem_ld16(t_row + (uint32_t)(gate_col + cb), vg[0]);
              tmem_ld16(t_row + (uint32_t)(gate_col + cb + 16), vg[1]);
              tmem_wait_ld_dep(va[0], va[1]);
              tmem_wait_ld_dep(vg[0], vg[1]);
              uint32_t o[16];
              // four columns at a time: the column parameters as 16-byte shared loads, the arithmetic on fp32 pairs
              // (each lane of an f32x2 FMA is one fmaf; a product alone is an FMA with a -0 addend, which rounds
              // like the multiply).  Per column: a = x * m + i, with m = 1/2 (bf16 weights), rstd / 2 (LayerNorm
              // folded), rstd * s / 2 (both) or s / 2 (scaled weights; W8A8: x = the s32 sum times the row scale),
              // and i = b / 2 - rstd * mean * colsum * m' (LayerNorm folded) or b / 2
              const pk2 rs2 = pk_make(rs, rs), rsh2 = pk_make(rsh, rsh), nrsm2 = pk_make(-rsm, -rsm);
              const pk2 half2 = pk_make(0.5f, 0.5f), nz2 = pk_make(-0.0f, -0.0f);
#pragma unroll
              for (int c = 0; c < 32; c += 4) {
                const float4 ba = *reinterpret_cast<const float4*>(&s.vb[cb + c]);
                const float4 bg = *reinterpret_cast<const float4*>(&s.vb[gate_col + cb + c]);
                pk2 ia[2] = {pk_make(ba.x, ba.y), pk_make(ba.z, ba.w)};
                pk2 ig[2] = {pk_make(bg.x, bg.y), pk_make(bg.z, bg.w)};
                if constexpr (LNF) {
                  const float4 ca = *reinterpret_cast<const float4*>(&s.vc[cb + c]);
                  const float4 cg = *reinterpret_cast<const float4*>(&s.vc[gate_col + cb + c]);
                  ia[0] = pk_fma(nrsm2, pk_make(ca.x, ca.y), ia[0]);
                  ia[1] = pk_fma(nrsm2, pk_make(ca.z, ca.w), ia[1]);
                  ig[0] = pk_fma(nrsm2, pk_make(cg.x, cg.y), ig[0]);
                  ig[1] = pk_fma(nrsm2, pk_make(cg.z, cg.w), ig[1]);
                }
                pk2 ma[2] = {LNF ? rsh2 : half2, LNF ? rsh2 : half2}, mg[2] = {ma[0], ma[1]};
                if constexpr (SCALED) {
                  const float4 sa = *reinterpret_cast<const float4*>(&s.vs[cb + c]);
                  const float4 sg = *reinterpret_cast<const float4*>(&s.vs[gate_col + cb + c]);
                  ma[0] = pk_make(sa.x, sa.y);
                  ma[1] = pk_make(sa.z, sa.w);
                  mg[0] = pk_make(sg.x, sg.y);
                  mg[1] = pk_make(sg.z, sg.w);
                  if constexpr (LNF) {
#pragma unroll
                    for (int z = 0; z < 2; ++z) {
                      ma[z] = pk_fma(rs2, ma[z], nz2);
                      mg[z] = pk_fma(rs2, mg[z], nz2);
                    }
                  }
                }
#pragma unroll
                for (int z = 0; z < 2; ++z) {
                  const int kk = c + 2 * z;
                  const uint32_t a0 = va[kk >> 4][kk & 15], a1 = va[kk >> 4][(kk & 15) + 1];
                  const uint32_t g0 = vg[kk >> 4][kk & 15], g1 = vg[kk >> 4][(kk & 15) + 1];
                  pk2 xa, xg;
                  if constexpr (A8) {
                    xa = pk_fma(pk_make((float)(int32_t)a0, (float)(int32_t)a1), rs2, nz2);
                    xg = pk_fma(pk_make((float)(int32_t)g0, (float)(int32_t)g1), rs2, nz2);
                  } else {
                    xa = pk_make(__uint_as_float(a0), __uint_as_float(a1));
                    xg = pk_make(__uint_as_float(g0), __uint_as_float(g1));
                  }
                  const pk2 a2 = pk_fma(xa, ma[z], ia[z]);
                  const float2 g2 = pk_split(pk_fma(xg, mg[z], ig[z]));
                  const float2 h2 = pk_split(pk_fma(a2, pk_make(tanh_approx(g2.x), tanh_approx(g2.y)), a2));
                  o[kk >> 1] = valid ? pack_bf16x2(h2.x, h2.y) : 0u;
                }
              }
#pragma unroll
              for (int c = 0; c < 4; ++c)
                *reinterpret_cast<uint4*>(wrow + cb * 2 + c * 16) =
                    make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
            }
          }
          // the accumulator buffer is free for the next tile's MMAs
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.tempty[acc]);
        } else if (et < 2 * HALO * 16) {
          // flush: the frames after the last tile are past the utterance, i.e. zero GLU rows
          const int r = 2 * HALO + (et >> 4), c = et & 15;
          *reinterpret_cast<uint4*>(s.win + r * WPITCH + c * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        epi_bar();

        // (2) depthwise + SiLU: output frame t0 - 7 + i reads window rows i .. i + 14.  Warp e owns i in
        // [16e, 16e + 16) (a half unit: 8 frames per half-warp); the flush only needs i in [0, 7).
        const int i_hi = flush ? HALO : BM;
        auto dw_rows = [&](auto nf_tag) {
          constexpr int NF = decltype(nf_tag)::value;
          const int i0 = e * FPW + (NF == FPW ? 0 : (lane >> 4) * NF);
          if (i0 >= i_hi) return;
          const uint8_t* xb = s.win + i0 * WPITCH + lch * 8;
          pk2 acc[NF][2];
#pragma unroll
          for (int r = 0; r < NF + 2 * HALO; ++r) {
            const uint2 v = *reinterpret_cast<const uint2*>(xb + r * WPITCH);
            const pk2 xv[2] = {pk_from_bf16x2(v.x), pk_from_bf16x2(v.y)};
#pragma unroll
            for (int f = 0; f < NF; ++f) {
              const int j = r - f;
              if (j >= 0 && j < KW) {
#pragma unroll
                for (int qq = 0; qq < 2; ++qq) acc[f][qq] = pk_fma(wr[j][qq], xv[qq], j == 0 ? wb[qq] : acc[f][qq]);
              }
            }
          }
          const int tf = t0 - HALO + i0;                 // the lane's first output frame
          const bool boxed = NF == FPW && !flush && tf >= 0 && tf + FPW <= store_end;   // warp-uniform
          uint8_t* ob = s.out[e];
          if (boxed) {
            if (lane == 0) bulk_wait_group_read<0>();  // the previous tile's box has been read by its store
            __syncwarp();
          }
#pragma unroll
          for (int f = 0; f < NF; ++f) {
            const int t = tf + f;
            uint32_t o[2];
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
              const float2 hh = pk_split(acc[f][qq]);
              const float2 s2 =
                  pk_split(pk_fma(acc[f][qq], pk_make(tanh_approx(hh.x), tanh_approx(hh.y)), acc[f][qq]));
              o[qq] = t < len ? pack_bf16x2(s2.x, s2.y) : 0u;
            }
            if (boxed)
              *reinterpret_cast<uint2*>(ob + f * (CH * 2) + lane * 8) = make_uint2(o[0], o[1]);
            else if (i0 + f < i_hi && t >= 0 && t < store_end)
              *reinterpret_cast<uint2*>(drow + (int64_t)t * inner) = make_uint2(o[0], o[1]);
          }
          if (boxed) {
            fence_proxy_async_smem();                    // generic-proxy writes -> visible to the TMA store
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmD, ob, c0, b * p.T + tf);
              bulk_commit_group();
            }
          }
        };
        if (ok && e * FPW < i_hi) {
          if (whole)
            dw_rows(std::integral_constant<int, FPW>{});
          else
            dw_rows(std::integral_constant<int, FPW / 2>{});
        }
        if (!flush && e == 0) {
          // (3) the tile's last 14 rows become the next window's left halo.  Window rows 0..13 are read by this
          // warp alone (output frames i < 16), so it moves them as soon as its own depthwise rows are done; the
          // barrier below then orders the move before the next tile's GLU rows are written
          __syncwarp();
          for (int q2 = lane; q2 < 2 * HALO * 16; q2 += 32) {
            const int r = q2 >> 4, c = q2 & 15;
            *reinterpret_cast<uint4*>(s.win + r * WPITCH + c * 16) =
                *reinterpret_cast<const uint4*>(s.win + (BM + r) * WPITCH + c * 16);
          }
        }
        epi_bar();
      }
    }
    if (lane == 0) bulk_wait_group<0>();   // this warp's output boxes have landed before the CTA ends
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gdw_impl

int launch_gemm_glu_dw(const GemmDwArgs& a, cudaStream_t stream) {
  namespace G = gdw_impl;
  if (a.B <= 0 || a.T <= 0) return 0;
  // W8A8: int8 operands, 128 elements (128 bytes) per box row
  const int kbe = a.a_int8 ? 2 * G::BK : G::BK;
  const int esz = a.a_int8 ? 1 : 2;
  const CUtensorMapDataType dt = a.a_int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (a.T % G::BM || a.K % kbe || a.N % G::BN) return (int)cudaErrorInvalidValue;
  if (a.a_int8 && (!a.col_scale || !a.row_scale || a.row_stats || a.row_partials)) return (int)cudaErrorInvalidValue;
  CUtensorMap tmA, tmW;
  const int64_t M = (int64_t)a.B * a.T;
  {
    const uint64_t dims[2] = {(uint64_t)a.K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)a.K * esz};
    const uint32_t box[2] = {(uint32_t)kbe, G::BM};
    if (int rc = encode_tmap(&tmA, dt, 2, a.a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  CUtensorMap tmW64;
  {
    const uint64_t dims[2] = {(uint64_t)a.K, (uint64_t)a.N};
    const uint64_t strides[1] = {(uint64_t)a.K * esz};
    const uint32_t box[2] = {(uint32_t)kbe, G::BN};
    if (int rc = encode_tmap(&tmW, dt, 2, a.w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    const uint32_t box64[2] = {(uint32_t)kbe, G::BN / 4};
    if (int rc = encode_tmap(&tmW64, dt, 2, a.w, dims, strides, box64, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  CUtensorMap tmD;
  {
    const uint64_t dims[2] = {(uint64_t)(a.N / 2), (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)(a.N / 2) * 2};
    const uint32_t box[2] = {G::CH, G::FPW};
    if (int rc = encode_tmap(&tmD, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.d, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  }
  G::Params p;
  p.bias = a.bias;
  p.col_scale = a.col_scale;
  p.dw_w = a.dw_w;
  p.dw_b = a.dw_b;
  p.d = a.d;
  p.lengths = a.lengths;
  p.row_stats = a.row_stats;
  p.colsum = a.colsum;
  p.row_scale = a.row_scale;
  p.row_partials = a.row_partials;
  p.ln_eps = a.ln_eps;
  p.B = a.B;
  p.T = a.T;
  p.K = a.K;
  p.N = a.N;
  const int smem = (int)sizeof(G::Smem) + 1024;
  if ((a.row_stats || a.row_partials) && !a.colsum) return (int)cudaErrorInvalidValue;
  if (a.row_partials && (a.row_stats || a.col_scale || a.K % 256 || a.K > 2048)) return (int)cudaErrorInvalidValue;
  auto kern = a.a_int8 ? G::gemm_glu_dw_kernel<true, 0, true>
             : a.col_scale ? (a.row_stats ? G::gemm_glu_dw_kernel<true, 1> : G::gemm_glu_dw_kernel<true, 0>)
             : a.row_partials ? G::gemm_glu_dw_kernel<false, 2>
                              : (a.row_stats ? G::gemm_glu_dw_kernel<false, 1> : G::gemm_glu_dw_kernel<false, 0>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return (int)e;
  const int64_t units = (int64_t)a.B * (a.N / G::BN);
  const int sms = device_sm_count();
  const int grid = (int)(units < sms ? units : sms);
  if (grid <= 0) return 0;
  kern<<<grid, G::THREADS, smem, stream>>>(tmA, tmW, tmW64, tmD, p);
  return (int)cudaGetLastError();
}

}  // namespace gsn
