// Pointwise (1x1) convolutions of the Conformer conv module as tcgen05 GEMMs on sm_100a.
//
//   up_conv   (models/granite_speech_nar/conformer.py:165,177) + GLU (:166,:181)  -> kEpiGlu
//   down_conv (conformer.py:170,187) + the block's residual add (conformer.py:207)  -> kEpiResidual
//   feed-forward up_proj + SiLU (conformer.py:27-29,35-36)                          -> kEpiSilu
//   feed-forward down_proj + the block's half-step residual (conformer.py:37,205)   -> kEpiResidual, out_scale 0.5
//
// Layout: A = activations [M, K] bf16 row-major (M = B*T frames, channels-last), W = weights [N, K] (the Conv1d
// weight [N, K, 1] as stored), both K-major, so D = A * W^T accumulates in TMEM in fp32.
//
// Two mainloops share one epilogue:
//  * single CTA per SM (every dtype): warp 0 TMA producer (A 128x64 + W 256x64 per stage, 128-byte swizzle,
//    4-stage ring), warp 1 TMEM allocator + single-thread UMMA issuer (M=128, N=256, K=16), warps 2-5 epilogue,
//    warps 6-9 (int8 weights only) dequantise the staged int8 W tile into the swizzled bf16 layout;
//  * CTA pairs (bf16 weights, compiled in with GSN_GEMM_PAIR=1): cta_group::2 MMA on 256 x 256 tiles, each CTA
//    loading its own halves of A and W (32 KB per K-block), 6-stage ring.
// Persistent grids; one CTA per SM (the shared-memory footprint guarantees it, and with it the 512 TMEM
// columns); the accumulator is double-buffered in TMEM (2 x 256 columns) so the epilogue of tile i overlaps the
// main loop of tile i+1.  Tiles are visited N-fastest so the CTAs sharing an A row-block run at the same time
// and read it from L2.
//
// Epilogue: a warp owns 32 accumulator rows (its TMEM lane quarter).  It keeps the tile's bias / scale columns
// in a shared slice (broadcast reads) and moves results through two 32 x 32 bf16 staging boxes in shared memory
// with the 64-byte swizzle: the residual sub-tile arrives there by TMA (prefetched one sub-tile ahead), each
// lane reads and overwrites its own row (conflict-free under the swizzle) and the box leaves by TMA store, so
// global memory only sees full, coalesced tiles.
//
// With per-utterance lengths (rows b*T .. b*T+T-1 belong to utterance b, T % 128 == 0), 128-row blocks made only
// of padding frames are skipped: the GLU GEMM leaves those rows unwritten (nothing downstream reads them) and the
// residual GEMM writes them as residual + bias, which is what a zero row of A produces.
#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

#ifndef GSN_GEMM_STAGES
#define GSN_GEMM_STAGES 4   // TMA ring depth of the bf16 single-CTA mainloop
#endif

namespace gsn {

namespace gemm_impl {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int A_BYTES = BM * BK * 2;      // 16 KB
constexpr int B_BYTES = BN * BK * 2;      // 32 KB (bf16, swizzled)
constexpr int B8_BYTES = BN * BK;         // 16 KB (int8 staging)
constexpr int BOX = 32;                   // epilogue box: 32 rows x 32 columns bf16
constexpr int BOX_BYTES = BOX * BOX * 2;
constexpr uint32_t TMEM_COLS = 512;

struct KParams {
  const float* bias;
  const float* col_scale;
  const float* row_scale;                 // W8A8: per-row scale of the int8 activations, else null
  const __nv_bfloat16* residual;
  __nv_bfloat16* out;
  const int* lengths;                     // per-utterance valid frames, or null (every row computed)
  int64_t ld_out, ld_res;
  int M, N, K;
  int T;                                  // frames per utterance when lengths != null (T % 128 == 0)
  float out_scale;                        // residual epilogue: out = out_scale * (acc * scale + bias) + residual
  unsigned long long* argmax_keys;        // ARGMAX: per row, the best (bf16 logit, lowest column) as one key
  int n_major;                            // walk tiles column block by column block (W read once)
  int withhold_load;                      // test only: operand load #k of every CTA armed but never issued (-1: none)
  float2* row_partials;                   // RESIDUAL: per row and 256-column block, (mean, M2) of the bf16 output
};

// 128-row block `blk` of the M range holds at least one valid frame (a block lies inside one utterance)
__device__ __forceinline__ bool rows_active(const KParams& p, int blk) {
  const int row = blk * 128;
  if (row >= p.M) return false;
  if (p.lengths == nullptr) return true;
  const int b = row / p.T;
  return row - b * p.T < __ldg(p.lengths + b);
}

__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Row statistics of a packed bf16 pair about the shift k (as fp32 pairs in 64-bit registers): with d = x - k,
// s += d and q += d * d, each lane of the f32x2 FMAs one fmaf (d = x * 1 - k is the rounded difference).
__device__ __forceinline__ void row_stats_pair(uint32_t w, uint64_t nk2, uint64_t& s2, uint64_t& q2) {
  asm("{\n\t.reg .b32 lo, hi;\n\t.reg .b64 x, one, d;\n\t"
      "shl.b32 lo, %2, 16;\n\tand.b32 hi, %2, 0xFFFF0000;\n\tmov.b64 x, {lo, hi};\n\t"
      "mov.b64 one, 0x3F8000003F800000;\n\t"
      "fma.rn.f32x2 d, x, one, %3;\n\t"
      "fma.rn.f32x2 %0, d, one, %0;\n\t"
      "fma.rn.f32x2 %1, d, d, %1;\n\t}"
      : "+l"(s2), "+l"(q2)
      : "r"(w), "l"(nk2));
}

// The tile list every role of a CTA walks (s = blockIdx.x + k * gridDim.x).  With lengths (B = M / T utterances of
// T % 128 == 0 frames), the list holds first the tiles of the 128-row blocks that contain valid frames, so those are
// dealt evenly over the CTAs whatever the utterance lengths, then the tiles of pure padding (only the residual
// epilogue touches them).  Per-utterance prefix counts of both kinds of blocks live in shared memory.
constexpr int kMapMaxB = 512;

struct TileMap {
  int num_n, num_tiles, active_tiles;
  int n_major, act_m;         // n-major walk over the act_m active 128-row blocks
  int mpu, B;                 // 128-row blocks per utterance, utterances (with the map)
  const int* act;             // act[b]: active blocks of utterances < b (B + 1 entries)
  const int* pad;             // pad[b]: padding blocks of utterances < b
  bool mapped;

  __device__ static int upper(const int* pref, int n, int v) {   // largest b with pref[b] <= v
    int lo = 0, hi = n;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (pref[mid] <= v) lo = mid; else hi = mid;
    }
    return lo;
  }

  // tile s -> (m_blk, n_blk); `active` false for a tile of pure padding (or past M)
  __device__ void get(int s, const KParams& p, int& m_blk, int& n_blk, bool& active) const {
    int mi;
    if (n_major) {                // only the active tiles are walked this way
      n_blk = s / act_m;
      mi = s - n_blk * act_m;
    } else {
      mi = s / num_n;
      n_blk = s - mi * num_n;
    }
    if (!mapped) {
      m_blk = mi;
      active = rows_active(p, m_blk);
      return;
    }
    const int na = act[B];
    if (mi < na) {
      const int b = upper(act, B, mi);
      m_blk = b * mpu + (mi - act[b]);
      active = true;
    } else {
      const int ip = mi - na;
      const int b = upper(pad, B, ip);
      m_blk = b * mpu + (act[b + 1] - act[b]) + (ip - pad[b]);
      active = false;
    }
  }
};

// Builds the prefix counts (all threads of the CTA take part; ends with __syncthreads).
__device__ void build_tile_map(TileMap& tm, int* act, int* pad, const KParams& p, int num_m, int num_n) {
  tm.num_n = num_n;
  tm.num_tiles = num_m * num_n;
  tm.mapped = p.lengths != nullptr && p.T > 0 && p.M % p.T == 0 && p.T % BM == 0 && p.M / p.T <= kMapMaxB;
  tm.act = act;
  tm.pad = pad;
  tm.B = tm.mapped ? p.M / p.T : 0;
  tm.mpu = p.T / BM;
  if (tm.mapped) {
    for (int b = threadIdx.x; b < tm.B; b += blockDim.x) {
      const int L = min(max(__ldg(p.lengths + b), 0), p.T);
      act[b + 1] = (L + BM - 1) / BM;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // inclusive scan in chunks of 32, carried across chunks
      int carry_a = 0, carry_p = 0;
      for (int base = 0; base < tm.B; base += 32) {
        const int b = base + (int)threadIdx.x;
        int a = b < tm.B ? act[b + 1] : 0;
        int q = b < tm.B ? tm.mpu - a : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int ya = __shfl_up_sync(0xffffffffu, a, o), yq = __shfl_up_sync(0xffffffffu, q, o);
          if ((int)threadIdx.x >= o) {
            a += ya;
            q += yq;
          }
        }
        if (b < tm.B) {
          act[b + 1] = carry_a + a;
          pad[b + 1] = carry_p + q;
        }
        carry_a += __shfl_sync(0xffffffffu, a, 31);
        carry_p += __shfl_sync(0xffffffffu, q, 31);
      }
      if (threadIdx.x == 0) {
        act[0] = 0;
        pad[0] = 0;
      }
    }
  }
  __syncthreads();
  tm.active_tiles = tm.mapped ? act[tm.B] * num_n : tm.num_tiles;
  tm.act_m = tm.mapped ? act[tm.B] : num_m;
  tm.n_major = p.n_major;
}

// Four signed int8 (one 32-bit word) -> two bf16x2 words, exactly.  Each byte is biased to unsigned
// (v + 128), placed in the low mantissa bits of the fp32 2^23, and the bias 2^23 + 128 is subtracted; every
// |v| <= 127 is exact in bf16.
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.0f;
  const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.0f;
  const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.0f;
  const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.0f;
  lo = pack_bf16x2(f0, f1);
  hi = pack_bf16x2(f2, f3);
}

// int8 -> bf16 (exact integers) for whole weight matrices: two arrays in one launch, 16 bytes per thread.
__global__ void __launch_bounds__(256) widen_i8_kernel(const int8_t* __restrict__ q0, __nv_bfloat16* __restrict__ o0,
                                                       int64_t n0, const int8_t* __restrict__ q1,
                                                       __nv_bfloat16* __restrict__ o1, int64_t n1) {
  const int64_t c0 = n0 / 16, c1 = n1 / 16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < c0 + c1; i += (int64_t)gridDim.x * blockDim.x) {
    const bool first = i < c0;
    const int64_t j = first ? i : i - c0;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(first ? q0 : q1) + j);
    uint4 lo, hi;
    i8x4_to_bf16x4(v.x, lo.x, lo.y);
    i8x4_to_bf16x4(v.y, lo.z, lo.w);
    i8x4_to_bf16x4(v.z, hi.x, hi.y);
    i8x4_to_bf16x4(v.w, hi.z, hi.w);
    uint4* dst = reinterpret_cast<uint4*>(first ? o0 : o1) + 2 * j;
    dst[0] = lo;
    dst[1] = hi;
  }
}

// Shared-memory area of the four epilogue warps.
struct __align__(1024) EpiSmem {
  uint8_t stage[4][2][BOX_BYTES];         // two staging boxes per warp, 64-byte swizzle
  float vec[4][2][BN];                    // per warp: the tile's bias and scale columns
  uint64_t res_full[4][2];                // residual box landed in stage[warp][buffer]
};

// ------------------------------------------------------------------------------------------------------------
// Epilogue of one warp (state lives in registers; one object per epilogue warp).  SCALED: the accumulator is
// multiplied by a per-output-column scale (int8 weights, staged as int8 or already widened to bf16).  A8: the
// accumulator is an s32 sum of int8 products (W8A8), converted to fp32 and multiplied by its row's scale first.
template <int EPI, bool SCALED, bool A8 = false>
struct Epilogue {
  static constexpr int NU = (EPI == kEpiGlu ? BN / 2 : BN) / BOX;   // 32-column output sub-tiles per tile
  float alpha;                            // residual epilogue: scale of acc * scale + bias
  const int* lengths;                     // SiLU epilogue: rows of padding frames are written as zero
  int T;
  float* vb;
  float* vs;
  uint8_t* stage0;                        // stage box b at stage0 + b * BOX_BYTES
  uint64_t* res0;                         // its barrier at res0 + b
  const CUtensorMap* tmO;
  const CUtensorMap* tmR;
  unsigned long long* argmax_keys;
  int M;
  const float* row_scale;
  float rs;                               // A8: this lane's row scale for the current tile
  float2* row_partials;                   // RESIDUAL: output row statistics per 256-column block, or null
  int n_part;
  bool has_res;
  int lane, swz;
  uint32_t su;                            // sub-tiles handled so far: buffer su & 1, its use count su >> 1
  uint32_t res_pend;                      // lane 0: buffers whose residual copy is issued and not yet waited for
  uint32_t res_par;                       //   and, bit b, the phase parity buffer b's copy completes

  __device__ void init(EpiSmem& e, int ew, const CUtensorMap* o, const CUtensorMap* r, const KParams& p) {
    vb = e.vec[ew][0];
    vs = e.vec[ew][1];
    stage0 = e.stage[ew][0];
    res0 = &e.res_full[ew][0];
    tmO = o;
    tmR = r;
    argmax_keys = p.argmax_keys;
    M = p.M;
    row_scale = p.row_scale;
    rs = 1.0f;
    row_partials = EPI == kEpiResidual ? p.row_partials : nullptr;
    n_part = p.N / BN;
    has_res = EPI == kEpiResidual && p.residual != nullptr;
    alpha = EPI == kEpiResidual ? p.out_scale : 1.0f;
    lengths = p.lengths;
    T = p.T;
    lane = threadIdx.x & 31;
    swz = (lane >> 1) & 3;
    su = 0;
    res_pend = 0;
    res_par = 0;
  }

  // The tile's 256 bias (and scale) values into the warp's slice.  For the GLU they are halved:
  // a * sigmoid(g) = a' + a' * tanh(g') with a' = a / 2 and g' = g / 2 (exact scalings).
  __device__ void load_vectors(const KParams& p, int nb) {
    // GLU works on halved pre-activations (a * sigmoid(g) = a' + a' * tanh(g')); SiLU and the residual
    // epilogue take the vectors as they are
    const float h = EPI == kEpiGlu ? 0.5f : 1.0f;
    __syncwarp();
    const float4* src = reinterpret_cast<const float4*>(p.bias + nb);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float4 b = __ldg(src + lane + 32 * i);
      b.x *= h; b.y *= h; b.z *= h; b.w *= h;
      reinterpret_cast<float4*>(vb)[lane + 32 * i] = b;
      if (SCALED) {
        float4 sc = __ldg(reinterpret_cast<const float4*>(p.col_scale + nb) + lane + 32 * i);
        sc.x *= h; sc.y *= h; sc.z *= h; sc.w *= h;
        reinterpret_cast<float4*>(vs)[lane + 32 * i] = sc;
      }
    }
    __syncwarp();
  }

  // accumulator word -> fp32 (A8: exact s32 sum, converted, times the row scale)
  __device__ __forceinline__ float accf(uint32_t bits) const {
    if constexpr (A8) return (float)(int32_t)bits * rs;
    return __uint_as_float(bits);
  }

  // residual of sub-tile `sub` (buffer sub & 1, completing that buffer's phase of parity (sub >> 1) & 1)
  __device__ void load_residual(uint32_t sub, int col, int row0) {
    const uint32_t buf = sub & 1;
    res_pend |= 1u << buf;
    res_par = (res_par & ~(1u << buf)) | (((sub >> 1) & 1u) << buf);
    mbar_arrive_expect_tx(res0 + buf, BOX_BYTES);
    tma_load_2d(stage0 + buf * BOX_BYTES, tmR, res0 + buf, col, row0);
  }

  // residual of the tile's first sub-tile, issued before the accumulator is waited for
  __device__ void prefetch_first(int ocol0, int row0) {
    if (has_res && lane == 0) {
      bulk_wait_group_read<0>();          // the buffer's previous store has read it
      load_residual(su, ocol0, row0);
    }
  }

  // Drain one tile: `t_row` is the TMEM address of this warp's accumulator rows (unused when !active, i.e. a
  // residual tile of pure padding).  Returns false if a wait ran out.
  __device__ bool run(int row0, int ocol0, bool active, uint32_t t_row, volatile int* abort_flag) {
    if constexpr (EPI == kEpiArgmax) {
      // best bf16-rounded logit of this lane's row over the tile's 256 columns (first column on ties), folded
      // into the row's key: (order-preserving bits of the value) << 32 | ~column, so atomicMax keeps the largest
      // value and, among equal values, the lowest column
      float best = -INFINITY;
      int best_col = ocol0;
      for (int u = 0; u < NU; ++u) {
        uint32_t v[2][16];
        tmem_ld16(t_row + (uint32_t)(u * BOX), v[0]);
        tmem_ld16(t_row + (uint32_t)(u * BOX + 16), v[1]);
        tmem_wait_ld_dep(v[0], v[1]);
#pragma unroll
        for (int k = 0; k < BOX; ++k) {
          const float x = bf16_round_f32(__uint_as_float(v[k >> 4][k & 15]) + vb[u * BOX + k]);
          if (x > best) {
            best = x;
            best_col = ocol0 + u * BOX + k;
          }
        }
      }
      const int row = row0 + lane;
      if (row < M && best_col >= 0) {
        uint32_t bits = __float_as_uint(best);
        bits = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
        const unsigned long long key =
            ((unsigned long long)bits << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)best_col);
        atomicMax(argmax_keys + row, key);
      }
      return true;
    }
    if constexpr (A8) {
      const int row = row0 + lane;
      rs = row < M ? __ldg(row_scale + row) : 0.f;
    }
    // SiLU: this lane's row is a padding frame -> zero, so the next GEMM sees what a masked input gives
    // RESIDUAL with row_partials: the tile row's 256 bf16 outputs as (mean, M2), summed about the row's first output
    // (a shift near the mean keeps the sum of squares free of cancellation); the next LayerNorm merges the blocks
    float ps_k = 0.f;
    uint64_t ps_nk2 = 0;                                // (-k, -k)
    uint64_t ps_s2[4] = {0, 0, 0, 0}, ps_q2[4] = {0, 0, 0, 0};   // four independent chains of fp32-pair sums
    bool row_valid = true;
    if (EPI == kEpiSilu && lengths != nullptr) {
      const int row = row0 + lane;
      const int b = row / T;
      row_valid = row - b * T < __ldg(lengths + b);
    }
    for (int u = 0; u < NU; ++u, ++su) {
      const uint32_t buf = su & 1;
      uint8_t* sb = stage0 + buf * BOX_BYTES;
      if (has_res) {
        if (lane == 0 && u + 1 < NU) {    // prefetch the next residual sub-tile into the other buffer
          bulk_wait_group_read<0>();
          load_residual(su + 1, ocol0 + (u + 1) * BOX, row0);
        }
      } else {
        if (lane == 0) bulk_wait_group_read<1>();   // the store that last used this buffer has read it
        __syncwarp();
      }
      float o[BOX];
      if (EPI == kEpiGlu) {
        // accumulator columns [0,128) = value channels, [128,256) = their gate channels
        uint32_t va[2][16], vg[2][16];
        tmem_ld16(t_row + (uint32_t)(u * BOX), va[0]);
        tmem_ld16(t_row + (uint32_t)(u * BOX + 16), va[1]);
        tmem_ld16(t_row + (uint32_t)(BN / 2 + u * BOX), vg[0]);
        tmem_ld16(t_row + (uint32_t)(BN / 2 + u * BOX + 16), vg[1]);
        tmem_wait_ld_dep(va[0], va[1]);
        tmem_wait_ld_dep(vg[0], vg[1]);
#pragma unroll
        for (int c4 = 0; c4 < BOX; c4 += 4) {
          const int j = u * BOX + c4;
          const float4 ba = lds4(vb + j), bg = lds4(vb + BN / 2 + j);
          float4 sa = make_float4(0.5f, 0.5f, 0.5f, 0.5f), sg = sa;
          if (SCALED) {
            sa = lds4(vs + j);
            sg = lds4(vs + BN / 2 + j);
          }
          const float bav[4] = {ba.x, ba.y, ba.z, ba.w}, bgv[4] = {bg.x, bg.y, bg.z, bg.w};
          const float sav[4] = {sa.x, sa.y, sa.z, sa.w}, sgv[4] = {sg.x, sg.y, sg.z, sg.w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int k = c4 + c;
            const float a = fmaf(accf(va[k >> 4][k & 15]), sav[c], bav[c]);   // value / 2
            const float g = fmaf(accf(vg[k >> 4][k & 15]), sgv[c], bgv[c]);   // gate / 2
            o[k] = fmaf(a, tanh_approx(g), a);
          }
        }
      } else {
        uint32_t v[2][16];
        if (active) {
          tmem_ld16(t_row + (uint32_t)(u * BOX), v[0]);
          tmem_ld16(t_row + (uint32_t)(u * BOX + 16), v[1]);
          tmem_wait_ld_dep(v[0], v[1]);
        } else {
#pragma unroll
          for (int c = 0; c < 16; ++c) v[0][c] = v[1][c] = 0u;   // padding rows: out = residual + bias
        }
#pragma unroll
        for (int c4 = 0; c4 < BOX; c4 += 4) {
          const int j = u * BOX + c4;
          const float4 bb = lds4(vb + j);
          float4 sc = make_float4(1.f, 1.f, 1.f, 1.f);
          if (SCALED) sc = lds4(vs + j);
          const float bv[4] = {bb.x, bb.y, bb.z, bb.w}, sv[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int k = c4 + c;
            o[k] = fmaf(accf(v[k >> 4][k & 15]), sv[c], bv[c]);
            if (EPI == kEpiSilu) {
              // the Linear output is a bf16 tensor before the SiLU (conformer.py:35-36): round it, then
              // silu(y) = h + h tanh(h) with h = y / 2
              const float hh = 0.5f * bf16_round_f32(o[k]);
              o[k] = row_valid ? fmaf(hh, tanh_approx(hh), hh) : 0.f;
            } else if (alpha != 1.0f) {
              // the scaled residual of the feed-forward halves: the Linear output is rounded to bf16 before the
              // 0.5 * ff(x) + x of ConformerBlock.forward (conformer.py:205)
              o[k] = alpha * bf16_round_f32(o[k]);
            }
          }
        }
        if (has_res) {
          bool got = mbar_wait_bounded(res0 + buf, (su >> 1) & 1, abort_flag, kStatusTimeoutEpilogue);
          got = __shfl_sync(0xffffffffu, got, 0);
          if (!got) return false;
          res_pend &= ~(1u << buf);
        }
      }
      // lane = row of the 32 x 32 box; 16-byte chunk c of the row sits at chunk c ^ ((row >> 1) & 3)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4* pc = reinterpret_cast<uint4*>(sb + lane * 64 + ((c ^ swz) << 4));
        float r[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (has_res) {
          const uint4 rv = *pc;
          const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            r[2 * i] = bf16lo_to_f32(rw[i]);
            r[2 * i + 1] = bf16hi_to_f32(rw[i]);
          }
        }
        uint4 w;
        w.x = pack_bf16x2(o[c * 8 + 0] + r[0], o[c * 8 + 1] + r[1]);
        w.y = pack_bf16x2(o[c * 8 + 2] + r[2], o[c * 8 + 3] + r[3]);
        w.z = pack_bf16x2(o[c * 8 + 4] + r[4], o[c * 8 + 5] + r[5]);
        w.w = pack_bf16x2(o[c * 8 + 6] + r[6], o[c * 8 + 7] + r[7]);
        *pc = w;
        if (EPI == kEpiResidual && row_partials != nullptr) {
          if (u == 0 && c == 0) {
            ps_k = bf16lo_to_f32(w.x);
            const uint32_t nk = __float_as_uint(-ps_k);
            ps_nk2 = ((uint64_t)nk << 32) | nk;
          }
          row_stats_pair(w.x, ps_nk2, ps_s2[0], ps_q2[0]);
          row_stats_pair(w.y, ps_nk2, ps_s2[1], ps_q2[1]);
          row_stats_pair(w.z, ps_nk2, ps_s2[2], ps_q2[2]);
          row_stats_pair(w.w, ps_nk2, ps_s2[3], ps_q2[3]);
        }
      }
      fence_proxy_async_smem();          // the generic-proxy writes are visible to the TMA store
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmO, sb, ocol0 + u * BOX, row0);
        bulk_commit_group();
      }
    }
    if (EPI == kEpiResidual && row_partials != nullptr && row0 + lane < M) {
      constexpr float inv = 1.0f / BN;
      float ps_s = 0.f, ps_q = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ps_s += __uint_as_float((uint32_t)ps_s2[i]) + __uint_as_float((uint32_t)(ps_s2[i] >> 32));
        ps_q += __uint_as_float((uint32_t)ps_q2[i]) + __uint_as_float((uint32_t)(ps_q2[i] >> 32));
      }
      const float mt = ps_s * inv;
      row_partials[(int64_t)(row0 + lane) * n_part + ocol0 / BN] =
          make_float2(ps_k + mt, fmaxf(fmaf(-ps_s, mt, ps_q), 0.f));
    }
    return true;
  }

  __device__ void finish() {
    if (lane == 0) {
      bulk_wait_group<0>();               // every store of this warp has landed before the CTA ends
      // after an unwind, residual copies still in flight land before the shared memory is released (bounded)
      for (uint32_t b = 0; b < 2; ++b)
        if (res_pend & (1u << b))
          mbar_wait_bounded(res0 + b, (res_par >> b) & 1u, nullptr, kStatusTimeoutEpilogue, 100000000ull);
    }
    __syncwarp();
  }
};

__device__ __forceinline__ void init_epi_barriers(EpiSmem& e) {
  for (int w = 0; w < 4; ++w) {
    mbar_init(&e.res_full[w][0], 1);
    mbar_init(&e.res_full[w][1], 1);
  }
}

// ================================================================================================================
// single CTA per SM
template <bool W_I8>
struct Cfg {
  static constexpr int STAGES = W_I8 ? 3 : GSN_GEMM_STAGES;
  static constexpr int THREADS = W_I8 ? 320 : 192;
};

template <bool W_I8>
struct __align__(1024) Smem {
  uint8_t a[Cfg<W_I8>::STAGES][A_BYTES];
  uint8_t b[Cfg<W_I8>::STAGES][B_BYTES];
  uint8_t b8[W_I8 ? Cfg<W_I8>::STAGES : 1][W_I8 ? B8_BYTES : 16];
  EpiSmem epi;
  uint64_t full[Cfg<W_I8>::STAGES];
  uint64_t full_b[Cfg<W_I8>::STAGES];     // int8: converted W tile ready
  uint64_t empty[Cfg<W_I8>::STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t mma_done;
  int map_act[kMapMaxB + 1];
  int map_pad[kMapMaxB + 1];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(offsetof(Smem<false>, b) % 1024 == 0 && offsetof(Smem<true>, b8) % 1024 == 0, "tile alignment");
static_assert(offsetof(Smem<false>, epi) % 1024 == 0 && offsetof(Smem<true>, epi) % 1024 == 0, "box alignment");
static_assert(sizeof(Smem<false>) + 1024 <= 232448 && sizeof(Smem<true>) + 1024 <= 232448, "shared memory size");

// A8 (W8A8): A and W are int8 with 128 elements (128 bytes) per K-block, the same bytes per stage and the same
// swizzled layout as 64 bf16; four kind::i8 MMAs of K = 32 per K-block, s32 accumulators.
template <int EPI, bool W_I8, bool SCALED, bool A8 = false>
__global__ void __launch_bounds__(Cfg<W_I8>::THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR, KParams p) {
  static_assert(!(A8 && W_I8), "W8A8 tiles are loaded as int8 and used as int8");
  constexpr int STAGES = Cfg<W_I8>::STAGES;
  constexpr uint32_t IDESC = A8 ? make_idesc_s8_s32(BM, BN) : make_idesc_bf16_f32(BM, BN);
  constexpr int KBE = A8 ? 2 * BK : BK;      // elements per K-block
  extern __shared__ uint8_t smem_raw[];
  Smem<W_I8>& s =
      *reinterpret_cast<Smem<W_I8>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = p.N / BN;
  const int num_kb = (p.K + KBE - 1) / KBE;   // a partial last K-block is completed with zeros by TMA

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.full_b[i], 4);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 4);
    }
    init_epi_barriers(s.epi);
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  TileMap tmap;
  build_tile_map(tmap, s.map_act, s.map_pad, p, num_m, num_n);
  const uint32_t tmem_base = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    const uint64_t pol_w = l2_policy_evict_last();
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tmap.active_tiles && ok; tile += gridDim.x) {
      int m_blk, n_blk;
      bool active;
      tmap.get(tile, p, m_blk, n_blk, active);
      if (!active) continue;
      for (int kb = 0; kb < num_kb; ++kb) {
        bool got = mbar_wait_bounded(&s.empty[stage], phase ^ 1u, abort_flag, kStatusTimeoutProducer);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
          ok = false;
          break;
        }
        if (lane == 0) {
          if (issued == p.withhold_load) {
            // test only: the stage is armed for its bytes but no copy is issued, so its phase never completes
            mbar_arrive_expect_tx(&s.full[stage], W_I8 ? A_BYTES + B8_BYTES : A_BYTES + B_BYTES);
          } else if (W_I8) {
            mbar_arrive_expect_tx(&s.full[stage], A_BYTES + B8_BYTES);
            tma_load_2d(s.a[stage], &tmA, &s.full[stage], kb * BK, m_blk * BM);
            tma_load_2d_hint(s.b8[stage], &tmW, &s.full[stage], kb * BK, n_blk * BN, pol_w);
          } else {
            mbar_arrive_expect_tx(&s.full[stage], A_BYTES + B_BYTES);
            tma_load_2d(s.a[stage], &tmA, &s.full[stage], kb * KBE, m_blk * BM);
            tma_load_2d_hint(s.b[stage], &tmW, &s.full[stage], kb * KBE, n_blk * BN, pol_w);
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
    if (!ok && lane == 0) {
      // Unwinding after a timeout: let the copies still in flight land before the CTA releases its shared
      // memory.  Only the last STAGES loads can be outstanding; wait for each with a short bound.
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
    for (int tile = blockIdx.x; tile < tmap.active_tiles && ok; tile += gridDim.x) {
      int m_blk, n_blk;
      bool active;
      tmap.get(tile, p, m_blk, n_blk, active);
      if (!active) continue;
      const int acc = local & 1;
      const uint32_t use_par = (uint32_t)((local >> 1) & 1);
      ++local;
      bool got = mbar_wait_bounded(&s.tempty[acc], use_par ^ 1u, abort_flag, kStatusTimeoutMma);
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
      for (int kb = 0; kb < num_kb; ++kb) {
        bool ready = mbar_wait_bounded(&s.full[stage], phase, abort_flag, kStatusTimeoutMma);
        if (W_I8 && ready) ready = mbar_wait_bounded(&s.full_b[stage], phase, abort_flag, kStatusTimeoutMma);
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
          for (int k = 0; k < BK / 16; ++k) {
            // +32 bytes per K=16 (bf16) or K=32 (int8) slice inside the 128-byte swizzled row: +2 in the
            // (addr >> 4) field
            if constexpr (A8)
              umma_i8(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), IDESC, (kb | k) != 0 ? 1u : 0u);
            else
              umma_f16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), IDESC,
                       (kb | k) != 0 ? 1u : 0u);
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
    // every MMA issued by this CTA has completed once mma_done flips (bounded: also the unwind path)
    if (lane == 0) umma_commit(&s.mma_done);
    __syncwarp();
    mbar_wait_bounded(&s.mma_done, 0, nullptr, kStatusTimeoutMma, 100000000ull);
  } else if (warp < 6) {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int q = warp & 3;           // a warp may only read its own 32-lane quarter of TMEM
    Epilogue<EPI, SCALED, A8> epi;
    epi.init(s.epi, warp - 2, &tmO, &tmR, p);
    int local = 0;
    const int epi_tiles = EPI == kEpiResidual ? tmap.num_tiles : tmap.active_tiles;
    for (int tile = blockIdx.x; tile < epi_tiles; tile += gridDim.x) {
      int m_blk, n_blk;
      bool active;
      tmap.get(tile, p, m_blk, n_blk, active);
      if (EPI != kEpiResidual && !active) continue;   // GLU / SiLU rows of padding frames are never read downstream
      const int nb = n_blk * BN;
      epi.load_vectors(p, nb);
      const int row0 = m_blk * BM + q * 32;
      const int ocol0 = EPI == kEpiGlu ? n_blk * (BN / 2) : nb;
      epi.prefetch_first(ocol0, row0);
      int acc = 0;
      uint32_t t_row = 0;
      if (active) {
        acc = local & 1;
        const uint32_t use_par = (uint32_t)((local >> 1) & 1);
        ++local;
        bool got = mbar_wait_bounded(&s.tfull[acc], use_par, abort_flag, kStatusTimeoutEpilogue);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) break;
        tc_fence_after();
        t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      }
      const bool ok = epi.run(row0, ocol0, active, t_row, abort_flag);
      if (active) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.tempty[acc]);
      }
      if (!ok) break;
    }
    epi.finish();
  } else if (W_I8) {
    // ---------------------------------------------------------------- int8 -> bf16 W converter (warps 6..9)
    const int ct = threadIdx.x - 192;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tmap.active_tiles && ok; tile += gridDim.x) {
      int m_blk, n_blk;
      bool active;
      tmap.get(tile, p, m_blk, n_blk, active);
      if (!active) continue;
      for (int kb = 0; kb < num_kb; ++kb) {
        bool got = mbar_wait_bounded(&s.full[stage], phase, abort_flag, kStatusTimeoutMma);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
          ok = false;
          break;
        }
        const uint8_t* src = s.b8[stage];
        uint8_t* dst = s.b[stage];
#pragma unroll 4
        for (int it = 0; it < (BN * 8) / 128; ++it) {
          const int task = it * 128 + ct;
          const int n = task >> 3;      // W row inside the tile
          const int c = task & 7;       // 8-element chunk along K
          const uint2 w8 = *reinterpret_cast<const uint2*>(src + n * BK + c * 8);
          uint4 o;
          i8x4_to_bf16x4(w8.x, o.x, o.y);
          i8x4_to_bf16x4(w8.y, o.z, o.w);
          // 128-byte swizzle: 16-byte chunk c of row n lands at chunk (c ^ (n % 8))
          *reinterpret_cast<uint4*>(dst + n * 128 + ((c ^ (n & 7)) << 4)) = o;
        }
        fence_proxy_async_smem();   // generic-proxy writes -> visible to the tensor core (async proxy)
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.full_b[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ================================================================================================================
// bf16 weights on CTA pairs: cta_group::2 MMA, 256 x 256 tiles per pair.
//
// The two CTAs of a cluster share one 256 x 256 output tile.  Each CTA loads its own half of A (128 rows) and its
// own half of W (128 rows) per K-block (16 KB + 16 KB), so a 6-stage ring fits.  The even CTA issues one M=256,
// N=256, K=16 MMA per slice that reads both CTAs' shared memory and writes both CTAs' TMEM (rows 0-127 in the
// even CTA, 128-255 in the odd one); each CTA's epilogue then drains its own 128 rows.  Synchronisation:
//   full[s]   (even CTA)  both CTAs' TMA bytes of stage s; armed by the even CTA's producer
//   empty[s]  (each CTA)  the pair's MMAs reading stage s completed (two commits from the even CTA)
//   tfull[a]  (each CTA)  accumulator buffer a complete (two commits)
//   tempty[a] (even CTA)  both CTAs' epilogues drained buffer a (8 warp arrivals, 4 of them remote)
// A cluster barrier ends the kernel so neither CTA leaves while the other may still touch its shared memory.
namespace pair_impl {

constexpr int STAGES = 6;
constexpr int HALF_BYTES = 128 * BK * 2;      // 16 KB: half of A or half of W per K-block

struct __align__(1024) Smem {
  uint8_t a[STAGES][HALF_BYTES];
  uint8_t b[STAGES][HALF_BYTES];
  EpiSmem epi;
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(offsetof(Smem, epi) % 1024 == 0 && offsetof(Smem, b) % 1024 == 0, "alignment");
static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory size");

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR, KParams p) {
  constexpr uint32_t IDESC = make_idesc_bf16_f32(256, 256);
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();      // 0: issues the MMAs; 1: peer
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;
  const int num_mp = (p.M + 255) / 256;
  const int num_n = p.N / BN;
  const int num_tiles = num_mp * num_n;
  const int num_kb = p.K / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 8);
    }
    init_epi_barriers(s.epi);
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc_pair(&s.tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();                               // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;
  auto pair_active = [&](int mp) { return rows_active(p, 2 * mp) || rows_active(p, 2 * mp + 1); };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    const uint64_t pol_w = l2_policy_evict_last();
    const uint64_t pol_a = l2_policy_evict_normal();   // A row-blocks are re-read by the pairs of the other N tiles
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int tile = pair; tile < num_tiles && ok; tile += n_pairs) {
      const int mp = tile / num_n;
      const int n_blk = tile - mp * num_n;
      if (!pair_active(mp)) continue;
      for (int kb = 0; kb < num_kb; ++kb) {
        bool got = mbar_wait_bounded(&s.empty[stage], phase ^ 1u, abort_flag, kStatusTimeoutProducer);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t full0 = mapa_shared(smem_u32(&s.full[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&s.full[stage], 4 * HALF_BYTES);
          tma_load_2d_pair(s.a[stage], &tmA, full0, kb * BK, mp * 256 + (int)rank * 128, pol_a);
          tma_load_2d_pair(s.b[stage], &tmW, full0, kb * BK, n_blk * BN + (int)rank * 128, pol_w);
        }
        __syncwarp();
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && lane == 0 && rank == 0) {
      // unwinding after a timeout: let the copies still counted on this CTA's full barriers land
      for (int back = 1; back <= STAGES && back <= issued; ++back) {
        const int idx = issued - back;
        mbar_wait_bounded(&s.full[idx % STAGES], (uint32_t)((idx / STAGES) & 1), nullptr, kStatusTimeoutProducer,
                          100000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- pair MMA issuer (even CTA only)
    if (rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int tile = pair; tile < num_tiles && ok; tile += n_pairs) {
        if (!pair_active(tile / num_n)) continue;
        const int acc = local & 1;
        const uint32_t use_par = (uint32_t)((local >> 1) & 1);
        ++local;
        bool got = mbar_wait_cluster_bounded(&s.tempty[acc], use_par ^ 1u, abort_flag, kStatusTimeoutMma);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) break;
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
            for (int k = 0; k < BK / 16; ++k)
              umma_f16_pair(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), IDESC,
                            (kb | k) != 0 ? 1u : 0u);
            const uint32_t e = smem_u32(&s.empty[stage]);
            umma_commit_pair(mapa_shared(e, 0));
            umma_commit_pair(mapa_shared(e, 1));
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (lane == 0) {
          const uint32_t t = smem_u32(&s.tfull[acc]);
          umma_commit_pair(mapa_shared(t, 0));
          umma_commit_pair(mapa_shared(t, 1));
        }
        __syncwarp();
      }
      if (lane == 0) umma_commit_pair(mapa_shared(smem_u32(&s.mma_done), 0));
      __syncwarp();
      mbar_wait_bounded(&s.mma_done, 0, nullptr, kStatusTimeoutMma, 100000000ull);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5, both CTAs)
    const int q = warp & 3;
    Epilogue<EPI, false> epi;
    epi.init(s.epi, warp - 2, &tmO, &tmR, p);
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += n_pairs) {
      const int mp = tile / num_n;
      const int n_blk = tile - mp * num_n;
      const bool active = pair_active(mp);
      if (EPI != kEpiResidual && !active) continue;
      const int nb = n_blk * BN;
      epi.load_vectors(p, nb);
      const int row0 = mp * 256 + (int)rank * 128 + q * 32;
      const int ocol0 = EPI == kEpiGlu ? n_blk * (BN / 2) : nb;
      epi.prefetch_first(ocol0, row0);
      int acc = 0;
      uint32_t t_row = 0;
      if (active) {
        acc = local & 1;
        const uint32_t use_par = (uint32_t)((local >> 1) & 1);
        ++local;
        bool got = mbar_wait_bounded(&s.tfull[acc], use_par, abort_flag, kStatusTimeoutEpilogue);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) break;
        tc_fence_after();
        t_row = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      }
      const bool ok = epi.run(row0, ocol0, active, t_row, abort_flag);
      if (active) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&s.tempty[acc]), 0));
      }
      if (!ok) break;
    }
    epi.finish();
  }

  tc_fence_before();
  cluster_sync();                               // the other CTA no longer reads or signals this CTA's memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace pair_impl

// ------------------------------------------------------------------------------------------------------------
// host side
int encode_operands(const GemmArgs& a, int epilogue, int a_rows, int w_rows, CUtensorMap* tmA, CUtensorMap* tmW,
                    CUtensorMap* tmO, CUtensorMap* tmR) {
  if (a.a_int8) {
    // W8A8: int8 A and W, 128 elements (128 bytes) per box row, 128-byte swizzle like the bf16 tiles
    const uint64_t adims[2] = {(uint64_t)a.K, (uint64_t)a.M};
    const uint64_t astrides[1] = {(uint64_t)a.K};
    const uint32_t abox[2] = {2 * BK, (uint32_t)a_rows};
    int rc = encode_tmap(tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a.a, adims, astrides, abox,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint64_t wdims[2] = {(uint64_t)a.K, (uint64_t)a.N};
    const uint32_t wbox[2] = {2 * BK, (uint32_t)w_rows};
    rc = encode_tmap(tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a.w, wdims, astrides, wbox, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    {
      const uint64_t dims[2] = {(uint64_t)a.K, (uint64_t)a.M};
      const uint64_t strides[1] = {(uint64_t)a.K * 2};
      const uint32_t box[2] = {BK, (uint32_t)a_rows};
      int rc = encode_tmap(tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.a, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    }
    {
      const uint64_t dims[2] = {(uint64_t)a.K, (uint64_t)a.N};
      const uint64_t strides[1] = {(uint64_t)a.K * (a.w_int8 ? 1 : 2)};
      const uint32_t box[2] = {BK, (uint32_t)w_rows};
      int rc = encode_tmap(tmW, a.w_int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.w,
                           dims, strides, box, a.w_int8 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    }
  }
  if (tmO == nullptr) return 0;   // no output tensor (argmax epilogue)
  {
    // output (and residual) move as 32 x 32 bf16 boxes with the 64-byte swizzle
    const uint64_t dims[2] = {(uint64_t)(epilogue == kEpiGlu ? a.N / 2 : a.N), (uint64_t)a.M};
    const uint64_t strides[1] = {(uint64_t)a.ld_out * 2};
    const uint32_t box[2] = {BOX, BOX};
    int rc = encode_tmap(tmO, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.out, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
  }
  if (epilogue == kEpiResidual && a.residual != nullptr) {
    const uint64_t dims[2] = {(uint64_t)a.N, (uint64_t)a.M};
    const uint64_t strides[1] = {(uint64_t)a.ld_res * 2};
    const uint32_t box[2] = {BOX, BOX};
    int rc = encode_tmap(tmR, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.residual, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
  } else {
    *tmR = *tmO;   // never read
  }
  return 0;
}

KParams make_params(const GemmArgs& a) {
  KParams p;
  p.bias = a.bias;
  p.col_scale = a.col_scale;
  p.row_scale = a.row_scale;
  p.residual = a.residual;
  p.out = a.out;
  p.lengths = a.lengths;
  p.ld_out = a.ld_out;
  p.ld_res = a.ld_res;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.T = a.T;
  p.out_scale = a.out_scale;
  p.argmax_keys = a.argmax_keys;
  p.n_major = a.n_major;
  p.withhold_load = a.withhold_load;
  p.row_partials = a.row_partials;
  return p;
}

template <int EPI, bool W_I8, bool SCALED, bool A8 = false>
int launch_single(const GemmArgs& a, cudaStream_t stream) {
  CUtensorMap tmA, tmW, tmO, tmR;
  if (EPI == kEpiArgmax) {
    // no output tensor: the keys are written by atomics (the store maps are never read)
    if (int rc = encode_operands(a, EPI, BM, BN, &tmA, &tmW, nullptr, nullptr)) return rc;
    tmO = tmA;
    tmR = tmA;
  } else if (int rc = encode_operands(a, EPI, BM, BN, &tmA, &tmW, &tmO, &tmR)) {
    return rc;
  }
  const KParams p = make_params(a);
  const int smem = (int)sizeof(Smem<W_I8>) + 1024;
  auto kern = gemm_kernel<EPI, W_I8, SCALED, A8>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return (int)e;
  const int tiles = ((a.M + BM - 1) / BM) * (a.N / BN);
  const int sms = device_sm_count();
  const int grid = tiles < sms ? tiles : sms;
  if (grid <= 0) return 0;
  kern<<<grid, Cfg<W_I8>::THREADS, smem, stream>>>(tmA, tmW, tmO, tmR, p);
  return (int)cudaGetLastError();
}

// Number of CTA pairs that can be resident at once (0 if the pair kernel cannot be scheduled).
template <int EPI>
int resident_pairs(int smem) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  static int cached[2][64] = {};
  if (dev < 64 && cached[EPI][dev] != 0) return cached[EPI][dev] > 0 ? cached[EPI][dev] : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, pair_impl::gemm_pair_kernel<EPI>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  if (dev < 64) cached[EPI][dev] = n > 0 ? n : -1;
  return n;
}

// Returns with *launched = false (and status 0) when no CTA pair can be scheduled.
template <int EPI>
int launch_pair(const GemmArgs& a, cudaStream_t stream, bool* launched) {
  *launched = false;
  const int smem = (int)sizeof(pair_impl::Smem) + 1024;
  auto kern = pair_impl::gemm_pair_kernel<EPI>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return (int)e;
  const int pairs = resident_pairs<EPI>(smem);
  if (pairs <= 0) return 0;
  CUtensorMap tmA, tmW, tmO, tmR;
  if (int rc = encode_operands(a, EPI, 128, 128, &tmA, &tmW, &tmO, &tmR)) return rc;
  const KParams p = make_params(a);
  const int tiles = ((a.M + 255) / 256) * (a.N / BN);
  const int n = tiles < pairs ? tiles : pairs;
  *launched = true;
  if (n <= 0) return 0;
  kern<<<2 * n, 192, smem, stream>>>(tmA, tmW, tmO, tmR, p);
  return (int)cudaGetLastError();
}

}  // namespace gemm_impl
using namespace gemm_impl;

// The CTA-pair mainloop is compiled in only when GSN_GEMM_PAIR is set to 1 (see the measurements of both
// mainloops on the conv-module shapes).
#ifndef GSN_GEMM_PAIR
#define GSN_GEMM_PAIR 0
#endif

int launch_widen_i8(const void* q0, void* o0, int64_t n0, const void* q1, void* o1, int64_t n1,
                    cudaStream_t stream) {
  if (n0 % 16 || n1 % 16) return (int)cudaErrorInvalidValue;
  const int64_t chunks = (n0 + n1) / 16;
  if (chunks == 0) return 0;
  const int64_t want = (chunks + 255) / 256;
  const int64_t cap = 8LL * device_sm_count();
  const int grid = (int)(want < cap ? want : cap);
  widen_i8_kernel<<<grid, 256, 0, stream>>>((const int8_t*)q0, (__nv_bfloat16*)o0, n0, (const int8_t*)q1,
                                            (__nv_bfloat16*)o1, n1);
  return (int)cudaGetLastError();
}

int launch_gemm(const GemmArgs& a, int epilogue, cudaStream_t stream) {
  if (a.a_int8) {
    // W8A8: int8 activations with per-row scales, int8 weights with per-column scales
    if (!a.w_int8 || !a.col_scale || !a.row_scale || a.K % 16 || a.out_scale != 1.0f ||
        (epilogue != kEpiGlu && epilogue != kEpiResidual))
      return (int)cudaErrorInvalidValue;
    return epilogue == kEpiGlu ? launch_single<kEpiGlu, false, true, true>(a, stream)
                               : launch_single<kEpiResidual, false, true, true>(a, stream);
  }
  if (GSN_GEMM_PAIR && !a.w_int8 && !a.col_scale && (epilogue == kEpiGlu || epilogue == kEpiResidual) &&
      a.out_scale == 1.0f && a.K % BK == 0) {
    bool launched = false;
    const int rc = epilogue == kEpiGlu ? launch_pair<kEpiGlu>(a, stream, &launched)
                                       : launch_pair<kEpiResidual>(a, stream, &launched);
    if (rc || launched) return rc;
  }
  // int8 weights staged as int8 (widened per tile in shared memory), bf16 weights with a column scale (int8
  // weights widened beforehand), plain bf16 weights
  if (epilogue == kEpiGlu) {
    if (a.w_int8) return launch_single<kEpiGlu, true, true>(a, stream);
    return a.col_scale ? launch_single<kEpiGlu, false, true>(a, stream) : launch_single<kEpiGlu, false, false>(a, stream);
  }
  if (epilogue == kEpiSilu) {
    if (a.w_int8 || a.col_scale) return (int)cudaErrorInvalidValue;
    return launch_single<kEpiSilu, false, false>(a, stream);
  }
  if (epilogue == kEpiLinear) {
    if (a.w_int8 || a.col_scale || a.residual) return (int)cudaErrorInvalidValue;
    return launch_single<kEpiLinear, false, false>(a, stream);
  }
  if (epilogue == kEpiArgmax) {
    if (a.w_int8 || a.col_scale || a.residual || !a.argmax_keys) return (int)cudaErrorInvalidValue;
    return launch_single<kEpiArgmax, false, false>(a, stream);
  }
  if (a.w_int8) return launch_single<kEpiResidual, true, true>(a, stream);
  return a.col_scale ? launch_single<kEpiResidual, false, true>(a, stream)
                     : launch_single<kEpiResidual, false, false>(a, stream);
}

}  // namespace gsn
