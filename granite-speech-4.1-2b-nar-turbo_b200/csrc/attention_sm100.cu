// Block-local attention with Shaw relative positions (the core of ConformerAttention), on sm_100a.
//
//   models/granite_speech_nar/conformer.py:61-131: frames are cut into blocks of context_size = 200; inside a
//   block, for every head h (dim_head 128),
//     logits[i, j] = scale * (q_i . k_j) + scale * (q_i . rel[i - j + max_pos_emb])            (:90-104)
//     keys (and queries) past the tensor's frames are masked (:108-112), softmax over j, ctx_i = sum_j p_ij v_j
//   (:114-128); the caller's to_out projection follows.
//
// Input: the fused q|k|v projection rows qkv[b, t, 0:3*inner] (inner = heads * 128), the table
// rel[2 * max_pos_emb + 1, 128].  Output ctx[b, t, h * 128 + d] (bf16), zero for frames t >= len[b] when lengths
// are given (those frames are also masked as keys, so each utterance's result equals the module run on the
// utterance alone).  Rows of qkv at frames t >= len[b] may hold anything (they are never used as values: the V
// rows of masked keys are zeroed in shared memory before P V).
//
// Work unit: (query tile q in {0, 1}, utterance b, block m, head h): the 100 query frames m*200 + 100 q + [0, 100)
// against the block's 200 keys.  One CTA per SM walks units blockIdx.x + k * gridDim.x (all q = 0 units first,
// so the positional table slice is loaded once per tile index).  Per unit, with TMEM holding 512 fp32 columns of
// 128 lanes (lane = query row r of the tile; rows 100..127 are computed and discarded):
//   Pos[r, c] = q_r . rel[max_pos - 199 + 100 q + c], c in [0, 304)   columns 208..511 (N = 160 + 144)
//   S[r, j]   = q_r . k_j, j in [0, 208)                                columns 0..207
// The positional bias of (r, j) is Pos[r, r - j + 199] (the Shaw skew).  The softmax warps read S by 32-key chunks
// and, per chunk, a 64-column window of Pos; each thread shifts the window by its own row (a 5-stage register
// barrel shift), adds, scales by scale * log2(e), masks, and writes the logits back over S.  A second pass turns
// them into bf16 probabilities (row max subtracted, ex2) stored into TMEM columns 224..327 as packed pairs (over
// the consumed Pos columns), the A operand of O = P V (V as an MN-major operand straight from its TMA tile, 13
// MMAs of K = 16), which lands in columns 0..127 (over the consumed S) and is scaled by 1 / row sum on the way out.
// With P in TMEM the Q/K tiles are free as soon as the S / Pos MMAs finish, so the next unit's Q/K loads run under
// the softmax, and the next unit's Pos MMAs are issued right behind P V, under this unit's output.
//
// Roles (320 threads): warp 0 TMA producer, warp 1 TMEM allocator + single-thread MMA issuer, warps 2-9 softmax /
// output: warp w reads TMEM lanes 32 (w % 4) ..; the two warps of a lane quarter take alternate key chunks and the
// two halves of the output columns, and exchange row max and row sum through shared memory.  Every wait is
// bounded; after a timeout the softmax warps keep meeting at their named barrier until the unit list ends.
#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

namespace gsn {

namespace attn_impl {

constexpr int DH = 128;                    // dim_head
constexpr int CTX = 200;                   // context_size (frames per block)
constexpr int QT = 100;                    // query frames per unit
constexpr int BM = 128;                    // MMA rows
constexpr int KEYS = 208;                  // keys per block rounded up to the MMA N granularity
constexpr int PCOLS = 304;                 // positional columns c = r - j + 199 in [0, 299), rounded up
constexpr int PN0 = 160, PN1 = PCOLS - PN0;
constexpr int S_COL = 0, POS_COL = KEYS;
constexpr int P_TCOL = 224;                // P: KEYS / 2 columns of packed bf16 pairs, over consumed Pos columns
constexpr int O_COL = 0;                   // O over the consumed S columns
constexpr int EPI_WARPS = 8;
constexpr int EPI_THREADS = 32 * EPI_WARPS;
constexpr int THREADS = 64 + EPI_THREADS;
constexpr int kEpiBar = 1;                 // named barrier of the softmax warps
constexpr uint32_t TMEM_COLS = 512;
constexpr int ROW_BYTES = 128;             // one 64-element half of a 128-wide row, 128-byte swizzle
constexpr int Q_BYTES = BM * ROW_BYTES;    // 16 KB per half
constexpr int KV_BYTES = KEYS * ROW_BYTES; // 26 KB per half
constexpr int E_BOX_ROWS = PCOLS / 2;      // 152 (a TMA box has at most 256 rows)
constexpr int E_BYTES = PCOLS * ROW_BYTES; // 38 KB per half
constexpr int P_STEPS = KEYS / 16;         // 13 MMAs of K = 16 for O = P V
static_assert(POS_COL + PCOLS == (int)TMEM_COLS, "S and the positional columns fill the tensor memory");
static_assert(P_TCOL >= POS_COL && P_TCOL + KEYS / 2 <= (int)TMEM_COLS && O_COL + DH <= POS_COL, "P, O placement");

struct __align__(1024) Smem {
  uint8_t q[2][Q_BYTES];
  uint8_t k[2][KV_BYTES];
  uint8_t v[2][KV_BYTES];
  uint8_t e[2][E_BYTES];
  float red_max[2][BM];      // the two warps of a lane quarter: partial row max, partial row sum
  float red_sum[2][BM];
  uint64_t qk_full, v_full, e_full, s_full, qk_free, p_full, o_full, v_free, tmem_free, mma_drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory");

struct Params {
  __nv_bfloat16* ctx;
  int64_t ld_ctx;
  const int* lengths;
  int B, T, H, nblk, n_units;
  int inner;
  int rel_row0;              // table row of c = 0 for query tile 0: max_pos_emb - (CTX - 1)
  float scale_log2;          // dim_head^-0.5 * log2(e)
};

struct Unit {
  int b, m, h, q, row0, L;
  bool exists, active;
};

__device__ __forceinline__ Unit decode(int u, const Params& p) {
  Unit x;
  const int per_q = p.B * p.nblk * p.H;
  x.q = u / per_q;
  int r = u - x.q * per_q;
  x.h = r % p.H;
  r /= p.H;
  x.m = r % p.nblk;
  x.b = r / p.nblk;
  x.row0 = x.m * CTX + x.q * QT;
  x.L = p.lengths ? min(max(__ldg(p.lengths + x.b), 0), p.T) : p.T;
  x.exists = x.row0 < p.T;
  x.active = x.row0 < x.L;
  return x;
}

// R[m] = w[sh + m] for m in [0, 32), sh in [0, 32): five conditional shifts with compile-time indices (selects).
__device__ __forceinline__ void barrel_shift(uint32_t (&w)[64], int sh) {
#pragma unroll
  for (int m = 0; m < 47; ++m) w[m] = (sh & 16) ? w[m + 16] : w[m];
#pragma unroll
  for (int m = 0; m < 39; ++m) w[m] = (sh & 8) ? w[m + 8] : w[m];
#pragma unroll
  for (int m = 0; m < 35; ++m) w[m] = (sh & 4) ? w[m + 4] : w[m];
#pragma unroll
  for (int m = 0; m < 33; ++m) w[m] = (sh & 2) ? w[m + 2] : w[m];
#pragma unroll
  for (int m = 0; m < 32; ++m) w[m] = (sh & 1) ? w[m + 1] : w[m];
}

__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync %0, %1;" ::"n"(kEpiBar), "n"(EPI_THREADS) : "memory");
}

__global__ void __launch_bounds__(THREADS, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                     const __grid_constant__ CUtensorMap tmE, Params p) {
  constexpr uint32_t IDESC_P0 = make_idesc_bf16_f32(BM, PN0);
  constexpr uint32_t IDESC_P1 = make_idesc_bf16_f32(BM, PN1);
  constexpr uint32_t IDESC_S = make_idesc_bf16_f32(BM, KEYS);
  constexpr uint32_t IDESC_O = make_idesc_bf16_f32(BM, DH) | (1u << 16);   // B (= V) MN-major
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = warp_id();
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&s.qk_full, 1);
    mbar_init(&s.v_full, 1);
    mbar_init(&s.e_full, 1);
    mbar_init(&s.s_full, 1);
    mbar_init(&s.qk_free, 1);
    mbar_init(&s.p_full, EPI_WARPS);
    mbar_init(&s.o_full, 1);
    mbar_init(&s.v_free, 1);
    mbar_init(&s.tmem_free, EPI_WARPS);
    mbar_init(&s.mma_drain, 1);
    s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKV);
    tma_prefetch_desc(&tmE);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  volatile int* abort_flag = &s.abort_flag;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (one thread)
    if (lane == 0) {
      int n = 0, ne = 0, nv = 0, cur_q = -1;
      bool ok = true;
      for (int u = blockIdx.x; u < p.n_units; u += gridDim.x) {
        const Unit x = decode(u, p);
        if (!x.active) continue;
        // the previous unit's S / Pos MMAs have read Q, K (and E)
        if (n > 0 && !mbar_wait_bounded(&s.qk_free, (uint32_t)((n - 1) & 1), abort_flag, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        if (x.q != cur_q) {
          cur_q = x.q;
          const int r0 = p.rel_row0 + QT * x.q;
          mbar_arrive_expect_tx(&s.e_full, 2 * E_BYTES);
          for (int kh = 0; kh < 2; ++kh)
            for (int rh = 0; rh < 2; ++rh)
              tma_load_2d(s.e[kh] + rh * E_BOX_ROWS * ROW_BYTES, &tmE, &s.e_full, 64 * kh, r0 + rh * E_BOX_ROWS);
          ++ne;
        }
        const int col = x.h * DH;
        mbar_arrive_expect_tx(&s.qk_full, 2 * Q_BYTES + 2 * KV_BYTES);
        for (int kh = 0; kh < 2; ++kh) tma_load_3d(s.q[kh], &tmQ, &s.qk_full, col + 64 * kh, x.row0, x.b);
        for (int kh = 0; kh < 2; ++kh)
          tma_load_3d(s.k[kh], &tmKV, &s.qk_full, p.inner + col + 64 * kh, x.m * CTX, x.b);
        ++n;
        // the previous unit's O = P V has read V
        if (nv > 0 && !mbar_wait_bounded(&s.v_free, (uint32_t)((nv - 1) & 1), abort_flag, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&s.v_full, 2 * KV_BYTES);
        for (int kh = 0; kh < 2; ++kh)
          tma_load_3d(s.v[kh], &tmKV, &s.v_full, 2 * p.inner + col + 64 * kh, x.m * CTX, x.b);
        ++nv;
      }
      if (!ok) {
        // unwinding after a timeout: let the loads in flight land before the CTA's shared memory goes away
        if (n > 0)
          mbar_wait_bounded(&s.qk_full, (uint32_t)((n - 1) & 1), nullptr, kStatusTimeoutProducer, 100000000ull);
        if (nv > 0)
          mbar_wait_bounded(&s.v_full, (uint32_t)((nv - 1) & 1), nullptr, kStatusTimeoutProducer, 100000000ull);
        if (ne > 0)
          mbar_wait_bounded(&s.e_full, (uint32_t)((ne - 1) & 1), nullptr, kStatusTimeoutProducer, 100000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (one thread)
    // Order per unit n: P V(n) -> Pos(n+1) -> [O(n) read out] -> S(n+1).  Pos(n+1) overwrites P(n), which P V(n)
    // (issued before it by this thread) reads first; O lives over S, so only S(n+1) waits for the output.
    if (lane == 0) {
      int ne = 0, cur_q = -1;
      bool ok = true;
      auto next_active = [&](int u) {
        for (; u < p.n_units; u += gridDim.x)
          if (decode(u, p).active) return u;
        return p.n_units;
      };
      auto issue_pos = [&](const Unit& x, int n) -> bool {
        if (x.q != cur_q) {
          cur_q = x.q;
          if (!mbar_wait_bounded(&s.e_full, (uint32_t)(ne & 1), abort_flag, kStatusTimeoutMma)) return false;
          ++ne;
        }
        if (!mbar_wait_bounded(&s.qk_full, (uint32_t)(n & 1), abort_flag, kStatusTimeoutMma)) return false;
        tc_fence_after();
        for (int kh = 0; kh < 2; ++kh) {
          const uint64_t qd = make_sw128_kmajor_desc(smem_u32(s.q[kh]));
          const uint64_t e0 = make_sw128_kmajor_desc(smem_u32(s.e[kh]));
          const uint64_t e1 = make_sw128_kmajor_desc(smem_u32(s.e[kh] + PN0 * ROW_BYTES));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t acc = (kh | k) != 0 ? 1u : 0u;
            umma_f16(tmem_base + POS_COL, qd + (uint64_t)(2 * k), e0 + (uint64_t)(2 * k), IDESC_P0, acc);
            umma_f16(tmem_base + POS_COL + PN0, qd + (uint64_t)(2 * k), e1 + (uint64_t)(2 * k), IDESC_P1, acc);
          }
        }
        return true;
      };
      auto issue_s = [&]() {
        for (int kh = 0; kh < 2; ++kh) {
          const uint64_t qd = make_sw128_kmajor_desc(smem_u32(s.q[kh]));
          const uint64_t kd = make_sw128_kmajor_desc(smem_u32(s.k[kh]));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem_base + S_COL, qd + (uint64_t)(2 * k), kd + (uint64_t)(2 * k), IDESC_S, (kh | k) != 0 ? 1u : 0u);
        }
        umma_commit(&s.s_full);
        umma_commit(&s.qk_free);
      };
      int u = next_active(blockIdx.x);
      int n = 0;
      if (u < p.n_units) {
        ok = issue_pos(decode(u, p), 0);
        if (ok) issue_s();
      }
      while (ok && u < p.n_units) {
        if (!mbar_wait_bounded(&s.p_full, (uint32_t)(n & 1), abort_flag, kStatusTimeoutMma) ||
            !mbar_wait_bounded(&s.v_full, (uint32_t)(n & 1), abort_flag, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t v0 = smem_u32(s.v[0]);
#pragma unroll 1
        for (int st = 0; st < P_STEPS; ++st) {
          const uint64_t vd = make_sw128_mnmajor_desc(v0 + (uint32_t)(st * 16 * ROW_BYTES), (uint32_t)KV_BYTES);
          umma_f16_ts(tmem_base + O_COL, tmem_base + P_TCOL + 8 * st, vd, IDESC_O, st != 0 ? 1u : 0u);
        }
        umma_commit(&s.o_full);
        umma_commit(&s.v_free);
        const int un = next_active(u + gridDim.x);
        if (un < p.n_units) {
          if (!issue_pos(decode(un, p), n + 1) ||
              !mbar_wait_bounded(&s.tmem_free, (uint32_t)(n & 1), abort_flag, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s();
        }
        u = un;
        ++n;
      }
      if (!ok) {
        // the MMAs already issued finish before the tensor memory is released
        umma_commit(&s.mma_drain);
        mbar_wait_bounded(&s.mma_drain, 0, nullptr, kStatusTimeoutMma, 100000000ull);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax and output (warps 2-9)
    const int e = warp - 2;
    const int qw = warp & 3;                            // TMEM lane quarter
    const int hh = e >> 2;                              // which of the quarter's two warps
    const int r = 32 * qw + lane;                       // MMA row = query frame row0 + r
    const uint32_t t_lane = tmem_base + ((uint32_t)(32 * qw) << 16);
    int n = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.n_units; u += gridDim.x) {
      const Unit x = decode(u, p);
      if (!x.exists) continue;
      const int t = x.row0 + r;
      const bool row_in = r < QT && t < p.T;
      uint4* crow = reinterpret_cast<uint4*>(p.ctx + ((int64_t)x.b * p.T + t) * p.ld_ctx + x.h * DH + 64 * hh);
      if (!x.active) {
        // every query frame of the unit is padding: zero context
        if (row_in)
          for (int c = 0; c < 8; ++c) crow[c] = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      const bool row_valid = row_in && t < x.L;
      if (ok) {
        bool got = mbar_wait_bounded(&s.s_full, (uint32_t)(n & 1), abort_flag, kStatusTimeoutEpilogue);
        ok = __shfl_sync(0xffffffffu, got, 0);
      }
      const int kv_lim = min(CTX, x.L - x.m * CTX);      // keys j < kv_lim are frames of the utterance

      // pass 1 (this warp's chunks J = hh, hh + 2, ...): logits in log2 units over the S columns, row max
      float mx = -INFINITY;
      if (ok) {
        tc_fence_after();
#pragma unroll 1
        for (int J = hh; J < 7; J += 2) {
          uint32_t sv[32];
          uint32_t w[64];
          const int wb = 32 * (qw - J) + 168;           // first Pos column any lane of the warp needs
          const int base = min(wb, PCOLS - 64);
          if (J < 6)
            tmem_ld32(t_lane + S_COL + 32 * J, sv);
          else
            tmem_ld8(t_lane + S_COL + 192, sv);
#pragma unroll
          for (int i = 0; i < 8; ++i) tmem_ld8(t_lane + POS_COL + base + 8 * i, w + 8 * i);
          tmem_wait_ld();
          tmem_regs_ready<32>(sv);
          tmem_regs_ready<64>(w);
          // lane row r needs column c = r - j + 199 = base + (wb - base + lane) + 31 - kk for key j = 32 J + kk
          barrel_shift(w, (wb - base + lane) & 31);
          const int nk = J < 6 ? 32 : 8;
#pragma unroll
          for (int kk = 0; kk < 32; ++kk) {
            if (kk < nk) {
              const int j = 32 * J + kk;
              float x2 = (__uint_as_float(sv[kk]) + __uint_as_float(w[31 - kk])) * p.scale_log2;
              x2 = j < kv_lim ? x2 : -INFINITY;
              mx = fmaxf(mx, x2);
              sv[kk] = __float_as_uint(x2);
            }
          }
          if (J < 6)
            tmem_st32(t_lane + S_COL + 32 * J, sv);
          else
            tmem_st8(t_lane + S_COL + 192, sv);
        }
        tmem_wait_st();
        tmem_wait_ld();
      }
      s.red_max[hh][r] = mx;
      tc_fence_before();
      epi_bar();                                        // both warps of the quarter are done with Pos
      mx = fmaxf(s.red_max[0][r], s.red_max[1][r]);

      // pass 2: bf16 probabilities as packed pairs into TMEM columns P_TCOL + j / 2, row sum
      float sum = 0.f;
      if (ok) {
        tc_fence_after();
#pragma unroll 1
        for (int J = hh; J < 7; J += 2) {
          uint32_t sv[32];
          if (J < 6)
            tmem_ld32(t_lane + S_COL + 32 * J, sv);
          else
            tmem_ld8(t_lane + S_COL + 192, sv);
          tmem_wait_ld();
          tmem_regs_ready<32>(sv);
          const int nk = J < 6 ? 32 : 8;
          uint32_t pk[16];
#pragma unroll
          for (int kk = 0; kk < 32; kk += 2) {
            float p0 = 0.f, p1 = 0.f;
            if (kk < nk && row_valid) {
              p0 = bf16_round_f32(ex2_approx(__uint_as_float(sv[kk]) - mx));
              p1 = bf16_round_f32(ex2_approx(__uint_as_float(sv[kk + 1]) - mx));
            }
            sum += p0 + p1;
            pk[kk >> 1] = pack_bf16x2(p0, p1);
          }
          if (J < 6)
            tmem_st16(t_lane + P_TCOL + 16 * J, pk);
          else
            tmem_st8(t_lane + P_TCOL + 96, pk);          // keys 192..207 (200..207 are zero)
        }
        tmem_wait_st();
        // V rows of keys past the utterance (or past the block) may hold anything: zero them before P V reads V
        bool got = mbar_wait_bounded(&s.v_full, (uint32_t)(n & 1), abort_flag, kStatusTimeoutEpilogue);
        ok = __shfl_sync(0xffffffffu, got, 0);
        if (ok) {
          const int et = e * 32 + lane;
          const int nz = (KEYS - kv_lim) * 16;          // 16-byte chunks: rows x 2 halves x 8
          for (int i = et; i < nz; i += EPI_THREADS) {
            const int row = kv_lim + (i >> 4), kh = (i >> 3) & 1, c = i & 7;
            *reinterpret_cast<uint4*>(s.v[kh] + row * ROW_BYTES + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
        }
      }
      s.red_sum[hh][r] = sum;
      tc_fence_before();
      epi_bar();
      sum = s.red_sum[0][r] + s.red_sum[1][r];
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&s.p_full);

      if (ok) {
        bool got = mbar_wait_bounded(&s.o_full, (uint32_t)(n & 1), abort_flag, kStatusTimeoutEpilogue);
        ok = __shfl_sync(0xffffffffu, got, 0);
      }
      if (ok) {
        tc_fence_after();
        const float inv = row_valid ? 1.0f / sum : 0.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[16];
          tmem_ld16(t_lane + O_COL + 64 * hh + 16 * c, ov);
          tmem_wait_ld();
          tmem_regs_ready<16>(ov);
          if (row_in) {
            uint32_t o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              o[i] = pack_bf16x2(__uint_as_float(ov[2 * i]) * inv, __uint_as_float(ov[2 * i + 1]) * inv);
            crow[2 * c] = make_uint4(o[0], o[1], o[2], o[3]);
            crow[2 * c + 1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.tmem_free);
      }
      ++n;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace attn_impl

int launch_attention(const AttnArgs& a, cudaStream_t stream) {
  namespace A = attn_impl;
  if (a.B <= 0 || a.T <= 0 || a.H <= 0) return 0;
  const int inner = a.H * A::DH;
  CUtensorMap tmQ, tmKV, tmE;
  {
    const uint64_t dims[3] = {(uint64_t)(3 * inner), (uint64_t)a.T, (uint64_t)a.B};
    const uint64_t strides[2] = {(uint64_t)a.ld_qkv * 2, (uint64_t)a.ld_qkv * 2 * (uint64_t)a.T};
    const uint32_t boxq[3] = {64, A::BM, 1};
    if (int rc = encode_tmap(&tmQ, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a.qkv, dims, strides, boxq,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    const uint32_t boxkv[3] = {64, A::KEYS, 1};
    if (int rc = encode_tmap(&tmKV, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a.qkv, dims, strides, boxkv,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)A::DH, (uint64_t)a.n_rel};
    const uint64_t strides[1] = {(uint64_t)A::DH * 2};
    const uint32_t box[2] = {64, A::E_BOX_ROWS};
    if (int rc = encode_tmap(&tmE, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.rel, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  A::Params p;
  p.ctx = a.ctx;
  p.ld_ctx = a.ld_ctx;
  p.lengths = a.lengths;
  p.B = a.B;
  p.T = a.T;
  p.H = a.H;
  p.nblk = (a.T + A::CTX - 1) / A::CTX;
  const int64_t units = 2LL * a.B * p.nblk * a.H;
  if (units > 0x7FFFFFFF) return (int)cudaErrorInvalidValue;
  p.n_units = (int)units;
  p.inner = inner;
  p.rel_row0 = a.max_pos - (A::CTX - 1);
  p.scale_log2 = a.scale * 1.4426950408889634f;
  const int smem = (int)sizeof(A::Smem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(A::attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return (int)e;
  const int sms = device_sm_count();
  const int grid = (int)(units < sms ? units : sms);
  A::attention_kernel<<<grid, A::THREADS, smem, stream>>>(tmQ, tmKV, tmE, p);
  return (int)cudaGetLastError();
}

}  // namespace gsn
