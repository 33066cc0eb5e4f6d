// Depthwise Conv1d k=15 (+ folded BatchNorm bias) + SiLU on the 5th-generation tensor cores, for the layout the
// reference op receives at its call site: x (B, C, T) with T innermost (script/models/granite_speech_nar/
// conformer.py:177-183, granite::dwconv_silu, script/cuda_kernels/conv1d.py:21-42).
//
// The convolution of one channel is a matrix product.  With the channel's frames [t0 - 8, t0 + 1040) contiguous in
// shared memory, the matrix A[m, k] = x[t0 - 8 + 8 m + k] (m < 128 rows, k < 32) is a Hankel matrix whose rows
// start 8 frames = 16 bytes apart: exactly the row pitch of a K-major core matrix without swizzle (8 rows x 16
// bytes), so the staged row itself is the A operand, described with a leading byte offset (next 8 k) of 16 bytes
// and a stride byte offset (next 8 rows) of 128 bytes.  B[n, k] = w[k - n - 1] (zero outside the 15 taps) is the
// channel's Toeplitz table, n < 16, so D[m, n] = sum_k A[m, k] B[n, k] = sum_j w[j] x[t0 + 8 m + n - 7 + j] =
// y[t0 + 8 m + n] before the bias.  One M=128, N=16, K=32 product (two K=16 MMAs) gives 1024 frames of one channel;
// rows overlap by 8 frames, and only D[m, 0..7] is read.  The weights are halved in the table (exact), so D holds
// y / 2 and silu(y) = h + h tanh(h) with h = D + b / 2.
//
// GLU form (granite::dwconv_silu_glu, x (B, 2C, T)): the item's value rows and gate rows are staged side by side
// and converter warps replace each value frame by bf16(a * sigmoid(g)) in place (the arithmetic of the CUDA-core
// kernels' GLU, one rounding to bf16 as script/cuda_kernels/conv1d.py:70-73), so the value rows become the A
// operand.  Without lengths the items stay 8 channels wide in 3 stages with one table slot (two CTAs still fit on
// an SM); with lengths they are 4 channels wide.
//
// Work item: 8 channels (GLU form with lengths: 4) x 1024 frames of one utterance.  Two CTAs per SM (at most 256
// tensor-memory columns and ~110 KB of shared memory each), so two independent load -> MMA -> epilogue pipelines
// overlap on every SM.  Roles (352 threads; the GLU form adds 4 converter warps):
//   warp 0      producer: per item, writes the parts of the staged rows outside the copied range (zeros before
//               frame 0 and from len on, the ragged last chunk of an utterance), then one bulk copy per row for the
//               rest (16-byte aligned: T % 8 == 0); builds a channel block's 16 Toeplitz tables (from weights
//               staged in shared memory) into one of two table slots when the block changes (the GLU form
//               without lengths: one slot); 5 stages (GLU form: 3 without lengths, 4 with)
//   warps 1-2   MMA issuers (warp 1 also allocates TMEM): each issues the 8 MMAs of its 4 channels per item into
//               one of two 128-column accumulators (16 columns per channel).  An M=128, N=16 MMA runs in a few
//               cycles but takes about a hundred to issue, so the issue is split
//   warps 3-10  epilogue: warp e reads TMEM lane quarter e % 4 (rows 32 (e % 4) .. + 31) and 4 of the channels:
//               per row 8 consecutive frames of a channel, bias + SiLU, one 16-byte store (a warp writes 512
//               contiguous bytes of a channel row)
//   warps 11-14 (GLU form) converters: per item, the GLU of every staged value / gate chunk pair into the value row
// Frames t >= len read as zero and are written as zero; frames >= T are neither read nor written.
//
// Accumulation happens inside the tensor core in fp32, in its own order, so results can differ from the CUDA-core
// kernels (fp32 FMA chains) in the last bits before the bf16 rounding: within the parity gates, not bit for bit.
#include <algorithm>

#include "gsn_kernels.cuh"
#include "gsn_ptx.cuh"

namespace gsn {

namespace dwm_impl {

constexpr int KW = 15;
constexpr int FR = 1024;                     // output frames per item (128 rows x 8)
constexpr int ROWF = FR + 24;                // staged frames per channel: t0 - 8 .. t0 + 1039
constexpr int ROW_BYTES = ROWF * 2;          // 2096 = 131 x 16
constexpr int TAB_BYTES = 16 * 32 * 2;       // one channel's Toeplitz table: 16 n x 32 k bf16
constexpr int NISS = 2;                      // MMA-issuing warps: an N=16 MMA is issued far slower than it runs, so
                                             //   each issuer takes CT / NISS channels of the item
constexpr int EPI_WARPS = 8;                 // each covers a TMEM lane quarter and CT * 4 / EPI_WARPS channels
constexpr int EPI_W0 = 1 + NISS;             // first epilogue warp
constexpr int CONV_W0 = EPI_W0 + EPI_WARPS;  // first converter warp (GLU form)
constexpr int MINB = 2;                      // CTAs per SM (registers, tensor memory and shared memory allow two)
constexpr uint32_t IDESC = make_idesc_bf16_f32(128, 16);
static_assert(ROW_BYTES % 16 == 0, "rows must stay 16-byte aligned");

// Shapes: the plain form; the GLU form without lengths (contiguous item ranges, so the channel block rarely
// changes: one table slot leaves room for 8-channel items of value + gate rows at two CTAs per SM); the GLU form
// with lengths (round-robin items, a new channel block nearly every item: two table slots, 4-channel items).
enum Form : int { kPlain = 0, kGluDense = 1, kGluMasked = 2 };

template <int FORM>
struct Cfg {
  static constexpr bool GLU = FORM != kPlain;
  static constexpr int CT = FORM == kGluMasked ? 4 : 8;   // channels per item
  static constexpr int ROWS = GLU ? 2 * CT : CT;         // staged rows per item: value rows, then gate rows
  static constexpr int STAGE_BYTES = ROWS * ROW_BYTES;
  static constexpr int STAGES = FORM == kGluDense ? 3 : (FORM == kPlain ? 5 : 4);
  static constexpr int TSLOTS = FORM == kGluDense ? 1 : 2;   // Toeplitz table slots (channel blocks kept)
  static constexpr int CPI = CT / NISS;
  static constexpr int EPI_CH = CT * 4 / EPI_WARPS;  // channels per epilogue warp, in batches of EB
  static constexpr int EB = EPI_CH < 8 ? EPI_CH : 8;
  static constexpr int CONV_WARPS = GLU ? 4 : 0;
  static constexpr int THREADS = 32 * (CONV_W0 + CONV_WARPS);
  static constexpr uint32_t TMEM_COLS = 2 * CT * 16;   // 2 accumulators x CT channels x 16 columns
  static_assert(CPI * NISS == CT && EPI_CH * EPI_WARPS == CT * 4, "channel split");
  static_assert(MINB * TMEM_COLS <= 512, "tensor memory");

  struct __align__(1024) Smem {
    uint8_t x[STAGES][STAGE_BYTES];
    uint8_t tab[TSLOTS][CT * TAB_BYTES];     // Toeplitz tables of the last channel blocks
    __nv_bfloat16 wst[CT * KW];              // a block's weights, staged for the table build
    int st_slot[STAGES];                     // table slot of the item in each stage
    uint64_t full[STAGES];                   // the stage's copies landed
    uint64_t cfull[STAGES];                  // GLU form: the stage's value rows converted
    uint64_t empty[STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort_flag;
  };
  static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory");
};

struct Params {
  const __nv_bfloat16* x;
  const __nv_bfloat16* w;                    // [C, 15]
  const __nv_bfloat16* bias;                 // [C]
  __nv_bfloat16* y;
  const int* lengths;
  int64_t sxB, sxC, syB, syC;                // element strides (T stride 1)
  int64_t gate_off;                          // GLU form: elements from a value row to its gate row (C * sxC)
  int B, C, T;
  int n_tt, per_cb, n_items;
  int withhold;                              // test only: item #k of every CTA armed but never copied (-1: none)
};

// K-major operand without swizzle: 16-byte rows, leading byte offset = next 8 k, stride byte offset = next 8 rows
__device__ __forceinline__ uint64_t make_noswz_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;                   // descriptor version; layout type 0 = no swizzle
  return d;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <int FORM>
__global__ void __launch_bounds__(Cfg<FORM>::THREADS, MINB) dwconv_cf_mma_kernel(Params p) {
  using K = Cfg<FORM>;
  constexpr bool GLU = K::GLU;
  using Smem = typename K::Smem;
  constexpr int CT = K::CT, ROWS = K::ROWS, STAGES = K::STAGES, CPI = K::CPI, EPI_CH = K::EPI_CH, EB = K::EB;
  constexpr uint32_t TMEM_COLS = K::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = warp_id();
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x, k = blockIdx.x;
  int first, step, n_items;
  if (p.lengths) {                           // round robin: tiles past utterance ends spread evenly
    first = k;
    step = G;
    n_items = p.n_items > k ? (p.n_items - k + G - 1) / G : 0;
  } else {                                   // contiguous range: the channel block rarely changes
    first = (int)((int64_t)k * p.n_items / G);
    step = 1;
    n_items = (int)((int64_t)(k + 1) * p.n_items / G) - first;
  }
  auto item = [&](int i, int& c0, int& b, int& t0) {
    const int g = first + i * step;
    const int cb = g / p.per_cb;
    const int r = g - cb * p.per_cb;
    c0 = cb * CT;
    b = r / p.n_tt;
    t0 = (r - b * p.n_tt) * FR;
  };
  auto len_of = [&](int b) { return p.lengths ? min(max(__ldg(p.lengths + b), 0), p.T) : p.T; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.cfull[i], K::CONV_WARPS > 0 ? K::CONV_WARPS : 1);
      mbar_init(&s.empty[i], NISS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], NISS);
      mbar_init(&s.tempty[i], EPI_WARPS);
    }
    mbar_init(&s.mma_done, NISS);
    s.abort_flag = 0;
    fence_mbar_init();
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
    // ------------------------------------------------------------------ producer
    int issued = 0;
    bool ok = true;
    int slot_c0a = -1, slot_c0b = -1, slot_lasta = -1, slot_lastb = -1;   // table slots 0 / 1: channel block, last
                                                                      //   item using it (scalars: kept in registers)
    for (int i = 0; i < n_items && ok; ++i) {
      const int st = i % STAGES;
      if (i >= STAGES) {
        bool got = mbar_wait_bounded(&s.empty[st], (uint32_t)(((i / STAGES) - 1) & 1), abort_flag,
                                     kStatusTimeoutProducer);
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) {
          ok = false;
          break;
        }
      }
      int c0, b, t0;
      item(i, c0, b, t0);
      const int len = len_of(b);
      if (t0 >= len) {                        // every frame of the item is padding: no operands, no MMAs
        ++issued;
        if (lane == 0) mbar_arrive(&s.full[st]);
        continue;
      }
      // staged frames [t0 - 8, t0 + 1040) of the ROWS rows (GLU form: CT value rows, then their CT gate rows):
      // frames [lo, hi8) by bulk copy, the ragged end [hi8, hi) of an utterance (len % 8 != 0) by a masked 16-byte
      // copy, zeros elsewhere (before frame 0, from len on; a zero value and gate give a zero GLU)
      const int f_begin = t0 - 8;
      const int lo = max(f_begin, 0);                        // multiple of 8
      const int hi = min(t0 + FR + 16, len);                 // > lo: t0 < len
      const int hi8 = hi & ~7;
      uint8_t* xs = s.x[st];
      // element offset of staged row r in x: value channel c0 + r, or the gate row of value channel c0 + r - CT
      auto row_off = [&](int r) {
        return (int64_t)b * p.sxB + (int64_t)(c0 + (r < CT ? r : r - CT)) * p.sxC + (r < CT ? 0 : p.gate_off);
      };
      // the bulk copies go first, so their latency runs under the table build and the hand-written chunks; the
      // stage's phase cannot complete before the arrive below (its one expected arrival), which also sets the
      // byte count the copies' completions are counted against
      const uint32_t row_bytes = hi8 > lo ? (uint32_t)(hi8 - lo) * 2 : 0u;
      ++issued;
      if (row_bytes > 0 && lane < ROWS && i != p.withhold) {   // test only: a withheld item's copies never start
        const __nv_bfloat16* src = p.x + row_off(lane) + lo;
        bulk_load(xs + lane * ROW_BYTES + (lo - f_begin) * 2, src, row_bytes, &s.full[st]);
      }
      // the channel block's Toeplitz tables: kept in TSLOTS slots; a new block takes the slot used longer ago,
      // after the MMAs of that slot's last item are done.  Channel c's table holds B[n, k] = w[k - n - 1] / 2 as
      // core matrices (n-group g, k-chunk h) at (2 h + g) * 128 bytes, row n % 8 at 16 (n % 8), element k % 8
      int slot = c0 == slot_c0a ? 0 : (K::TSLOTS > 1 && c0 == slot_c0b ? 1 : -1);
      if (slot < 0) {
        slot = K::TSLOTS == 1 || slot_lasta <= slot_lastb ? 0 : 1;
        const int last = slot ? slot_lastb : slot_lasta;
        if (last >= 0 && i - last < STAGES) {                // its stage not reused yet: wait for that item's MMAs
          bool got = mbar_wait_bounded(&s.empty[last % STAGES], (uint32_t)((last / STAGES) & 1), abort_flag,
                                       kStatusTimeoutProducer);
          got = __shfl_sync(0xffffffffu, got, 0);
          if (!got) {
            // the copies just issued are counted on this stage's barrier, so the unwind below waits for them
            if (lane == 0) mbar_arrive_expect_tx(&s.full[st], row_bytes * ROWS);
            ok = false;
            break;
          }
        }
        for (int q = lane; q < CT * KW; q += 32) s.wst[q] = p.w[(int64_t)c0 * KW + q];   // rows c0.. are contiguous
        __syncwarp();
        uint8_t* tab = s.tab[slot];
        for (int q = lane; q < CT * 64; q += 32) {           // (channel, n, h): 16 rows x 4 chunks per channel
          const int c = q >> 6, nn = (q >> 2) & 15, h = q & 3;
          const __nv_bfloat16* wc = s.wst + c * KW;
          uint32_t wd[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int ja = 8 * h + 2 * e - nn - 1, jb = ja + 1;
            const uint32_t lo = (ja >= 0 && ja < KW)
                                    ? __bfloat16_as_ushort(__float2bfloat16_rn(0.5f * __bfloat162float(wc[ja]))) : 0u;
            const uint32_t hi = (jb >= 0 && jb < KW)
                                    ? __bfloat16_as_ushort(__float2bfloat16_rn(0.5f * __bfloat162float(wc[jb]))) : 0u;
            wd[e] = lo | (hi << 16);
          }
          *reinterpret_cast<uint4*>(tab + c * TAB_BYTES + (2 * h + (nn >> 3)) * 128 + (nn & 7) * 16) =
              make_uint4(wd[0], wd[1], wd[2], wd[3]);
        }
        __syncwarp();
        if (slot) slot_c0b = c0; else slot_c0a = c0;
      }
      if (slot) slot_lastb = i; else slot_lasta = i;
      if (lane == 0) s.st_slot[st] = slot;                   // read by the issuers after the stage's full barrier
      // chunks to write by hand: the head chunk (frames -8 .. -1) when t0 = 0, and from hi8 on the tail (the ragged
      // chunk [hi8, hi), then zeros); a tile inside the utterance has neither
      const int head = lo > f_begin ? 1 : 0;
      const int tail0 = (hi8 - f_begin) / 8;                 // first tail chunk of a row
      const int per_row = head + (ROWF / 8 - tail0);
      for (int q = lane; q < ROWS * per_row; q += 32) {
        const int c = q / per_row, j = q - c * per_row;
        const int ch = (j < head) ? 0 : tail0 + (j - head);  // chunk index within the row
        const int t = f_begin + ch * 8;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (t == hi8 && hi8 < hi) {                          // the ragged end: frames hi8 .. hi - 1 of 8 (in bounds:
          v = __ldg(reinterpret_cast<const uint4*>(p.x + row_off(c) + t));
          const int keep = hi - hi8;                         //  hi8 + 8 <= round_up(len, 8) <= T)
          uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (2 * e >= keep) w4[e] = 0u;
            else if (2 * e + 1 >= keep) w4[e] &= 0xFFFFu;
          }
          v = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
        *reinterpret_cast<uint4*>(xs + c * ROW_BYTES + ch * 16) = v;
      }
      fence_proxy_async_smem();               // generic writes (zeros, tables) before the tensor core reads them
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&s.full[st], row_bytes * ROWS);
      __syncwarp();
    }
    if (!ok && lane == 0) {
      // unwinding: the copies of the last STAGES items may still be in flight
      for (int back = 1; back <= STAGES && back <= issued; ++back) {
        const int idx = issued - back;
        mbar_wait_bounded(&s.full[idx % STAGES], (uint32_t)((idx / STAGES) & 1), nullptr, kStatusTimeoutProducer,
                          100000000ull);
      }
    }
  } else if (warp <= NISS) {
    // ------------------------------------------------------------------ MMA issuers: warp 1 + j, channels CPI j ..
    const int cfirst = CPI * (warp - 1);
    for (int i = 0; i < n_items; ++i) {
      const int st = i % STAGES;
      const int acc = i & 1;
      bool got = true;
      if (i >= 2)
        got = mbar_wait_bounded(&s.tempty[acc], (uint32_t)(((i >> 1) - 1) & 1), abort_flag, kStatusTimeoutMma);
      if (got)
        got = mbar_wait_bounded(GLU ? &s.cfull[st] : &s.full[st], (uint32_t)((i / STAGES) & 1), abort_flag,
                                kStatusTimeoutMma);
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      tc_fence_after();
      int c0, b, t0;
      item(i, c0, b, t0);
      if (lane == 0) {
        if (t0 < len_of(b)) {
          const uint32_t xa = smem_u32(s.x[st]);
          const uint32_t ta = smem_u32(s.tab[s.st_slot[st]]);
          const uint32_t d0 = tmem_base + (uint32_t)(acc * CT * 16);
#pragma unroll
          for (int c = cfirst; c < cfirst + CPI; ++c) {
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const uint64_t ad = make_noswz_desc(xa + c * ROW_BYTES + 32 * kk, 16, 128);
              const uint64_t bd = make_noswz_desc(ta + c * TAB_BYTES + 512 * kk, 256, 128);
              umma_f16(d0 + (uint32_t)(16 * c), ad, bd, IDESC, (uint32_t)kk);
            }
          }
        }
        umma_commit(&s.empty[st]);            // the stage is free once these MMAs (if any) have read it
        umma_commit(&s.tfull[acc]);
      }
      __syncwarp();
    }
    if (lane == 0) umma_commit(&s.mma_done);
    __syncwarp();
    mbar_wait_bounded(&s.mma_done, 0, nullptr, kStatusTimeoutMma, 100000000ull);
  } else if (warp < CONV_W0) {
    // ------------------------------------------------------------------ epilogue
    const int e = warp - EPI_W0;
    const int q = warp & 3;                  // TMEM lane quarter this warp may read
    const int cg = e >> 2;                   // channels EPI_CH cg .. EPI_CH cg + EPI_CH - 1 of the item
    const int m = q * 32 + lane;             // row: frames t0 + 8 m .. + 7
    int bias_c0 = -1;                        // channel block whose halved biases are in bh_all
    float bh_all[EPI_CH];
    for (int i = 0; i < n_items; ++i) {
      const int acc = i & 1;
      // the item's length and (when its channel block changed) biases are read before the accumulator wait, so
      // their latency overlaps it
      int c0, b, t0;
      item(i, c0, b, t0);
      const int len = len_of(b);
      if (!GLU && c0 != bias_c0) {           // (the GLU forms have no registers to spare: they load per batch)
#pragma unroll
        for (int cc = 0; cc < EPI_CH; ++cc) bh_all[cc] = 0.5f * __bfloat162float(__ldg(p.bias + c0 + EPI_CH * cg + cc));
        bias_c0 = c0;
      }
      bool got = mbar_wait_bounded(&s.tfull[acc], (uint32_t)((i >> 1) & 1), abort_flag, kStatusTimeoutEpilogue);
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      tc_fence_after();
      const int tf = t0 + 8 * m;             // this lane's first frame
      const bool live = t0 < len;            // warp-uniform: the MMAs ran
      const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * CT * 16);
#pragma unroll
      for (int cb8 = 0; cb8 < EPI_CH; cb8 += EB) {
        const int cfirst = EPI_CH * cg + cb8;              // first of this batch's EB channels
        __nv_bfloat16* yrow = p.y + (int64_t)b * p.syB + (int64_t)(c0 + cfirst) * p.syC + tf;
        // the batch's accumulator columns in flight at once, one wait
        uint32_t v[EB][8];
        float bh[EB];
        if (live) {
#pragma unroll
          for (int cc = 0; cc < EB; ++cc) tmem_ld8(trow + (uint32_t)(16 * (cfirst + cc)), v[cc]);
#pragma unroll
          for (int cc = 0; cc < EB; ++cc)
            bh[cc] = GLU ? 0.5f * __bfloat162float(__ldg(p.bias + c0 + cfirst + cc)) : bh_all[cb8 + cc];
          tmem_wait_ld();
#pragma unroll
          for (int cc = 0; cc < EB; ++cc) tmem_regs_ready<8>(v[cc]);
        }
#pragma unroll
        for (int cc = 0; cc < EB; ++cc) {
          uint32_t o[4] = {0u, 0u, 0u, 0u};
          if (live) {
#pragma unroll
            for (int f = 0; f < 8; f += 2) {
              const float h0 = __uint_as_float(v[cc][f]) + bh[cc], h1 = __uint_as_float(v[cc][f + 1]) + bh[cc];
              const float s0 = tf + f < len ? fmaf(h0, tanh_approx(h0), h0) : 0.f;
              const float s1 = tf + f + 1 < len ? fmaf(h1, tanh_approx(h1), h1) : 0.f;
              o[f >> 1] = pack_bf16x2(s0, s1);
            }
          }
          if (tf < p.T) *reinterpret_cast<uint4*>(yrow + (int64_t)cc * p.syC) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.tempty[acc]);
    }
  } else if constexpr (GLU) {
    // ------------------------------------------------------------------ converters (GLU form)
    // every 16-byte chunk of the staged value rows becomes the GLU of itself and the gate chunk CT rows below;
    // chunks the producer zeroed stay zero (0 * sigmoid(0))
    const int ct = threadIdx.x - 32 * CONV_W0;
    constexpr int CHUNKS = ROWF / 8;
    for (int i = 0; i < n_items; ++i) {
      const int st = i % STAGES;
      bool got = mbar_wait_bounded(&s.full[st], (uint32_t)((i / STAGES) & 1), abort_flag, kStatusTimeoutEpilogue);
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      int c0, b, t0;
      item(i, c0, b, t0);
      if (t0 < len_of(b)) {
        uint8_t* xs = s.x[st];
        for (int q = ct; q < CT * CHUNKS; q += 32 * K::CONV_WARPS) {
          uint4* vp = reinterpret_cast<uint4*>(xs + q * 16);    // row q / CHUNKS, chunk q % CHUNKS: rows are
          const uint4 g = *reinterpret_cast<const uint4*>(xs + CT * ROW_BYTES + q * 16);   // CHUNKS chunks long
          const uint4 a = *vp;
          *vp = make_uint4(glu_word(a.x, g.x), glu_word(a.y, g.y), glu_word(a.z, g.z), glu_word(a.w, g.w));
        }
        fence_proxy_async_smem();           // the converted rows, written by this proxy, are read by the MMAs
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.cfull[st]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace dwm_impl

// channels-first depthwise on the tensor cores; x (B, C, T) (GLU form: (B, 2C, T), value rows then gate rows) with T
// innermost, C % 16 == 0, T % 8 == 0, 16-byte aligned rows
template <int FORM>
int launch_cf_mma(const DwArgs& a, cudaStream_t stream) {
  namespace W = dwm_impl;
  using K = W::Cfg<FORM>;
  W::Params p;
  p.x = a.x;
  p.w = a.w;
  p.bias = a.bias;
  p.y = a.y;
  p.lengths = a.lengths;
  p.sxB = a.sxB;
  p.sxC = a.sxC;
  p.syB = a.syB;
  p.syC = a.syC;
  p.gate_off = (int64_t)a.C * a.sxC;
  p.B = a.B;
  p.C = a.C;
  p.T = a.T;
  p.n_tt = (a.T + W::FR - 1) / W::FR;
  const int64_t per_cb = (int64_t)a.B * p.n_tt;
  const int64_t items = per_cb * (a.C / K::CT);
  if (items > (1 << 30)) return (int)cudaErrorInvalidValue;
  p.per_cb = (int)per_cb;
  p.n_items = (int)items;
  p.withhold = a.withhold_tile;
  const int smem = (int)sizeof(typename K::Smem) + 1024;
  auto kern = W::dwconv_cf_mma_kernel<FORM>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return (int)e;
  // the whole unified L1 / shared array as shared memory, so two CTAs fit on every SM
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return (int)e;
  // one CTA per resident slot: __launch_bounds__ gives MINB CTAs their registers, the tensor memory holds MINB
  // accumulator pairs, and MINB copies of the shared memory fit in the SM's 228 KB (1 KB reserved per CTA)
  constexpr int kSmemPerSm = 233472;
  const int per_sm = std::min<int>(W::MINB, kSmemPerSm / (smem + 1024));
  const int64_t slots = (int64_t)device_sm_count() * per_sm;
  const int grid = (int)(items < slots ? items : slots);
  if (grid <= 0) return 0;
  kern<<<grid, K::THREADS, smem, stream>>>(p);
  return (int)cudaGetLastError();
}

int launch_dwconv_cf_mma(const DwArgs& a, cudaStream_t stream) {
  namespace W = dwm_impl;
  if (!a.glu) return launch_cf_mma<W::kPlain>(a, stream);
  return a.lengths ? launch_cf_mma<W::kGluMasked>(a, stream) : launch_cf_mma<W::kGluDense>(a, stream);
}

}  // namespace gsn
