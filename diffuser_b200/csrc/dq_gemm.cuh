// dq_gemm.cuh -- fused dequantize + tcgen05 GEMM for weight-only NF4 / fp8.
//
// Computes one output tile Y^T[n0:n0+128, m0:m0+BM] = W_tile . X_tile^T with
// the 5th-generation tensor cores:
//   * the dequantized weight tile (128 rows x 64 K per k-block, bf16) is the
//     MMA A operand and lives in TENSOR MEMORY: dequant warps decode packed
//     NF4 / e4m3 bytes in registers and write them with tcgen05.st, so the
//     bf16 weight never touches shared or global memory;
//   * the activation tile X[m0:m0+BM, k:k+64] is the MMA B operand, staged in
//     shared memory by TMA (128-byte swizzle, K-major);
//   * the f32 accumulator (128 lanes = weight rows, BM columns = tokens) is in
//     tensor memory, double-buffered when it fits, and drained by epilogue
//     warps that add the bias, round to bf16 and store Y row-major.
// Warp roles (one persistent CTA per SM, static round-robin over tiles):
//   warps 0-3     epilogue (warp w owns TMEM lanes 32w..32w+31)
//   warps 4..     dequant, G groups of four (G = 2, or 4 for BM <= 64); the
//                 groups take turns by k-block (warp w writes TMEM lanes
//                 32(w%4)..)
//   then          weight producer (TMA of the packed weight, deep ring),
//                 MMA warp (elected lane issues; TMEM allocator),
//                 activation producer (TMA of X tiles)
// Three rings decouple the operands' lifetimes: packed-weight stages are
// released as soon as the dequant warps have read them, so the weight ring
// runs far ahead; X stages and TMEM A stages are released per ROUND by one
// tcgen05.commit of the MMA thread.  A round is kRound k-blocks: the MMA
// thread waits once and commits once per round, because a thread that touches
// shared memory after a tcgen05.commit pays a fixed latency of several hundred
// cycles, which per-k-block handshakes would add to every 64-deep MMA step.
// Every mbarrier wait is bounded (dq_ptx.cuh); on expiry the CTA unwinds,
// drains its in-flight copies and MMAs (bounded), frees TMEM and records
// DQ_ERR_TIMEOUT in g_dq_error.
#pragma once

#include <cuda_bf16.h>

#include "dq_codec.cuh"
#include "dq_epilogue.cuh"
#include "dq_ptx.cuh"

namespace dq {

enum : int { kFmtNF4 = 0, kFmtFP8 = 1 };
enum : unsigned int { kErrTimeout = 5u };

// Per-device kernel error word (bit kErrTimeout: a bounded wait expired).
// The library is a single translation unit, so it is defined here.
__device__ unsigned int g_dq_error = 0;

// Optional per-role timestamps (SM clock) of CTA 0, for pipeline analysis.
// Compiled out unless DQ_TRACE is defined; a tracing build supplies
// g_dq_trace[slot][index].
#ifdef DQ_TRACE
constexpr int kTraceLen = 4096;
constexpr int kTraceSlots = 32;  // 0-4 producers/MMA, 5+5g..9+5g dequant group g, 25
__device__ long long g_dq_trace[kTraceSlots][kTraceLen];
// Per CTA: globaltimer at start and end, and the SM it ran on.
__device__ unsigned long long g_dq_cta_trace[1024][3];
#define DQ_TRACE_CTA(field, value)                                                 \
  do {                                                                             \
    if (threadIdx.x == 0 && blockIdx.x < 1024) g_dq_cta_trace[blockIdx.x][field] = (value); \
  } while (0)
#define DQ_TRACE_POINT(slot, idx)                                   \
  do {                                                              \
    if (blockIdx.x == 0 && (idx) < kTraceLen) g_dq_trace[slot][idx] = clock64(); \
  } while (0)
#else
#define DQ_TRACE_POINT(slot, idx) \
  do {                            \
  } while (0)
#define DQ_TRACE_CTA(field, value) \
  do {                             \
  } while (0)
#endif

constexpr int kMaxRanks = 8;  // column-parallel ranks one launch can write to

struct GemmArgs {
  const float* absmax;        // NF4: [N, K/64] block scales, f32 (or bf16: scale_bf16)
  int scale_bf16;             // NF4: absmax holds bf16 scales
  const __nv_bfloat16* bias;  // [N] or nullptr
  void* out;                  // f32 partials [splits, M, N] when splits > 1
  int M, N, K;
  int num_n_tiles, num_tiles;
  int tile_n;                 // weight rows per tile: 128 (one CTA) or 256 (CTA pair)
  int splits, kb_per_split;
  int group_n;                // > 0: tiles visit group_n weight tiles x all token tiles at a time
  int act;                    // kActNone or kActGeluTanh (bf16 output only)
  float fp8_scale;            // fp8: per-tensor scale (rounded to bf16 in-kernel)
  int vec_ok;                 // 16-byte vector stores are aligned for every destination
  // bf16 Y destinations (splits == 1): element (m, n) goes to
  // outs[d][m * ldy + col0 + n] for every d < n_out.  One destination with
  // col0 = 0 and the caller's row stride ldy (N unless y is a column range of
  // a wider buffer) normally; every rank's y [M, N_total] (possibly peer
  // memory) in the column-parallel linear.
  void* outs[kMaxRanks];
  int n_out, ldy, col0;
  // column-parallel through a multicast mapping: when out_mc != nullptr the
  // 16-byte stores go once to out_mc[m * ldy + col0 + n] (multimem.st, all
  // ranks' y at once) instead of to each outs[d]
  void* out_mc;
  // Column-parallel completion: when tp_counter != nullptr every CTA fences
  // its stores system-wide and counts itself done; the last one raises flag
  // tp_rank of every rank's flag array (tp_flags[d]) to tp_epoch.
  unsigned int* tp_counter;
  unsigned int* tp_flags[kMaxRanks];
  int tp_rank;
  unsigned int tp_epoch;
  // Grouped order: the first group spans group0_n weight tiles (<= group_n;
  // 0 means group_n), the later ones group_n.
  int group0_n;
  // bf16 pair GEMM that dequantizes its own weight (bf16_gemm2_kernel<BM,
  // FMT>, FMT >= 0): dq_w is the packed NF4 / e4m3 weight (with absmax or
  // fp8_scale above), dq_out the bf16 scratch [N, K] its TMA loads read, and
  // dq_ready[g] counts the dequantizing warps that finished weight group g.
  const uint8_t* dq_w;
  __nv_bfloat16* dq_out;
  unsigned int* dq_ready;
};

// Column-parallel completion signal (every thread of the CTA calls it after
// the teardown barrier; the epilogue threads have already fenced their stores
// system-wide).
__device__ __forceinline__ void tp_signal_done(const GemmArgs& a) {
  if (a.tp_counter == nullptr || threadIdx.x != 0) return;
  __threadfence();  // this CTA's error-word update precedes its count
  const unsigned int done = atomicAdd(a.tp_counter, 1u);
  if (done != gridDim.x - 1) return;
  __threadfence();  // ... and is seen by the last CTA after it reads the count
  *a.tp_counter = 0u;  // ready for the next launch (stream-ordered)
  // A CTA that gave up on a wait left its tiles unwritten: raise no flag, so
  // the other ranks' bounded waits report the failure too.
  if (atomicOr(&g_dq_error, 0u) & (1u << kErrTimeout)) return;
  __threadfence_system();
#pragma unroll
  for (int d = 0; d < kMaxRanks; ++d)
    if (d < a.n_out)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.tp_flags[d] + a.tp_rank),
                   "r"(a.tp_epoch)
                   : "memory");
}

template <int FMT, int BM>
struct GemmCfg {
  static_assert(BM % 16 == 0 && BM >= 16 && BM <= 256, "BM must be a multiple of 16 in [16,256]");
  static constexpr int kBN = 128;                               // weight rows per tile (MMA M)
  static constexpr int kWBytes = FMT == kFmtNF4 ? 32 : 64;      // packed bytes per row per k-block
  static constexpr int kNumAcc = BM <= 192 ? 2 : 1;             // accumulator buffers
  static constexpr int kAccStride = BM < 32 ? 32 : BM;          // TMEM columns per accumulator
  static constexpr int kACol0 = ((kNumAcc * kAccStride + 31) / 32) * 32;
  // k-blocks per MMA round (the measured best: 2, and 1 for BM=256).
  static constexpr int kRound = BM >= 256 ? 1 : 2;
  // Small tiles carry little MMA work per k-block, so the decode rate sets the
  // pace: four groups of dequant warps (and deeper rings) for BM <= 64.
  static constexpr bool kSmall = BM <= 64;
  static constexpr int kDqGroups = kSmall ? 4 : 2;
  static constexpr int kDqWarps = 4 * kDqGroups;
  static constexpr int kWProducerWarp = 4 + kDqWarps;
  static constexpr int kMmaWarp = 5 + kDqWarps;
  static constexpr int kXProducerWarp = 6 + kDqWarps;
  static constexpr int kThreads = (7 + kDqWarps) * 32;
  static constexpr int kXStageBytes = BM * 128;
  static constexpr int kWStageBytes = kBN * kWBytes;
  static constexpr int kEpiCols = BM % 32 == 0 ? 32 : 16;       // accumulator columns per drain step
  static constexpr int kEpiBytes = 4 * kEpiCols * 32 * 4;       // per-warp [cols][32] f32 staging
  static constexpr int kSmemLimit = 227 * 1024;
  // NF4 decodes through a 32 KB shared byte LUT (dq_codec.cuh)
  static constexpr int kLutBytes = FMT == kFmtNF4 ? kNf4LutBytes : 0;
  // weight ring: 32 KB (NF4) / 48 KB (fp8) of packed tiles, 96 / 128 KB for small tiles
  static constexpr int kWStages =
      ((kSmall ? (FMT == kFmtNF4 ? 96 : 128) : (FMT == kFmtNF4 ? 32 : 48)) * 1024) / kWStageBytes;
  // activation ring: rounds of X tiles in the rest
  static constexpr int kXRoundsFit =
      (kSmemLimit - kEpiBytes - 2048 - kLutBytes - kWStages * kWStageBytes) / (kRound * kXStageBytes);
  static constexpr int kXRoundsMax = kSmall ? 8 : 4;
  static constexpr int kXRounds = kXRoundsFit > kXRoundsMax ? kXRoundsMax : kXRoundsFit;
  static_assert(kXRounds >= 2, "need two rounds of X tiles in flight");
  static constexpr int kXStages = kXRounds * kRound;
  // TMEM A ring
  static constexpr int kARoundsFit = (512 - kACol0) / 32 / kRound;
  static constexpr int kARoundsMax = kSmall ? 8 : 4;
  static constexpr int kARounds = kARoundsFit > kARoundsMax ? kARoundsMax : kARoundsFit;
  static_assert(kARounds >= 2, "need two rounds of TMEM A stages");
  static constexpr int kAStages = kARounds * kRound;
  // one completion barrier per round, shared by the X and A rings
  static constexpr int kDoneBars = kXRounds > kARounds ? kXRounds : kARounds;
  static constexpr int kNumBars = 2 * kWStages + kXStages + kDoneBars + kARounds + 2 * kNumAcc + 1;
  static constexpr int kOffW = kXStages * kXStageBytes;
  static constexpr int kOffLut = kOffW + kWStages * kWStageBytes;
  static constexpr int kOffEpi = kOffLut + kLutBytes;
  static constexpr int kOffBar = kOffEpi + kEpiBytes;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  // Padded so that one CTA fills an SM: the CTA allocates all 512 TMEM columns.
  static constexpr int kSmemUsed = kOffMisc + 16 + 1024;
  static constexpr int kSmemBytes = kSmemUsed < 120 * 1024 ? 120 * 1024 : kSmemUsed;
  static_assert(kSmemBytes <= kSmemLimit, "shared memory over the per-CTA limit");
  static constexpr uint32_t kIdesc = make_idesc_bf16(kBN, BM);
};

struct TileCoord {
  int m0, n0, kb0, kb1, split;
  int group;  // weight group of the grouped order (0 otherwise)
};

// Width of the first weight group of the grouped order.
__host__ __device__ __forceinline__ int first_group_width(int group_n, int group0_n, int n_tiles) {
  const int g0 = group0_n > 0 ? (group0_n < group_n ? group0_n : group_n) : group_n;
  return g0 < n_tiles ? g0 : n_tiles;
}

__device__ __forceinline__ TileCoord tile_coord(const GemmArgs& a, int t, int KB) {
  TileCoord c;
  c.split = t % a.splits;
  c.group = 0;
  const int mn = t / a.splits;
  if (a.group_n > 0) {
    // Grouped order: token tiles run fastest over a group of weight tiles, so
    // the tiles in flight share a few weight tiles (kept in L2) instead of
    // streaming every weight row once per token tile.  The first group may be
    // narrower (group0_n) so that the weight it needs is ready sooner.
    const int m_tiles = a.num_tiles / (a.splits * a.num_n_tiles);
    const int g0 = first_group_width(a.group_n, a.group0_n, a.num_n_tiles);
    int nb, gn, r;
    if (mn < g0 * m_tiles) {
      nb = 0;
      gn = g0;
      r = mn;
    } else {
      const int per_group = a.group_n * m_tiles;
      const int q = (mn - g0 * m_tiles) / per_group;
      c.group = 1 + q;
      nb = g0 + q * a.group_n;
      gn = min(a.group_n, a.num_n_tiles - nb);
      r = mn - g0 * m_tiles - q * per_group;
    }
    c.n0 = (nb + r % gn) * a.tile_n;
    c.m0 = r / gn;
  } else {
    c.n0 = (mn % a.num_n_tiles) * a.tile_n;
    c.m0 = (mn / a.num_n_tiles);
  }
  c.kb0 = c.split * a.kb_per_split;
  c.kb1 = min(KB, c.kb0 + a.kb_per_split);
  return c;
}

// Position in this CTA's sequence of rounds: tile t, first k-block kb of the
// round (k-blocks kb .. kb+R-1, those >= tc.kb1 are absent).
struct RoundCursor {
  int t, kb, stride;
  TileCoord tc;
  bool valid;
};

// Tiles first, first + stride, ... belong to this CTA (or CTA pair).
__device__ __forceinline__ RoundCursor round_begin(const GemmArgs& a, int KB, int first,
                                                   int stride) {
  RoundCursor c;
  c.t = first;
  c.stride = stride;
  c.valid = c.t < a.num_tiles;
  if (c.valid) {
    c.tc = tile_coord(a, c.t, KB);
    c.kb = c.tc.kb0;
  }
  return c;
}

template <int R>
__device__ __forceinline__ void round_advance(RoundCursor& c, const GemmArgs& a, int KB) {
  if (!c.valid) return;
  c.kb += R;
  if (c.kb >= c.tc.kb1) {
    c.t += c.stride;
    c.valid = c.t < a.num_tiles;
    if (c.valid) {
      c.tc = tile_coord(a, c.t, KB);
      c.kb = c.tc.kb0;
    }
  }
}

// absmax of (row r of the round's tile, k-block kb); 0 when absent.
__device__ __forceinline__ float load_absmax(const GemmArgs& a, const RoundCursor& c, int kb, int r,
                                             int KB) {
  const int n = c.tc.n0 + r;
  if (!c.valid || n >= a.N || kb >= c.tc.kb1) return 0.f;
  return load_scale(a.absmax, static_cast<int64_t>(n) * KB + kb, a.scale_bf16 != 0);
}

// VAR: 0 = plain epilogue (no activation or GELU-tanh), 1 = column-parallel
// (every rank's y, then the completion flags), 2 = gated epilogue (SwiGLU /
// GeGLU-tanh; its own instantiation, which keeps the extra epilogue code out
// of the other two: compiled into the plain kernel it cost 4-7% at M = 512).
template <int FMT, int BM, int VAR>
__global__ void __launch_bounds__(GemmCfg<FMT, BM>::kThreads, 1)
    dq_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                   const __grid_constant__ CUtensorMap tmap_w, const GemmArgs args) {
  using C = GemmCfg<FMT, BM>;
  constexpr bool TP = VAR == 1;
  constexpr bool GATED = VAR == 2;
  constexpr int R = C::kRound;
  constexpr int XR = C::kXRounds;
  constexpr int AR = C::kARounds;
  constexpr int DB = C::kDoneBars;
  constexpr int WS = C::kWStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::kOffBar;
  // barriers: wfull[WS], wempty[WS], xfull[XS], done[DB], afull[AR], acc_full, acc_empty, drain
  auto wfull_bar = [&](int s) { return bar0 + 8u * s; };
  auto wempty_bar = [&](int s) { return bar0 + 8u * (WS + s); };
  auto xfull_bar = [&](int s) { return bar0 + 8u * (2 * WS + s); };
  auto done_bar = [&](int d) { return bar0 + 8u * (2 * WS + C::kXStages + d); };
  auto afull_bar = [&](int a) { return bar0 + 8u * (2 * WS + C::kXStages + DB + a); };
  auto accfull_bar = [&](int a) { return bar0 + 8u * (2 * WS + C::kXStages + DB + AR + a); };
  auto accempty_bar = [&](int a) {
    return bar0 + 8u * (2 * WS + C::kXStages + DB + AR + C::kNumAcc + a);
  };
  const uint32_t drain_bar = bar0 + 8u * (C::kNumBars - 1);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);
  // Wait until round qq's MMAs have retired (no wait for qq < 0).
  auto wait_done = [&](int qq) -> bool {
    if (qq < 0) return true;
    return mbar_wait(done_bar(qq % DB), static_cast<uint32_t>((qq / DB) & 1), abort_flag);
  };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KB = (args.K + 63) / 64;  // fp8 allows a ragged last k-block (TMA zero-fills it)

  if (warp == C::kWProducerWarp && lane == 0) {
    for (int s = 0; s < WS; ++s) {
      mbar_init(wfull_bar(s), 1);
      mbar_init(wempty_bar(s), 4);  // the four warps of the group that decoded it
    }
    for (int s = 0; s < C::kXStages; ++s) mbar_init(xfull_bar(s), 1);
    for (int d = 0; d < DB; ++d) mbar_init(done_bar(d), 1);
    for (int a = 0; a < AR; ++a) mbar_init(afull_bar(a), 4 * R);  // four warps per k-block
    for (int a = 0; a < C::kNumAcc; ++a) {
      mbar_init(accfull_bar(a), 1);
      mbar_init(accempty_bar(a), 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmap_x);
    prefetch_tensormap(&tmap_w);
  }
  if (warp == C::kMmaWarp) {
    tmem_alloc(smem_u32(tmem_holder), 512);
    tmem_relinquish();
  }
  if constexpr (FMT == kFmtNF4) nf4_lut_fill(reinterpret_cast<uint32_t*>(smem + C::kOffLut));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  DQ_TRACE_CTA(0, globaltimer_ns());

  if (warp == C::kWProducerWarp) {
    // ----------------------------------------------------- weight producer
    if (lane == 0) {
      int iw = 0;  // running count of present k-blocks = weight ring position
      for (RoundCursor rc = round_begin(args, KB, blockIdx.x, gridDim.x); rc.valid; round_advance<R>(rc, args, KB)) {
        for (int j = 0; j < R; ++j) {
          const int kb = rc.kb + j;
          if (kb >= rc.tc.kb1) break;
          const int s = iw % WS;
          if (!mbar_wait(wempty_bar(s), static_cast<uint32_t>(((iw / WS) & 1) ^ 1), abort_flag)) break;
          DQ_TRACE_POINT(0, iw);
          mbar_arrive_expect_tx(wfull_bar(s), C::kWStageBytes);
          tma_load_2d(sbase + C::kOffW + s * C::kWStageBytes, &tmap_w, wfull_bar(s), kb * C::kWBytes,
                      rc.tc.n0);
          ++iw;
        }
        if (*abort_flag) break;
      }
      if (*abort_flag) {
        // Let issued copies land before shared memory is released (bounded).
        for (int i = 1; i <= WS && i <= iw; ++i) {
          volatile int never = 0;
          mbar_wait(wfull_bar((iw - i) % WS), static_cast<uint32_t>(((iw - i) / WS) & 1), &never,
                    100000000ull);
        }
      }
    }
    __syncwarp();
  } else if (warp == C::kXProducerWarp) {
    // ------------------------------------------------- activation producer
    if (lane == 0) {
      int q = 0;
      for (RoundCursor rc = round_begin(args, KB, blockIdx.x, gridDim.x); rc.valid; round_advance<R>(rc, args, KB), ++q) {
        // X slots of round q were last used by round q - XR.
        if (!wait_done(q - XR)) break;
        DQ_TRACE_POINT(1, q);
        const int m0 = rc.tc.m0 * BM;
#pragma unroll
        for (int j = 0; j < R; ++j) {
          const int slot = (q % XR) * R + j;
          const int kb = rc.kb + j;
          if (kb < rc.tc.kb1) {
            mbar_arrive_expect_tx(xfull_bar(slot), C::kXStageBytes);
            tma_load_2d(sbase + slot * C::kXStageBytes, &tmap_x, xfull_bar(slot), kb * 64, m0);
          } else {
            mbar_arrive(xfull_bar(slot));  // absent k-block: complete the phase with no data
          }
        }
      }
      if (*abort_flag) {
        for (int i = 1; i <= XR && i <= q; ++i) {
          const int qq = q - i;
          for (int j = 0; j < R; ++j) {
            volatile int never = 0;
            mbar_wait(xfull_bar((qq % XR) * R + j), static_cast<uint32_t>((qq / XR) & 1), &never,
                      100000000ull);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == C::kMmaWarp) {
    // ------------------------------------------------------------------ MMA
    // The whole warp runs the loop (warp-uniform state); one elected lane
    // issues each tcgen05.mma / commit.  Wait outcomes are agreed warp-wide.
    int q = 0, acc = 0;
    uint32_t accphase = 0;
    uint32_t d_tmem = 0;
    for (RoundCursor rc = round_begin(args, KB, blockIdx.x, gridDim.x); rc.valid; ++q) {
      if (rc.kb == rc.tc.kb0) {
        if (!__all_sync(0xffffffffu, mbar_wait(accempty_bar(acc), accphase ^ 1u, abort_flag))) break;
        tc_fence_after();
        d_tmem = tmem_base + static_cast<uint32_t>(acc * C::kAccStride);
      }
      // The dequant warps arrive only after observing the round's X tiles
      // land, so this one wait covers both operands.
      if (lane == 0) DQ_TRACE_POINT(2, q);
      if (!__all_sync(0xffffffffu,
                      mbar_wait(afull_bar(q % AR), static_cast<uint32_t>((q / AR) & 1), abort_flag)))
        break;
      if (lane == 0) DQ_TRACE_POINT(3, q);
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const int kb = rc.kb + j;
        if (kb < rc.tc.kb1) {
          const uint64_t bdesc = make_sw128_kmajor_desc(sbase + ((q % XR) * R + j) * C::kXStageBytes);
          const uint32_t a_tmem =
              tmem_base + static_cast<uint32_t>(C::kACol0 + ((q % AR) * R + j) * 32);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // K step k: 16 bf16 = 8 TMEM columns of A, 32 bytes along the swizzled B rows.
            tc_mma_ts_elect(d_tmem, a_tmem + 8u * k, bdesc + static_cast<uint64_t>(2 * k), C::kIdesc,
                            (kb > rc.tc.kb0 || k > 0) ? 1u : 0u);
          }
        }
      }
      tc_commit_elect(done_bar(q % DB));
      if (lane == 0) DQ_TRACE_POINT(4, q);
      const int t_now = rc.t;
      round_advance<R>(rc, args, KB);
      if (!rc.valid || rc.t != t_now) {
        tc_commit_elect(accfull_bar(acc));
        if (++acc == C::kNumAcc) { acc = 0; accphase ^= 1u; }
      }
      __syncwarp();
    }
    if (*abort_flag) {
      // Wait (bounded) until every MMA this warp issued has retired.
      __syncwarp();
      tc_commit_elect(drain_bar);
      volatile int never = 0;
      mbar_wait(drain_bar, 0, &never, 100000000ull);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // -------------------------------------------------------------- dequant
    const int dw = warp - 4;
    const int quad = warp & 3;           // TMEM lane quadrant this warp may access
    const int group = dw >> 2;           // this warp decodes k-blocks j = group, group + G, ...
    const int r = quad * 32 + lane;      // weight row within the tile
    // The weight tile lands with the TMA 32-byte (NF4) / 64-byte (fp8)
    // swizzle: 16-byte chunk c of row r sits at chunk c ^ (r>>2 & 1) /
    // c ^ (r>>1 & 3), so the eight lanes of each 128-bit load phase hit
    // distinct banks.
    const uint32_t wsw = FMT == kFmtNF4 ? ((r >> 2) & 1) : ((r >> 1) & 3);
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    float sfp8 = 0.f;
    if constexpr (FMT == kFmtFP8) sfp8 = __bfloat162float(__float2bfloat16_rn(args.fp8_scale));
    constexpr int G = C::kDqGroups;
    // k-block j of round q belongs to group (q * R + j) % G, so the groups
    // alternate k-blocks whatever the round length.
    auto mine = [&](int qq, int j) { return ((qq * R + j) % G) == group; };
    RoundCursor rc = round_begin(args, KB, blockIdx.x, gridDim.x);
    // Block scales are fetched one round ahead of their use.
    float am[R];
#pragma unroll
    for (int j = 0; j < R; ++j)
      am[j] = (FMT == kFmtNF4 && mine(0, j)) ? load_absmax(args, rc, rc.kb + j, r, KB) : 0.f;
    int iw = 0;  // weight ring position of the round's first k-block
    bool ok = true;
    for (int q = 0; rc.valid && ok; ++q) {
      RoundCursor nx = rc;
      round_advance<R>(nx, args, KB);
      float am_next[R];
#pragma unroll
      for (int j = 0; j < R; ++j)
        am_next[j] = (FMT == kFmtNF4 && mine(q + 1, j)) ? load_absmax(args, nx, nx.kb + j, r, KB) : 0.f;
      const int present = min(R, rc.tc.kb1 - rc.kb);
      const bool row_ok = (rc.tc.n0 + r) < args.N;
      bool tmem_free = false;
#pragma unroll
      for (int j = 0; j < R; ++j) {
        if (!mine(q, j)) continue;
        if (j < present) {
          const int ws = (iw + j) % WS;
          if (!mbar_wait(wfull_bar(ws), static_cast<uint32_t>(((iw + j) / WS) & 1), abort_flag)) {
            ok = false;
            break;
          }
          const bool tp = lane == 0 && quad == 0;
          if (tp) DQ_TRACE_POINT(5 + 5 * group, q * R + j);
          const uint32_t wrow = sbase + C::kOffW + ws * C::kWStageBytes + r * C::kWBytes;
          uint4 pk[C::kWBytes / 16];
#pragma unroll
          for (int i = 0; i < C::kWBytes / 16; ++i) pk[i] = lds128(wrow + 16u * (i ^ wsw));
          // the producer's next TMA into this stage must not overtake these reads
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(wempty_bar(ws));
          if (tp && group == 0) DQ_TRACE_POINT(25, q * R + j);
          uint32_t out[32];
          const uint32_t* pw = reinterpret_cast<const uint32_t*>(pk);
          if constexpr (FMT == kFmtNF4) {
            const uint32_t sc2 = nf4_scale2(am[j]);
            const uint32_t lut_lane = sbase + C::kOffLut + 4u * lane;
#pragma unroll
            for (int i = 0; i < 8; ++i) nf4_decode_word_lut(pw[i], lut_lane, sc2, out + 4 * i);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) fp8_decode_word(pw[i], sfp8, out + 2 * i);
          }
          if (!row_ok) {
#pragma unroll
            for (int i = 0; i < 32; ++i) out[i] = 0u;
          }
          if (tp) DQ_TRACE_POINT(6 + 5 * group, q * R + j);
          // The MMA thread waits only on afull: make sure this k-block's X
          // tile has landed before vouching for it.
          if (!mbar_wait(xfull_bar((q % XR) * R + j), static_cast<uint32_t>((q / XR) & 1),
                         abort_flag)) {
            ok = false;
            break;
          }
          if (tp) DQ_TRACE_POINT(7 + 5 * group, q * R + j);
          if (!tmem_free) {
            // TMEM A stages of this round were last read by round q - AR.
            if (!wait_done(q - AR)) { ok = false; break; }
            tc_fence_after();
            tmem_free = true;
          }
          tmem_st_x32(tmem_base + lane_addr +
                          static_cast<uint32_t>(C::kACol0 + ((q % AR) * R + j) * 32),
                      out);
          tmem_wait_st();
          tc_fence_before();
          if (tp) DQ_TRACE_POINT(8 + 5 * group, q * R + j);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(afull_bar(q % AR));
        if (lane == 0 && quad == 0) DQ_TRACE_POINT(9 + 5 * group, q * R + j);
      }
#pragma unroll
      for (int j = 0; j < R; ++j) am[j] = am_next[j];
      iw += present;
      rc = nx;
    }
  } else {
    // ------------------------------------------------------------- epilogue
    constexpr int EC = C::kEpiCols;
    const int quad = warp;  // warps 0..3
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    uint8_t* stg = smem + C::kOffEpi + quad * (EC * 32 * 4);
    const uint32_t stg_s = sbase + C::kOffEpi + quad * (EC * 32 * 4);
    int acc = 0;
    uint32_t accphase = 0;
    const bool f32_out = args.splits > 1;
    for (int t = blockIdx.x; t < args.num_tiles; t += gridDim.x) {
      const TileCoord tc = tile_coord(args, t, KB);
      const int m0 = tc.m0 * BM;
      const int n = tc.n0 + quad * 32 + lane;
      float bias = 0.f;
      if (!f32_out && args.bias != nullptr && n < args.N) bias = __bfloat162float(args.bias[n]);
      if (!mbar_wait(accfull_bar(acc), accphase, abort_flag)) break;
      tc_fence_after();
      const uint32_t d_addr = tmem_base + lane_addr + static_cast<uint32_t>(acc * C::kAccStride);
      const int ncol0 = tc.n0 + quad * 32;
      constexpr int NC = BM / EC;
      // Double-buffered drain: the TMEM load of chunk c+1 is in flight while
      // chunk c is converted and stored.
      uint32_t v[2][32];
      auto tmem_load = [&](int c, uint32_t* dst) {
        if constexpr (EC == 32) {
          tmem_ld_x32(d_addr + 32u * c, dst);
        } else {
          tmem_ld_x16(d_addr + 16u * c, *reinterpret_cast<uint32_t(*)[16]>(dst));
        }
      };
      tmem_load(0, v[0]);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        tmem_wait_ld();
        if (c + 1 < NC) {
          tmem_load(c + 1, v[(c + 1) & 1]);
        } else {
          // The whole accumulator has been read: hand it back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(accempty_bar(acc));
        }
        const uint32_t* vc = v[c & 1];
        const int mrow0 = m0 + EC * c;  // token of staging row 0
        if (!f32_out) {
          // stage [EC tokens][32 outputs] bf16 per warp, then write 64-byte
          // row segments of Y (to every rank's y in the column-parallel
          // instantiation; the store loop is compiled only there: even an
          // untaken one costs ~10% at BM=256, where the drain is exposed)
          __nv_bfloat16* sb = reinterpret_cast<__nv_bfloat16*>(stg);
          if constexpr (GATED) {
            gated_chunk_store<EC>(vc, bias, args.act, stg_s, sb,
                                  reinterpret_cast<__nv_bfloat16*>(args.outs[0]) + args.col0, args.ldy, args.M,
                                  args.N / 2, mrow0, ncol0 / 2, args.vec_ok, lane);
          } else {
            if (args.act == kActNone) {
#pragma unroll
              for (int j = 0; j < EC; ++j)
                sts16(stg_s + 2u * (j * 32 + lane),
                      __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(vc[j]) + bias)));
            } else {
#pragma unroll
              for (int j = 0; j < EC; ++j)
                sts16(stg_s + 2u * (j * 32 + lane),
                      __bfloat16_as_ushort(__float2bfloat16_rn(
                          apply_act(__uint_as_float(vc[j]) + bias, args.act))));
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < EC / 8; ++i) {
              const int row = (lane >> 2) + 8 * i;
              const int col = (lane & 3) * 8;
              const int m = mrow0 + row;
              const int nc = ncol0 + col;
              if (m < args.M) {
                const size_t off = static_cast<size_t>(m) * args.ldy + args.col0 + nc;
                if (args.vec_ok && nc + 8 <= args.N) {
                  const uint4 v16 = lds128(stg_s + 2u * (row * 32 + col));
                  if constexpr (TP) {
                    if (args.out_mc != nullptr) {
                      multimem_st16(reinterpret_cast<__nv_bfloat16*>(args.out_mc) + off, v16);
                    } else {
#pragma unroll
                      for (int d = 0; d < kMaxRanks; ++d)
                        if (d < args.n_out)
                          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(args.outs[d]) + off) = v16;
                    }
                  } else {
                    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(args.outs[0]) + off) = v16;
                  }
                } else {
                  const __nv_bfloat16* src = sb + row * 32 + col;
#pragma unroll
                  for (int d = 0; d < (TP ? kMaxRanks : 1); ++d) {
                    if (d >= args.n_out) break;
                    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.outs[d]) + off;
                    for (int e = 0; e < 8; ++e)
                      if (nc + e < args.N) dst[e] = src[e];
                  }
                }
              }
            }
            __syncwarp();
          }
        } else {
          // split-K partial: stage [EC][32] f32, write 128-byte row segments
          float* sf = reinterpret_cast<float*>(stg);
#pragma unroll
          for (int j = 0; j < EC; ++j) sts32(stg_s + 4u * (j * 32 + lane), vc[j]);
          __syncwarp();
          float* part = reinterpret_cast<float*>(args.out) +
                        static_cast<size_t>(tc.split) * args.M * args.N;
#pragma unroll
          for (int i = 0; i < EC / 4; ++i) {
            const int row = (lane >> 3) + 4 * i;
            const int col = (lane & 7) * 4;
            const int m = mrow0 + row;
            const int nc = ncol0 + col;
            if (m < args.M) {
              float* dst = part + static_cast<size_t>(m) * args.N + nc;
              const float* src = sf + row * 32 + col;
              if (args.vec_ok && nc + 4 <= args.N) {
                const uint4 q4 = lds128(stg_s + 4u * (row * 32 + col));
                *reinterpret_cast<uint4*>(dst) = q4;
              } else {
                for (int e = 0; e < 4; ++e)
                  if (nc + e < args.N) dst[e] = src[e];
              }
            }
          }
          __syncwarp();
        }
      }
      if (++acc == C::kNumAcc) { acc = 0; accphase ^= 1u; }
    }
    // Column-parallel output: this thread's peer stores are visible system-wide
    // before its CTA counts itself done.
    if constexpr (TP) __threadfence_system();
  }

  // ------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == C::kMmaWarp) tmem_dealloc(tmem_base, 512);
  if (threadIdx.x == 0 && *abort_flag) atomicOr(&g_dq_error, 1u << kErrTimeout);
  if constexpr (TP) tp_signal_done(args);
#ifdef DQ_TRACE
  {
    unsigned int smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    DQ_TRACE_CTA(1, globaltimer_ns());
    DQ_TRACE_CTA(2, smid);
  }
#endif
}

}  // namespace dq
