// dq_gemm2.cuh -- the fused dequantize + tcgen05 GEMM on a CTA PAIR (cluster of
// two CTAs on two SMs, tcgen05 cta_group::2).
//
// One pair computes Y^T[n0:n0+256, m0:m0+BM] with M = 256 MMAs: CTA r of the
// pair dequantizes weight rows n0+128r .. n0+128r+127 into its own tensor
// memory (the MMA A operand, as in dq_gemm.cuh) and stages token rows
// m0+r*BM/2 .. m0+(r+1)*BM/2-1 of X in its own shared memory (half of the B
// operand).  The leader CTA (rank 0) issues the pair MMAs, which read the A
// halves from both CTAs' tensor memory and the B halves from both CTAs' shared
// memory, and accumulate each CTA's 128 weight rows x BM tokens in that CTA's
// tensor memory.  Relative to one CTA per tile, every SM stages and streams
// half as many activation bytes per MMA, which leaves shared-memory bandwidth
// for the dequant warps' byte-LUT lookups.
//
// Cross-CTA protocol (the peer is rank 1):
//   * X halves: both CTAs TMA their half with .cta_group::2, completing on the
//     LEADER's xfull barrier; the leader's producer alone posts expect_tx for
//     both halves.
//   * A stages: both CTAs' dequant warps arrive on the LEADER's afull barrier
//     (mapa + mbarrier.arrive.release.cluster); only the leader's dequant warps
//     wait on xfull first, so one wait by the MMA thread covers every operand.
//   * Round completion and accumulator-full: the leader's tcgen05.commit is
//     multicast to the barrier at the same offset in both CTAs.
//   * Accumulator-empty: both CTAs' epilogue warps arrive on the LEADER's
//     accempty barrier.
//   * A cluster barrier after barrier initialization and another before TMEM
//     deallocation keep remote arrivals off uninitialized or released memory.
// No TMA load here is a cluster-multicast load: each CTA fetches its own half.
#pragma once

#include "dq_gemm.cuh"

namespace dq {

template <int FMT, int BM>
struct Gemm2Cfg {
  static_assert(BM % 32 == 0 && BM >= 64 && BM <= 256, "pair tiles need BM in {64..256}, /32");
  static constexpr int kHalfBM = BM / 2;                        // token rows staged per CTA
  static constexpr int kWBytes = FMT == kFmtNF4 ? 32 : 64;
  static constexpr int kNumAcc = BM <= 192 ? 2 : 1;
  static constexpr int kAccStride = BM;
  static constexpr int kACol0 = ((kNumAcc * kAccStride + 31) / 32) * 32;
  // k-blocks per MMA round.  Two k-blocks even at BM=256 (1024 cycles of
  // tensor work per round): one k-block per round leaves the tensor core idle
  // during the MMA warp's per-round wait + commit handshake.
  static constexpr int kRound = BM >= 128 ? 2 : 4;
  static constexpr int kDqGroups = 2;
  static constexpr int kDqWarps = 4 * kDqGroups;
  static constexpr int kWProducerWarp = 4 + kDqWarps;
  static constexpr int kMmaWarp = 5 + kDqWarps;
  static constexpr int kXProducerWarp = 6 + kDqWarps;
  static constexpr int kThreads = (7 + kDqWarps) * 32;
  static constexpr int kXStageBytes = kHalfBM * 128;
  static constexpr int kWStageBytes = 128 * kWBytes;
  static constexpr int kEpiCols = 32;
  static constexpr int kEpiBytes = 4 * kEpiCols * 32 * 4;
  static constexpr int kLutBytes = FMT == kFmtNF4 ? kNf4LutBytes : 0;
  static constexpr int kSmemLimit = 227 * 1024;
  static constexpr int kWStages = ((FMT == kFmtNF4 ? 32 : 48) * 1024) / kWStageBytes;
  static constexpr int kXRoundsFit =
      (kSmemLimit - kEpiBytes - 2048 - kLutBytes - kWStages * kWStageBytes) / (kRound * kXStageBytes);
  static constexpr int kXRounds = kXRoundsFit > 6 ? 6 : kXRoundsFit;
  static_assert(kXRounds >= 2, "need two rounds of X tiles in flight");
  static constexpr int kXStages = kXRounds * kRound;
  static constexpr int kARoundsFit = (512 - kACol0) / 32 / kRound;
  static constexpr int kARounds = kARoundsFit > 4 ? 4 : kARoundsFit;
  static_assert(kARounds >= 2, "need two rounds of TMEM A stages");
  static constexpr int kAStages = kARounds * kRound;
  static constexpr int kDoneBars = kXRounds > kARounds ? kXRounds : kARounds;
  static constexpr int kNumBars = 2 * kWStages + kXStages + kDoneBars + kARounds + 2 * kNumAcc + 1;
  static constexpr int kOffW = kXStages * kXStageBytes;
  static constexpr int kOffLut = kOffW + kWStages * kWStageBytes;
  static constexpr int kOffEpi = kOffLut + kLutBytes;
  static constexpr int kOffBar = kOffEpi + kEpiBytes;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemUsed = kOffMisc + 16 + 1024;
  static constexpr int kSmemBytes = kSmemUsed < 120 * 1024 ? 120 * 1024 : kSmemUsed;
  static_assert(kSmemBytes <= kSmemLimit, "shared memory over the per-CTA limit");
  static constexpr uint32_t kIdesc = make_idesc_bf16(256, BM);
  static constexpr uint32_t kXTxBytes = BM * 128;               // both halves of a k-block
};

// VAR: 0 = plain epilogue (no activation or GELU-tanh), 1 = column-parallel
// (every rank's y, then the completion flags), 2 = gated epilogue (SwiGLU /
// GeGLU-tanh; its own instantiation, which keeps the extra epilogue code out
// of the other two: compiled into the plain kernel it cost 4-7% at M = 512).
template <int FMT, int BM, int VAR>
__global__ void __launch_bounds__(Gemm2Cfg<FMT, BM>::kThreads, 1)
    dq_gemm2_kernel(const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_w, const GemmArgs args) {
  using C = Gemm2Cfg<FMT, BM>;
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

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int KB = (args.K + 63) / 64;
  // Round completions are committed by the leader to both CTAs: wait with
  // cluster-scope acquire.
  auto wait_done = [&](int qq) -> bool {
    if (qq < 0) return true;
    return mbar_wait_cluster(done_bar(qq % DB), static_cast<uint32_t>((qq / DB) & 1), abort_flag);
  };

  if (warp == C::kWProducerWarp && lane == 0) {
    for (int s = 0; s < WS; ++s) {
      mbar_init(wfull_bar(s), 1);
      mbar_init(wempty_bar(s), 4);
    }
    for (int s = 0; s < C::kXStages; ++s) mbar_init(xfull_bar(s), 1);
    for (int d = 0; d < DB; ++d) mbar_init(done_bar(d), 1);
    for (int a = 0; a < AR; ++a) mbar_init(afull_bar(a), 2 * 4 * R);  // 4 warps x R k-blocks x 2 CTAs
    for (int a = 0; a < C::kNumAcc; ++a) {
      mbar_init(accfull_bar(a), 1);
      mbar_init(accempty_bar(a), 2 * 4);                                // 4 epilogue warps x 2 CTAs
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmap_x);
    prefetch_tensormap(&tmap_w);
  }
  if (warp == C::kMmaWarp) {
    tmem_alloc_pair(smem_u32(tmem_holder), 512);
    tmem_relinquish_pair();
  }
  if constexpr (FMT == kFmtNF4) nf4_lut_fill(reinterpret_cast<uint32_t*>(smem + C::kOffLut));
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before anyone signals across the pair
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  DQ_TRACE_CTA(0, globaltimer_ns());

  if (warp == C::kWProducerWarp) {
    // ----------------------------------------------------- weight producer
    if (lane == 0) {
      int iw = 0;
      for (RoundCursor rc = round_begin(args, KB, pair, npairs); rc.valid; round_advance<R>(rc, args, KB)) {
        for (int j = 0; j < R; ++j) {
          const int kb = rc.kb + j;
          if (kb >= rc.tc.kb1) break;
          const int s = iw % WS;
          if (!mbar_wait(wempty_bar(s), static_cast<uint32_t>(((iw / WS) & 1) ^ 1), abort_flag)) break;
          DQ_TRACE_POINT(0, iw);
          mbar_arrive_expect_tx(wfull_bar(s), C::kWStageBytes);
          tma_load_2d(sbase + C::kOffW + s * C::kWStageBytes, &tmap_w, wfull_bar(s), kb * C::kWBytes,
                      rc.tc.n0 + 128 * static_cast<int>(rank));
          ++iw;
        }
        if (*abort_flag) break;
      }
      if (*abort_flag) {
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
      for (RoundCursor rc = round_begin(args, KB, pair, npairs); rc.valid;
           round_advance<R>(rc, args, KB), ++q) {
        if (!wait_done(q - XR)) break;
        DQ_TRACE_POINT(1, q);
        const int m_half = rc.tc.m0 * BM + static_cast<int>(rank) * C::kHalfBM;
#pragma unroll
        for (int j = 0; j < R; ++j) {
          const int slot = (q % XR) * R + j;
          const uint32_t lead_bar = mapa_shared(xfull_bar(slot), 0);
          const int kb = rc.kb + j;
          if (kb < rc.tc.kb1) {
            if (leader) mbar_arrive_expect_tx(xfull_bar(slot), C::kXTxBytes);
            tma_load_2d_pair(sbase + slot * C::kXStageBytes, &tmap_x, lead_bar, kb * 64, m_half);
          } else if (leader) {
            mbar_arrive(xfull_bar(slot));  // absent k-block: complete the phase with no data
          }
        }
      }
      // In-flight copies of this CTA complete on the leader's barriers, which
      // the leader drains; both CTAs meet at the cluster barrier before exit.
      if (*abort_flag && leader) {
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
    // ------------------------------------------------------- MMA (leader)
    // Whole-warp loop, one elected lane issues (see the one-CTA kernel).
    if (leader) {
      int q = 0, acc = 0;
      uint32_t accphase = 0;
      uint32_t d_tmem = 0;
      for (RoundCursor rc = round_begin(args, KB, pair, npairs); rc.valid; ++q) {
        if (rc.kb == rc.tc.kb0) {
          if (!__all_sync(0xffffffffu, mbar_wait_cluster(accempty_bar(acc), accphase ^ 1u, abort_flag)))
            break;
          tc_fence_after();
          d_tmem = tmem_base + static_cast<uint32_t>(acc * C::kAccStride);
        }
        if (lane == 0) DQ_TRACE_POINT(2, q);
        if (!__all_sync(0xffffffffu, mbar_wait_cluster(afull_bar(q % AR),
                                                       static_cast<uint32_t>((q / AR) & 1), abort_flag)))
          break;
        if (lane == 0) DQ_TRACE_POINT(3, q);
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < R; ++j) {
          const int kb = rc.kb + j;
          if (kb < rc.tc.kb1) {
            const uint64_t bdesc =
                make_sw128_kmajor_desc(sbase + ((q % XR) * R + j) * C::kXStageBytes);
            const uint32_t a_tmem =
                tmem_base + static_cast<uint32_t>(C::kACol0 + ((q % AR) * R + j) * 32);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma_ts_pair_elect(d_tmem, a_tmem + 8u * k, bdesc + static_cast<uint64_t>(2 * k),
                                   C::kIdesc, (kb > rc.tc.kb0 || k > 0) ? 1u : 0u);
          }
        }
        tc_commit_pair_elect(done_bar(q % DB));
        if (lane == 0) DQ_TRACE_POINT(4, q);
        const int t_now = rc.t;
        round_advance<R>(rc, args, KB);
        if (!rc.valid || rc.t != t_now) {
          tc_commit_pair_elect(accfull_bar(acc));
          if (++acc == C::kNumAcc) { acc = 0; accphase ^= 1u; }
        }
        __syncwarp();
      }
      if (*abort_flag) {
        __syncwarp();
        tc_commit_pair_elect(drain_bar);
        volatile int never = 0;
        mbar_wait(drain_bar, 0, &never, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // -------------------------------------------------------------- dequant
    const int dw = warp - 4;
    const int quad = warp & 3;
    const int group = dw >> 2;
    const int r = quad * 32 + lane;      // weight row within this CTA's 128
    // The weight tile lands with the TMA 32-byte (NF4) / 64-byte (fp8)
    // swizzle: 16-byte chunk c of row r sits at chunk c ^ (r>>2 & 1) /
    // c ^ (r>>1 & 3), so the eight lanes of each 128-bit load phase hit
    // distinct banks.
    const uint32_t wsw = FMT == kFmtNF4 ? ((r >> 2) & 1) : ((r >> 1) & 3);
    const int r_tile = static_cast<int>(rank) * 128 + r;  // row within the pair's 256
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    float sfp8 = 0.f;
    if constexpr (FMT == kFmtFP8) sfp8 = __bfloat162float(__float2bfloat16_rn(args.fp8_scale));
    constexpr int G = C::kDqGroups;
    auto mine = [&](int qq, int j) { return ((qq * R + j) % G) == group; };
    RoundCursor rc = round_begin(args, KB, pair, npairs);
    float am[R];
#pragma unroll
    for (int j = 0; j < R; ++j)
      am[j] = (FMT == kFmtNF4 && mine(0, j)) ? load_absmax(args, rc, rc.kb + j, r_tile, KB) : 0.f;
    int iw = 0;
    bool ok = true;
    for (int q = 0; rc.valid && ok; ++q) {
      RoundCursor nx = rc;
      round_advance<R>(nx, args, KB);
      float am_next[R];
#pragma unroll
      for (int j = 0; j < R; ++j)
        am_next[j] =
            (FMT == kFmtNF4 && mine(q + 1, j)) ? load_absmax(args, nx, nx.kb + j, r_tile, KB) : 0.f;
      const int present = min(R, rc.tc.kb1 - rc.kb);
      const bool row_ok = (rc.tc.n0 + r_tile) < args.N;
      bool tmem_free = false;
      const uint32_t lead_afull = mapa_shared(afull_bar(q % AR), 0);
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
          if (leader) {
            // The leader vouches for both X halves (they complete on its barrier).
            if (!mbar_wait(xfull_bar((q % XR) * R + j), static_cast<uint32_t>((q / XR) & 1),
                           abort_flag)) {
              ok = false;
              break;
            }
          }
          if (tp) DQ_TRACE_POINT(7 + 5 * group, q * R + j);
          if (!tmem_free) {
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
        if (lane == 0) mbar_arrive_cluster(lead_afull);
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
    const int quad = warp;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    uint8_t* stg = smem + C::kOffEpi + quad * (EC * 32 * 4);
    const uint32_t stg_s = sbase + C::kOffEpi + quad * (EC * 32 * 4);
    int acc = 0;
    uint32_t accphase = 0;
    const bool f32_out = args.splits > 1;
    for (int t = pair; t < args.num_tiles; t += npairs) {
      const TileCoord tc = tile_coord(args, t, KB);
      const int m0 = tc.m0 * BM;
      const int nbase = tc.n0 + static_cast<int>(rank) * 128;
      const int n = nbase + quad * 32 + lane;
      float bias = 0.f;
      if (!f32_out && args.bias != nullptr && n < args.N) bias = __bfloat162float(args.bias[n]);
      if (!mbar_wait_cluster(accfull_bar(acc), accphase, abort_flag)) break;
      tc_fence_after();
      const uint32_t d_addr = tmem_base + lane_addr + static_cast<uint32_t>(acc * C::kAccStride);
      const uint32_t lead_accempty = mapa_shared(accempty_bar(acc), 0);
      const int ncol0 = nbase + quad * 32;
      constexpr int NC = BM / EC;
      uint32_t v[2][32];
      tmem_ld_x32(d_addr, v[0]);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        tmem_wait_ld();
        if (c + 1 < NC) {
          tmem_ld_x32(d_addr + 32u * (c + 1), v[(c + 1) & 1]);
        } else {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(lead_accempty);
        }
        const uint32_t* vc = v[c & 1];
        const int mrow0 = m0 + EC * c;
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
  cluster_sync();  // every cross-CTA arrival and pair MMA is done in both CTAs
  tc_fence_after();
  if (warp == C::kMmaWarp) tmem_dealloc_pair(tmem_base, 512);
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
