// dq_bf16gemm2.cuh -- bf16 x bf16 tcgen05 GEMM on CTA pairs, the second phase
// of the large-token-batch plan: the NF4 / fp8 weight is first dequantized
// once into a bf16 scratch [N, K] (dequant_*_kernel, bit-exact with the
// reference's dequantization), then this kernel computes
// Y^T[n0:n0+256, m0:m0+BM] = W_tile . X_tile^T with M = 256 pair MMAs whose A
// (128 weight rows per CTA) and B (BM/2 token rows per CTA) both come from
// shared memory.  At large M the fused kernels decode every weight tile once
// per token tile; here each weight element is decoded once per call, and with
// no weight in tensor memory both 256-column accumulators fit, so the epilogue
// of one tile overlaps the MMAs of the next.
//
// Warps: 0-7 epilogue (two per TMEM lane quadrant, each draining half of the
// tile's columns), 8 producer (TMA of the A and X halves of each stage), 9 MMA
// (leader CTA; elected lane issues).  Eight epilogue warps keep the drain of
// one tile shorter than the next tile's MMAs even with an activation in the
// epilogue; with four, a GELU-tanh epilogue outlasted them.
//
// With FMT >= 0 (kFmtNF4 / kFmtFP8) the launch also dequantizes the weight:
// four more warps per CTA decode the packed weight into the bf16 scratch
// (the arithmetic of dequant_nf4_kernel / dequant_fp8_kernel, bit-exact with
// the reference's dequantization) one weight group of the grouped tile order
// at a time, every warp counting itself done on dq_ready[g]; the producer
// waits (bounded) for a group's count before its first TMA load of that
// group.  The decode then runs under the MMAs of the earlier groups instead
// of before the GEMM; the first group is made narrow so the first MMAs start
// after a short decode.  The dequantizing warps wait on nothing.
//
// Cross-CTA protocol as in
// dq_gemm2.cuh: both CTAs' TMA loads complete on the leader's full barrier,
// the leader's commits multicast stage-empty and accumulator-full to both
// CTAs, both CTAs' epilogue warps arrive on the leader's accumulator-empty
// barrier.  No TMA load here is a cluster-multicast load.
#pragma once

#include "dq_gemm.cuh"

namespace dq {

template <int BM, int FMT = -1>
struct Bf16PairCfg {
  static_assert(BM % 32 == 0 && BM >= 64 && BM <= 256, "pair tiles need BM in {64..256}, /32");
  static constexpr int kHalfBM = BM / 2;
  static constexpr int kNumAcc = 2;
  static constexpr int kAccStride = BM;
  static constexpr int kAStageBytes = 128 * 128;  // 128 weight rows x 64 bf16, SW128 K-major
  static constexpr int kXStageBytes = kHalfBM * 128;
  static constexpr int kEpiWarps = 8;
  static constexpr int kEpiCols = 32;
  static constexpr int kEpiWarpBytes = kEpiCols * 32 * 2;  // [32 tokens][32 outputs] bf16
  static constexpr int kEpiBytes = kEpiWarps * kEpiWarpBytes;
  static constexpr int kSmemLimit = 227 * 1024;
  static constexpr int kStagesFit =
      (kSmemLimit - kEpiBytes - 2048 - 1024) / (kAStageBytes + kXStageBytes);
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static_assert(kStages >= 3, "need three stages in flight");
  static constexpr int kProducerWarp = kEpiWarps;
  static constexpr int kMmaWarp = kEpiWarps + 1;
  static constexpr int kDqWarp0 = kEpiWarps + 2;
  static constexpr int kDqWarps = FMT >= 0 ? 4 : 0;
  static constexpr int kThreads = (kEpiWarps + 2 + kDqWarps) * 32;
  static_assert(BM % (2 * kEpiCols) == 0, "each epilogue warp drains whole 32-column chunks");
  static constexpr int kNumBars = 2 * kStages + 2 * kNumAcc + 1;
  static constexpr int kOffA = 0;
  static constexpr int kOffX = kStages * kAStageBytes;
  static constexpr int kOffEpi = kOffX + kStages * kXStageBytes;
  static constexpr int kOffBar = kOffEpi + kEpiBytes;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemUsed = kOffMisc + 16 + 1024;
  // Padded so that one CTA fills an SM: the CTA allocates all 512 TMEM columns.
  static constexpr int kSmemBytes = kSmemUsed < 120 * 1024 ? 120 * 1024 : kSmemUsed;
  static_assert(kSmemBytes <= kSmemLimit, "shared memory over the per-CTA limit");
  static constexpr uint32_t kIdesc = make_idesc_bf16(256, BM);
  static constexpr uint32_t kTxBytes = 2 * (kAStageBytes + kXStageBytes);  // both CTAs
};

// Decode weight rows [r0, r1) of the flat packed weight into dq_out: the
// calling thread's share (thread tid of nthr) of the 16-byte chunks.
template <int FMT>
__device__ __forceinline__ void dequant_rows(const GemmArgs& a, int64_t r0, int64_t r1, int tid,
                                             int nthr, uint4* stage) {
  const int64_t K = a.K;
  if constexpr (FMT == kFmtNF4) {
    dequant_nf4_chunks(reinterpret_cast<const uint4*>(a.dq_w), a.absmax,
                       reinterpret_cast<uint4*>(a.dq_out), r0 * K / 32, r1 * K / 32, tid, nthr,
                       stage, a.scale_bf16 != 0);
  } else {
    // K % 16 == 0, so rows hold whole chunks
    dequant_fp8_chunks(reinterpret_cast<const uint4*>(a.dq_w),
                       __bfloat162float(__float2bfloat16_rn(a.fp8_scale)),
                       reinterpret_cast<uint4*>(a.dq_out), r0 * K / 16, r1 * K / 16, tid, nthr,
                       stage);
  }
}

// TP: the column-parallel instantiation -- every output row segment goes to
// every rank's y (args.outs, column offset args.col0, possibly peer memory),
// and after the teardown the CTAs count themselves done and the last raises
// this rank's completion flag on every rank (tp_signal_done).
template <int BM, int FMT = -1, bool TP = false>
__global__ void __launch_bounds__(Bf16PairCfg<BM, FMT>::kThreads, 1)
    bf16_gemm2_kernel(const __grid_constant__ CUtensorMap tmap_x,
                      const __grid_constant__ CUtensorMap tmap_a, const GemmArgs args) {
  using C = Bf16PairCfg<BM, FMT>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::kOffBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (S + s); };
  auto accfull_bar = [&](int a) { return bar0 + 8u * (2 * S + a); };
  auto accempty_bar = [&](int a) { return bar0 + 8u * (2 * S + C::kNumAcc + a); };
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

  if (warp == C::kProducerWarp && lane == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);   // the leader's producer (with both CTAs' bytes)
      mbar_init(empty_bar(s), 1);  // the leader's MMA commit, multicast to both CTAs
    }
    for (int a = 0; a < C::kNumAcc; ++a) {
      mbar_init(accfull_bar(a), 1);
      mbar_init(accempty_bar(a), 2 * C::kEpiWarps);  // every epilogue warp of both CTAs
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmap_x);
    prefetch_tensormap(&tmap_a);
  }
  if (warp == C::kMmaWarp) {
    tmem_alloc_pair(smem_u32(tmem_holder), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before anyone signals across the pair
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == C::kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      int ready_group = -1;  // weight groups up to this one are decoded
      for (int t = pair; t < args.num_tiles && ok; t += npairs) {
        const TileCoord tc = tile_coord(args, t, KB);
        if constexpr (FMT >= 0) {
          if (tc.group > ready_group) {
            const unsigned int target = gridDim.x * C::kDqWarps;
            if (!wait_count_geq(args.dq_ready + tc.group, target, abort_flag)) break;
            fence_proxy_async_global();
            ready_group = tc.group;
          }
        }
        const int m_half = tc.m0 * BM + static_cast<int>(rank) * C::kHalfBM;
        const int n_row = tc.n0 + 128 * static_cast<int>(rank);
        for (int kb = tc.kb0; kb < tc.kb1; ++kb, ++it) {
          const int s = it % S;
          // stage s was last read by the MMAs of k-block it - S
          if (!mbar_wait_cluster(empty_bar(s), static_cast<uint32_t>(((it / S) & 1) ^ 1), abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t lead_full = mapa_shared(full_bar(s), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(s), C::kTxBytes);
          tma_load_2d_pair(sbase + C::kOffA + s * C::kAStageBytes, &tmap_a, lead_full, kb * 64, n_row);
          tma_load_2d_pair(sbase + C::kOffX + s * C::kXStageBytes, &tmap_x, lead_full, kb * 64, m_half);
        }
      }
      // In-flight copies of both CTAs complete on the leader's barriers, which
      // the leader drains (bounded); both CTAs meet at the cluster barrier.
      if (*abort_flag && leader) {
        for (int i = 1; i <= S && i <= it; ++i) {
          volatile int never = 0;
          mbar_wait_cluster(full_bar((it - i) % S), static_cast<uint32_t>(((it - i) / S) & 1), &never,
                            100000000ull);
        }
      }
    }
    __syncwarp();
  } else if (warp == C::kMmaWarp) {
    // -------------------------------------------------------- MMA (leader)
    if (leader) {
      int it = 0, acc = 0;
      uint32_t accphase = 0;
      bool ok = true;
      for (int t = pair; t < args.num_tiles && ok; t += npairs) {
        const TileCoord tc = tile_coord(args, t, KB);
        if (!__all_sync(0xffffffffu, mbar_wait_cluster(accempty_bar(acc), accphase ^ 1u, abort_flag)))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::kAccStride);
        for (int kb = tc.kb0; kb < tc.kb1; ++kb, ++it) {
          const int s = it % S;
          if (!__all_sync(0xffffffffu,
                          mbar_wait_cluster(full_bar(s), static_cast<uint32_t>((it / S) & 1), abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = make_sw128_kmajor_desc(sbase + C::kOffA + s * C::kAStageBytes);
          const uint64_t bdesc = make_sw128_kmajor_desc(sbase + C::kOffX + s * C::kXStageBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma_ss_pair_elect(d_tmem, adesc + static_cast<uint64_t>(2 * k),
                                 bdesc + static_cast<uint64_t>(2 * k), C::kIdesc,
                                 (kb > tc.kb0 || k > 0) ? 1u : 0u);
          tc_commit_pair_elect(empty_bar(s));
          __syncwarp();
        }
        if (!ok) break;
        tc_commit_pair_elect(accfull_bar(acc));
        if (++acc == C::kNumAcc) { acc = 0; accphase ^= 1u; }
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
  } else if (FMT >= 0 && warp >= C::kDqWarp0) {
    // ------------------------------------------------------ weight decode
    if constexpr (FMT >= 0) {
      const int nthr = static_cast<int>(gridDim.x) * C::kDqWarps * 32;
      const int tid = static_cast<int>(blockIdx.x) * C::kDqWarps * 32 + threadIdx.x - C::kDqWarp0 * 32;
      const int g0 = first_group_width(args.group_n, args.group0_n, args.num_n_tiles);
      int nb = 0;
      for (int g = 0; nb < args.num_n_tiles; ++g) {
        const int gn = g == 0 ? g0 : min(args.group_n, args.num_n_tiles - nb);
        const int64_t r0 = static_cast<int64_t>(nb) * 256;
        const int64_t r1 = min(static_cast<int64_t>(args.N), static_cast<int64_t>(nb + gn) * 256);
        // stores go out directly: staging them through shared memory (as the
        // standalone decode does) measured no faster beside the GEMM
        dequant_rows<FMT>(args, r0, r1, tid, nthr, nullptr);
        // every lane's stores, then the warp's count (release)
        fence_proxy_async_global();
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(args.dq_ready + g, 1u);
        nb += gn;
      }
    }
  } else if (warp < C::kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    constexpr int EC = C::kEpiCols;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int half = warp >> 2;  // which half of the tile's columns it drains
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    uint8_t* stg = smem + C::kOffEpi + warp * C::kEpiWarpBytes;
    const uint32_t stg_s = sbase + C::kOffEpi + warp * C::kEpiWarpBytes;
    int acc = 0;
    uint32_t accphase = 0;
    for (int t = pair; t < args.num_tiles; t += npairs) {
      const TileCoord tc = tile_coord(args, t, KB);
      const int m0 = tc.m0 * BM;
      const int nbase = tc.n0 + static_cast<int>(rank) * 128;
      const int n = nbase + quad * 32 + lane;
      float bias = 0.f;
      if (args.bias != nullptr && n < args.N) bias = __bfloat162float(args.bias[n]);
      if (!mbar_wait_cluster(accfull_bar(acc), accphase, abort_flag)) break;
      tc_fence_after();
      const uint32_t d_addr = tmem_base + lane_addr + static_cast<uint32_t>(acc * C::kAccStride);
      const uint32_t lead_accempty = mapa_shared(accempty_bar(acc), 0);
      const int ncol0 = nbase + quad * 32;
      constexpr int NC = BM / EC / 2;  // chunks per warp
      const int c0 = half * NC;
      uint32_t v[2][32];
      tmem_ld_x32(d_addr + 32u * c0, v[0]);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        tmem_wait_ld();
        if (c + 1 < NC) {
          tmem_ld_x32(d_addr + 32u * (c0 + c + 1), v[(c + 1) & 1]);
        } else {
          // the whole accumulator has been read: hand it back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(lead_accempty);
        }
        const uint32_t* vc = v[c & 1];
        const int mrow0 = m0 + EC * (c0 + c);
        // stage [EC tokens][32 outputs] bf16, then write 64-byte row segments
        __nv_bfloat16* sb = reinterpret_cast<__nv_bfloat16*>(stg);
        if (act_is_gated(args.act)) {
          gated_chunk_store<EC>(vc, bias, args.act, stg_s, sb,
                                reinterpret_cast<__nv_bfloat16*>(args.outs[0]), args.ldy, args.M,
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
                if (TP && args.out_mc != nullptr) {
                  multimem_st16(reinterpret_cast<__nv_bfloat16*>(args.out_mc) + off, v16);
                } else {
#pragma unroll
                  for (int d = 0; d < (TP ? kMaxRanks : 1); ++d)
                    if (d < args.n_out)
                      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(args.outs[d]) + off) = v16;
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
      }
      if (++acc == C::kNumAcc) { acc = 0; accphase ^= 1u; }
    }
    // column-parallel: this thread's peer stores are visible system-wide
    // before its CTA counts itself done
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
}

}  // namespace dq
