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
//   warps 0-3            epilogue (warp w owns TMEM lanes 32w..32w+31)
//   warps 4..4+DQ-1      dequant  (warp w writes lanes 32(w%4).., column half (w-4)/4)
//   warp 4+DQ            producer (TMA for X and packed W; cp.async for absmax)
//   warp 5+DQ            MMA issuer (one thread) and TMEM allocator
// Every mbarrier wait is bounded (dq_ptx.cuh); on expiry the CTA unwinds,
// drains its in-flight copies and MMAs (bounded), frees TMEM and records
// DQ_ERR_TIMEOUT in g_dq_error.
#pragma once

#include <cuda_bf16.h>

#include "dq_codec.cuh"
#include "dq_ptx.cuh"

namespace dq {

enum : int { kFmtNF4 = 0, kFmtFP8 = 1 };
enum : unsigned int { kErrTimeout = 5u };

// Per-device kernel error word (bit kErrTimeout: a bounded wait expired).
// The library is a single translation unit, so it is defined here.
__device__ unsigned int g_dq_error = 0;

struct GemmArgs {
  const float* absmax;        // NF4: [N, K/64] f32 block scales
  const __nv_bfloat16* bias;  // [N] or nullptr
  void* out;                  // bf16 Y [M, N] (splits == 1) or f32 partials [splits, M, N]
  int M, N, K;
  int num_n_tiles, num_tiles;
  int splits, kb_per_split;
  float fp8_scale;            // fp8: per-tensor scale (rounded to bf16 in-kernel)
  int vec_ok;                 // 16-byte vector stores are aligned for `out`
};

template <int FMT, int BM>
struct GemmCfg {
  static_assert(BM % 16 == 0 && BM >= 16 && BM <= 256, "BM must be a multiple of 16 in [16,256]");
  static constexpr int kBN = 128;                               // weight rows per tile (MMA M)
  static constexpr int kBK = 64;                                // K per k-block
  static constexpr int kWBytes = FMT == kFmtNF4 ? 32 : 64;      // packed bytes per row per k-block
  static constexpr int kNumAcc = BM <= 192 ? 2 : 1;             // accumulator buffers
  static constexpr int kAccStride = BM < 32 ? 32 : BM;          // TMEM columns per accumulator
  static constexpr int kACol0 = ((kNumAcc * kAccStride + 31) / 32) * 32;
  static constexpr int kAStagesFit = (512 - kACol0) / 32;
  static constexpr int kAStages = kAStagesFit > 8 ? 8 : kAStagesFit;
  static_assert(kAStages >= 2, "not enough TMEM for the A ring");
  static constexpr int kDqWarps = BM <= 64 ? 8 : 4;
  static constexpr int kColsPerDqThread = 32 / (kDqWarps / 4);  // TMEM columns per k-block
  static constexpr int kBytesPerDqThread = kWBytes / (kDqWarps / 4);
  static constexpr int kProducerWarp = 4 + kDqWarps;
  static constexpr int kMmaWarp = 5 + kDqWarps;
  static constexpr int kThreads = (6 + kDqWarps) * 32;
  static constexpr int kXStageBytes = BM * 128;
  static constexpr int kWStageBytes = kBN * kWBytes;
  static constexpr int kAmStageBytes = FMT == kFmtNF4 ? kBN * 4 : 0;
  static constexpr int kStageBytes = kXStageBytes + kWStageBytes + kAmStageBytes;
  static constexpr int kEpiBytes = 4 * 16 * 32 * 4;             // per-warp 16x32 f32 staging
  static constexpr int kSmemBudget = 200 * 1024;
  static constexpr int kStagesFit = (kSmemBudget - kEpiBytes - 1024) / kStageBytes;
  static constexpr int kStages = kStagesFit > 16 ? 16 : kStagesFit;
  static_assert(kStages >= 2, "shared memory too small for two stages");
  static constexpr int kNumBars = 2 * kStages + 2 * kAStages + 2 * kNumAcc + 1;
  static constexpr int kOffW = kStages * kXStageBytes;
  static constexpr int kOffAm = kOffW + kStages * kWStageBytes;
  static constexpr int kOffEpi = kOffAm + kStages * kAmStageBytes;
  static constexpr int kOffBar = kOffEpi + kEpiBytes;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  // Padded so that one CTA fills an SM: the CTA allocates all 512 TMEM columns.
  static constexpr int kSmemUsed = kOffMisc + 16 + 1024;
  static constexpr int kSmemBytes = kSmemUsed < 120 * 1024 ? 120 * 1024 : kSmemUsed;
  static constexpr uint32_t kIdesc = make_idesc_bf16(kBN, BM);
  static constexpr uint32_t kTxBytes = kXStageBytes + kWStageBytes;
};

struct TileCoord {
  int m0, n0, kb0, kb1, split;
};

__device__ __forceinline__ TileCoord tile_coord(const GemmArgs& a, int t, int KB) {
  TileCoord c;
  c.split = t % a.splits;
  const int mn = t / a.splits;
  c.n0 = (mn % a.num_n_tiles) * 128;
  c.m0 = (mn / a.num_n_tiles);
  c.kb0 = c.split * a.kb_per_split;
  c.kb1 = min(KB, c.kb0 + a.kb_per_split);
  return c;
}

template <int FMT, int BM>
__global__ void __launch_bounds__(GemmCfg<FMT, BM>::kThreads, 1)
    dq_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                   const __grid_constant__ CUtensorMap tmap_w, const GemmArgs args) {
  using C = GemmCfg<FMT, BM>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::kOffBar;
  // barrier layout: full[S], empty[S], a_full[A], a_empty[A], acc_full[ACC], acc_empty[ACC], drain
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::kStages + s); };
  auto afull_bar = [&](int s) { return bar0 + 8u * (2 * C::kStages + s); };
  auto aempty_bar = [&](int s) { return bar0 + 8u * (2 * C::kStages + C::kAStages + s); };
  auto accfull_bar = [&](int s) { return bar0 + 8u * (2 * C::kStages + 2 * C::kAStages + s); };
  auto accempty_bar = [&](int s) {
    return bar0 + 8u * (2 * C::kStages + 2 * C::kAStages + C::kNumAcc + s);
  };
  const uint32_t drain_bar = bar0 + 8u * (C::kNumBars - 1);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KB = (args.K + 63) / 64;  // fp8 allows a ragged last k-block (TMA zero-fills it)

  if (warp == C::kProducerWarp && lane == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1 + C::kDqWarps);
    }
    for (int s = 0; s < C::kAStages; ++s) {
      mbar_init(afull_bar(s), C::kDqWarps);
      mbar_init(aempty_bar(s), 1);
    }
    for (int s = 0; s < C::kNumAcc; ++s) {
      mbar_init(accfull_bar(s), 1);
      mbar_init(accempty_bar(s), 4);
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == C::kProducerWarp) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < args.num_tiles && ok; t += gridDim.x) {
      const TileCoord tc = tile_coord(args, t, KB);
      const int m0 = tc.m0 * BM;
      for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
        if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) { ok = false; break; }
        const uint32_t xs = sbase + stage * C::kXStageBytes;
        const uint32_t ws = sbase + C::kOffW + stage * C::kWStageBytes;
        if constexpr (FMT == kFmtNF4) {
          const uint32_t ams = sbase + C::kOffAm + stage * C::kAmStageBytes;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = lane + 32 * i;
            const int n = tc.n0 + r;
            if (n < args.N) cp_async_4(ams + 4u * r, args.absmax + static_cast<size_t>(n) * KB + kb);
          }
          cp_async_mbar_arrive(full_bar(stage));
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_expect_tx(full_bar(stage), C::kTxBytes);
          tma_load_2d(xs, &tmap_x, full_bar(stage), kb * 64, m0);
          tma_load_2d(ws, &tmap_w, full_bar(stage), kb * C::kWBytes, tc.n0);
        }
        ++issued;
        if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
      }
    }
    if (*abort_flag) {
      // Let the copies already issued land before the CTA's shared memory is
      // released (bounded: a copy that never lands is abandoned after 100 ms).
      int st = stage;
      uint32_t ph = phase;
      const int pending = issued < C::kStages ? issued : C::kStages;
      for (int i = 0; i < pending; ++i) {
        if (--st < 0) { st = C::kStages - 1; ph ^= 1u; }
        volatile int never = 0;
        mbar_wait(full_bar(st), ph, &never, 100000000ull);
      }
    }
  } else if (warp == C::kMmaWarp) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      int stage = 0, astage = 0, acc = 0;
      uint32_t phase = 0, aphase = 0, accphase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < args.num_tiles && ok; t += gridDim.x) {
        const TileCoord tc = tile_coord(args, t, KB);
        if (!mbar_wait(accempty_bar(acc), accphase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::kAccStride);
        for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag)) { ok = false; break; }
          if (!mbar_wait(afull_bar(astage), aphase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t bdesc = make_sw128_kmajor_desc(sbase + stage * C::kXStageBytes);
          const uint32_t a_tmem = tmem_base + static_cast<uint32_t>(C::kACol0 + astage * 32);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // K step j: 16 bf16 = 8 TMEM columns of A, 32 bytes along the swizzled B rows.
            tc_mma_ts(d_tmem, a_tmem + 8u * j, bdesc + static_cast<uint64_t>(2 * j), C::kIdesc,
                      (kb > tc.kb0 || j > 0) ? 1u : 0u);
          }
          tc_commit(empty_bar(stage));
          tc_commit(aempty_bar(astage));
          if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
          if (++astage == C::kAStages) { astage = 0; aphase ^= 1u; }
        }
        if (!ok) break;
        tc_commit(accfull_bar(acc));
        if (++acc == C::kNumAcc) { acc = 0; accphase ^= 1u; }
      }
      if (*abort_flag) {
        // Wait (bounded) until every MMA this thread issued has retired.
        tc_commit(drain_bar);
        volatile int never = 0;
        mbar_wait(drain_bar, 0, &never, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // -------------------------------------------------------------- dequant
    const int dw = warp - 4;
    const int quad = warp & 3;           // TMEM lane quadrant this warp may access
    const int half = dw >> 2;            // which column slice of the k-block
    const int r = quad * 32 + lane;      // weight row within the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    float sfp8 = 0.f;
    if constexpr (FMT == kFmtFP8) sfp8 = __bfloat162float(__float2bfloat16_rn(args.fp8_scale));
    int stage = 0, astage = 0;
    uint32_t phase = 0, aphase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < args.num_tiles && ok; t += gridDim.x) {
      const TileCoord tc = tile_coord(args, t, KB);
      const bool row_ok = (tc.n0 + r) < args.N;
      for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
        if (!mbar_wait(full_bar(stage), phase, abort_flag)) { ok = false; break; }
        const uint8_t* wrow = smem + C::kOffW + stage * C::kWStageBytes + r * C::kWBytes +
                              half * C::kBytesPerDqThread;
        uint4 pk[C::kBytesPerDqThread / 16];
#pragma unroll
        for (int i = 0; i < C::kBytesPerDqThread / 16; ++i)
          pk[i] = *reinterpret_cast<const uint4*>(wrow + 16 * i);
        float am = 0.f;
        if constexpr (FMT == kFmtNF4)
          am = *reinterpret_cast<const float*>(smem + C::kOffAm + stage * C::kAmStageBytes + 4 * r);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(stage));
        if (++stage == C::kStages) { stage = 0; phase ^= 1u; }

        uint32_t out[32];
        const uint32_t* pw = reinterpret_cast<const uint32_t*>(pk);
        if constexpr (FMT == kFmtNF4) {
          const uint32_t sc2 = nf4_scale2(am);
#pragma unroll
          for (int i = 0; i < C::kBytesPerDqThread / 4; ++i) nf4_decode_word(pw[i], sc2, out + 4 * i);
        } else {
#pragma unroll
          for (int i = 0; i < C::kBytesPerDqThread / 4; ++i) fp8_decode_word(pw[i], sfp8, out + 2 * i);
        }
        if (!row_ok) {
#pragma unroll
          for (int i = 0; i < C::kColsPerDqThread; ++i) out[i] = 0u;
        }
        if (!mbar_wait(aempty_bar(astage), aphase ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = tmem_base + lane_addr +
                                static_cast<uint32_t>(C::kACol0 + astage * 32 + half * C::kColsPerDqThread);
#pragma unroll
        for (int c = 0; c < C::kColsPerDqThread / 16; ++c)
          tmem_st_x16(a_addr + 16u * c, *reinterpret_cast<const uint32_t(*)[16]>(out + 16 * c));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(afull_bar(astage));
        if (++astage == C::kAStages) { astage = 0; aphase ^= 1u; }
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int quad = warp;  // warps 0..3
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    uint8_t* stg = smem + C::kOffEpi + quad * (16 * 32 * 4);
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
#pragma unroll 1
      for (int c = 0; c < BM / 16; ++c) {
        uint32_t v[16];
        tmem_ld_x16(d_addr + 16u * c, v);
        tmem_wait_ld();
        if (c == BM / 16 - 1) {
          // The whole accumulator has been read: hand it back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(accempty_bar(acc));
        }
        const int mrow0 = m0 + 16 * c;  // token of staging row 0
        const int ncol0 = tc.n0 + quad * 32;
        if (!f32_out) {
          // stage [16 tokens][32 outputs] bf16, then write 64-byte row segments
          __nv_bfloat16* sb = reinterpret_cast<__nv_bfloat16*>(stg);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            sb[j * 32 + lane] = __float2bfloat16_rn(__uint_as_float(v[j]) + bias);
          __syncwarp();
          __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(args.out);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int row = (lane >> 2) + 8 * i;
            const int col = (lane & 3) * 8;
            const int m = mrow0 + row;
            const int nc = ncol0 + col;
            if (m < args.M) {
              __nv_bfloat16* dst = y + static_cast<size_t>(m) * args.N + nc;
              const __nv_bfloat16* src = sb + row * 32 + col;
              if (args.vec_ok && nc + 8 <= args.N) {
                *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
              } else {
                for (int e = 0; e < 8; ++e)
                  if (nc + e < args.N) dst[e] = src[e];
              }
            }
          }
          __syncwarp();
        } else {
          // split-K partial: stage [16][32] f32, write 128-byte row segments
          float* sf = reinterpret_cast<float*>(stg);
#pragma unroll
          for (int j = 0; j < 16; ++j) sf[j * 32 + lane] = __uint_as_float(v[j]);
          __syncwarp();
          float* part = reinterpret_cast<float*>(args.out) +
                        static_cast<size_t>(tc.split) * args.M * args.N;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int row = (lane >> 3) + 4 * i;
            const int col = (lane & 7) * 4;
            const int m = mrow0 + row;
            const int nc = ncol0 + col;
            if (m < args.M) {
              float* dst = part + static_cast<size_t>(m) * args.N + nc;
              const float* src = sf + row * 32 + col;
              if (args.vec_ok && nc + 4 <= args.N) {
                *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(src);
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
  }

  // ------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == C::kMmaWarp) tmem_dealloc(tmem_base, 512);
  if (threadIdx.x == 0 && *abort_flag) atomicOr(&g_dq_error, 1u << kErrTimeout);
}

}  // namespace dq
