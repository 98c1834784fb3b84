// dq_smallm2.cuh -- the NF4 / fp8 linear for decode-sized token counts
// (M <= 16) with the weight streamed through a TMA ring in shared memory.
//
// The bound is HBM: every weight byte is read once and the tensor-core work is
// tiny (3072 -> 18432 NF4 at M = 1: 31.9 MB, ~4.9 us at the measured copy
// bandwidth).  What decides the time is how many weight bytes are in flight
// per SM.  smallm_kernel (dq_smallm.cuh) loads the weights straight into
// registers, so its bytes in flight are bounded by registers and by each
// warp's load -> decode -> MMA sequence.  Here one producer thread per CTA
// keeps a ring of stages full with 2-D TMA tile copies (one weight tile of
// 16 * R16 rows x 128 bytes per box, 128-byte swizzle, plus the rows' NF4
// block scales), independent of the decode: with two CTAs per SM (eight
// stages each) about 140 KB of NF4 weight are in flight per SM, with three
// (four stages each) about 100 KB.  The planner picks the row groups per CTA
// (R16) and the CTAs per SM (CPS) that fill the most resident slots in one
// wave: the consumers' decode, not the weight stream, sets the pace once the
// ring is deep enough, so filling every SM's warp slots matters most.
//
// Work split.  A stage holds the weight bytes of eight 16-row x 128-k work
// items: R16 row groups x (8 / R16) k-groups (NF4: 256 k per box row, fp8:
// 128 k).  Consumer warp w always takes row group w % R16 and the k-group
// w / R16 of every stage, so each warp accumulates one 16-row block over its
// share of K.  Inside an item a thread decodes its two 32-weight runs (rows
// g4 and g4 + 8, k 32*tig..32*tig+31 of the k-group) exactly as smallm_kernel
// does -- the per-lane shared-memory byte LUT times the bf16 block scale for
// NF4, the exact e4m3 -> bf16 scaling for fp8 -- into the A fragments of
// warp-level m16n8k16 bf16 MMAs with f32 accumulation, under the same k
// permutation (dq_smallm.cuh), alternating two accumulator sets so that
// consecutive MMAs do not wait on each other.  A warp releases a stage as
// soon as its bytes are in registers.  Partial sums of the warps sharing a
// row group meet in shared memory, where bias and activation are added.
//
// Launch overlap: the launch carries the programmatic stream serialization
// attribute, so when the kernel before it on the stream is another decode-
// sized linear (which releases its dependents at its start), this grid is
// scheduled while that one still runs: barrier set-up, the LUT fill and the
// first stages of the weight stream overlap its tail.  The consumers wait
// for the preceding grid to complete (griddepcontrol.wait) before the first
// read of x, so only the weight and its scales are read early: they must not
// be outputs of the immediately preceding decode-sized linear call.
//
// Two token tiles (9-16 tokens): x is staged with the weights -- per stage,
// 16-row x 64-k TMA boxes of x (128-byte swizzle, rows past M zero-filled),
// read by the consumers from shared memory instead of through L1 -- in 64-row
// CTAs, two per SM, four stages.  The producer then waits for the preceding
// grid before its first copy (x may be that grid's output).
//
// Requirements: at most 16 tokens, K % 128 == 0 (fp8) / K % 256 == 0 with
// 16-byte aligned f32 block scales (NF4: the scale tile is a TMA copy; a
// stage's rows of scales must be whole 16-byte units).  Loading the scales
// with plain per-thread loads instead measured 19% slower (3072 -> 18432,
// M = 1: 13.7 against 11.5 us): their latency lands in the decode.  Every
// wait is bounded (2 s); on expiry the CTA drains its copies, writes nothing
// and records DQ_ERR_TIMEOUT.  One launch, no workspace.
#pragma once

#include "dq_codec.cuh"
#include "dq_ptx.cuh"
#include "dq_smallm.cuh"

namespace dq {

template <int FMT, int MT, int R16, int CPS>
struct SmallM2Cfg {
  static constexpr int kConsumerWarps = 8;
  static constexpr int kThreads = (kConsumerWarps + 1) * 32;  // + the producer warp
  static constexpr int kRows = 16 * R16;
  static constexpr int kKgPerBox = FMT == kFmtNF4 ? 2 : 1;  // 128-k groups per 128-byte row
  static constexpr int kKgPerStage = 8 / R16;                // one work item per consumer warp
  static constexpr int kBoxes = kKgPerStage / kKgPerBox;     // weight boxes per stage
  static constexpr int kBoxBytes = 128 * kRows;
  static constexpr int kWStageBytes = kBoxes * kBoxBytes;    // 8 KB NF4, 16 KB fp8
  static constexpr int kAbsPerRow = FMT == kFmtNF4 ? 2 * kKgPerStage : 0;  // f32 block scales
  static constexpr int kAStageBytes = kAbsPerRow * 4 * kRows;              // 1 KB NF4
  // Two token tiles (up to 16 tokens): x travels with the stage, as 16-row x
  // 64-k boxes (128-byte swizzle, rows past M zero-filled), two per k-group
  static constexpr bool kXStaged = MT == 2;
  static constexpr int kXBoxBytes = 16 * 128;
  static constexpr int kXStageBytes = kXStaged ? 2 * kKgPerStage * kXBoxBytes : 0;
  static constexpr int kOffXInStage = kWStageBytes + kAStageBytes;
  static constexpr int kStageBytes = kWStageBytes + kAStageBytes + kXStageBytes;
  // CPS resident CTAs per SM: CPS x (smem + 1 KB reserved) <= 228 KB
  static constexpr int kStages = kXStaged ? 4
                                 : CPS == 2 ? (FMT == kFmtNF4 ? 8 : 6)
                                            : 4;
  static constexpr int kLutBytes = FMT == kFmtNF4 ? kNf4LutBytes : 0;
  static constexpr int kRedBytes = kConsumerWarps * MT * 128 * 4;
  // offsets from the 1024-byte aligned base (128-byte swizzled boxes)
  static constexpr int kOffRing = 0;
  static constexpr int kOffLut = kStages * kStageBytes;
  static constexpr int kOffRed = kOffLut + kLutBytes;
  static constexpr int kOffBar = kOffRed + kRedBytes;
  static constexpr int kOffFlag = kOffBar + 2 * kStages * 8;
  static constexpr int kSmemBytes = kOffFlag + 16 + 1024;  // + alignment slack
  static_assert(kBoxes >= 1 && kBoxes * kKgPerBox == kKgPerStage, "stage shape");
  static_assert(kStageBytes % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
  static_assert(kOffXInStage % 1024 == 0, "x boxes keep the 1024-byte swizzle alignment");
  static_assert(!kXStaged || (R16 == 4 && CPS == 2), "two token tiles: 64-row CTAs, two per SM");
  static_assert(CPS * (kSmemBytes + 1024) <= 228 * 1024, "CPS CTAs per SM");
};

template <int FMT, int MT, int R16, int CPS>
__global__ void __launch_bounds__(SmallM2Cfg<FMT, MT, R16, CPS>::kThreads, CPS)
    smallm2_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_x, const __nv_bfloat16* __restrict__ x,
                   float fp8_scale,
                   const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ y, int M,
                   int N, int K, int act, int64_t ldy) {
  using C = SmallM2Cfg<FMT, MT, R16, CPS>;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KG = K / 128;
  const int S = (KG + C::kKgPerStage - 1) / C::kKgPerStage;
  const int row0 = blockIdx.x * C::kRows;
  const uint32_t bar0 = sbase + C::kOffBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::kStages + s); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffFlag);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), C::kConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  // Programmatic dependent launch: a following kernel launched with the
  // programmatic-serialization attribute may start its prologue (and its own
  // weight stream) now; it reads x and writes y only after this grid is done.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == C::kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&tmap_w);
      if constexpr (FMT == kFmtNF4) prefetch_tensormap(&tmap_a);
      if constexpr (C::kXStaged) {
        prefetch_tensormap(&tmap_x);
        // x may be the output of the kernel before this one on the stream
        asm volatile("griddepcontrol.wait;" ::: "memory");
      }
      int s = 0;
      for (; s < S; ++s) {
        const int slot = s % C::kStages;
        if (!mbar_wait(empty_bar(slot), static_cast<uint32_t>(((s / C::kStages) & 1) ^ 1), abort_flag))
          break;
        // boxes reaching past K or N are zero-filled and still count in full
        mbar_arrive_expect_tx(full_bar(slot), C::kStageBytes);
        const uint32_t dst = sbase + C::kOffRing + slot * C::kStageBytes;
#pragma unroll
        for (int b = 0; b < C::kBoxes; ++b)
          tma_load_2d(dst + b * C::kBoxBytes, &tmap_w, full_bar(slot), (s * C::kBoxes + b) * 128, row0);
        if constexpr (FMT == kFmtNF4)
          tma_load_2d(dst + C::kWStageBytes, &tmap_a, full_bar(slot), s * C::kAbsPerRow, row0);
        if constexpr (C::kXStaged) {
#pragma unroll
          for (int b = 0; b < 2 * C::kKgPerStage; ++b)
            tma_load_2d(dst + C::kOffXInStage + b * C::kXBoxBytes, &tmap_x, full_bar(slot),
                        (s * 2 * C::kKgPerStage + b) * 64, 0);
        }
      }
      if (*abort_flag) {
        // let issued copies land before shared memory is released (bounded)
        for (int i = 1; i <= C::kStages && i <= s; ++i) {
          volatile int never = 0;
          mbar_wait(full_bar((s - i) % C::kStages), static_cast<uint32_t>(((s - i) / C::kStages) & 1),
                    &never, 100000000ull);
        }
      }
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- consumers
    if constexpr (FMT == kFmtNF4) {
      uint32_t* lut = reinterpret_cast<uint32_t*>(smem + C::kOffLut);
      for (int i = threadIdx.x; i < 256 * 32; i += 32 * C::kConsumerWarps) {
        const int b = i >> 5;
        lut[i] = static_cast<uint32_t>(c_nf4_level_bits[b >> 4]) |
                 (static_cast<uint32_t>(c_nf4_level_bits[b & 15]) << 16);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * C::kConsumerWarps) : "memory");
    }
    // x (and y) may belong to the kernel before this one on the stream: wait
    // for it to complete (a no-op unless launched as a programmatic dependent)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t lut_lane = sbase + C::kOffLut + 4u * lane;
    const float fp8_s = __bfloat162float(__float2bfloat16_rn(fp8_scale));
    const int rg = warp % R16;   // row group of this warp
    const int kgl = warp / R16;  // its k-group within every stage
    const int bx = kgl / C::kKgPerBox, kk = kgl % C::kKgPerBox;
    const int g4 = lane >> 2, tig = lane & 3;
    const int r_lo = 16 * rg + g4;  // rows of the CTA tile: r_lo and r_lo + 8
    // 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r % 8)
    const uint32_t row_off = static_cast<uint32_t>(r_lo) * 128u;

    float acc[2][MT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[a][mt][i] = 0.f;

    for (int s = 0; s < S; ++s) {
      const int slot = s % C::kStages;
      const int g = s * C::kKgPerStage + kgl;  // global k-group
      const bool present = g < KG;
      const int64_t k0 = 128ll * g + 32 * tig;
      // x of this thread's tokens at k0 .. k0 + 31 (bf16 pairs xw[mt][0..15]):
      // independent of the stage, so its latency overlaps the stage wait
      uint32_t xw[MT][16];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int t = 8 * mt + g4;
        if constexpr (C::kXStaged) break;  // read from the stage below
        if (present && t < M) {
          const uint4* src = reinterpret_cast<const uint4*>(x + t * static_cast<int64_t>(K) + k0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 v = __ldg(src + q);
            xw[mt][4 * q] = v.x; xw[mt][4 * q + 1] = v.y; xw[mt][4 * q + 2] = v.z; xw[mt][4 * q + 3] = v.w;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) xw[mt][e] = 0u;
        }
      }
      if (!mbar_wait(full_bar(slot), static_cast<uint32_t>((s / C::kStages) & 1), abort_flag)) break;
      const uint32_t stage = sbase + C::kOffRing + slot * C::kStageBytes;
      const uint32_t box = stage + bx * C::kBoxBytes;
      if constexpr (C::kXStaged) {
        // this thread's 32-k run of x (k 128 g + 32 tig ..) for tokens g4 and
        // 8 + g4: box 2 kgl + tig / 2, bytes 64 (tig % 2) .. of the row, in
        // 16-byte chunks c at c ^ (row % 8); rows past M arrived as zeros
        const uint32_t xbox = stage + C::kOffXInStage + (2 * kgl + (tig >> 1)) * C::kXBoxBytes;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int t = 8 * mt + g4;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t ch = static_cast<uint32_t>((4 * (tig & 1) + q) ^ (t & 7)) * 16u;
            const uint4 v = present ? lds128(xbox + static_cast<uint32_t>(t) * 128u + ch)
                                    : make_uint4(0u, 0u, 0u, 0u);
            xw[mt][4 * q] = v.x; xw[mt][4 * q + 1] = v.y; xw[mt][4 * q + 2] = v.z; xw[mt][4 * q + 3] = v.w;
          }
        }
      }
      uint32_t plo[FMT == kFmtNF4 ? 4 : 8], phi[FMT == kFmtNF4 ? 4 : 8];
      uint32_t sc_lo = 0, sc_hi = 0;
      if (present) {
        if constexpr (FMT == kFmtNF4) {
          const uint32_t ch = static_cast<uint32_t>((4 * kk + tig) ^ g4) * 16u;
          const uint4 a = lds128(box + row_off + ch);
          const uint4 b = lds128(box + row_off + 1024u + ch);  // row + 8: same swizzle phase
          plo[0] = a.x; plo[1] = a.y; plo[2] = a.z; plo[3] = a.w;
          phi[0] = b.x; phi[1] = b.y; phi[2] = b.z; phi[3] = b.w;
          const uint32_t sc = stage + C::kWStageBytes +
                              4u * static_cast<uint32_t>(r_lo * C::kAbsPerRow + 2 * kgl + (tig >> 1));
          sc_lo = nf4_scale2(__uint_as_float(lds32(sc)));
          sc_hi = nf4_scale2(__uint_as_float(lds32(sc + 4u * 8u * C::kAbsPerRow)));
        } else {
          const uint32_t c0 = static_cast<uint32_t>((2 * tig) ^ g4) * 16u;
          const uint32_t c1 = static_cast<uint32_t>((2 * tig + 1) ^ g4) * 16u;
          const uint4 a0 = lds128(box + row_off + c0), a1 = lds128(box + row_off + c1);
          const uint4 b0 = lds128(box + row_off + 1024u + c0), b1 = lds128(box + row_off + 1024u + c1);
          plo[0] = a0.x; plo[1] = a0.y; plo[2] = a0.z; plo[3] = a0.w;
          plo[4] = a1.x; plo[5] = a1.y; plo[6] = a1.z; plo[7] = a1.w;
          phi[0] = b0.x; phi[1] = b0.y; phi[2] = b0.z; phi[3] = b0.w;
          phi[4] = b1.x; phi[5] = b1.y; phi[6] = b1.z; phi[7] = b1.w;
        }
      }
      // the stage's bytes are in registers: hand it back to the producer
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(slot));
      if (!present) continue;

#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t w0[8], w1[8];
        if constexpr (FMT == kFmtNF4) {
          nf4_decode_word_lut(plo[2 * h], lut_lane, sc_lo, w0);
          nf4_decode_word_lut(plo[2 * h + 1], lut_lane, sc_lo, w0 + 4);
          nf4_decode_word_lut(phi[2 * h], lut_lane, sc_hi, w1);
          nf4_decode_word_lut(phi[2 * h + 1], lut_lane, sc_hi, w1 + 4);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            fp8_decode_word(plo[4 * h + q], fp8_s, w0 + 2 * q);
            fp8_decode_word(phi[4 * h + q], fp8_s, w1 + 2 * q);
          }
        }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            mma_16816_bf16(acc[jj & 1][mt], w0[2 * jj], w1[2 * jj], w0[2 * jj + 1], w1[2 * jj + 1],
                           xw[mt][8 * h + 2 * jj], xw[mt][8 * h + 2 * jj + 1]);
      }
    }

    // partial sums -> shared memory, fragment element (token, row)
    float* red = reinterpret_cast<float*>(smem + C::kOffRed);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      float* dst = red + (warp * MT + mt) * 128;
      dst[(2 * tig) * 16 + g4] = acc[0][mt][0] + acc[1][mt][0];
      dst[(2 * tig + 1) * 16 + g4] = acc[0][mt][1] + acc[1][mt][1];
      dst[(2 * tig) * 16 + g4 + 8] = acc[0][mt][2] + acc[1][mt][2];
      dst[(2 * tig + 1) * 16 + g4 + 8] = acc[0][mt][3] + acc[1][mt][3];
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * C::kConsumerWarps) : "memory");
    if (!*abort_flag && act_is_gated(act)) {
      // gated row order: row groups 2p (gate) and 2p + 1 (up) of this CTA
      // give output features row0 / 2 + 16 p .. +15 (R16 is even here)
      for (int o = threadIdx.x; o < (R16 / 2) * MT * 128; o += 32 * C::kConsumerWarps) {
        const int row = o & 15;
        const int tok = (o >> 4) & 7;
        const int pm = o >> 7;  // pair * MT + mt
        const int pr = pm / MT, mt = pm - pr * MT;
        float g = 0.f, u = 0.f;
#pragma unroll
        for (int q = 0; q < C::kKgPerStage; ++q) {
          g += red[((q * R16 + 2 * pr) * MT + mt) * 128 + tok * 16 + row];
          u += red[((q * R16 + 2 * pr + 1) * MT + mt) * 128 + tok * 16 + row];
        }
        const int64_t ng = row0 + 32 * pr + row;  // gate row; its up row is ng + 16
        const int m = 8 * mt + tok;
        if (ng < N && m < M) {
          if (bias != nullptr) {
            g += __bfloat162float(bias[ng]);
            u += __bfloat162float(bias[ng + 16]);
          }
          y[static_cast<int64_t>(m) * ldy + row0 / 2 + 16 * pr + row] = __float2bfloat16_rn(gated_value(g, u, act));
        }
      }
    } else if (!*abort_flag) {
      // output o = (rg * MT + mt) * 128 + token * 16 + row: consecutive threads
      // store consecutive output features of one token
      for (int o = threadIdx.x; o < R16 * MT * 128; o += 32 * C::kConsumerWarps) {
        const int row = o & 15;
        const int tok = (o >> 4) & 7;
        const int rm = o >> 7;  // rg * MT + mt
        const int orow = rm / MT, mt = rm - orow * MT;
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < C::kKgPerStage; ++q) v += red[((q * R16 + orow) * MT + mt) * 128 + tok * 16 + row];
        const int64_t n = row0 + 16 * orow + row;
        const int m = 8 * mt + tok;
        if (n < N && m < M) {
          if (bias != nullptr) v += __bfloat162float(bias[n]);
          y[static_cast<int64_t>(m) * ldy + n] = __float2bfloat16_rn(apply_act(v, act));
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) atomicOr(&g_dq_error, 1u << kErrTimeout);
}

}  // namespace dq
