// dq_smallm.cuh -- the NF4 / fp8 linear for decode-sized token counts
// (M <= 16): y[M, N] = x[M, K] . dequant(W)[N, K]^T, HBM-bound on the weight.
//
// At these sizes the weight bytes set the time (3072 -> 18432 NF4: 31.9 MB,
// ~5 us at the HBM rate) and the tensor-core work is tiny.  The tcgen05 path
// needs every decoded weight tile in tensor memory before a 128-row MMA can be
// issued, and its per-MMA issue cost at N = 16 outlasts the weight stream;
// here the decoded weights go straight from the decode into the A operand
// registers of warp-level m16n8k16 bf16 MMAs (f32 accumulation), so the
// weight never touches shared or tensor memory.
//
// K permutation: a sum over k may visit k in any order as long as A and B use
// the same order.  Thread (g4 = lane / 4, tig = lane % 4) of a warp owns, per
// group of 128 k, the 32 consecutive weights k0 + 32*tig .. +31 of rows g4
// and g4 + 8 of a 16-row group (16 packed NF4 bytes or 32 e4m3 bytes per
// row), decodes them to 16 bf16 pairs w[0..15] (w[i] = elements 2i, 2i+1),
// and MMA j (j = 0..7) takes w[2j] / w[2j+1] of both rows as its A fragment:
// MMA k-slot 2*tig + e is element 4j + e of that run, slot 2*tig + 8 + e
// element 4j + 2 + e -- a function of the slot alone, so thread tig's B
// fragment (x of token g4 at the same k) is the same 4j.. run of x.
//
// A CTA (8 warps) owns 16 * R16 weight rows; its warps split the 128-k
// groups round-robin and their partial sums meet in shared memory, where the
// bias and activation are added and y is stored.  No workspace, one launch.
//
// Weight stream: plain 16-byte loads that bypass L1 (x lives there) straight
// into registers.  With one row group per CTA the next k-group is prefetched
// while this one is decoded; with two or four, the row groups' loads of one
// k-group are the bytes in flight.  (A shared-memory ring fed by cp.async
// measured slower: once enough rows share a CTA, the warp MMAs, not the
// loads, set the pace.)
#pragma once

#include "dq_codec.cuh"

namespace dq {

__device__ __forceinline__ void mma_16816_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Streaming 16-byte weight load (read once: not kept in L1, where x lives).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <int FMT, int MT, int R16>
struct SmallMCfg {
  static constexpr int kWarps = 8;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kRows = 16 * R16;
  static constexpr bool kPrefetch = R16 == 1;
  // resident CTAs per SM the register budget is sized for: three where the
  // accumulators and weight runs fit in 85 registers without spilling
  static constexpr int kMinCtas = (MT == 1 && R16 <= 2) ? 3 : 2;
  static constexpr int kLutBytes = FMT == kFmtNF4 ? kNf4LutBytes : 0;
  // per warp, row group and token tile: a 16 x 8 f32 fragment
  static constexpr int kRedBytes = kWarps * R16 * MT * 128 * 4;
  static constexpr int kSmemBytes = kLutBytes + kRedBytes;
};

// One k-group (128 k) of one row: this thread's 32-weight run.
template <int FMT>
struct RowRun {
  uint32_t p[FMT == kFmtNF4 ? 4 : 8];
  float am;
};

template <int FMT, bool SBF>
__device__ __forceinline__ void load_run(RowRun<FMT>& r, const uint8_t* w, const void* absmax,
                                         int64_t row, bool valid, int K, int g, int tig) {
  if (!valid) {
#pragma unroll
    for (int i = 0; i < (FMT == kFmtNF4 ? 4 : 8); ++i) r.p[i] = 0u;
    r.am = 0.f;
    return;
  }
  if constexpr (FMT == kFmtNF4) {
    const uint4 v = ld_stream16(w + row * (K / 2) + 64 * g + 16 * tig);
    r.p[0] = v.x; r.p[1] = v.y; r.p[2] = v.z; r.p[3] = v.w;
    r.am = load_scale(absmax, row * (K / 64) + 2 * g + (tig >> 1), SBF);
  } else {
    const uint8_t* src = w + row * K + 128 * g + 32 * tig;
    const uint4 v0 = ld_stream16(src);
    const uint4 v1 = ld_stream16(src + 16);
    r.p[0] = v0.x; r.p[1] = v0.y; r.p[2] = v0.z; r.p[3] = v0.w;
    r.p[4] = v1.x; r.p[5] = v1.y; r.p[6] = v1.z; r.p[7] = v1.w;
    r.am = 0.f;
  }
}

// Decode half h (weights 16h .. 16h+15 of the run) into w[0..7] (bf16 pairs).
template <int FMT>
__device__ __forceinline__ void decode_half(const RowRun<FMT>& r, int h, uint32_t lut_lane,
                                            float fp8_s, uint32_t* w) {
  if constexpr (FMT == kFmtNF4) {
    const uint32_t sc2 = nf4_scale2(r.am);
    nf4_decode_word_lut(r.p[2 * h], lut_lane, sc2, w);
    nf4_decode_word_lut(r.p[2 * h + 1], lut_lane, sc2, w + 4);
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) fp8_decode_word(r.p[4 * h + q], fp8_s, w + 2 * q);
  }
}

// SBF: the NF4 block scales are bf16 (repacked at load time), else f32.
template <int FMT, int MT, int R16, bool SBF>
__global__ void __launch_bounds__(SmallMCfg<FMT, MT, R16>::kThreads, SmallMCfg<FMT, MT, R16>::kMinCtas)
    smallm_kernel(const __nv_bfloat16* __restrict__ x, const uint8_t* __restrict__ w,
                  const void* __restrict__ absmax, float fp8_scale,
                  const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ y, int M,
                  int N, int K, int act, int64_t ldy) {
  using C = SmallMCfg<FMT, MT, R16>;
  constexpr bool PF = C::kPrefetch;
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g4 = lane >> 2, tig = lane & 3;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * C::kRows;
  const int KG = K / 128;
  uint32_t lut_lane = 0;
  if constexpr (FMT == kFmtNF4) {
    nf4_lut_fill(reinterpret_cast<uint32_t*>(smem));
    lut_lane = smem_u32(smem) + 4u * lane;
    __syncthreads();
  }
  const float fp8_s = __bfloat162float(__float2bfloat16_rn(fp8_scale));

  float acc[R16][MT][4];
#pragma unroll
  for (int rr = 0; rr < R16; ++rr)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[rr][mt][i] = 0.f;

  RowRun<FMT> cur[R16][2], nxt[R16][PF ? 2 : 1];
  auto load_group = [&](RowRun<FMT>(&r)[R16][2], int g) {
#pragma unroll
    for (int rr = 0; rr < R16; ++rr)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int64_t row = row0 + 16 * rr + g4 + 8 * hh;
        load_run<FMT, SBF>(r[rr][hh], w, absmax, row, row < N, K, g, tig);
      }
  };
  if (PF && warp < KG) load_group(cur, warp);
  for (int g = warp; g < KG; g += C::kWarps) {
    if constexpr (PF) {
      if (g + C::kWarps < KG) load_group(nxt, g + C::kWarps);
    } else {
      load_group(cur, g);
    }
    const int64_t k0 = 128ll * g + 32 * tig;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // x of this thread's tokens at k0 + 16h .. +15 (bf16 pairs xw[0..7])
      uint32_t xw[MT][8];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int t = 8 * mt + g4;
        if (t < M) {
          const uint4* src =
              reinterpret_cast<const uint4*>(x + t * static_cast<int64_t>(K) + k0 + 16 * h);
          const uint4 a = __ldg(src), b = __ldg(src + 1);
          xw[mt][0] = a.x; xw[mt][1] = a.y; xw[mt][2] = a.z; xw[mt][3] = a.w;
          xw[mt][4] = b.x; xw[mt][5] = b.y; xw[mt][6] = b.z; xw[mt][7] = b.w;
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) xw[mt][e] = 0u;
        }
      }
#pragma unroll
      for (int rr = 0; rr < R16; ++rr) {
        uint32_t w0[8], w1[8];
        decode_half<FMT>(cur[rr][0], h, lut_lane, fp8_s, w0);
        decode_half<FMT>(cur[rr][1], h, lut_lane, fp8_s, w1);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            mma_16816_bf16(acc[rr][mt], w0[2 * jj], w1[2 * jj], w0[2 * jj + 1], w1[2 * jj + 1],
                           xw[mt][2 * jj], xw[mt][2 * jj + 1]);
      }
    }
    if constexpr (PF) {
#pragma unroll
      for (int rr = 0; rr < R16; ++rr)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) cur[rr][hh] = nxt[rr][hh];
    }
  }

  // partial sums of the 8 warps -> shared memory, fragment element (row, token)
  float* red = reinterpret_cast<float*>(smem + C::kLutBytes);
#pragma unroll
  for (int rr = 0; rr < R16; ++rr)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      float* dst = red + ((warp * R16 + rr) * MT + mt) * 128;
      dst[(2 * tig) * 16 + g4] = acc[rr][mt][0];
      dst[(2 * tig + 1) * 16 + g4] = acc[rr][mt][1];
      dst[(2 * tig) * 16 + g4 + 8] = acc[rr][mt][2];
      dst[(2 * tig + 1) * 16 + g4 + 8] = acc[rr][mt][3];
    }
  __syncthreads();
  if (act_is_gated(act)) {
    // gated row order: row groups 2p (gate) and 2p + 1 (up) give output
    // features row0 / 2 + 16 p .. +15 (R16 is even here)
    for (int o = threadIdx.x; o < (R16 / 2) * MT * 128; o += C::kThreads) {
      const int row = o & 15;
      const int tok = (o >> 4) & 7;
      const int pm = o >> 7;  // pair * MT + mt
      const int pr = pm / MT, mt = pm - pr * MT;
      float g = 0.f, u = 0.f;
#pragma unroll
      for (int wp = 0; wp < C::kWarps; ++wp) {
        g += red[((wp * R16 + 2 * pr) * MT + mt) * 128 + tok * 16 + row];
        u += red[((wp * R16 + 2 * pr + 1) * MT + mt) * 128 + tok * 16 + row];
      }
      const int64_t ng = row0 + 32 * pr + row;
      const int m = 8 * mt + tok;
      if (ng < N && m < M) {
        if (bias != nullptr) {
          g += __bfloat162float(bias[ng]);
          u += __bfloat162float(bias[ng + 16]);
        }
        y[static_cast<int64_t>(m) * ldy + row0 / 2 + 16 * pr + row] = __float2bfloat16_rn(gated_value(g, u, act));
      }
    }
    return;
  }
  // element o = ((rr * MT + mt) * 8 + token) * 16 + row: consecutive threads
  // store consecutive output features of one token
  for (int o = threadIdx.x; o < R16 * MT * 128; o += C::kThreads) {
    float s = 0.f;
#pragma unroll
    for (int wp = 0; wp < C::kWarps; ++wp) s += red[wp * R16 * MT * 128 + o];
    const int row = o & 15;
    const int tok = (o >> 4) & 7;
    const int rm = o >> 7;  // rr * MT + mt
    const int rr = rm / MT, mt = rm - rr * MT;
    const int64_t n = row0 + 16 * rr + row;
    const int m = 8 * mt + tok;
    if (n < N && m < M) {
      if (bias != nullptr) s += __bfloat162float(bias[n]);
      y[static_cast<int64_t>(m) * ldy + n] = __float2bfloat16_rn(apply_act(s, act));
    }
  }
}

}  // namespace dq
