// dq_codec.cuh -- register-level NF4 / fp8-e4m3 codecs shared by the fused
// GEMM, the standalone dequantizers and the quantizers.
//
// NF4 decode follows diffuseR's byte-LUT dequantizer (R/nf4_ltx23.R:77-115,
// table R/jit_ltx23.R:270-281): w = RNE_bf16(bf16(level) * bf16(absmax)).
// Here, per 64-element block, the 16 levels are first multiplied by the bf16
// block scale with the packed bf16 multiply (one RNE rounding of an exact
// product, as in the reference), then split into byte planes held in eight
// 32-bit registers, and every 4-bit code is looked up with byte permutes
// instead of a memory table.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "dq_ptx.cuh"

namespace dq {

// bf16 bit patterns of the 16 NF4 levels of R/nf4_ltx23.R:15-21
// (double literal -> float -> bf16, round to nearest even).
constexpr uint16_t kNf4LevelBits[16] = {0xBF80, 0xBF32, 0xBF06, 0xBECA, 0xBE92, 0xBE3D,
                                        0xBDBA, 0x0000, 0x3DA3, 0x3E25, 0x3E7C, 0x3EAD,
                                        0x3EE2, 0x3F10, 0x3F39, 0x3F80};

// Four bytes (byte `hi` selects the high or low byte of each level pattern)
// of levels first..first+3, packed little-endian into one register.
__host__ __device__ constexpr uint32_t nf4_plane(int first, bool hi) {
  uint32_t r = 0;
  for (int i = 0; i < 4; ++i) {
    const uint32_t b = hi ? (kNf4LevelBits[first + i] >> 8) : (kNf4LevelBits[first + i] & 0xFFu);
    r |= b << (8 * i);
  }
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// The 16 levels multiplied by one bf16 block scale and rounded once
// (RNE_bf16(bf16(level) * bf16(absmax)), the reference's dequantized value),
// split into byte planes for the permute lookups: ha..hd hold the high bytes of
// levels 0-3, 4-7, 8-11, 12-15 and la..ld the low bytes.
struct Nf4Planes {
  uint32_t ha, hb, hc, hd, la, lb, lc, ld;
};

__host__ __device__ constexpr uint32_t nf4_level_pair(int i) {
  return static_cast<uint32_t>(kNf4LevelBits[2 * i]) |
         (static_cast<uint32_t>(kNf4LevelBits[2 * i + 1]) << 16);
}

__device__ __forceinline__ Nf4Planes nf4_scaled_planes(uint32_t sc2) {
  constexpr uint32_t kPairs[8] = {nf4_level_pair(0), nf4_level_pair(1), nf4_level_pair(2),
                                  nf4_level_pair(3), nf4_level_pair(4), nf4_level_pair(5),
                                  nf4_level_pair(6), nf4_level_pair(7)};
  uint32_t q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = bf16x2_mul(kPairs[i], sc2);
  Nf4Planes p;
  p.ha = prmt(q[0], q[1], 0x7531u);
  p.la = prmt(q[0], q[1], 0x6420u);
  p.hb = prmt(q[2], q[3], 0x7531u);
  p.lb = prmt(q[2], q[3], 0x6420u);
  p.hc = prmt(q[4], q[5], 0x7531u);
  p.lc = prmt(q[4], q[5], 0x6420u);
  p.hd = prmt(q[6], q[7], 0x7531u);
  p.ld = prmt(q[6], q[7], 0x6420u);
  return p;
}

// Decode one 32-bit word of packed NF4 (bytes b0..b3 in memory order, i.e.
// elements 0..7 with element 2j in the high nibble of byte j) into four
// bf16x2 words in element order (element 2i in the low half of o[i]), looking
// each code up in the scaled planes.
__device__ __forceinline__ void nf4_decode_word(uint32_t w, const Nf4Planes& P, uint32_t* o) {
  // Selector nibbles: code & 7 picks one of 8 bytes of a register pair.
  const uint32_t s7 = w & 0x77777777u;
  // Byte masks for codes >= 8: prmt in sign-replicate mode (selector bit 3
  // set) copies a byte's msb over the whole byte.  The msb of byte j of w is
  // bit 3 of its high nibble; the msb of byte j of (w << 4) is bit 3 of its
  // low nibble.
  const uint32_t w4 = w << 4;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint32_t sel = half ? (s7 >> 16) : s7;
    // Output byte order of the lookups below: b.lo, b.hi, b'.lo, b'.hi for
    // the two bytes b, b' of this half.
    const uint32_t m = prmt(w, w4, half ? 0xBFAEu : 0x9D8Cu);
    const uint32_t h = (prmt(P.ha, P.hb, sel) & ~m) | (prmt(P.hc, P.hd, sel) & m);
    const uint32_t l = (prmt(P.la, P.lb, sel) & ~m) | (prmt(P.lc, P.ld, sel) & m);
    // Interleave low/high bytes into bf16 pairs: (hi nibble, lo nibble) of b,
    // then of b'.
    o[2 * half + 0] = prmt(l, h, 0x4051u);
    o[2 * half + 1] = prmt(l, h, 0x6273u);
  }
}

// Shared-memory byte LUT for NF4: entry b is the bf16 pair (level[b >> 4] in
// the low half, level[b & 15] in the high half), i.e. the two elements of a
// packed byte in order -- the reference's [256, 2] byte table
// (R/jit_ltx23.R:270-281).  It is replicated once per lane, entry b of lane l
// at word b * 32 + l, so 32 lanes looking up arbitrary bytes hit 32 distinct
// banks.  32 KB.
constexpr int kNf4LutBytes = 256 * 32 * 4;

// The 16 level patterns in constant memory: the LUT fill reads them with a
// warp-uniform index (a broadcast), where a per-thread copy of the table would
// be indexed dynamically and live in local memory.
__constant__ uint16_t c_nf4_level_bits[16] = {
    kNf4LevelBits[0],  kNf4LevelBits[1],  kNf4LevelBits[2],  kNf4LevelBits[3],
    kNf4LevelBits[4],  kNf4LevelBits[5],  kNf4LevelBits[6],  kNf4LevelBits[7],
    kNf4LevelBits[8],  kNf4LevelBits[9],  kNf4LevelBits[10], kNf4LevelBits[11],
    kNf4LevelBits[12], kNf4LevelBits[13], kNf4LevelBits[14], kNf4LevelBits[15]};

// Fill the LUT (called by every thread of the CTA; caller synchronizes).
// Entry b of lane l is word b * 32 + l: each warp writes one byte value b for
// all 32 lanes per iteration (blockDim.x is a multiple of 32).
__device__ __forceinline__ void nf4_lut_fill(uint32_t* lut) {
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) {
    const int b = i >> 5;
    lut[i] = static_cast<uint32_t>(c_nf4_level_bits[b >> 4]) |
             (static_cast<uint32_t>(c_nf4_level_bits[b & 15]) << 16);
  }
}

// Decode one 32-bit word of packed NF4 through the shared LUT: four
// conflict-free lookups, each multiplied by the bf16 block scale (sc2, held
// twice) with one RNE rounding.  lut_lane = shared-window address of this
// lane's entry 0 (LUT base + 4 * lane); entry b is 128 bytes further per b.
__device__ __forceinline__ void nf4_decode_word_lut(uint32_t w, uint32_t lut_lane, uint32_t sc2,
                                                    uint32_t* o) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t b = prmt(w, 0u, 0x4440u + i);  // byte i, zero-extended
    o[i] = bf16x2_mul(lds32(lut_lane + b * 128u), sc2);
  }
}

__device__ __forceinline__ uint32_t bf16_bits(float v) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
}

// Block scale i of an NF4 weight whose scales are f32 (the reference's
// absmax buffer) or bf16 (repacked at load time: bf16(absmax), the value the
// forward casts to anyway, so both give the same dequantized weights).
__device__ __forceinline__ float load_scale(const void* absmax, int64_t i, bool bf16) {
  return bf16 ? __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(absmax) + i))
              : __ldg(static_cast<const float*>(absmax) + i);
}

// absmax$to(bf16), replicated into both halves.
__device__ __forceinline__ uint32_t nf4_scale2(float absmax) {
  const uint32_t b = bf16_bits(absmax);
  return b | (b << 16);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Decode one 32-bit word of e4m3 (elements 0..3 in memory order) into two
// bf16x2 words: RNE_bf16(e4m3 * s) where s is the bf16-rounded scale held as
// f32.  e4m3 -> f16 -> f32 is exact and the f32 product of a 4-bit and an
// 8-bit significand is exact, so the final conversion is the only rounding,
// as in R/fp8_ltx23.R:79-80.
__device__ __forceinline__ void fp8_decode_word(uint32_t w, float s, uint32_t* o) {
  const __half2_raw h01 =
      __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w & 0xFFFFu), __NV_E4M3);
  const __half2_raw h23 =
      __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w >> 16), __NV_E4M3);
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
  o[0] = pack_bf16x2(f01.x * s, f01.y * s);
  o[1] = pack_bf16x2(f23.x * s, f23.y * s);
}

// bucketize(v, midpoints, right = FALSE): number of midpoints strictly below v.
// The midpoints are (level[i] + level[i+1]) / 2 computed in float32 exactly as
// R/nf4_ltx23.R:46 does.
__device__ __forceinline__ uint32_t nf4_code(float v) {
  constexpr float kMid[15] = {
      -0x1.b239b0p-1f, -0x1.38a4e0p-1f, -0x1.d70900p-2f, -0x1.5bd4ecp-2f, -0x1.e079d8p-3f,
      -0x1.1a7178p-3f, -0x1.74f0e2p-5f, 0x1.45f5fep-5f,  0x1.ec90c4p-4f,  0x1.a0cfc0p-3f,
      0x1.2b05a8p-2f,  0x1.8ea7f2p-2f,  0x1.00da08p-1f,  0x1.491b5ep-1f,  0x1.b913b4p-1f};
  uint32_t c = 0;
#pragma unroll
  for (int i = 0; i < 15; ++i) c += (kMid[i] < v) ? 1u : 0u;
  return c;
}

// float32 -> e4m3fn, round to nearest even; magnitudes above 464 become NaN
// as in c10::Float8_e4m3fn (a quantized weight never reaches them).
__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  if (fabsf(v) > 464.0f) return static_cast<uint8_t>(0x7Fu | (v < 0.0f ? 0x80u : 0u));
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

// ------------------------------------------------------------ activation
// Decode 16-byte chunks c0 + tid, c0 + tid + nthr, ... (< c1) of a flat
// packed weight into bf16, four chunks in flight per thread (the loads of all
// four are issued before any is decoded).  NF4: a chunk is 32 weights of one
// 64-block (block scale index c >> 1) and decodes to 4 x 16 bytes; fp8: 16
// weights times the bf16-rounded scale s, 2 x 16 bytes.
//
// Called by whole warps whose lanes hold consecutive tids (tid % 32 == lane):
// a warp's 32 consecutive chunks decode to one contiguous run (2 KB NF4, 1 KB
// fp8), which goes through `stage` (the warp's own 128 / 64 x 16 bytes of
// shared memory, XOR-swizzled) so that each store instruction writes 512
// contiguous bytes; a warp whose 32 chunks straddle c1, or one given no stage
// (nullptr), stores each chunk directly.
__device__ __forceinline__ void dequant_nf4_chunks(const uint4* __restrict__ src,
                                                   const void* __restrict__ absmax,
                                                   uint4* __restrict__ dst, int64_t c0, int64_t c1,
                                                   int64_t tid, int64_t nthr, uint4* stage,
                                                   bool scale_bf16 = false) {
  const int lane = threadIdx.x & 31;
  for (int64_t c = c0 + tid; c - lane < c1; c += 4 * nthr) {
    uint4 p[4];
    float am[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t cu = c + u * nthr;
      if (cu < c1) {
        p[u] = __ldg(src + cu);
        am[u] = load_scale(absmax, cu >> 1, scale_bf16);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t cu = c + u * nthr;
      const int64_t cbase = cu - lane;  // the warp's first chunk
      if (cbase >= c1) break;            // warp-uniform
      uint32_t o[16];
      if (cu < c1) {
        const Nf4Planes planes = nf4_scaled_planes(nf4_scale2(am[u]));
        nf4_decode_word(p[u].x, planes, o + 0);
        nf4_decode_word(p[u].y, planes, o + 4);
        nf4_decode_word(p[u].z, planes, o + 8);
        nf4_decode_word(p[u].w, planes, o + 12);
      }
      if (stage != nullptr && cbase + 31 < c1) {
        // piece j of chunk q lives at stage[q * 4 + (j ^ (q & 3))]
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 4; ++j)
          stage[lane * 4 + (j ^ (lane & 3))] =
              make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int e = 32 * j + lane;  // 16-byte piece e of the warp's 2 KB
          const int q = e >> 2;
          dst[4 * cbase + e] = stage[q * 4 + ((e & 3) ^ (q & 3))];
        }
      } else if (cu < c1) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dst[4 * cu + j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
      }
    }
  }
}

__device__ __forceinline__ void dequant_fp8_chunks(const uint4* __restrict__ src, float s,
                                                   uint4* __restrict__ dst, int64_t c0, int64_t c1,
                                                   int64_t tid, int64_t nthr, uint4* stage) {
  const int lane = threadIdx.x & 31;
  for (int64_t c = c0 + tid; c - lane < c1; c += 4 * nthr) {
    uint4 p[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t cu = c + u * nthr;
      if (cu < c1) p[u] = __ldg(src + cu);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t cu = c + u * nthr;
      const int64_t cbase = cu - lane;
      if (cbase >= c1) break;  // warp-uniform
      uint32_t o[8];
      if (cu < c1) {
        fp8_decode_word(p[u].x, s, o + 0);
        fp8_decode_word(p[u].y, s, o + 2);
        fp8_decode_word(p[u].z, s, o + 4);
        fp8_decode_word(p[u].w, s, o + 6);
      }
      if (stage != nullptr && cbase + 31 < c1) {
        // piece j of chunk q lives at stage[q * 2 + (j ^ (q & 1))]
        __syncwarp();
        stage[lane * 2 + (lane & 1)] = make_uint4(o[0], o[1], o[2], o[3]);
        stage[lane * 2 + (1 ^ (lane & 1))] = make_uint4(o[4], o[5], o[6], o[7]);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int e = 32 * j + lane;  // 16-byte piece e of the warp's 1 KB
          const int q = e >> 1;
          dst[2 * cbase + e] = stage[q * 2 + ((e & 1) ^ (q & 1))];
        }
      } else if (cu < c1) {
        dst[2 * cu] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[2 * cu + 1] = make_uint4(o[4], o[5], o[6], o[7]);
      }
    }
  }
}

// Epilogue activations.  The gated ones (SwiGLU: silu(gate) * up, as the
// FLUX.2 / Z-Image feed-forward, R/dit_flux2_modules.R:77-84; GeGLU-tanh:
// gelu_tanh(gate) * up) take the weight in the gated row order: per group of
// 32 weight rows, rows 0-15 are the gate rows of 16 output features and rows
// 16-31 the up rows of the same features, so y has half as many columns.
enum : int { kActNone = 0, kActGeluTanh = 1, kActSwiGlu = 2, kActGeGluTanh = 3 };

__host__ __device__ __forceinline__ bool act_is_gated(int act) { return act >= kActSwiGlu; }

// GELU, tanh approximation, in float32: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))),
// with tanh(u) = 1 - 2 / (exp(2u) + 1) on the exp intrinsic: a few instructions
// instead of a full tanhf (32 copies of which, unrolled into the epilogue,
// slowed the whole kernel), accurate to ~1e-7 absolute, far below the bf16
// rounding that follows.  The exponent is clamped so exp never overflows.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float x_cube = x * x * x;
  const float inner = 0.7978845608028654f * (x + 0.044715f * x_cube);
  const float e = __expf(2.0f * fminf(fmaxf(inner, -20.0f), 20.0f));
  const float t = 1.0f - __fdividef(2.0f, e + 1.0f);
  return 0.5f * x * (1.0f + t);
}

// The epilogue value of an up-projection followed by GELU-tanh: the
// reference rounds the projection to bf16 before the activation
// (nnf_gelu(approximate = "tanh") on the bf16 output).
__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == kActGeluTanh) return gelu_tanh(__bfloat162float(__float2bfloat16_rn(v)));
  return v;
}

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// One output of a gated activation from the f32 sums of its gate and up rows
// (bias included), rounded as the reference's tensor chain rounds: the
// projection to bf16, the activation of the bf16 gate to bf16 (SiLU
// x / (1 + e^-x) in f32, as torch evaluates it), then the bf16 product.
__device__ __forceinline__ float gated_value(float gate, float up, int act) {
  const float g = round_bf16(gate);
  const float a = act == kActSwiGlu ? g / (1.0f + expf(-g)) : gelu_tanh(g);
  return round_bf16(a) * round_bf16(up);
}

}  // namespace dq
