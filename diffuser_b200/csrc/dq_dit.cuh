// dq_dit.cuh -- attention prologue / epilogue of the FLUX DiT blocks that call
// the quantized linears: one pass instead of the reference's chain of tensor
// ops (R/dit_flux_modules.R:161-212 with ltx23_rms_norm, R/dit_ltx23_modules.R
// :25-46, and flux_apply_rotary_emb, R/rope_flux.R:96-110).
//
//   qk_norm_rope_kernel: per (batch, token, head) vector of D features from the
//     text and image projections (token-major [B, S, H*D] bf16): RMS-normalize
//     in float32 (x * rsqrt(mean(x^2) + eps), rounded to bf16, times the bf16
//     weight, rounded to bf16), then rotate pairs with the float32 cos/sin
//     table (x*cos and rot(x)*sin each rounded to float32, summed, rounded to
//     bf16), writing the head-major [B, H, S_txt + S_img, D] layout the
//     attention reads, text tokens first.  Without a weight the norm is
//     skipped, without a table the rotation: the value tensor uses it as a
//     pure concatenate + transpose.
//   heads_to_tokens_kernel: the attention output [B, H, S, D] back to
//     token-major [B, S_txt, H*D] and [B, S_img, H*D].
// One warp per (token, head) vector, one CTA per token; lane l holds
// features EPL*l .. EPL*l+EPL-1 (pairs stay within a lane).  With VEC the lane moves its EPL features with the widest
// aligned accesses (16 / 8 / 4-byte bf16 runs, 16 / 8-byte float runs; the
// host checks the alignment), else one element at a time; the arithmetic is
// the same either way.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace dq {

// EPL consecutive bf16 values -> float (exact).
template <int EPL, bool VEC>
__device__ __forceinline__ void load_bf16_run(const __nv_bfloat16* p, float* v) {
  if constexpr (VEC) {
    constexpr int W = EPL % 8 == 0 ? 4 : EPL % 4 == 0 ? 2 : 1;  // 32-bit words per access
    uint32_t u[EPL / 2];
#pragma unroll
    for (int i = 0; i < EPL / (2 * W); ++i) {
      if constexpr (W == 4) {
        const uint4 q = reinterpret_cast<const uint4*>(p)[i];
        u[4 * i] = q.x; u[4 * i + 1] = q.y; u[4 * i + 2] = q.z; u[4 * i + 3] = q.w;
      } else if constexpr (W == 2) {
        const uint2 q = reinterpret_cast<const uint2*>(p)[i];
        u[2 * i] = q.x; u[2 * i + 1] = q.y;
      } else {
        u[i] = reinterpret_cast<const uint32_t*>(p)[i];
      }
    }
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
      v[2 * i] = __uint_as_float(u[i] << 16);
      v[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = __bfloat162float(p[i]);
  }
}

// EPL floats, already rounded to bf16-representable values or not: RNE to bf16.
template <int EPL, bool VEC>
__device__ __forceinline__ void store_bf16_run(__nv_bfloat16* p, const float* v) {
  if constexpr (VEC) {
    constexpr int W = EPL % 8 == 0 ? 4 : EPL % 4 == 0 ? 2 : 1;
    uint32_t u[EPL / 2];
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      u[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
#pragma unroll
    for (int i = 0; i < EPL / (2 * W); ++i) {
      if constexpr (W == 4)
        reinterpret_cast<uint4*>(p)[i] = make_uint4(u[4 * i], u[4 * i + 1], u[4 * i + 2], u[4 * i + 3]);
      else if constexpr (W == 2)
        reinterpret_cast<uint2*>(p)[i] = make_uint2(u[2 * i], u[2 * i + 1]);
      else
        reinterpret_cast<uint32_t*>(p)[i] = u[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) p[i] = __float2bfloat16_rn(v[i]);
  }
}

template <int EPL, bool VEC>
__device__ __forceinline__ void load_f32_run(const float* p, float* v) {
  if constexpr (VEC && EPL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < EPL / 4; ++i) {
      const float4 q = reinterpret_cast<const float4*>(p)[i];
      v[4 * i] = q.x; v[4 * i + 1] = q.y; v[4 * i + 2] = q.z; v[4 * i + 3] = q.w;
    }
  } else if constexpr (VEC) {
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
      const float2 q = reinterpret_cast<const float2*>(p)[i];
      v[2 * i] = q.x; v[2 * i + 1] = q.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = p[i];
  }
}

// One CTA per token (b, s) of the [text; image] sequence; warp w owns heads
// w*HPW .. w*HPW+HPW-1 (then the next round of nwarps*HPW heads) and issues
// all their loads before computing, so HPW vectors per warp are in flight.
// The token's cos / sin slice is loaded once per warp.
constexpr int kHeadsPerWarp = 4;

template <int EPL, bool VEC>
__global__ void __launch_bounds__(512)
    qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ img, int64_t ld_img,
                        const __nv_bfloat16* __restrict__ txt, int64_t ld_txt, int B, int S_img,
                        int S_txt, int H, const __nv_bfloat16* __restrict__ w_img,
                        const __nv_bfloat16* __restrict__ w_txt, const float* __restrict__ cos_t,
                        const float* __restrict__ sin_t, float eps, __nv_bfloat16* __restrict__ out) {
  constexpr int D = EPL * 32;
  constexpr int HPW = kHeadsPerWarp;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int S = S_txt + S_img;
  const int b = static_cast<int>(blockIdx.x) / S;
  const int s = static_cast<int>(blockIdx.x) - b * S;
  const bool is_txt = s < S_txt;
  const __nv_bfloat16* row = is_txt ? txt + (static_cast<int64_t>(b) * S_txt + s) * ld_txt
                                    : img + (static_cast<int64_t>(b) * S_img + (s - S_txt)) * ld_img;
  const __nv_bfloat16* w = is_txt ? w_txt : w_img;
  float wv[EPL], c[EPL], sn[EPL];
  if (w != nullptr) load_bf16_run<EPL, VEC>(w + EPL * lane, wv);
  if (cos_t != nullptr) {
    load_f32_run<EPL, VEC>(cos_t + static_cast<int64_t>(s) * D + EPL * lane, c);
    load_f32_run<EPL, VEC>(sin_t + static_cast<int64_t>(s) * D + EPL * lane, sn);
  }
  for (int h0 = warp * HPW; h0 < H; h0 += nwarps * HPW) {
    float x[HPW][EPL];
#pragma unroll
    for (int j = 0; j < HPW; ++j)
      if (h0 + j < H) load_bf16_run<EPL, VEC>(row + static_cast<int64_t>(h0 + j) * D + EPL * lane, x[j]);
#pragma unroll
    for (int j = 0; j < HPW; ++j) {
      const int h = h0 + j;
      if (h >= H) break;  // warp-uniform
      if (w != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < EPL; ++i) ss += x[j][i] * x[j][i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float r = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const float n = __bfloat162float(__float2bfloat16_rn(x[j][i] * r));
          x[j][i] = __bfloat162float(__float2bfloat16_rn(n * wv[i]));
        }
      }
      __nv_bfloat16* dst = out + ((static_cast<int64_t>(b) * H + h) * S + s) * D + EPL * lane;
      if (cos_t != nullptr) {
        float o[EPL];
#pragma unroll
        for (int i = 0; i < EPL; i += 2) {
          // rotated pair: (-x[i+1], x[i])
          o[i] = __fadd_rn(__fmul_rn(x[j][i], c[i]), __fmul_rn(-x[j][i + 1], sn[i]));
          o[i + 1] = __fadd_rn(__fmul_rn(x[j][i + 1], c[i + 1]), __fmul_rn(x[j][i], sn[i + 1]));
        }
        store_bf16_run<EPL, VEC>(dst, o);
      } else {
        store_bf16_run<EPL, VEC>(dst, x[j]);
      }
    }
  }
}

// q, k and v of one attention in one launch.  Part p (0..nparts-1) reads its
// image / text token rows from its own pointers (column views of the
// concatenated q/k/v projection output or separate tensors), normalizes with
// its own weights when it has them, rotates when `rope` is set, and writes its
// own head-major [B, H, S_txt + S_img, D] output -- per part exactly the
// arithmetic of qk_norm_rope_kernel, so the bits are the same.  Work items are
// (token, part, group of HPW heads), taken by warps in a grid-stride loop:
// every warp of the resident grid keeps its HPW head vectors (plus the
// token's cos / sin slice) in flight, instead of the short-lived per-token
// CTAs of the one-part kernel.
struct QkvPart {
  const __nv_bfloat16* img;
  const __nv_bfloat16* txt;
  const __nv_bfloat16* w_img;
  const __nv_bfloat16* w_txt;
  __nv_bfloat16* out;
  int64_t ld_img, ld_txt;
  int rope;
};
struct QkvParts {
  QkvPart p[3];
  int nparts;
};

template <int EPL, bool VEC>
__global__ void __launch_bounds__(256)
    qkv_norm_rope_kernel(const QkvParts parts, int B, int S_img, int S_txt, int H,
                         const float* __restrict__ cos_t, const float* __restrict__ sin_t, float eps) {
  constexpr int D = EPL * 32;
  constexpr int HPW = kHeadsPerWarp;
  const int lane = threadIdx.x & 31;
  const int S = S_txt + S_img;
  const int G = (H + HPW - 1) / HPW;
  const int64_t per_token = static_cast<int64_t>(parts.nparts) * G;
  const int64_t items = static_cast<int64_t>(B) * S * per_token;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t it = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items;
       it += nwarps) {
    const int64_t bs = it / per_token;  // b * S + s
    const int rem = static_cast<int>(it - bs * per_token);
    const int pi = rem / G;
    const int h0 = (rem - pi * G) * HPW;
    const int b = static_cast<int>(bs / S);
    const int s = static_cast<int>(bs - static_cast<int64_t>(b) * S);
    // select the part without indexing the parameter array dynamically
    const QkvPart P = pi == 0 ? parts.p[0] : (pi == 1 ? parts.p[1] : parts.p[2]);
    const bool is_txt = s < S_txt;
    const __nv_bfloat16* row = is_txt ? P.txt + (static_cast<int64_t>(b) * S_txt + s) * P.ld_txt
                                      : P.img + (static_cast<int64_t>(b) * S_img + (s - S_txt)) * P.ld_img;
    const __nv_bfloat16* w = is_txt ? P.w_txt : P.w_img;
    float x[HPW][EPL], wv[EPL], c[EPL], sn[EPL];
#pragma unroll
    for (int j = 0; j < HPW; ++j)
      if (h0 + j < H) load_bf16_run<EPL, VEC>(row + static_cast<int64_t>(h0 + j) * D + EPL * lane, x[j]);
    if (w != nullptr) load_bf16_run<EPL, VEC>(w + EPL * lane, wv);
    if (P.rope) {
      load_f32_run<EPL, VEC>(cos_t + static_cast<int64_t>(s) * D + EPL * lane, c);
      load_f32_run<EPL, VEC>(sin_t + static_cast<int64_t>(s) * D + EPL * lane, sn);
    }
#pragma unroll
    for (int j = 0; j < HPW; ++j) {
      const int h = h0 + j;
      if (h >= H) break;  // warp-uniform
      if (w != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < EPL; ++i) ss += x[j][i] * x[j][i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float r = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const float n = __bfloat162float(__float2bfloat16_rn(x[j][i] * r));
          x[j][i] = __bfloat162float(__float2bfloat16_rn(n * wv[i]));
        }
      }
      __nv_bfloat16* dst = P.out + ((static_cast<int64_t>(b) * H + h) * S + s) * D + EPL * lane;
      if (P.rope) {
        float o[EPL];
#pragma unroll
        for (int i = 0; i < EPL; i += 2) {
          o[i] = __fadd_rn(__fmul_rn(x[j][i], c[i]), __fmul_rn(-x[j][i + 1], sn[i]));
          o[i + 1] = __fadd_rn(__fmul_rn(x[j][i + 1], c[i + 1]), __fmul_rn(x[j][i], sn[i + 1]));
        }
        store_bf16_run<EPL, VEC>(dst, o);
      } else {
        store_bf16_run<EPL, VEC>(dst, x[j]);
      }
    }
  }
}

// One CTA per token, warps over groups of HPW heads (as above).
template <int EPL, bool VEC>
__global__ void __launch_bounds__(512)
    heads_to_tokens_kernel(const __nv_bfloat16* __restrict__ in, int B, int H, int S_txt, int S_img,
                           __nv_bfloat16* __restrict__ out_txt, int64_t ld_txt,
                           __nv_bfloat16* __restrict__ out_img, int64_t ld_img) {
  constexpr int D = EPL * 32;
  constexpr int HPW = kHeadsPerWarp;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int S = S_txt + S_img;
  const int b = static_cast<int>(blockIdx.x) / S;
  const int s = static_cast<int>(blockIdx.x) - b * S;
  __nv_bfloat16* drow = s < S_txt ? out_txt + (static_cast<int64_t>(b) * S_txt + s) * ld_txt
                                  : out_img + (static_cast<int64_t>(b) * S_img + (s - S_txt)) * ld_img;
  for (int h0 = warp * HPW; h0 < H; h0 += nwarps * HPW) {
    float v[HPW][EPL];
#pragma unroll
    for (int j = 0; j < HPW; ++j)
      if (h0 + j < H)
        load_bf16_run<EPL, VEC>(in + ((static_cast<int64_t>(b) * H + h0 + j) * S + s) * D + EPL * lane,
                                v[j]);
#pragma unroll
    for (int j = 0; j < HPW; ++j) {
      if (h0 + j >= H) break;
      // bf16 -> float -> bf16 is exact: a plain copy
      store_bf16_run<EPL, VEC>(drow + static_cast<int64_t>(h0 + j) * D + EPL * lane, v[j]);
    }
  }
}

// ---------------------------------------------------------- AdaLN glue
// adaln_modulate_kernel: the AdaLN-Zero modulation of the FLUX blocks
// (R/dit_flux_modules.R:26-42, 54-70, and the norm2 lines of the double
// block): out = bf16(bf16(bf16(LN(x)) * bf16(1 + scale)) + shift), LN a
// LayerNorm without affine (eps), statistics in float32 (two passes over the
// row held in registers).  One CTA (256 threads) per token row; each thread
// owns up to NPT runs of 4 features (8-byte accesses).
// gated_residual_kernel: out = bf16(x + bf16(gate * y)), the gated residual
// adds of the same blocks.  scale / shift / gate are [B, D] rows (row stride
// ld_mod) broadcast over the S tokens of each batch element.
__device__ __forceinline__ void unpack_bf16x4(uint2 u, float* v) {
  v[0] = __uint_as_float(u.x << 16);
  v[1] = __uint_as_float(u.x & 0xFFFF0000u);
  v[2] = __uint_as_float(u.y << 16);
  v[3] = __uint_as_float(u.y & 0xFFFF0000u);
}
__device__ __forceinline__ uint2 pack_bf16x4(const float* v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
  const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}
__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Sum over the CTA (256 threads); red holds 8 floats.
__device__ __forceinline__ float block_sum_256(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5;
  __syncthreads();  // red may still be read from a previous call
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) t += red[i];
  return t;
}

template <int NPT>
__global__ void __launch_bounds__(256)
    adaln_modulate_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x, int S, int D,
                          const __nv_bfloat16* __restrict__ scale,
                          const __nv_bfloat16* __restrict__ shift, int64_t ld_mod, float eps,
                          __nv_bfloat16* __restrict__ out, int64_t ld_out) {
  __shared__ float red[8];
  const int64_t t = blockIdx.x;
  const int b = static_cast<int>(t / S);
  const int nrun = D / 4;
  const __nv_bfloat16* xr = x + t * ld_x;
  float v[NPT][4];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int r = threadIdx.x + 256 * j;
    if (r < nrun) {
      unpack_bf16x4(reinterpret_cast<const uint2*>(xr)[r], v[j]);
      sum += (v[j][0] + v[j][1]) + (v[j][2] + v[j][3]);
    }
  }
  const float mean = block_sum_256(sum, red) / static_cast<float>(D);
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int r = threadIdx.x + 256 * j;
    if (r < nrun) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float d = v[j][e] - mean;
        sq += d * d;
      }
    }
  }
  const float rstd = rsqrtf(block_sum_256(sq, red) / static_cast<float>(D) + eps);
  const uint2* sc = reinterpret_cast<const uint2*>(scale + b * ld_mod);
  const uint2* sh = reinterpret_cast<const uint2*>(shift + b * ld_mod);
  uint2* o = reinterpret_cast<uint2*>(out + t * ld_out);
#pragma unroll
  for (int j = 0; j < NPT; ++j) {
    const int r = threadIdx.x + 256 * j;
    if (r < nrun) {
      float a[4], c[4], y[4];
      unpack_bf16x4(sc[r], a);
      unpack_bf16x4(sh[r], c);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float n = bf16r((v[j][e] - mean) * rstd);
        y[e] = bf16r(n * bf16r(a[e] + 1.0f)) + c[e];
      }
      o[r] = pack_bf16x4(y);
    }
  }
}

// Gated residual with 16-byte accesses (rows, gate and output 16-byte
// aligned, D a multiple of 8): each thread takes two 8-feature runs per
// iteration, so four 16-byte loads are in flight per thread.
__global__ void __launch_bounds__(256)
    gated_residual16_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x,
                            const __nv_bfloat16* __restrict__ gate, int64_t ld_mod,
                            const __nv_bfloat16* __restrict__ y, int64_t ld_y, int64_t T, int S, int D,
                            __nv_bfloat16* out, int64_t ld_out) {
  const int nrun = D / 8;
  const int64_t total = T * nrun;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i0 < total;
       i0 += 2 * stride) {
    uint4 xu[2], yu[2], gu[2];
    int64_t tt[2];
    int rr[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int64_t i = i0 + q * stride;
      tt[q] = i / nrun;
      rr[q] = static_cast<int>(i - tt[q] * nrun);
      if (i < total) {
        const int b = static_cast<int>(tt[q] / S);
        xu[q] = reinterpret_cast<const uint4*>(x + tt[q] * ld_x)[rr[q]];
        yu[q] = reinterpret_cast<const uint4*>(y + tt[q] * ld_y)[rr[q]];
        gu[q] = reinterpret_cast<const uint4*>(gate + b * ld_mod)[rr[q]];
      }
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (i0 + q * stride >= total) break;
      float xv[8], gv[8], yv[8], o[8];
      unpack_bf16x4(make_uint2(xu[q].x, xu[q].y), xv);
      unpack_bf16x4(make_uint2(xu[q].z, xu[q].w), xv + 4);
      unpack_bf16x4(make_uint2(gu[q].x, gu[q].y), gv);
      unpack_bf16x4(make_uint2(gu[q].z, gu[q].w), gv + 4);
      unpack_bf16x4(make_uint2(yu[q].x, yu[q].y), yv);
      unpack_bf16x4(make_uint2(yu[q].z, yu[q].w), yv + 4);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = xv[e] + bf16r(gv[e] * yv[e]);
      const uint2 lo = pack_bf16x4(o), hi = pack_bf16x4(o + 4);
      reinterpret_cast<uint4*>(out + tt[q] * ld_out)[rr[q]] = make_uint4(lo.x, lo.y, hi.x, hi.y);
    }
  }
}

__global__ void __launch_bounds__(256)
    gated_residual_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld_x,
                          const __nv_bfloat16* __restrict__ gate, int64_t ld_mod,
                          const __nv_bfloat16* __restrict__ y, int64_t ld_y, int64_t T, int S, int D,
                          __nv_bfloat16* out, int64_t ld_out) {
  const int nrun = D / 4;
  const int64_t total = T * nrun;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / nrun;
    const int r = static_cast<int>(i - t * nrun);
    const int b = static_cast<int>(t / S);
    float xv[4], gv[4], yv[4], o[4];
    unpack_bf16x4(reinterpret_cast<const uint2*>(x + t * ld_x)[r], xv);
    unpack_bf16x4(reinterpret_cast<const uint2*>(gate + b * ld_mod)[r], gv);
    unpack_bf16x4(reinterpret_cast<const uint2*>(y + t * ld_y)[r], yv);
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = xv[e] + bf16r(gv[e] * yv[e]);
    reinterpret_cast<uint2*>(out + t * ld_out)[r] = pack_bf16x4(o);
  }
}

}  // namespace dq
