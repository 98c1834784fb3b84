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
// One warp per vector; lane l holds features EPL*l .. EPL*l+EPL-1 (pairs stay
// within a lane).
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace dq {

template <int EPL>
__global__ void __launch_bounds__(256)
    qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ img, int64_t ld_img,
                        const __nv_bfloat16* __restrict__ txt, int64_t ld_txt, int B, int S_img,
                        int S_txt, int H, const __nv_bfloat16* __restrict__ w_img,
                        const __nv_bfloat16* __restrict__ w_txt, const float* __restrict__ cos_t,
                        const float* __restrict__ sin_t, float eps, __nv_bfloat16* __restrict__ out) {
  constexpr int D = EPL * 32;
  const int lane = threadIdx.x & 31;
  const int64_t S = static_cast<int64_t>(S_txt) + S_img;
  const int64_t vec = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (vec >= static_cast<int64_t>(B) * S * H) return;
  // vec enumerates (b, s, h) with h fastest: consecutive warps read
  // consecutive heads of one token row
  const int h = static_cast<int>(vec % H);
  const int64_t bs = vec / H;
  const int64_t s = bs % S;
  const int b = static_cast<int>(bs / S);
  const bool is_txt = s < S_txt;
  const __nv_bfloat16* src = is_txt ? txt + (static_cast<int64_t>(b) * S_txt + s) * ld_txt
                                    : img + (static_cast<int64_t>(b) * S_img + (s - S_txt)) * ld_img;
  src += static_cast<int64_t>(h) * D + EPL * lane;
  const __nv_bfloat16* w = is_txt ? w_txt : w_img;
  float x[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) x[i] = __bfloat162float(src[i]);
  if (w != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) ss += x[i] * x[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const float n = __bfloat162float(__float2bfloat16_rn(x[i] * r));
      x[i] = __bfloat162float(__float2bfloat16_rn(n * __bfloat162float(w[EPL * lane + i])));
    }
  }
  __nv_bfloat16* dst = out + ((static_cast<int64_t>(b) * H + h) * S + s) * D + EPL * lane;
  if (cos_t != nullptr) {
    const float* c = cos_t + s * D + EPL * lane;
    const float* sn = sin_t + s * D + EPL * lane;
#pragma unroll
    for (int i = 0; i < EPL; i += 2) {
      // rotated pair: (-x[i+1], x[i])
      const float o0 = __fadd_rn(__fmul_rn(x[i], c[i]), __fmul_rn(-x[i + 1], sn[i]));
      const float o1 = __fadd_rn(__fmul_rn(x[i + 1], c[i + 1]), __fmul_rn(x[i], sn[i + 1]));
      dst[i] = __float2bfloat16_rn(o0);
      dst[i + 1] = __float2bfloat16_rn(o1);
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) dst[i] = __float2bfloat16_rn(x[i]);
  }
}

template <int EPL>
__global__ void __launch_bounds__(256)
    heads_to_tokens_kernel(const __nv_bfloat16* __restrict__ in, int B, int H, int S_txt, int S_img,
                           __nv_bfloat16* __restrict__ out_txt, __nv_bfloat16* __restrict__ out_img) {
  constexpr int D = EPL * 32;
  const int lane = threadIdx.x & 31;
  const int64_t S = static_cast<int64_t>(S_txt) + S_img;
  const int64_t vec = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (vec >= static_cast<int64_t>(B) * S * H) return;
  const int h = static_cast<int>(vec % H);
  const int64_t bs = vec / H;
  const int64_t s = bs % S;
  const int b = static_cast<int>(bs / S);
  const __nv_bfloat16* src = in + ((static_cast<int64_t>(b) * H + h) * S + s) * D + EPL * lane;
  __nv_bfloat16* dst =
      s < S_txt ? out_txt + (static_cast<int64_t>(b) * S_txt + s) * H * D
                : out_img + (static_cast<int64_t>(b) * S_img + (s - S_txt)) * H * D;
  dst += static_cast<int64_t>(h) * D + EPL * lane;
#pragma unroll
  for (int i = 0; i < EPL; ++i) dst[i] = src[i];
}

}  // namespace dq
