// dq_epilogue.cuh -- the gated-activation epilogue shared by the tensor-memory
// GEMM kernels (fused one-CTA, fused CTA-pair and the two-phase bf16 pair
// GEMM).
//
// In those kernels an epilogue warp drains the accumulator rows of 32 weight
// rows (one per lane) EC token columns at a time.  With the weight in the
// gated row order (dq_codec.cuh) lanes 0-15 hold the gate rows of 16 output
// features and lanes 16-31 the up rows of the same features: each gate lane
// takes its up value with one shuffle, forms the gated output, and the warp
// stores [EC tokens][16 outputs] as 32-byte row segments.
#pragma once

#include "dq_codec.cuh"
#include "dq_ptx.cuh"

namespace dq {

// vc[j]: f32 accumulator bits of this lane's row at token mrow0 + j; bias:
// this lane's row bias; stg_s / sb: the warp's staging (>= EC * 16 bf16);
// y: output base (row stride ldy, n_out columns); ocol0: the warp's first
// output column (its first weight row / 2).
template <int EC>
__device__ __forceinline__ void gated_chunk_store(const uint32_t* vc, float bias, int act,
                                                  uint32_t stg_s, const __nv_bfloat16* sb,
                                                  __nv_bfloat16* y, int64_t ldy, int M, int n_out,
                                                  int mrow0, int ocol0, bool vec_ok, int lane) {
  static_assert(EC % 16 == 0, "two lanes per token row");
#pragma unroll
  for (int j = 0; j < EC; ++j) {
    const float v = __uint_as_float(vc[j]) + bias;
    const float u = __shfl_down_sync(0xffffffffu, v, 16);
    if (lane < 16)
      sts16(stg_s + 2u * (j * 16 + lane), __bfloat16_as_ushort(__float2bfloat16_rn(gated_value(v, u, act))));
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < EC / 16; ++i) {
    const int row = (lane >> 1) + 16 * i;
    const int col = (lane & 1) * 8;
    const int m = mrow0 + row;
    const int oc = ocol0 + col;
    if (m < M) {
      __nv_bfloat16* dst = y + static_cast<size_t>(m) * ldy + oc;
      if (vec_ok && oc + 8 <= n_out) {
        *reinterpret_cast<uint4*>(dst) = lds128(stg_s + 2u * (row * 16 + col));
      } else {
        const __nv_bfloat16* src = sb + row * 16 + col;
        for (int e = 0; e < 8; ++e)
          if (oc + e < n_out) dst[e] = src[e];
      }
    }
  }
  __syncwarp();
}

}  // namespace dq
