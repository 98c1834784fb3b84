/* dq_dit.h -- fused attention prologue / epilogue for the FLUX DiT blocks
 * that call the quantized linears (same library as dq_linear.h).
 *
 * These have no single reference counterpart: each replaces a chain of the
 * reference's tensor ops around the attention (R/dit_flux_modules.R:161-212:
 * per-head ltx23_rms_norm, the [text; image] concatenation, the transpose to
 * head-major, flux_apply_rotary_emb R/rope_flux.R:96-110, and the way back).
 * bf16 tensors, device pointers, the given stream; for the attention glue D
 * (the head dimension) is a multiple of 64 up to 256.  The AdaLN glue below
 * fuses the modulation and gated-residual tensor ops around the blocks. */
#ifndef DQ_DIT_H
#define DQ_DIT_H

#include <stdint.h>
#include "dq_linear.h"

#ifdef __cplusplus
extern "C" {
#endif

/* img [B, S_img, H*D] (row stride ld_img elements) and, if txt != NULL, txt
 * [B, S_txt, H*D] (row stride ld_txt) -> out [B, H, S_txt + S_img, D], text
 * first.  w_img / w_txt: RMS-norm weights [D] (NULL: no norm; eps as the
 * module's); cos_t / sin_t: float32 rotary tables [S_txt + S_img, D] (NULL: no
 * rotation). */
int dq_qk_norm_rope(const void* img, int64_t ld_img, const void* txt, int64_t ld_txt, int B,
                    int S_img, int S_txt, int H, int D, const void* w_img, const void* w_txt,
                    const float* cos_t, const float* sin_t, float eps, void* out,
                    dq_stream_t stream);

/* The q, k and v of one attention in one launch: part p (p < nparts <= 3)
 * reads img[p] [B, S_img, H*D] (row stride ld_img[p]) and, if S_txt > 0,
 * txt[p] [B, S_txt, H*D] (row stride ld_txt[p]), normalizes with
 * w_img[p] / w_txt[p] when w_img[p] != NULL, rotates with cos_t / sin_t when
 * rope[p] != 0, and writes out[p] [B, H, S_txt + S_img, D] -- the same bits as
 * one dq_qk_norm_rope call per part.  The pointer arrays are host arrays. */
int dq_qkv_norm_rope(int nparts, const void* const* img, const int64_t* ld_img,
                     const void* const* txt, const int64_t* ld_txt, int B, int S_img, int S_txt,
                     int H, int D, const void* const* w_img, const void* const* w_txt,
                     const int* rope, const float* cos_t, const float* sin_t, float eps,
                     void* const* out, dq_stream_t stream);

/* in [B, H, S_txt + S_img, D] -> out_txt [B, S_txt, H*D] (if S_txt > 0) and
 * out_img [B, S_img, H*D]. */
int dq_heads_to_tokens(const void* in, int B, int H, int S_txt, int S_img, int D, void* out_txt,
                       void* out_img, dq_stream_t stream);

/* dq_heads_to_tokens with the outputs' row strides (elements, >= H*D): the
 * tokens can land in a column range of a wider buffer. */
int dq_heads_to_tokens_ld(const void* in, int B, int H, int S_txt, int S_img, int D, void* out_txt,
                          int64_t ld_txt, void* out_img, int64_t ld_img, dq_stream_t stream);

/* AdaLN-Zero modulation (R/dit_flux_modules.R:26-42 and 54-70; the norm2
 * lines of flux_double_block): x [T, D] (row stride ld_x, T = B * S tokens,
 * batch element t / S) -> out = bf16(bf16(bf16(LayerNorm(x)) * bf16(1 +
 * scale)) + shift), LayerNorm without affine with eps, statistics in float32;
 * scale / shift [B, D] rows with row stride ld_mod.  D a multiple of 4 up to
 * 8192; every row start 8-byte aligned. */
int dq_adaln_modulate(const void* x, int64_t ld_x, int64_t T, int S, int D, const void* scale,
                      const void* shift, int64_t ld_mod, float eps, void* out, int64_t ld_out,
                      dq_stream_t stream);

/* Gated residual of the same blocks: out = bf16(x + bf16(gate * y)), gate
 * [B, D] (row stride ld_mod) broadcast over each batch element's S tokens;
 * out may be x.  D a multiple of 4; every row start 8-byte aligned. */
int dq_gated_residual(const void* x, int64_t ld_x, const void* gate, int64_t ld_mod, const void* y,
                      int64_t ld_y, int64_t T, int S, int D, void* out, int64_t ld_out,
                      dq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DQ_DIT_H */
