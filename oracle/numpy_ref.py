"""Bit-level numpy restatement of diffuseR's NF4 / fp8 weight-only linear.

TEST INFRASTRUCTURE ONLY (the checker; never the product path).

Every function cites the reference file:line it restates (paths relative to
the diffuseR 0.2.2 source tree).

Conventions (same as the reference):
  * a weight ``W`` is ``[N, K]`` (out_features, in_features), row-major;
  * NF4 blocks are 64 consecutive elements of the flattened weight; with
    ``K % 64 == 0`` every block lies inside one output row;
  * packed byte ``j`` holds element ``2j`` in its HIGH nibble and ``2j+1`` in
    its LOW nibble;
  * bf16 values are carried as ``uint16`` bit patterns; rounding is
    round-to-nearest-even, exactly as c10::BFloat16 does.
"""
from __future__ import annotations

import numpy as np

# R/nf4_ltx23.R:15-21 -- the 16 QLoRA NormalFloat levels (double literals).
NF4_LEVELS_F64 = np.array([
    -1.0, -0.6961928009986877, -0.5250730514526367,
    -0.39491748809814453, -0.28444138169288635,
    -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725,
    0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941,
    0.7229568362236023, 1.0], dtype=np.float64)

# R/nf4_ltx23.R:23
NF4_BLOCK = 64

FP8_MAX = 448.0           # R/fp8_ltx23.R:180, R/quantize_flux.R:407 ("/ 448")
SCALE_FLOOR = 1e-12       # clamp(min = 1e-12) in both quantizers


# ---------------------------------------------------------------- bf16 helpers
def f32_to_bf16_bits(a) -> np.ndarray:
    """Round float32 -> bf16 (RNE), returned as uint16 bit patterns."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(a) -> np.ndarray:
    """float32 -> nearest bf16, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


# ------------------------------------------------------------------ NF4 codec
def nf4_levels_f32() -> np.ndarray:
    """torch_tensor(.ltx23_nf4_table, dtype = float32) (R/nf4_ltx23.R:43-45)."""
    return NF4_LEVELS_F64.astype(np.float32)


def nf4_levels_bf16_bits() -> np.ndarray:
    """The levels as the LUT holds them in bf16 (R/jit_ltx23.R:270-281).

    The double literal goes double -> float -> bf16; for these 16 values that
    equals direct double -> bf16 rounding (checked in tests).
    """
    return f32_to_bf16_bits(nf4_levels_f32())


def nf4_midpoints_f32() -> np.ndarray:
    """Decision boundaries, computed in float32 (R/nf4_ltx23.R:46)."""
    t = nf4_levels_f32()
    return ((t[:15] + t[1:]) / np.float32(2)).astype(np.float32)


def nf4_quantize(w) -> tuple[np.ndarray, np.ndarray]:
    """ltx23_nf4_quantize (R/nf4_ltx23.R:35-61).

    Returns (packed uint8 [n/2], absmax float32 [n/64]).
      absmax = max|block| in float32, clamped to >= 1e-12      (:48-49)
      normalized = block / absmax (IEEE float32 division)       (:50)
      idx = bucketize(normalized, midpoints, right=FALSE)       (:52)
            i.e. the number of midpoints strictly below the value, so a
            value equal to a midpoint takes the lower level
      packed = idx[2j] * 16 + idx[2j+1]                         (:55-58)
    """
    w = np.asarray(w, dtype=np.float32).reshape(-1)
    n = w.size
    if n % NF4_BLOCK != 0:
        raise ValueError(f"Tensor length must be a multiple of {NF4_BLOCK}")
    blocks = w.reshape(-1, NF4_BLOCK)
    absmax = np.maximum(np.abs(blocks).max(axis=1), np.float32(SCALE_FLOOR)).astype(np.float32)
    normalized = (blocks / absmax[:, None]).astype(np.float32).reshape(-1)
    idx = np.searchsorted(nf4_midpoints_f32(), normalized, side="left").astype(np.uint8)
    pairs = idx.reshape(-1, 2)
    packed = (pairs[:, 0] * np.uint8(16) + pairs[:, 1]).astype(np.uint8)
    return packed, absmax


def nf4_byte_lut_f32() -> np.ndarray:
    """Byte LUT [256, 2] = (level[b >> 4], level[b & 15]) (R/jit_ltx23.R:274-277)."""
    t = nf4_levels_f32()
    b = np.arange(256)
    return np.stack([t[b >> 4], t[b & 15]], axis=1)


def nf4_dequantize_bf16_bits(packed, absmax) -> np.ndarray:
    """ltx23_nf4_dequantize with dtype = bf16 (R/nf4_ltx23.R:77-115).

    w = RNE_bf16( bf16(level) * bf16(absmax) ): the LUT is built in bf16
    (R/jit_ltx23.R:276) and absmax is cast with absmax$to(dtype) (:97) before
    the in-place mul_ (:109-110).  The product of two bf16 values is exact in
    float32, so a single RNE rounding of the float32 product is bit-exact.
    Returns the flat uint16 bit patterns.
    """
    packed = np.asarray(packed, dtype=np.uint8).reshape(-1)
    absmax = np.asarray(absmax, dtype=np.float32).reshape(-1)
    lv = bf16_bits_to_f32(nf4_levels_bf16_bits())
    vals = np.empty(packed.size * 2, dtype=np.float32)
    vals[0::2] = lv[packed >> 4]
    vals[1::2] = lv[packed & 15]
    am = bf16_bits_to_f32(f32_to_bf16_bits(absmax))
    prod = (vals.reshape(-1, NF4_BLOCK) * am[:, None]).astype(np.float32)
    return f32_to_bf16_bits(prod).reshape(-1)


def nf4_dequantize_f32(packed, absmax) -> np.ndarray:
    """ltx23_nf4_dequantize with dtype = float32 (the reference's CPU mode)."""
    packed = np.asarray(packed, dtype=np.uint8).reshape(-1)
    absmax = np.asarray(absmax, dtype=np.float32).reshape(-1)
    lv = nf4_levels_f32()
    vals = np.empty(packed.size * 2, dtype=np.float32)
    vals[0::2] = lv[packed >> 4]
    vals[1::2] = lv[packed & 15]
    return (vals.reshape(-1, NF4_BLOCK) * absmax[:, None]).astype(np.float32).reshape(-1)


# ------------------------------------------------------------------ fp8 codec
def _e4m3_code_values() -> np.ndarray:
    """float64 value of every e4m3fn code 0..255 (0x7F / 0xFF are NaN)."""
    codes = np.arange(256)
    s = (codes >> 7) & 1
    e = (codes >> 3) & 15
    m = codes & 7
    mag = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1 + m / 8.0) * 2.0 ** (e - 7.0))
    v = np.where(s == 1, -mag, mag)
    v = v.astype(np.float64)
    v[(codes & 0x7F) == 0x7F] = np.nan
    return v


E4M3_VALUES = _e4m3_code_values()


def f32_to_e4m3(a) -> np.ndarray:
    """float32 -> float8_e4m3fn bits, round-to-nearest-even.

    Magnitudes above 464 (the midpoint between 448 and the absent 480) map to
    NaN (0x7F) and 464 itself rounds to 448, as c10::Float8_e4m3fn does; the quantizer below never
    produces them (|W / scale| <= 448 up to one float32 ulp).
    """
    a = np.asarray(a, dtype=np.float32)
    mag = np.abs(a).astype(np.float64)
    pos = E4M3_VALUES[:127]                       # codes 0..126, increasing
    i = np.searchsorted(pos, mag, side="left")     # pos[i-1] < mag <= pos[i]
    i = np.clip(i, 1, 126)
    lo, hi = pos[i - 1], pos[i]
    code = np.where(mag - lo < hi - mag, i - 1, i)
    tie = (mag - lo) == (hi - mag)
    code = np.where(tie, np.where(((i - 1) & 1) == 0, i - 1, i), code)
    code = np.where(mag <= 0, 0, code)
    code = np.where(mag > 464.0, 0x7F, code)
    code = np.where(np.isnan(mag), 0x7F, code).astype(np.uint8)
    sign = (np.signbit(a)).astype(np.uint8) << 7
    return (code | sign).astype(np.uint8)


def e4m3_to_f32(b) -> np.ndarray:
    return E4M3_VALUES[np.asarray(b, dtype=np.uint8)].astype(np.float32)


def fp8_quantize(w) -> tuple[np.ndarray, np.float32]:
    """Per-tensor e4m3 quantizer (R/quantize_flux.R:406-409, R/fp8_ltx23.R:178-181).

    scale = max|W| (as float32) clamped to >= 1e-12, divided by 448 (float32);
    W8 = e4m3fn(W_f32 / scale).
    """
    w = np.asarray(w, dtype=np.float32)
    amax = np.float32(np.abs(w).max()) if w.size else np.float32(0)
    scale = np.float32(np.maximum(amax, np.float32(SCALE_FLOOR)) / np.float32(FP8_MAX))
    w8 = f32_to_e4m3((w / scale).astype(np.float32))
    return w8, scale


def fp8_dequantize_bf16_bits(w8, scale) -> np.ndarray:
    """ltx23_fp8_linear forward dequant (R/fp8_ltx23.R:79-80).

    w$copy_(w8) is an exact e4m3 -> bf16 upcast; w$mul_(scale$to(bf16)) gives
    RNE_bf16(e4m3 * bf16(scale)) -- a single rounding of an exact product.
    """
    v = e4m3_to_f32(w8)
    s = bf16_bits_to_f32(f32_to_bf16_bits(np.float32(scale)))
    return f32_to_bf16_bits((v * s).astype(np.float32))


def fp8_dequantize_f32(w8, scale) -> np.ndarray:
    return (e4m3_to_f32(w8) * np.float32(scale)).astype(np.float32)


# ------------------------------------------------------------------- linear
def linear_bf16(x_bits, w_bits, bias_bits=None) -> np.ndarray:
    """torch::nnf_linear(x, w, bias) in bf16 (R/nf4_ltx23.R:245, R/fp8_ltx23.R:82).

    bf16 operands, float accumulation (float64 here), bias added before the
    single rounding to bf16.  Returns uint16 bit patterns [M, N].
    """
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    w = bf16_bits_to_f32(w_bits).astype(np.float64)
    y = x @ w.T
    if bias_bits is not None:
        y = y + bf16_bits_to_f32(bias_bits).astype(np.float64)[None, :]
    return f32_to_bf16_bits(y.astype(np.float32))


def nf4_linear_bf16(x_bits, packed, absmax, n, k, bias_bits=None) -> np.ndarray:
    """ltx23_nf4_linear$forward in bf16 (R/nf4_ltx23.R:235-246)."""
    w = nf4_dequantize_bf16_bits(packed, absmax).reshape(n, k)
    return linear_bf16(np.asarray(x_bits).reshape(-1, k), w, bias_bits)


def fp8_linear_bf16(x_bits, w8, scale, n, k, bias_bits=None) -> np.ndarray:
    """ltx23_fp8_linear$forward in bf16 (R/fp8_ltx23.R:70-83)."""
    w = fp8_dequantize_bf16_bits(w8, scale).reshape(n, k)
    return linear_bf16(np.asarray(x_bits).reshape(-1, k), w, bias_bits)


def gated_bf16(y_bits, act="swiglu") -> np.ndarray:
    """The gated activation of a [gate; up] projection in bf16, as the
    reference's tensor chain rounds it (R/dit_flux2_modules.R:80-83:
    nnf_silu(x$narrow(-1, 1, half)) * x$narrow(-1, half + 1, half)): the
    activation of the bf16 gate computed in float32 (SiLU x / (1 + e^-x);
    for "geglu_tanh" GELU with the tanh approximation) rounded to bf16, then
    the bf16 product rounded to bf16.  y_bits [M, 2H] -> bits [M, H]."""
    y = bf16_bits_to_f32(y_bits)
    h = y.shape[-1] // 2
    g = y[..., :h].astype(np.float32)
    u = y[..., h:].astype(np.float32)
    if act == "swiglu":
        a = g / (np.float32(1) + np.exp(-g))
    elif act == "geglu_tanh":
        a = np.float32(0.5) * g * (np.float32(1) + np.tanh(
            np.float32(0.7978845608028654) * (g + np.float32(0.044715) * g * g * g)))
    else:
        raise ValueError(act)
    a = bf16_bits_to_f32(f32_to_bf16_bits(a.astype(np.float32)))
    return f32_to_bf16_bits((a * u).astype(np.float32))


def rel_err(y_bits, ref_bits) -> float:
    """max|y - ref| / max|ref| -- the norm used for the 1e-2 GEMM tolerance."""
    y = bf16_bits_to_f32(y_bits).astype(np.float64)
    r = bf16_bits_to_f32(ref_bits).astype(np.float64)
    return float(np.abs(y - r).max() / max(np.abs(r).max(), 1e-30))
