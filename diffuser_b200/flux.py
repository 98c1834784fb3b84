"""FLUX.1 DiT on the quantized-linear engine: the consumer of the hot path.

A PyTorch restatement of the reference's FLUX transformer (R/dit_flux.R:43-150,
R/dit_flux_modules.R:26-321, the LTX primitives it reuses in
R/dit_ltx23_modules.R:25-105,500-526), rotary embedding (R/rope_flux.R:28-114),
latent packing (R/txt2img_flux.R:21-31) and the flow-match Euler step
(R/flowmatch_scheduler.R:236-264).  Module names follow the diffusers state
dict exactly as the reference's do, so one checkpoint loads into both.  The 494
cast-set linears (R/checkpoint_flux.R:21-42) become fused NF4 linears through
``modules.swap_quant_linears``; attention runs on torch's fused SDPA.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib, modules


# ------------------------------------------------------ fused attention glue
def _fused_ok(x, dim_head: int) -> bool:
    """The CUDA prologue / epilogue kernels serve bf16 CUDA tensors with a head
    dimension that is a multiple of 64 (FLUX: 128); other cases (the float32
    CPU fixture model) take the tensor-op path."""
    return x.is_cuda and x.dtype == torch.bfloat16 and dim_head % 64 == 0 and dim_head <= 256


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def qk_norm_rope(img, txt, heads: int, w_img=None, w_txt=None, rope=None, eps: float = 1e-6):
    """Per-head RMS norm + [text; image] concatenation + transpose + rotary
    embedding in one kernel: img [B, S_img, H*D] (and txt [B, S_txt, H*D]) ->
    [B, H, S_txt + S_img, D] bf16."""
    b, s_img, hd = img.shape
    d = hd // heads
    s_txt = 0 if txt is None else txt.shape[1]
    img = img if img.stride(-1) == 1 else img.contiguous()
    if txt is not None and txt.stride(-1) != 1:
        txt = txt.contiguous()
    out = torch.empty((b, heads, s_txt + s_img, d), dtype=torch.bfloat16, device=img.device)
    cos = sin = None
    if rope is not None:
        cos, sin = rope[0].contiguous(), rope[1].contiguous()
    stream = ctypes.c_void_p(torch.cuda.current_stream(img.device).cuda_stream)
    rc = _lib.lib().dq_qk_norm_rope(
        _ptr(img), img.stride(1), _ptr(txt), 0 if txt is None else txt.stride(1), b, s_img, s_txt,
        heads, d, _ptr(w_img), _ptr(w_txt), _ptr(cos), _ptr(sin), ctypes.c_float(eps), _ptr(out), stream)
    _lib.check("dq_qk_norm_rope", rc)
    return out


def qkv_norm_rope(parts_img, parts_txt, heads: int, norms_img, norms_txt, ropes, rope=None,
                  eps: float = 1e-6):
    """qk_norm_rope for up to three tensors (q, k, v) of one attention in one
    launch: part p reads parts_img[p] (and parts_txt[p]), normalizes with
    norms_img[p] / norms_txt[p] when given, rotates when ropes[p] is set, and
    returns its own [B, H, S_txt + S_img, D] tensor -- the same bits as one
    qk_norm_rope call per part."""
    n = len(parts_img)
    b, s_img, hd = parts_img[0].shape
    d = hd // heads
    s_txt = 0 if parts_txt[0] is None else parts_txt[0].shape[1]
    imgs = [t if t.stride(-1) == 1 else t.contiguous() for t in parts_img]
    txts = [None if t is None else (t if t.stride(-1) == 1 else t.contiguous()) for t in parts_txt]
    outs = [torch.empty((b, heads, s_txt + s_img, d), dtype=torch.bfloat16, device=imgs[0].device)
            for _ in range(n)]
    cos = sin = None
    if rope is not None:
        cos, sin = rope[0].contiguous(), rope[1].contiguous()
    P = ctypes.c_void_p * n
    L = ctypes.c_int64 * n
    stream = ctypes.c_void_p(torch.cuda.current_stream(imgs[0].device).cuda_stream)
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    rc = _lib.lib().dq_qkv_norm_rope(
        n, P(*[ptr(t) for t in imgs]), L(*[t.stride(1) for t in imgs]),
        P(*[ptr(t) for t in txts]) if s_txt else None,
        L(*[0 if t is None else t.stride(1) for t in txts]) if s_txt else None,
        b, s_img, s_txt, heads, d, P(*[ptr(w) for w in norms_img]), P(*[ptr(w) for w in norms_txt]),
        (ctypes.c_int * n)(*[1 if r else 0 for r in ropes]), _ptr(cos), _ptr(sin), ctypes.c_float(eps),
        P(*[t.data_ptr() for t in outs]), stream)
    _lib.check("dq_qkv_norm_rope", rc)
    return outs


def heads_to_tokens(x, s_txt: int, img_out=None):
    """[B, H, S_txt + S_img, D] -> (txt [B, S_txt, H*D] or None, img [B, S_img, H*D]);
    img_out, if given, is a [B, S_img, H*D] view (e.g. the first columns of a
    wider buffer) that receives the image tokens."""
    b, h, s, d = x.shape
    x = x if x.is_contiguous() else x.contiguous()
    s_img = s - s_txt
    if img_out is None:
        img = torch.empty((b, s_img, h * d), dtype=torch.bfloat16, device=x.device)
        ld_img = h * d
    else:
        img, ld_img = _rows(img_out)
        if img.data_ptr() != img_out.data_ptr():
            raise ValueError("img_out must have evenly spaced rows with unit feature stride")
    txt = torch.empty((b, s_txt, h * d), dtype=torch.bfloat16, device=x.device) if s_txt else None
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    rc = _lib.lib().dq_heads_to_tokens_ld(_ptr(x), b, h, s_txt, s_img, d, _ptr(txt), h * d,
                                          _ptr(img), ld_img, stream)
    _lib.check("dq_heads_to_tokens_ld", rc)
    return txt, img


# AdaLN modulation and gated residuals as one kernel each (False: the
# reference's chain of tensor ops).
FUSED_ADALN = True
# q/k/v projections through one concatenated NF4 linear where fuse_qkv_projections
# built it (False: three linears, as the reference calls them).
FUSED_QKV = True
# Single blocks: attention and MLP outputs written into the two column ranges
# of proj_out's input (False: torch.cat of the two, as the reference does).
FUSED_CONCAT = True


def _rows(t):
    """(tensor, row stride) with unit stride along the last dim and rows of a
    [B, S, D] tensor evenly spaced; copies only when they are not."""
    if t.stride(-1) != 1 or (t.dim() == 3 and t.stride(0) != t.shape[1] * t.stride(1)):
        t = t.contiguous()
    return t, t.stride(-2)


def adaln_modulate(x, scale, shift, eps: float = 1e-6):
    """LayerNorm(x) * (1 + scale[:, None]) + shift[:, None] for x [B, S, D]
    bf16, scale / shift [B, D], rounded to bf16 after each op like the tensor
    chain (R/dit_flux_modules.R:26-42), in one kernel."""
    b, s, d = x.shape
    x, ldx = _rows(x)
    scale, ldm = _rows(scale)
    shift, ldm2 = _rows(shift)
    if ldm2 != ldm:
        scale, shift = scale.contiguous(), shift.contiguous()
        ldm = d
    out = torch.empty((b, s, d), dtype=torch.bfloat16, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    rc = _lib.lib().dq_adaln_modulate(_ptr(x), ldx, b * s, s, d, _ptr(scale), _ptr(shift), ldm,
                                      ctypes.c_float(eps), _ptr(out), d, stream)
    _lib.check("dq_adaln_modulate", rc)
    return out


def gated_residual(x, gate, y):
    """x + gate[:, None] * y for x, y [B, S, D] bf16 and gate [B, D], rounded
    like the two tensor ops, in one kernel."""
    b, s, d = x.shape
    x, ldx = _rows(x)
    y, ldy = _rows(y)
    gate, ldm = _rows(gate)
    out = torch.empty((b, s, d), dtype=torch.bfloat16, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    rc = _lib.lib().dq_gated_residual(_ptr(x), ldx, _ptr(gate), ldm, _ptr(y), ldy, b * s, s, d,
                                      _ptr(out), d, stream)
    _lib.check("dq_gated_residual", rc)
    return out


def _adaln_ok(x):
    return FUSED_ADALN and x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 3 and x.shape[-1] % 4 == 0


def _modulate(norm, x, scale, shift):
    if _adaln_ok(x) and norm.weight is None and norm.bias is None:
        return adaln_modulate(x, scale, shift, norm.eps)
    return norm(x) * (scale[:, None] + 1) + shift[:, None]


def _gated_add(x, gate, y):
    if _adaln_ok(x) and y.shape == x.shape:
        return gated_residual(x, gate, y)
    return x + gate[:, None] * y


# GELU-tanh after the up-projections runs in the quantized linear's epilogue
# (False: a separate activation pass, as the reference does).
FUSED_GELU = True


def _proj_gelu_tanh(proj, x, out=None):
    """GELU-tanh of a projection; fused into the quantized linear's epilogue on
    the engine (the projection is still rounded to bf16 before the activation).
    With `out` the result is written there."""
    if FUSED_GELU and isinstance(proj, (modules.Ltx23Nf4Linear, modules.Ltx23Fp8Linear)) and x.is_cuda:
        if out is None:  # forwards that predate `out` keep working
            return proj(x, act="gelu_tanh")
        return proj(x, act="gelu_tanh", out=out)
    y = F.gelu(proj(x), approximate="tanh")
    if out is None:
        return y
    out.copy_(y)
    return out


# --------------------------------------------------------------- primitives
class RMSNorm(nn.Module):
    """ltx23_rms_norm (R/dit_ltx23_modules.R:25-46): normalize in float32, then
    cast to the weight dtype and scale."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        variance = x.to(torch.float32).pow(2).mean(dim=-1, keepdim=True)
        x = x * torch.rsqrt(variance + self.eps)
        return x.to(self.weight.dtype) * self.weight


def timestep_sinusoid(timesteps, dim: int, flip_sin_to_cos=True, downscale_freq_shift=0.0,
                      max_period=10000.0):
    """ltx23_get_timestep_embedding (R/dit_ltx23_modules.R:62-88)."""
    half = dim // 2
    exponent = -math.log(max_period) * torch.arange(0, half, dtype=torch.float32,
                                                    device=timesteps.device)
    exponent = exponent / (half - downscale_freq_shift)
    emb = timesteps[:, None].to(torch.float32) * torch.exp(exponent)[None, :]
    emb = torch.cat([torch.sin(emb), torch.cos(emb)], dim=-1)
    if flip_sin_to_cos:
        emb = torch.cat([emb[:, half:], emb[:, :half]], dim=-1)
    if dim % 2 == 1:
        emb = F.pad(emb, (0, 1, 0, 0))
    return emb


class TimestepEmbedding(nn.Module):
    """linear_1 -> silu -> linear_2 (R/dit_ltx23_modules.R:91-100)."""

    def __init__(self, in_channels: int, dim: int):
        super().__init__()
        self.linear_1 = nn.Linear(in_channels, dim)
        self.linear_2 = nn.Linear(dim, dim)

    def forward(self, x):
        return self.linear_2(F.silu(self.linear_1(x)))


class TimeTextEmbed(nn.Module):
    """flux_time_text_embed (R/dit_flux.R:17-31)."""

    def __init__(self, dim: int, pooled_dim: int):
        super().__init__()
        self.timestep_embedder = TimestepEmbedding(256, dim)
        self.text_embedder = TimestepEmbedding(pooled_dim, dim)

    def forward(self, timestep, pooled):
        proj = timestep_sinusoid(timestep, 256, flip_sin_to_cos=True, downscale_freq_shift=0)
        return self.timestep_embedder(proj.to(pooled.dtype)) + self.text_embedder(pooled)


class GeluProj(nn.Module):
    def __init__(self, dim_in: int, dim_out: int):
        super().__init__()
        self.proj = nn.Linear(dim_in, dim_out)

    def forward(self, x):
        return _proj_gelu_tanh(self.proj, x)


class FeedForward(nn.Module):
    """ltx23_feed_forward (R/dit_ltx23_modules.R:500-526): net.0 = GELU-tanh
    projection, net.1 = dropout slot (identity), net.2 = down projection."""

    def __init__(self, dim: int, mult: int = 4):
        super().__init__()
        inner = dim * mult
        self.net = nn.ModuleList([GeluProj(dim, inner), nn.Identity(), nn.Linear(inner, dim)])

    def forward(self, x):
        return self.net[2](self.net[0](x))


class AdaLayerNormZero(nn.Module):
    """flux_ada_layer_norm_zero (R/dit_flux_modules.R:26-42)."""

    def __init__(self, dim: int):
        super().__init__()
        self.linear = nn.Linear(dim, 6 * dim)
        self.norm = nn.LayerNorm(dim, eps=1e-6, elementwise_affine=False)

    def forward(self, x, emb):
        p = self.linear(F.silu(emb)).chunk(6, dim=1)
        x = _modulate(self.norm, x, p[1], p[0])
        return x, p[2], p[3], p[4], p[5]


class AdaLayerNormZeroSingle(nn.Module):
    """flux_ada_layer_norm_zero_single (R/dit_flux_modules.R:54-70)."""

    def __init__(self, dim: int):
        super().__init__()
        self.linear = nn.Linear(dim, 3 * dim)
        self.norm = nn.LayerNorm(dim, eps=1e-6, elementwise_affine=False)

    def forward(self, x, emb):
        p = self.linear(F.silu(emb)).chunk(3, dim=1)
        return _modulate(self.norm, x, p[1], p[0]), p[2]


class AdaLayerNormContinuous(nn.Module):
    """flux_ada_layer_norm_continuous (R/dit_flux_modules.R:87-103): scale
    first, then shift."""

    def __init__(self, dim: int, cond_dim: int):
        super().__init__()
        self.linear = nn.Linear(cond_dim, 2 * dim)
        self.norm = nn.LayerNorm(dim, eps=1e-6, elementwise_affine=False)

    def forward(self, x, cond):
        scale, shift = self.linear(F.silu(cond).to(x.dtype)).chunk(2, dim=1)
        return self.norm(x) * (scale[:, None] + 1) + shift[:, None]


# ------------------------------------------------------------------- rotary
def prepare_latent_image_ids(height: int, width: int, device=None):
    """flux_prepare_latent_image_ids (R/rope_flux.R:28-40): (0, row, col)."""
    ids = torch.zeros(height, width, 3, dtype=torch.float32, device=device)
    ids[..., 1] += torch.arange(height, dtype=torch.float32, device=device)[:, None]
    ids[..., 2] += torch.arange(width, dtype=torch.float32, device=device)[None, :]
    return ids.reshape(height * width, 3)


def pos_embed(ids, axes_dim=(16, 56, 56), theta=10000.0):
    """flux_pos_embed (R/rope_flux.R:56-85): per-axis frequencies in float64
    on the host, cos/sin repeated pairwise, returned as float32 on ids' device."""
    pos = ids.to(device="cpu", dtype=torch.float64)
    cos_out, sin_out = [], []
    for i, d in enumerate(axes_dim):
        freqs = 1.0 / torch.pow(theta, torch.arange(0, d, 2, dtype=torch.float64) / d)
        f = pos[:, i][:, None] * freqs[None, :]
        cos_out.append(f.cos().repeat_interleave(2, dim=1))
        sin_out.append(f.sin().repeat_interleave(2, dim=1))
    return (torch.cat(cos_out, dim=-1).to(dtype=torch.float32, device=ids.device),
            torch.cat(sin_out, dim=-1).to(dtype=torch.float32, device=ids.device))


def apply_rotary_emb(x, freqs):
    """flux_apply_rotary_emb (R/rope_flux.R:96-110); x [B, H, S, D]."""
    cos = freqs[0][None, None]
    sin = freqs[1][None, None]
    pairs = x.unflatten(-1, (-1, 2))
    rotated = torch.stack([-pairs[..., 1], pairs[..., 0]], dim=-1).flatten(3)
    out = x.to(torch.float32) * cos + rotated.to(torch.float32) * sin
    return out.to(x.dtype)


# ---------------------------------------------------------------- attention
class FluxAttention(nn.Module):
    """flux_attention (R/dit_flux_modules.R:127-213)."""

    def __init__(self, dim: int, heads: int, dim_head: int, added_kv=False, pre_only=False):
        super().__init__()
        inner = heads * dim_head
        self.heads = heads
        self.pre_only = pre_only
        self.norm_q = RMSNorm(dim_head)
        self.norm_k = RMSNorm(dim_head)
        self.to_q = nn.Linear(dim, inner)
        self.to_k = nn.Linear(dim, inner)
        self.to_v = nn.Linear(dim, inner)
        if not pre_only:
            self.to_out = nn.ModuleList([nn.Linear(inner, dim)])
        self.added_kv = added_kv
        if added_kv:
            self.norm_added_q = RMSNorm(dim_head)
            self.norm_added_k = RMSNorm(dim_head)
            self.add_q_proj = nn.Linear(dim, inner)
            self.add_k_proj = nn.Linear(dim, inner)
            self.add_v_proj = nn.Linear(dim, inner)
            self.to_add_out = nn.Linear(inner, dim)

    def forward(self, x, ctx=None, rope=None, out=None):
        h = self.heads
        if _fused_ok(x, self.norm_q.weight.shape[0]):
            return self._forward_fused(x, ctx, rope, out)
        q = self.norm_q(self.to_q(x).unflatten(-1, (h, -1)))
        k = self.norm_k(self.to_k(x).unflatten(-1, (h, -1)))
        v = self.to_v(x).unflatten(-1, (h, -1))
        txt_len = 0
        if ctx is not None:
            txt_len = ctx.shape[1]
            eq = self.norm_added_q(self.add_q_proj(ctx).unflatten(-1, (h, -1)))
            ek = self.norm_added_k(self.add_k_proj(ctx).unflatten(-1, (h, -1)))
            ev = self.add_v_proj(ctx).unflatten(-1, (h, -1))
            q = torch.cat([eq, q], dim=1)  # text tokens first
            k = torch.cat([ek, k], dim=1)
            v = torch.cat([ev, v], dim=1)
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if rope is not None:
            q = apply_rotary_emb(q, rope)
            k = apply_rotary_emb(k, rope)
        out = F.scaled_dot_product_attention(q, k, v, dropout_p=0.0, is_causal=False)
        out = out.transpose(1, 2).flatten(2).to(x.dtype)
        if ctx is not None:
            img = out[:, txt_len:].contiguous()
            txt = out[:, :txt_len].contiguous()
            return self.to_out[0](img), self.to_add_out(txt)
        if self.pre_only:
            return out
        return self.to_out[0](out)

    @staticmethod
    def _qkv(x, fused, q_proj, k_proj, v_proj):
        """q, k, v projections of x: one concatenated NF4 linear (column views
        of its output, read in place by the attention glue) or three."""
        if FUSED_QKV and fused is not None:
            y = fused(x)
            n = q_proj.out_features
            return y[..., :n], y[..., n:2 * n], y[..., 2 * n:]
        return q_proj(x), k_proj(x), v_proj(x)

    def _forward_fused(self, x, ctx, rope, out=None):
        """The same computation with the norm / concat / transpose / rotary
        chain in one kernel per tensor and the split back in one more."""
        h = self.heads
        q_t = k_t = v_t = None
        wq_t = wk_t = None
        if ctx is not None:
            q_t, k_t, v_t = self._qkv(ctx, getattr(self, "add_qkv", None), self.add_q_proj,
                                      self.add_k_proj, self.add_v_proj)
            wq_t, wk_t = self.norm_added_q.weight, self.norm_added_k.weight
        q_i, k_i, v_i = self._qkv(x, getattr(self, "to_qkv", None), self.to_q, self.to_k, self.to_v)
        if self.norm_q.eps == self.norm_k.eps:
            q, k, v = qkv_norm_rope((q_i, k_i, v_i), (q_t, k_t, v_t), h,
                                    (self.norm_q.weight, self.norm_k.weight, None), (wq_t, wk_t, None),
                                    (rope is not None, rope is not None, False), rope, self.norm_q.eps)
        else:
            q = qk_norm_rope(q_i, q_t, h, self.norm_q.weight, wq_t, rope, self.norm_q.eps)
            k = qk_norm_rope(k_i, k_t, h, self.norm_k.weight, wk_t, rope, self.norm_k.eps)
            v = qk_norm_rope(v_i, v_t, h)
        att = F.scaled_dot_product_attention(q, k, v, dropout_p=0.0, is_causal=False)
        txt_len = 0 if ctx is None else ctx.shape[1]
        # `out` (pre-only attention): the image tokens go straight there
        txt, img = heads_to_tokens(att, txt_len, out if (self.pre_only and ctx is None) else None)
        if ctx is not None:
            return self.to_out[0](img), self.to_add_out(txt)
        if self.pre_only:
            return img
        return self.to_out[0](img)


class DoubleBlock(nn.Module):
    """flux_double_block (R/dit_flux_modules.R:230-274)."""

    def __init__(self, dim: int, heads: int, dim_head: int):
        super().__init__()
        self.norm1 = AdaLayerNormZero(dim)
        self.norm1_context = AdaLayerNormZero(dim)
        self.attn = FluxAttention(dim, heads, dim_head, added_kv=True)
        self.norm2 = nn.LayerNorm(dim, eps=1e-6, elementwise_affine=False)
        self.ff = FeedForward(dim)
        self.norm2_context = nn.LayerNorm(dim, eps=1e-6, elementwise_affine=False)
        self.ff_context = FeedForward(dim)

    def forward(self, x, ctx, temb, rope):
        nx, g_msa, sh_mlp, sc_mlp, g_mlp = self.norm1(x, temb)
        nc, cg_msa, csh_mlp, csc_mlp, cg_mlp = self.norm1_context(ctx, temb)
        a_img, a_txt = self.attn(nx, nc, rope)
        x = _gated_add(x, g_msa, a_img)
        x = _gated_add(x, g_mlp, self.ff(_modulate(self.norm2, x, sc_mlp, sh_mlp)))
        ctx = _gated_add(ctx, cg_msa, a_txt)
        ctx = _gated_add(ctx, cg_mlp, self.ff_context(
            _modulate(self.norm2_context, ctx, csc_mlp, csh_mlp)))
        if ctx.dtype == torch.float16:
            ctx = ctx.clamp(-65504, 65504)
        return ctx, x


class SingleBlock(nn.Module):
    """flux_single_block (R/dit_flux_modules.R:296-321)."""

    def __init__(self, dim: int, heads: int, dim_head: int, mlp_ratio: float = 4.0):
        super().__init__()
        hidden = int(dim * mlp_ratio)
        self.norm = AdaLayerNormZeroSingle(dim)
        self.proj_mlp = nn.Linear(dim, hidden)
        self.proj_out = nn.Linear(dim + hidden, dim)
        self.attn = FluxAttention(dim, heads, dim_head, pre_only=True)

    def forward(self, x, temb, rope):
        n, gate = self.norm(x, temb)
        if FUSED_CONCAT and _fused_ok(n, self.attn.norm_q.weight.shape[0]) and \
                isinstance(self.proj_mlp, (modules.Ltx23Nf4Linear, modules.Ltx23Fp8Linear)):
            # attention and MLP outputs land in the two column ranges of the
            # proj_out input, which is then read whole (no concatenation pass)
            d_attn = self.attn.to_q.out_features
            cat = torch.empty(*n.shape[:-1], d_attn + self.proj_mlp.out_features,
                              dtype=torch.bfloat16, device=n.device)
            _proj_gelu_tanh(self.proj_mlp, n, out=cat[..., d_attn:])
            self.attn(n, rope=rope, out=cat[..., :d_attn])
            return _gated_add(x, gate, self.proj_out(cat))
        mlp = _proj_gelu_tanh(self.proj_mlp, n)
        a = self.attn(n, rope=rope)
        x = _gated_add(x, gate, self.proj_out(torch.cat([a, mlp], dim=2)))
        if x.dtype == torch.float16:
            x = x.clamp(-65504, 65504)
        return x


class FluxTransformer(nn.Module):
    """flux_transformer (R/dit_flux.R:43-150); defaults = FLUX.1 (schnell)."""

    def __init__(self, in_channels=64, num_layers=19, num_single_layers=38, attention_head_dim=128,
                 num_attention_heads=24, joint_attention_dim=4096, pooled_projection_dim=768,
                 axes_dims_rope=(16, 56, 56), out_channels=None):
        super().__init__()
        dim = num_attention_heads * attention_head_dim
        self.inner_dim = dim
        self.axes_dims_rope = tuple(axes_dims_rope)
        self.out_channels = out_channels or in_channels
        self.time_text_embed = TimeTextEmbed(dim, pooled_projection_dim)
        self.context_embedder = nn.Linear(joint_attention_dim, dim)
        self.x_embedder = nn.Linear(in_channels, dim)
        self.transformer_blocks = nn.ModuleList(
            [DoubleBlock(dim, num_attention_heads, attention_head_dim) for _ in range(num_layers)])
        self.single_transformer_blocks = nn.ModuleList(
            [SingleBlock(dim, num_attention_heads, attention_head_dim) for _ in range(num_single_layers)])
        self.norm_out = AdaLayerNormContinuous(dim, dim)
        self.proj_out = nn.Linear(dim, self.out_channels)

    def forward(self, hidden_states, encoder_hidden_states, pooled_projections, timestep, rope):
        x = self.x_embedder(hidden_states)
        t = timestep.to(x.dtype) * 1000
        temb = self.time_text_embed(t, pooled_projections)
        ctx = self.context_embedder(encoder_hidden_states)
        for blk in self.transformer_blocks:
            ctx, x = blk(x, ctx, temb, rope)
        txt_len = ctx.shape[1]
        x = torch.cat([ctx, x], dim=1)
        for blk in self.single_transformer_blocks:
            x = blk(x, temb, rope)
        x = x[:, txt_len:]
        return self.proj_out(self.norm_out(x, temb))


# ------------------------------------------------------------ latents, steps
def pack_latents(latents):
    """flux_pack_latents (R/txt2img_flux.R:21-31): [B, C, H, W] ->
    [B, (H/2)(W/2), 4C]."""
    b, c, h, w = latents.shape
    x = latents.view(b, c, h // 2, 2, w // 2, 2).permute(0, 2, 4, 1, 3, 5)
    return x.reshape(b, (h // 2) * (w // 2), c * 4)


def unpack_latents(x, height: int, width: int, channels: int):
    """Inverse of pack_latents (R/txt2img_flux.R:44-56)."""
    b = x.shape[0]
    x = x.view(b, height // 2, width // 2, channels, 2, 2).permute(0, 3, 1, 4, 2, 5)
    return x.reshape(b, channels, height, width)


def euler_step(v, sigma: float, sigma_next: float, sample):
    """flowmatch_scheduler_step (R/flowmatch_scheduler.R:236-264): float32
    update, cast back to the model dtype."""
    return (sample.to(torch.float32) + (sigma_next - sigma) * v).to(v.dtype)


def sample(model, latents_packed, text_states, pooled, rope, sigmas):
    """Euler flow-match loop over `sigmas` (a trailing 0 is appended)."""
    x = latents_packed
    sig = list(sigmas) + [0.0]
    for i in range(len(sigmas)):
        t = torch.full((x.shape[0],), sig[i], dtype=torch.float32, device=x.device)
        v = model(x, text_states, pooled, t, rope)
        x = euler_step(v, sig[i], sig[i + 1], x)
    return x


# ------------------------------------------------------ full-size random model
def init_random_(model: nn.Module, seed: int = 0, std: float = 0.02):
    """Linear weights ~ N(0, std), biases 0, norm weights 1 (the synthetic
    FLUX configuration), from one seeded generator on the model's device."""
    dev = next(model.parameters()).device
    g = torch.Generator(device=dev).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm_q.weight") or name.endswith("norm_k.weight") or \
                    name.endswith("norm_added_q.weight") or name.endswith("norm_added_k.weight"):
                p.fill_(1.0)
            elif name.endswith(".bias"):
                p.zero_()
            else:
                p.copy_(torch.randn(p.shape, generator=g, device=dev, dtype=torch.float32) * std)
    return model


def concat_nf4_linears(mods):
    """modules.concat_nf4_linears: NF4 rows are contiguous byte ranges, so
    concatenating the buffers concatenates the rows (q/k/v of one stream)."""
    return modules.concat_nf4_linears(mods)


def fuse_qkv_projections(model):
    """Give every attention of `model` a concatenated q/k/v NF4 linear per
    stream (``to_qkv``, and ``add_qkv`` for the text stream): one wider GEMM
    instead of three, its output read in place by the attention glue.  The
    separate projections stay (the tensor-op path and the reference-algorithm
    timing use them)."""
    attns = [m for m in model.modules() if isinstance(m, FluxAttention)]
    for a in attns:
        f = concat_nf4_linears([a.to_q, a.to_k, a.to_v])
        if f is not None:
            a.to_qkv = f
        if a.added_kv:
            f = concat_nf4_linears([a.add_q_proj, a.add_k_proj, a.add_v_proj])
            if f is not None:
                a.add_qkv = f
    return model


def build_flux_nf4(device="cuda", seed: int = 0, fuse_qkv: bool = True, **config) -> FluxTransformer:
    """FLUX.1 transformer in bf16 with random weights and its 494 cast-set
    linears replaced by fused NF4 linears (R/quantize_flux.R:541-576); with
    fuse_qkv each attention also gets its concatenated q/k/v linears."""
    with torch.device(device):
        model = FluxTransformer(**config).to(torch.bfloat16)
    init_random_(model, seed)
    modules.swap_quant_linears(model, modules.flux_is_quant_key, "nf4")
    if fuse_qkv:
        fuse_qkv_projections(model)
    torch.cuda.empty_cache()
    return model.eval()
