"""Drop-in module mirrors of diffuseR's quantized linears.

``ltx23_nf4_linear`` / ``ltx23_fp8_linear`` keep the reference's constructor,
setters, buffers and forward contract (R/nf4_ltx23.R:211-247,
R/fp8_ltx23.R:49-84), with forward() running the fused sm_100a kernel instead
of dequantize-into-a-buffer + cuBLAS.  ``swap_quant_linears`` mirrors the
loader swap ``do.call(`$<-`, list(parent, leaf, quant_mod))``
(R/quantize_flux.R:541-576).
"""
from __future__ import annotations

import re

import torch
from torch import nn

from . import ops

NF4_BLOCK = ops.NF4_BLOCK


class Ltx23Nf4Linear(nn.Module):
    """NF4 linear (R/nf4_ltx23.R:211-247).

    Buffers ``weight_nf4`` (uint8 [N*K/2]) and ``weight_absmax`` (float32
    [N*K/64]) move with the module; uint8 survives dtype casts and absmax is
    kept float32 (the forward uses bf16(absmax), which a cast would not change).
    """

    def __init__(self, out_features: int, in_features: int, bias: bool = True):
        super().__init__()
        self.out_features = int(out_features)
        self.in_features = int(in_features)
        n = self.out_features * self.in_features
        self.register_buffer("weight_nf4", torch.zeros(n // 2, dtype=torch.uint8))
        self.register_buffer("weight_absmax", torch.ones(n // NF4_BLOCK, dtype=torch.float32))
        self.scales_bf16 = False
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)
        self.gated_act = None

    def set_nf4_weight(self, packed: torch.Tensor, absmax: torch.Tensor):
        """Copy packed codes and block scales into the buffers (R/nf4_ltx23.R:228-234)."""
        with torch.no_grad():
            self.weight_nf4.copy_(packed.reshape(-1))
            self.weight_absmax.copy_(absmax.reshape(-1))
        return self

    def _apply(self, fn, recurse=True):
        super()._apply(fn, recurse)
        want = torch.bfloat16 if getattr(self, "scales_bf16", False) else torch.float32
        if self.weight_absmax.dtype != want:
            self.weight_absmax = self.weight_absmax.to(want)
        return self

    def repack_scales_bf16(self):
        """Load-time repack of the block scales to bf16 (half the scale
        bytes).  The forward casts absmax to bf16 before scaling
        (R/nf4_ltx23.R:97), so the dequantized weights are unchanged."""
        self.weight_absmax = self.weight_absmax.to(torch.bfloat16)
        self.scales_bf16 = True
        return self

    def to_gated(self, act: str = "swiglu"):
        """Reorder the rows of a [gate; up] projection into the gated row
        order and fuse `act` ("swiglu": silu(gate) * up, "geglu_tanh") into
        every forward, which then returns out_features / 2 columns."""
        if act not in ops.GATED_ACTS:
            raise ValueError(f"act must be one of {ops.GATED_ACTS}")
        with torch.no_grad():
            p, a = ops.to_gated_rows_nf4(self.weight_nf4, self.weight_absmax, self.out_features,
                                         self.in_features)
            self.weight_nf4.copy_(p)
            self.weight_absmax.copy_(a)
            if self.bias is not None:
                self.bias.copy_(ops.to_gated_rows(self.bias.detach(), self.out_features))
        self.gated_act = act
        return self

    def forward(self, x: torch.Tensor, act: str | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        return ops.nf4_linear(x, self.weight_nf4, self.weight_absmax, self.out_features, self.bias,
                              act=act or self.gated_act, out=out)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, format=nf4"


class Ltx23Fp8Linear(nn.Module):
    """fp8-e4m3 linear with a per-tensor scale (R/fp8_ltx23.R:49-84).

    As in the reference, the fp8 weight and its scale are plain attributes, not
    buffers, so ``.to()`` moves only the bias.  The reference streams them to
    the device on every forward; here the first forward on a device copies them
    once and keeps that copy resident (B200 holds every weight in HBM).
    """

    def __init__(self, out_features: int, in_features: int, bias: bool = True):
        super().__init__()
        self.out_features = int(out_features)
        self.in_features = int(in_features)
        self.weight_fp8 = None
        self.weight_scale = None
        self._resident = None
        self._scale_f = None
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)
        self.gated_act = None

    def set_fp8_weight(self, weight: torch.Tensor, scale, pin: bool = False):
        """Store the e4m3 weight and float32 scale (R/fp8_ltx23.R:60-68)."""
        if weight.dtype != torch.float8_e4m3fn:
            raise TypeError("weight must be float8_e4m3fn")
        if pin and not weight.is_cuda and torch.cuda.is_available():
            weight = weight.pin_memory()
        self.weight_fp8 = weight
        scale_t = torch.as_tensor(scale).detach().to(device="cpu", dtype=torch.float32)
        self.weight_scale = scale_t
        self._scale_f = float(scale_t)
        self._resident = weight if weight.is_cuda else None
        return self

    def to_gated(self, act: str = "swiglu"):
        """As Ltx23Nf4Linear.to_gated: rows into the gated row order, `act`
        fused into every forward (out_features / 2 output columns)."""
        if act not in ops.GATED_ACTS:
            raise ValueError(f"act must be one of {ops.GATED_ACTS}")
        if self.weight_fp8 is None:
            raise RuntimeError("set_fp8_weight() has not been called")
        self.weight_fp8 = ops.to_gated_rows(self.weight_fp8, self.out_features)
        self._resident = self.weight_fp8 if self.weight_fp8.is_cuda else None
        if self.bias is not None:
            with torch.no_grad():
                self.bias.copy_(ops.to_gated_rows(self.bias.detach(), self.out_features))
        self.gated_act = act
        return self

    def forward(self, x: torch.Tensor, act: str | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        act = act or self.gated_act
        if self.weight_fp8 is None:
            raise RuntimeError("set_fp8_weight() has not been called")
        w8 = self._resident
        if w8 is None or w8.device != x.device:
            w8 = self.weight_fp8.to(device=x.device, non_blocking=True)
            self._resident = w8
        return ops.fp8_linear(x, w8, self._scale_f, self.bias, act=act, out=out)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, format=fp8"


def concat_nf4_linears(mods):
    """One NF4 linear whose output features are those of `mods`, in order.
    NF4 blocks of 64 never straddle a weight row, so a row range's packed codes
    and block scales are contiguous: concatenating the buffers concatenates
    the rows, with no repacking.  None unless every module is NF4 with the same
    in_features and scale dtype."""
    if not mods or any(not isinstance(m, Ltx23Nf4Linear) for m in mods):
        return None
    k = mods[0].in_features
    if any(m.in_features != k or m.weight_absmax.dtype != mods[0].weight_absmax.dtype for m in mods):
        return None
    dev = mods[0].weight_nf4.device
    fused = Ltx23Nf4Linear(sum(m.out_features for m in mods), k, bias=False).to(dev)
    if mods[0].scales_bf16:
        fused.repack_scales_bf16()
    fused.set_nf4_weight(torch.cat([m.weight_nf4 for m in mods]),
                         torch.cat([m.weight_absmax for m in mods]))
    if any(m.bias is not None for m in mods):
        dt = next(m.bias.dtype for m in mods if m.bias is not None)
        fused.bias = nn.Parameter(torch.cat([
            m.bias.detach().to(dt) if m.bias is not None
            else torch.zeros(m.out_features, dtype=dt, device=dev) for m in mods]), requires_grad=False)
    return fused


def fuse_gated_pair(gate: nn.Module, up: nn.Module, act: str = "geglu_tanh"):
    """One NF4 linear computing act(gate(x)) * up(x) with the gate fused into
    its epilogue (the gated MLP of a Gemma-style text encoder, whose gate_proj
    and up_proj are separate checkpoint weights, R/quantize_gemma3.R:126-130):
    the two weights' rows concatenated as [gate; up] and put in the gated row
    order.  NF4 only (fp8's per-tensor scales differ between the two)."""
    fused = concat_nf4_linears([gate, up])
    if fused is None or gate.out_features != up.out_features:
        raise ValueError("fuse_gated_pair needs two NF4 linears of the same shape")
    return fused.to_gated(act)


class Flux2FeedForward(nn.Module):
    """flux2_feed_forward (R/dit_flux2_modules.R:73-87) on quantized linears:
    ``linear_in`` (dim -> 2 * inner, [gate; up]) runs in the gated row order
    with SiLU(gate) * up fused into its epilogue, then ``linear_out``
    (inner -> dim_out).  Build it from the reference module's two linears with
    ``from_linears``; forward(x) returns the same values as
    linear_out(silu(h[..., :inner]) * h[..., inner:]) with h = linear_in(x)."""

    def __init__(self, linear_in: nn.Module, linear_out: nn.Module):
        super().__init__()
        self.linear_in = linear_in
        self.linear_out = linear_out

    @classmethod
    def from_linears(cls, linear_in: nn.Linear, linear_out: nn.Linear, fmt: str = "nf4"):
        holder = nn.Module()
        holder.linear_in, holder.linear_out = linear_in, linear_out
        swap_quant_linears(holder, lambda key: True, fmt)
        holder.linear_in.to_gated("swiglu")
        return cls(holder.linear_in, holder.linear_out)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.linear_out(self.linear_in(x))


# Reference-spelled aliases, so callers read like the R API.
ltx23_nf4_linear = Ltx23Nf4Linear
ltx23_fp8_linear = Ltx23Fp8Linear


def _walk(module: nn.Module, segments):
    cur = module
    for seg in segments:
        cur = cur[int(seg)] if seg.isdigit() else getattr(cur, seg, None)
        if cur is None:
            return None
    return cur


def swap_quant_linears(model: nn.Module, is_quant_key, fmt: str = "nf4",
                       device=None) -> list[str]:
    """Replace every ``nn.Linear`` whose ``<name>.weight`` key matches
    ``is_quant_key`` by an NF4 / fp8 module holding its quantized weight,
    adopting the original bias parameter (R/quantize_flux.R:541-576).

    Quantization runs on the GPU kernels of this package.  Returns the swapped
    keys.
    """
    if fmt not in ("nf4", "fp8"):
        raise ValueError("fmt must be 'nf4' or 'fp8'")
    swapped = []
    for name, mod in list(model.named_modules()):
        if not isinstance(mod, nn.Linear) or not is_quant_key(name + ".weight"):
            continue
        segs = name.split(".")
        parent = _walk(model, segs[:-1]) if len(segs) > 1 else model
        leaf = segs[-1]
        w = mod.weight.detach()
        dev = torch.device(device) if device is not None else w.device
        w = w.to(dev)
        n_out, n_in = w.shape
        has_bias = mod.bias is not None
        if fmt == "nf4":
            q = Ltx23Nf4Linear(n_out, n_in, bias=has_bias).to(dev)
            packed, absmax = ops.ltx23_nf4_quantize(w)
            q.set_nf4_weight(packed, absmax)
        else:
            q = Ltx23Fp8Linear(n_out, n_in, bias=has_bias).to(dev)
            w8, scale = ops.fp8_quantize(w)
            q.set_fp8_weight(w8, scale.cpu())
        if has_bias:
            q.bias = mod.bias
        if leaf.isdigit():
            parent[int(leaf)] = q
        else:
            setattr(parent, leaf, q)
        swapped.append(name + ".weight")
    return swapped


# R/checkpoint_flux.R:21-32 -- the FLUX.1 cast set (494 weights at full size).
FLUX_QUANT_CAST_PATTERN = re.compile(
    r"^("
    r"transformer_blocks\.[0-9]+\.("
    r"attn\.(to_q|to_k|to_v|add_q_proj|add_k_proj|add_v_proj|to_out\.0|to_add_out)"
    r"|ff\.net\.(0\.proj|2)|ff_context\.net\.(0\.proj|2)"
    r"|norm1\.linear|norm1_context\.linear"
    r")"
    r"|single_transformer_blocks\.[0-9]+\.("
    r"attn\.(to_q|to_k|to_v)|proj_mlp|proj_out|norm\.linear"
    r")"
    r")\.weight$")

# R/fp8_ltx23.R:15-18 -- the official LTX fp8 cast set.
LTX23_FP8_CAST_PATTERN = re.compile(
    r"^transformer_blocks\.[0-9]+\..*"
    r"(to_q|to_k|to_v|to_out\.0|ff\.net\.0\.proj|ff\.net\.2)\.weight$")


def flux_is_quant_key(key: str) -> bool:
    """R/checkpoint_flux.R:41-42."""
    return FLUX_QUANT_CAST_PATTERN.search(key) is not None


def ltx23_is_fp8_cast_key(key: str) -> bool:
    """R/fp8_ltx23.R:28-30."""
    return LTX23_FP8_CAST_PATTERN.search(key) is not None
