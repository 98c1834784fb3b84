"""The reference's on-disk quantized artifacts: write, open, and load them into
a module tree as the engine's quantized linears.

An artifact is a directory of safetensors shards plus ``manifest.json``
(R/quantize_flux.R:366-444 for FLUX / Z-Image, R/quantize_gemma3.R:29-123 for
the Gemma3 text encoder; read back by ltx23_open_fp8_checkpoint,
R/fp8_ltx23.R:230-265).  Every weight the model's cast-set selector picks is
stored quantized:

* NF4: ``<key>`` uint8 [N*K/2] (two codes per byte, the first element in the
  high nibble) and ``<key>_absmax`` f32 [N*K/64];
* fp8: ``<key>`` e4m3 [N, K] and ``<key>_scale`` f32 (0-d);

every other tensor ("resident") in bf16.  The manifest records the format
(``"nf4"`` / ``"fp8"``), the shard file names, the tensor and cast counts, the
model config and, for Gemma3, ``model: "gemma3"``.

``load_quantized`` mirrors the reference's loaders (flux_load_transformer,
R/quantize_flux.R:488-627; load_gemma3_nf4, R/quantize_gemma3.R:150-215):
each quantized key replaces the linear at that module path by an NF4 / fp8
module filled from the artifact, residents are copied into the remaining
parameters and buffers, and any parameter left unfilled, or any artifact key
that lands nowhere, is an error.  Optionally the NF4 block scales are repacked
to bf16 at load time (bit-identical dequantized weights, half the scale
bytes).
"""
from __future__ import annotations

import json
import os
import re

import torch
from torch import nn

from . import modules

MANIFEST = "manifest.json"


# ----------------------------------------------------------------- selectors
# R/quantize_gemma3.R:126-130 -- the seven per-layer projections.
GEMMA3_QUANT_PATTERN = re.compile(
    r"^layers\.[0-9]+\.(self_attn\.(q|k|v|o)_proj|mlp\.(gate|up|down)_proj)\.weight$")


def gemma3_is_quant_key(key: str) -> bool:
    """R/quantize_gemma3.R:126-130 (keys normalized as gemma3_normalize_key)."""
    return GEMMA3_QUANT_PATTERN.search(key) is not None


def gemma3_normalize_key(key: str):
    """The key the Gemma3 artifact stores for a HuggingFace checkpoint key
    (``language_model.`` / ``model.`` stripped), or None for the tensors the
    text encoder never uses (R/quantize_gemma3.R:91-95)."""
    if re.match(r"^(vision_tower|multi_modal_projector|lm_head)\.", key):
        return None
    return re.sub(r"^model\.", "", re.sub(r"^language_model\.", "", key))


# -------------------------------------------------------------------- write
def quantize_state(state: dict, is_quant_key, fmt: str, quantize_nf4=None, quantize_fp8=None,
                   resident_dtype=torch.bfloat16) -> tuple[dict, int]:
    """Artifact tensors of a state dict: cast keys quantized, residents cast
    to `resident_dtype`.  The quantizers default to the engine's GPU kernels
    (bit-exact with ltx23_nf4_quantize and the fp8 cast, R/quantize_flux.R:
    400-410); each takes a tensor and returns (packed, absmax) / (w8, scale).
    Returns (tensors on the CPU, number of cast keys)."""
    from . import ops
    if fmt not in ("nf4", "fp8"):
        raise ValueError("fmt must be 'nf4' or 'fp8'")
    quantize_nf4 = quantize_nf4 or ops.ltx23_nf4_quantize
    quantize_fp8 = quantize_fp8 or ops.fp8_quantize
    out, n_cast = {}, 0
    for key, t in state.items():
        if is_quant_key(key):
            if fmt == "nf4":
                packed, absmax = quantize_nf4(t)
                out[key] = packed.reshape(-1).cpu()
                out[key + "_absmax"] = absmax.reshape(-1).float().cpu()
            else:
                w8, scale = quantize_fp8(t)
                out[key] = w8.cpu()
                out[key + "_scale"] = torch.as_tensor(scale, dtype=torch.float32).reshape(()).cpu()
            n_cast += 1
        else:
            out[key] = t.detach().to(resident_dtype).cpu()
    return out, n_cast


def write_artifact(out_dir: str, tensors: dict, fmt: str, n_cast: int, config=None,
                   shard_bytes: float = 1.9e9, shard_prefix: str = "transformer",
                   extra: dict | None = None) -> dict:
    """Write artifact tensors (from quantize_state) as shards of at most about
    `shard_bytes` plus manifest.json; returns the manifest."""
    from safetensors.torch import save_file
    os.makedirs(out_dir, exist_ok=True)
    shards, cur, size = [], {}, 0

    def flush():
        nonlocal cur, size
        if not cur:
            return
        name = f"{shard_prefix}-{fmt}-{len(shards) + 1:05d}.safetensors"
        save_file(cur, os.path.join(out_dir, name))
        shards.append(name)
        cur, size = {}, 0

    for key, t in tensors.items():
        cur[key] = t.contiguous()
        size += t.numel() * t.element_size()
        if size >= shard_bytes:
            flush()
    flush()
    manifest = {"format": fmt, "shards": shards, "tensors": len(tensors) - n_cast, "cast": n_cast,
                "config": config}
    if extra:
        manifest.update(extra)
    with open(os.path.join(out_dir, MANIFEST), "w") as f:
        json.dump(manifest, f, indent=2)
    return manifest


# --------------------------------------------------------------------- open
class Artifact:
    """An opened artifact: ``keys``, ``get_tensor(key)``, ``manifest``,
    ``format`` and ``config`` (ltx23_open_fp8_checkpoint, R/fp8_ltx23.R:
    230-265)."""

    def __init__(self, path: str):
        from safetensors import safe_open
        mpath = os.path.join(path, MANIFEST)
        if not os.path.exists(mpath):
            raise FileNotFoundError(f"no {MANIFEST} in {path}: not a quantized artifact")
        with open(mpath) as f:
            self.manifest = json.load(f)
        self.path = path
        self.format = self.manifest.get("format", "fp8")
        self.config = self.manifest.get("config")
        self._where = {}
        for shard in self.manifest["shards"]:
            sp = os.path.join(path, shard)
            with safe_open(sp, framework="pt") as h:
                for k in h.keys():
                    self._where[k] = sp
        self.keys = list(self._where)

    def get_tensor(self, key: str) -> torch.Tensor:
        from safetensors import safe_open
        sp = self._where.get(key)
        if sp is None:
            raise KeyError(f"key not found in the artifact's shards: {key}")
        with safe_open(sp, framework="pt") as h:
            return h.get_tensor(key)

    def cast_keys(self) -> list[str]:
        """Weights stored quantized (those with an _absmax or _scale companion)."""
        return [k[:-len("_absmax")] for k in self.keys if k.endswith("_absmax")] + \
               [k[:-len("_scale")] for k in self.keys if k.endswith("_scale")]


def open_artifact(path: str) -> Artifact:
    return Artifact(path)


# --------------------------------------------------------------------- load
def _parent_and_leaf(model: nn.Module, module_path: str):
    segs = module_path.split(".")
    parent = modules._walk(model, segs[:-1]) if len(segs) > 1 else model
    if parent is None:
        raise KeyError(f"artifact key has no module in the model: {module_path}")
    return parent, segs[-1]


def load_quantized(model: nn.Module, art: Artifact, device=None, scales: str = "f32",
                   strict: bool = True) -> dict:
    """Swap every quantized key of `art` into `model` as an NF4 / fp8 linear
    and copy the residents; hard errors (strict) on an artifact key that lands
    nowhere or a model parameter the artifact leaves unfilled.  scales="bf16"
    repacks the NF4 block scales to bf16 at load time.  Returns a report
    {"cast": [...], "residents": [...]}."""
    if scales not in ("f32", "bf16"):
        raise ValueError("scales must be 'f32' or 'bf16'")
    cast = art.cast_keys()
    used = set()
    for key in cast:
        if not key.endswith(".weight"):
            raise KeyError(f"quantized key is not a weight: {key}")
        parent, leaf = _parent_and_leaf(model, key[:-len(".weight")])
        old = parent[int(leaf)] if leaf.isdigit() else getattr(parent, leaf, None)
        if old is None:
            raise KeyError(f"artifact key has no module in the model: {key}")
        if isinstance(old, nn.Linear):
            n_out, n_in = old.weight.shape
        else:
            n_out, n_in = old.out_features, old.in_features
        has_bias = getattr(old, "bias", None) is not None
        dev = torch.device(device) if device is not None else next(
            (p.device for p in old.parameters()), torch.device("cpu"))
        if key + "_absmax" in art._where:
            q = modules.Ltx23Nf4Linear(n_out, n_in, bias=has_bias)
            packed, absmax = art.get_tensor(key), art.get_tensor(key + "_absmax")
            if packed.numel() * 2 != n_out * n_in:
                raise ValueError(f"{key}: packed size does not match the module's [{n_out}, {n_in}]")
            q.set_nf4_weight(packed, absmax)
            used.update((key, key + "_absmax"))
            q = q.to(dev)
            if scales == "bf16":
                q.repack_scales_bf16()
        else:
            q = modules.Ltx23Fp8Linear(n_out, n_in, bias=has_bias)
            w8 = art.get_tensor(key)
            if tuple(w8.shape) != (n_out, n_in):
                raise ValueError(f"{key}: e4m3 shape {tuple(w8.shape)} != [{n_out}, {n_in}]")
            q.set_fp8_weight(w8.to(dev), art.get_tensor(key + "_scale"))
            used.update((key, key + "_scale"))
            q = q.to(dev)
        if has_bias:
            q.bias = old.bias
        if leaf.isdigit():
            parent[int(leaf)] = q
        else:
            setattr(parent, leaf, q)
    # residents into parameters and buffers
    targets = dict(model.named_parameters())
    targets.update(dict(model.named_buffers()))
    quant_bufs = {n for n, _ in model.named_buffers()
                  if n.endswith((".weight_nf4", ".weight_absmax"))}
    filled, unknown = [], []
    with torch.no_grad():
        for key in art.keys:
            if key in used:
                continue
            dst = targets.get(key)
            if dst is None:
                unknown.append(key)
                continue
            src = art.get_tensor(key)
            if tuple(src.shape) != tuple(dst.shape):
                raise ValueError(f"{key}: artifact shape {tuple(src.shape)} != model {tuple(dst.shape)}")
            dst.copy_(src.to(device=dst.device, dtype=dst.dtype))
            filled.append(key)
    missing = [n for n in targets if n not in filled and n not in quant_bufs and n not in used]
    if strict and unknown:
        raise KeyError(f"artifact keys with no place in the model: {unknown[:8]}")
    if strict and missing:
        raise KeyError(f"model tensors the artifact does not fill: {missing[:8]}")
    return {"cast": cast, "residents": filled, "unknown": unknown, "missing": missing}
