"""Torch-facing wrappers over the C ABI: every op runs the sm_100a kernels.

These mirror the functional half of diffuseR's quantized-linear API
(R/nf4_ltx23.R, R/fp8_ltx23.R).  Tensors are passed to the library as raw
device pointers with torch's current CUDA stream.  There is no CPU path: a
CPU tensor, a non-bf16 activation or a missing library raises.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

NF4_BLOCK = 64  # R/nf4_ltx23.R:23


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor: the engine has no CPU path")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return _lib.DQ_DTYPE_F32
    if t.dtype == torch.bfloat16:
        return _lib.DQ_DTYPE_BF16
    raise TypeError(f"unsupported weight dtype {t.dtype}; expected float32 or bfloat16")


# ------------------------------------------------------------- workspaces
_WS_LOCK = threading.Lock()
_WS: dict = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    """Per-device scratch for split-K partial sums, grown on demand and reused
    (the analogue of the reference's per-shape dequant buffers,
    R/nf4_ltx23.R:160-175, except that it holds f32 partials, not weights)."""
    if nbytes == 0:
        return None
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _WS_LOCK:
        buf = _WS.get(idx)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
            _WS[idx] = buf
        return buf


def release_workspaces() -> None:
    """Drop the cached scratch (ltx23_release_dequant_buffers, R/nf4_ltx23.R:185-194)."""
    with _WS_LOCK:
        _WS.clear()


def workspace_size(M: int, N: int, K: int, fmt: int = _lib.DQ_FMT_NF4) -> int:
    return int(_lib.lib().dq_workspace_size(M, N, K, fmt))


# ----------------------------------------------------------------- quantize
def ltx23_nf4_quantize(x: torch.Tensor):
    """NF4-quantize a CUDA tensor (R/nf4_ltx23.R:35-61).

    Returns ``(packed uint8 [n/2], absmax float32 [n/64])``; ``n`` must be a
    multiple of 64 (the reference's error otherwise).
    """
    _require_cuda(x, "x")
    n = x.numel()
    if n % NF4_BLOCK != 0:
        raise ValueError(f"Tensor length must be a multiple of {NF4_BLOCK}")
    src = x.detach()
    if src.dtype not in (torch.float32, torch.bfloat16):
        src = src.to(torch.float32)
    src = src.contiguous()
    packed = torch.empty(n // 2, dtype=torch.uint8, device=x.device)
    absmax = torch.empty(n // NF4_BLOCK, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check("dq_quantize_nf4", _lib.lib().dq_quantize_nf4(
            _ptr(src), _dtype_code(src), n, _ptr(packed), _ptr(absmax), _stream(x.device)))
    return packed, absmax


def fp8_quantize(x: torch.Tensor):
    """Per-tensor e4m3 quantization (R/quantize_flux.R:406-409).

    Returns ``(w8 float8_e4m3fn, scale float32 0-d tensor)``, both on x's device.
    """
    _require_cuda(x, "x")
    src = x.detach()
    if src.dtype not in (torch.float32, torch.bfloat16):
        src = src.to(torch.float32)
    src = src.contiguous()
    w8 = torch.empty(src.shape, dtype=torch.uint8, device=x.device)
    scale = torch.empty((), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check("dq_quantize_fp8", _lib.lib().dq_quantize_fp8(
            _ptr(src), _dtype_code(src), src.numel(), _ptr(w8), _ptr(scale), _stream(x.device)))
    return w8.view(torch.float8_e4m3fn), scale


# --------------------------------------------------------------- dequantize
def ltx23_nf4_dequantize(packed: torch.Tensor, absmax: torch.Tensor, shape,
                         dtype=torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
    """NF4 -> bf16 (R/nf4_ltx23.R:77-115), bit-exact with the byte-LUT path."""
    _require_cuda(packed, "packed")
    if dtype != torch.bfloat16:
        raise TypeError("the engine dequantizes to bfloat16 only")
    n = 1
    for s in shape:
        n *= int(s)
    if packed.numel() * 2 != n or absmax.numel() * NF4_BLOCK != n:
        raise ValueError("packed / absmax sizes do not match shape")
    if out is None:
        out = torch.empty(tuple(shape), dtype=torch.bfloat16, device=packed.device)
    if absmax.dtype == torch.bfloat16:
        with torch.cuda.device(packed.device):
            _lib.check("dq_dequant_nf4_scaled", _lib.lib().dq_dequant_nf4_scaled(
                _ptr(packed.contiguous()), _ptr(absmax.contiguous()), _lib.DQ_DTYPE_BF16, n,
                _ptr(out), _stream(packed.device)))
        return out
    am = absmax if absmax.dtype == torch.float32 else absmax.float()
    with torch.cuda.device(packed.device):
        _lib.check("dq_dequant_nf4", _lib.lib().dq_dequant_nf4(
            _ptr(packed.contiguous()), _ptr(am.contiguous()), n, _ptr(out), _stream(packed.device)))
    return out


def fp8_dequantize(w8: torch.Tensor, scale, dtype=torch.bfloat16,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """e4m3 -> bf16 times bf16(scale) (R/fp8_ltx23.R:79-80), bit-exact."""
    _require_cuda(w8, "w8")
    if dtype != torch.bfloat16:
        raise TypeError("the engine dequantizes to bfloat16 only")
    s = float(scale)
    if out is None:
        out = torch.empty(w8.shape, dtype=torch.bfloat16, device=w8.device)
    raw = w8.contiguous().view(torch.uint8)
    with torch.cuda.device(w8.device):
        _lib.check("dq_dequant_fp8", _lib.lib().dq_dequant_fp8(
            _ptr(raw), ctypes.c_float(s), raw.numel(), _ptr(out), _stream(w8.device)))
    return out


# ------------------------------------------------------------------- linear
def _prep_x(x: torch.Tensor, k: int) -> torch.Tensor:
    _require_cuda(x, "x")
    if x.dtype != torch.bfloat16:
        raise TypeError(f"activations must be bfloat16 on the GPU path, got {x.dtype}")
    if x.shape[-1] != k:
        raise ValueError(f"last dim of x is {x.shape[-1]}, expected in_features={k}")
    x2 = x.reshape(-1, k)
    if not x2.is_contiguous() or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    return x2


def _prep_bias(bias, n: int, device):
    if bias is None:
        return None
    b = bias.detach()
    if b.dtype != torch.bfloat16:
        b = b.to(torch.bfloat16)
    if b.device != device:
        b = b.to(device)
    if b.numel() != n:
        raise ValueError("bias size does not match out_features")
    return b.contiguous()


_ACTS = {None: _lib.DQ_ACT_NONE, "gelu_tanh": _lib.DQ_ACT_GELU_TANH, "swiglu": _lib.DQ_ACT_SWIGLU,
         "geglu_tanh": _lib.DQ_ACT_GEGLU_TANH}
GATED_ACTS = ("swiglu", "geglu_tanh")


def _act_code(act, n: int) -> tuple[int, int]:
    """(C-ABI activation code, output width) of a linear with n weight rows."""
    if act not in _ACTS:
        raise ValueError(f"unknown activation {act!r}; expected one of {list(_ACTS)}")
    if act in GATED_ACTS:
        if n % 32 != 0:
            raise ValueError("a gated activation needs out_features % 32 == 0 (gated row order)")
        return _ACTS[act], n // 2
    return _ACTS[act], n


# ------------------------------------------------------------ gated rows
def gated_row_order(n: int, device=None) -> torch.Tensor:
    """Row permutation from the reference's [gate; up] halves of an n-row
    weight (R/dit_flux2_modules.R:77-84: silu(first half) * second half) to
    the gated row order of the epilogue: for each block b of 16 output
    features, rows 32b .. 32b+15 are gate rows 16b .. 16b+15 and rows
    32b+16 .. 32b+31 the up rows n/2 + 16b .. n/2 + 16b+15."""
    if n % 32 != 0:
        raise ValueError("the gated row order needs n % 32 == 0")
    h = n // 2
    b = torch.arange(n // 32).view(-1, 1) * 16
    i = torch.arange(16).view(1, -1)
    order = torch.stack([b + i, h + b + i], dim=1).reshape(-1)
    return order if device is None else order.to(device)


def to_gated_rows_nf4(packed: torch.Tensor, absmax: torch.Tensor, n: int, k: int):
    """NF4 buffers of a [gate; up] weight reordered into the gated row order:
    rows are whole byte ranges of the packed codes and of the block scales
    (K % 64 == 0), so the reorder is a row gather."""
    order = gated_row_order(n, packed.device)
    p = packed.reshape(n, k // 2).index_select(0, order).reshape(-1)
    a = absmax.reshape(n, k // NF4_BLOCK).index_select(0, order.to(absmax.device)).reshape(-1)
    return p, a


def to_gated_rows(t: torch.Tensor, n: int) -> torch.Tensor:
    """Rows of an fp8 weight [n, K] (or a bias [n]) in the gated row order."""
    order = gated_row_order(n, t.device)
    raw = t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t
    out = raw.index_select(0, order)
    return out.view(torch.float8_e4m3fn) if t.dtype == torch.float8_e4m3fn else out


def _out_rows(out: torch.Tensor, m: int, n: int) -> int:
    """Row stride (elements) of a caller-given output viewed as [m, n] rows,
    which must be evenly spaced with unit stride along the features."""
    if out.dtype != torch.bfloat16 or not out.is_cuda:
        raise TypeError("out must be a bfloat16 CUDA tensor")
    if out.shape[-1] != n or out.numel() != m * n or out.stride(-1) != 1:
        raise ValueError(f"out must hold [{m}, {n}] with unit stride along the last dimension")
    ld = out.stride(-2) if out.dim() >= 2 else n
    for d in range(out.dim() - 2):
        if out.stride(d) != out.shape[d + 1] * out.stride(d + 1):
            raise ValueError("out's rows must be evenly spaced")
    return ld


def nf4_linear(x: torch.Tensor, packed: torch.Tensor, absmax: torch.Tensor,
               out_features: int, bias: torch.Tensor | None = None, act: str | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x . dequant_nf4(W)^T + bias (R/nf4_ltx23.R:235-246); act="gelu_tanh"
    applies GELU-tanh in the epilogue, as gelu_proj does after the projection;
    act="swiglu" / "geglu_tanh" gate a weight in the gated row order
    (to_gated_rows_nf4) and return out_features / 2 columns.  With `out`
    (e.g. a column range of a wider buffer) y is written there."""
    n = int(out_features)
    k = packed.numel() * 2 // n
    code, n_out = _act_code(act, n)
    x2 = _prep_x(x, k)
    m = x2.shape[0]
    b = _prep_bias(bias, n, x.device)
    if absmax.dtype == torch.bfloat16:
        # block scales repacked to bf16 at load time (bf16(absmax), the value
        # the forward uses): the dtype-tagged entry point
        y = out if out is not None else torch.empty((m, n_out), dtype=torch.bfloat16, device=x.device)
        ldy = _out_rows(y, m, n_out)
        with torch.cuda.device(x.device):
            ws_bytes = workspace_size(m, n, k, _lib.DQ_FMT_NF4)
            ws = workspace(x.device, ws_bytes)
            _lib.check("dq_linear_nf4_scaled", _lib.lib().dq_linear_nf4_scaled(
                _ptr(x2), m, k, _ptr(packed), _ptr(absmax), _lib.DQ_DTYPE_BF16, _ptr(b), n, code,
                _ptr(y), ldy, _ptr(ws), ws_bytes, _stream(x.device)))
        return y if out is not None else y.reshape(*x.shape[:-1], n_out)
    am = absmax if absmax.dtype == torch.float32 else absmax.float()
    if out is not None:
        ldy = _out_rows(out, m, n_out)
        with torch.cuda.device(x.device):
            ws_bytes = workspace_size(m, n, k, _lib.DQ_FMT_NF4)
            ws = workspace(x.device, ws_bytes)
            _lib.check("dq_linear_nf4_ld", _lib.lib().dq_linear_nf4_ld(
                _ptr(x2), m, k, _ptr(packed), _ptr(am), _ptr(b), n, code, _ptr(out), ldy,
                _ptr(ws), ws_bytes, _stream(x.device)))
        return out
    y = torch.empty((m, n_out), dtype=torch.bfloat16, device=x.device)
    with torch.cuda.device(x.device):
        ws_bytes = workspace_size(m, n, k, _lib.DQ_FMT_NF4)
        ws = workspace(x.device, ws_bytes)
        if act is None:
            _lib.check("dq_linear_nf4", _lib.lib().dq_linear_nf4(
                _ptr(x2), m, k, _ptr(packed), _ptr(am), _ptr(b), n, _ptr(y),
                _ptr(ws), ws_bytes, _stream(x.device)))
        else:
            _lib.check("dq_linear_nf4_ex", _lib.lib().dq_linear_nf4_ex(
                _ptr(x2), m, k, _ptr(packed), _ptr(am), _ptr(b), n, code, _ptr(y),
                _ptr(ws), ws_bytes, _stream(x.device)))
    return y.reshape(*x.shape[:-1], n_out)


def fp8_linear(x: torch.Tensor, w8: torch.Tensor, scale: float,
               bias: torch.Tensor | None = None, act: str | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x . (e4m3(W) * bf16(scale))^T + bias fused (R/fp8_ltx23.R:70-83);
    act="gelu_tanh" applies GELU-tanh in the epilogue, act="swiglu" /
    "geglu_tanh" gate a weight in the gated row order (to_gated_rows) and
    return half as many columns; with `out` y is written there (its rows may
    be spaced wider than the output width)."""
    n, k = int(w8.shape[0]), int(w8.shape[1])
    code, n_out = _act_code(act, n)
    x2 = _prep_x(x, k)
    m = x2.shape[0]
    b = _prep_bias(bias, n, x.device)
    raw = w8.view(torch.uint8)
    if out is not None:
        ldy = _out_rows(out, m, n_out)
        with torch.cuda.device(x.device):
            ws_bytes = workspace_size(m, n, k, _lib.DQ_FMT_FP8)
            ws = workspace(x.device, ws_bytes)
            _lib.check("dq_linear_fp8_ld", _lib.lib().dq_linear_fp8_ld(
                _ptr(x2), m, k, _ptr(raw), ctypes.c_float(float(scale)), _ptr(b), n, code,
                _ptr(out), ldy, _ptr(ws), ws_bytes, _stream(x.device)))
        return out
    y = torch.empty((m, n_out), dtype=torch.bfloat16, device=x.device)
    with torch.cuda.device(x.device):
        ws_bytes = workspace_size(m, n, k, _lib.DQ_FMT_FP8)
        ws = workspace(x.device, ws_bytes)
        if act is None:
            _lib.check("dq_linear_fp8", _lib.lib().dq_linear_fp8(
                _ptr(x2), m, k, _ptr(raw), ctypes.c_float(float(scale)), _ptr(b), n, _ptr(y),
                _ptr(ws), ws_bytes, _stream(x.device)))
        else:
            _lib.check("dq_linear_fp8_ex", _lib.lib().dq_linear_fp8_ex(
                _ptr(x2), m, k, _ptr(raw), ctypes.c_float(float(scale)), _ptr(b), n, code,
                _ptr(y), _ptr(ws), ws_bytes, _stream(x.device)))
    return y.reshape(*x.shape[:-1], n_out)


def device_error(device=None) -> int:
    """Read and clear the device's kernel error word (DQ_OK or DQ_ERR_TIMEOUT)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    code = ctypes.c_int(0)
    with torch.cuda.device(dev):
        _lib.check("dq_device_error", _lib.lib().dq_device_error(ctypes.byref(code), _stream(dev)))
    return code.value


def set_pair_mode(mode: int = 0) -> None:
    """0 = automatic, 1 = fused one-CTA tiles, 2 = fused CTA-pair tiles,
    3 = two-phase (the bf16 pair GEMM launch dequantizes the weight into bf16
    scratch one group of weight tiles ahead of its MMAs), 4 = two-phase with
    the dequantization as a separate launch before the GEMM, 5 = the small-M
    kernels (M <= 16, K % 128 == 0; the TMA-ring one where it applies),
    6 = the small-M kernel that loads the weight into registers."""
    _lib.check("dq_set_pair_mode", _lib.lib().dq_set_pair_mode(int(mode)))


def set_tile_override(bm: int = 0, splits: int = 0) -> None:
    """Force the x-tile height / split-K count (0 = automatic); for sweeps."""
    _lib.check("dq_set_tile_override", _lib.lib().dq_set_tile_override(int(bm), int(splits)))


def plan_info(M: int, N: int, K: int, fmt: int = _lib.DQ_FMT_NF4) -> dict:
    """The launch plan the linear uses for this shape on the current device."""
    vals = [ctypes.c_int(0) for _ in range(4)]
    _lib.check("dq_plan_info", _lib.lib().dq_plan_info(int(M), int(N), int(K), int(fmt),
                                                       *[ctypes.byref(v) for v in vals]))
    pair, bm, splits, grid = (v.value for v in vals)
    kernel = {0: "dq_gemm_kernel (one CTA)", 1: "dq_gemm2_kernel (CTA pair)",
              2: "bf16_gemm2_kernel (CTA pair, decoding its weight in-launch)",
              3: "smallm_kernel (weights loaded into registers, decoded into warp-MMA operands)",
              4: "smallm2_kernel (weights streamed through a TMA ring, decoded into warp-MMA "
                 "operands)"}[pair]
    return {"kernel": kernel, "pair": pair in (1, 2), "twophase": pair == 2, "smallm": pair in (3, 4),
            "ring": pair == 4,
            "bm": bm, "splits": splits, "grid": grid}
