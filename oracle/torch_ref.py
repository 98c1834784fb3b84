"""Line-by-line libtorch transcription of diffuseR's quantized linears.

TEST INFRASTRUCTURE ONLY: the second leg of the oracle and the timed CPU
port of the reference (``bench.py --impl reference``).

The reference is R on the ``torch`` package, whose ops are libtorch's.  Each
function below issues the same libtorch ops in the same order as the R
function it cites, with R's 1-based index shift removed.  It runs wherever
PyTorch runs; on CPU it is the reference's own CPU algorithm.
"""
from __future__ import annotations

import torch

# R/nf4_ltx23.R:15-21
NF4_TABLE = [-1.0, -0.6961928009986877, -0.5250730514526367,
             -0.39491748809814453, -0.28444138169288635,
             -0.18477343022823334, -0.09105003625154495, 0.0,
             0.07958029955625534, 0.16093020141124725,
             0.24611230194568634, 0.33791524171829224,
             0.44070982933044434, 0.5626170039176941,
             0.7229568362236023, 1.0]
NF4_BLOCK = 64  # R/nf4_ltx23.R:23


def ltx23_nf4_quantize(x: torch.Tensor):
    """R/nf4_ltx23.R:35-61."""
    n = x.numel()
    block = NF4_BLOCK
    if n % block != 0:
        raise ValueError(f"Tensor length must be a multiple of {block}")
    table = torch.tensor(NF4_TABLE, dtype=torch.float32, device=x.device)
    midpoints = (table.narrow(0, 0, 15) + table.narrow(0, 1, 15)) / 2
    blocks = x.detach().to(dtype=torch.float32).reshape(-1, block)
    absmax = blocks.abs().amax(dim=1).clamp(min=1e-12)
    normalized = blocks / absmax.unsqueeze(1)
    idx = torch.bucketize(normalized.flatten(), midpoints)  # 0..15
    idx = idx.to(dtype=torch.uint8)
    pairs = idx.reshape(-1, 2)
    packed = pairs.narrow(1, 0, 1).squeeze(1) * 16 + pairs.narrow(1, 1, 1).squeeze(1)
    return packed, absmax


_LUT_CACHE: dict = {}


def ltx23_jit_table(device, dtype):
    """Byte LUT [256, 2] in the compute dtype (R/jit_ltx23.R:270-281)."""
    key = (str(device), dtype)
    tbl = _LUT_CACHE.get(key)
    if tbl is None:
        pairs = [[NF4_TABLE[b // 16], NF4_TABLE[b % 16]] for b in range(256)]
        tbl = torch.tensor(pairs, dtype=dtype, device=device)
        _LUT_CACHE[key] = tbl
    return tbl


def ltx23_nf4_dequantize(packed, absmax, shape, dtype=torch.bfloat16,
                         chunk_elements=8388608, out=None):
    """R/nf4_ltx23.R:77-115 (chunked byte-LUT gather, then per-block mul_)."""
    block = NF4_BLOCK
    if out is None:
        out = torch.empty(shape, dtype=dtype, device=packed.device)
    out_pairs = out.view(-1, 2)
    out_blocks = out.view(-1, block)
    n_bytes = packed.shape[0]
    bytes_per_chunk = max(chunk_elements // 2, block)
    idx_scratch = torch.empty(min(bytes_per_chunk, n_bytes), dtype=torch.long,
                              device=packed.device)
    tbl = ltx23_jit_table(packed.device, dtype)
    am = absmax.to(dtype=dtype)
    start = 0
    with torch.no_grad():
        while start < n_bytes:
            ln = min(bytes_per_chunk, n_bytes - start)
            idx = idx_scratch.narrow(0, 0, ln)
            idx.copy_(packed.narrow(0, start, ln))
            torch.index_select(tbl, 0, idx, out=out_pairs.narrow(0, start, ln))
            block_start = (start * 2) // block
            n_blocks = (ln * 2) // block
            out_blocks.narrow(0, block_start, n_blocks).mul_(
                am.narrow(0, block_start, n_blocks).unsqueeze(1))
            start += ln
    return out


def nf4_lin(x, packed, absmax, bias, table2):
    """TorchScript nf4_lin (R/jit_ltx23.R:40-50)."""
    rows = bias.size(0)
    vals = torch.embedding(table2, packed.int())
    w = vals.reshape([-1, 64]) * absmax.type_as(table2).unsqueeze(1)
    return torch.nn.functional.linear(x, w.reshape([rows, -1]).type_as(x), bias)


def nf4_linear_forward(x, packed, absmax, n, k, bias=None, w_buffer=None):
    """ltx23_nf4_linear$forward (R/nf4_ltx23.R:235-246)."""
    w = w_buffer if w_buffer is not None else torch.empty((n, k), dtype=x.dtype, device=x.device)
    ltx23_nf4_dequantize(packed, absmax, (n, k), dtype=x.dtype, out=w)
    return torch.nn.functional.linear(x, w, bias)


def fp8_quantize(tensor):
    """R/quantize_flux.R:406-409 and R/fp8_ltx23.R:178-181 (per-tensor)."""
    scale = tensor.abs().max().to(dtype=torch.float32).clamp(min=1e-12) / 448
    w8 = (tensor.to(dtype=torch.float32) / scale).to(dtype=torch.float8_e4m3fn)
    return w8, scale


def fp8_linear_forward(x, w8, scale, bias=None, w_buffer=None):
    """ltx23_fp8_linear$forward (R/fp8_ltx23.R:70-83)."""
    w8 = w8.to(device=x.device, non_blocking=True)
    w = w_buffer if w_buffer is not None else torch.empty(w8.shape, dtype=x.dtype, device=x.device)
    with torch.no_grad():
        w.copy_(w8)
        w.mul_(scale.to(device=x.device, dtype=x.dtype))
    return torch.nn.functional.linear(x, w, bias)


# TorchScript source of nf4_lin (R/jit_ltx23.R:40-50) and of the linear
# followed by GELU-tanh (R/jit_ltx23.R:97-99), for compiling the block stack
# with the reference's own linear as the comparison.
NF4_LIN_TS_SOURCE = '''
def REF_LIN(x: Tensor, packed: Tensor, absmax: Tensor, bias: Tensor, table2: Tensor) -> Tensor:
    rows = bias.size(0)
    vals = torch.embedding(table2, packed.int())
    w = vals.reshape([-1, 64]) * absmax.type_as(table2).unsqueeze(1)
    return torch.nn.functional.linear(x, w.reshape([rows, -1]).type_as(x), bias)

def LIN_GELU_FN(x: Tensor, packed: Tensor, absmax: Tensor, bias: Tensor, table2: Tensor) -> Tensor:
    return torch.nn.functional.gelu(REF_LIN(x, packed, absmax, bias, table2), approximate="tanh")
'''
