"""GPU parity of the gated epilogue (SwiGLU / GeGLU-tanh) on every plan.

The FLUX.2 / Z-Image feed-forward computes linear_in, then silu(first half) *
second half (R/dit_flux2_modules.R:77-84).  The engine fuses the gate into the
epilogue of linear_in with the weight rows in the gated row order.  Checked
against (1) the same engine's plain linear on the [gate; up] weight followed
by torch's bf16 silu and product -- bitwise up to rare last-bit differences of
the activation arithmetic -- and (2) the float64 oracle linear followed by the
oracle's gated activation, within the linear tolerance (1e-2).
"""
import numpy as np
import pytest
import torch

from diffuser_b200 import modules, ops
from oracle import numpy_ref as R
from tests.gpu_util import seeded_bf16, seeded_f32, to_bits

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _weights(fmt, n, k, seed):
    w = seeded_f32((n, k), seed, 0.02)
    if fmt == "nf4":
        p, a = R.nf4_quantize(w.numpy())
        return (torch.from_numpy(p).cuda(), torch.from_numpy(a).cuda()), (p, a)
    w8, s = R.fp8_quantize(w.numpy())
    return (torch.from_numpy(w8).cuda().view(torch.float8_e4m3fn), float(s)), (w8, s)


def _linear(fmt, x, wd, n, bias, act=None, out=None):
    if fmt == "nf4":
        return ops.nf4_linear(x, wd[0], wd[1], n, bias, act=act, out=out)
    return ops.fp8_linear(x, wd[0], wd[1], bias, act=act, out=out)


def _gated_weights(fmt, wd, n, k):
    if fmt == "nf4":
        return ops.to_gated_rows_nf4(wd[0], wd[1], n, k)
    return ops.to_gated_rows(wd[0], n), wd[1]


def _close_bitwise(y, ref):
    # the gate's activation is evaluated in f32 by both sides; where its bf16
    # rounding is a near-tie a one-step difference can appear
    yf, rf = y.float(), ref.float()
    step = rf.abs() * 2.0 ** -7 + 1e-6
    assert ((yf - rf).abs() <= step).all()
    assert (y != ref).float().mean().item() < 0.02


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("mode,bm,splits,m", [
    (1, 128, 0, 300),   # fused one-CTA tiles
    (2, 192, 0, 300),   # fused CTA pairs
    (3, 256, 0, 1100),  # two-phase, decode in the GEMM launch
    (4, 256, 0, 300),   # two-phase, separate decode launch
    (1, 0, 3, 16),      # split-K partials + gated reduce
    (5, 0, 0, 4),       # small-M, TMA ring
    (5, 0, 0, 13),      # small-M, TMA ring, two token tiles (x staged in the ring)
    (6, 0, 0, 12),      # small-M, weights loaded into registers
])
def test_swiglu_epilogue_every_plan(fmt, mode, bm, splits, m):
    n, k = 640, 1024
    h = n // 2
    wd, wh = _weights(fmt, n, k, 500 + m)
    x = seeded_bf16((m, k), 600 + m)
    bias = seeded_bf16((n,), 700, 0.5)
    xc, bc = x.cuda(), bias.cuda()
    gw = _gated_weights(fmt, wd, n, k)
    gb = ops.to_gated_rows(bc, n)
    ops.set_pair_mode(mode)
    ops.set_tile_override(bm, splits)
    try:
        plain = _linear(fmt, xc, wd, n, bc)
        y = _linear(fmt, xc, gw, n, gb, act="swiglu")
        y2 = _linear(fmt, xc, gw, n, gb, act="swiglu")
        torch.cuda.synchronize()
    finally:
        ops.set_tile_override(0, 0)
        ops.set_pair_mode(0)
    assert y.shape == (m, h)
    assert torch.equal(y, y2)
    ref = torch.nn.functional.silu(plain[:, :h]) * plain[:, h:]
    _close_bitwise(y, ref)
    if fmt == "nf4":
        lin = R.nf4_linear_bf16(to_bits(x), wh[0], wh[1], n, k, to_bits(bias))
    else:
        lin = R.fp8_linear_bf16(to_bits(x), wh[0], wh[1], n, k, to_bits(bias))
    assert R.rel_err(to_bits(y), R.gated_bf16(lin, "swiglu")) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
def test_geglu_and_output_column_range(fmt):
    # GELU-tanh gate (a Gemma-style MLP), written into columns of a wider buffer
    m, n, k = 200, 1024, 512
    h = n // 2
    wd, wh = _weights(fmt, n, k, 41)
    x = seeded_bf16((m, k), 42).cuda()
    gw = _gated_weights(fmt, wd, n, k)
    plain = _linear(fmt, x, wd, n, None)
    buf = torch.full((m, h + 96), 3.0, dtype=torch.bfloat16, device="cuda")
    _linear(fmt, x, gw, n, None, act="geglu_tanh", out=buf[:, 32:32 + h])
    torch.cuda.synchronize()
    ref = torch.nn.functional.gelu(plain[:, :h], approximate="tanh") * plain[:, h:]
    _close_bitwise(buf[:, 32:32 + h], ref)
    assert (buf[:, :32] == 3.0).all() and (buf[:, 32 + h:] == 3.0).all()


def test_gated_shape_rules():
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device="cuda")
    p = torch.zeros(48 * 128, dtype=torch.uint8, device="cuda")
    a = torch.ones(48 * 4, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):  # 48 rows: not a whole number of 32-row groups
        ops.nf4_linear(x, p, a, 48, act="swiglu")


def test_flux2_feed_forward_matches_reference_chain():
    # flux2_feed_forward (R/dit_flux2_modules.R:73-87): linear_out(silu(a) * b),
    # [a, b] = linear_in(x), here on NF4 linears with the gate fused
    torch.manual_seed(5)
    dim, inner, m = 512, 768, 300
    lin_in = torch.nn.Linear(dim, 2 * inner, bias=False).cuda().to(torch.bfloat16)
    lin_out = torch.nn.Linear(inner, dim, bias=False).cuda().to(torch.bfloat16)
    with torch.no_grad():
        lin_in.weight.normal_(0, 0.02)
        lin_out.weight.normal_(0, 0.02)
    x = torch.randn(m, dim, device="cuda").to(torch.bfloat16)
    ff = modules.Flux2FeedForward.from_linears(lin_in, lin_out, "nf4")
    y = ff(x)
    # the reference chain on the same NF4 weights (dequantized, bf16, torch)
    wi = ops.ltx23_nf4_quantize(lin_in.weight.float())
    hid = torch.nn.functional.linear(x, ops.ltx23_nf4_dequantize(*wi, (2 * inner, dim)))
    act = torch.nn.functional.silu(hid[:, :inner]) * hid[:, inner:]
    wo = ops.ltx23_nf4_quantize(lin_out.weight.float())
    ref = torch.nn.functional.linear(act, ops.ltx23_nf4_dequantize(*wo, (dim, inner)))
    torch.cuda.synchronize()
    err = ((y.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
    assert err <= TOL, err
