"""GPU parity: quantizers and dequantizers against the oracle, bit for bit."""
import os

import numpy as np
import pytest
import torch

from oracle import numpy_ref as R
from tests.gpu_util import from_bits, seeded_f32, to_bits

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quant_linear_golden.npz")


@pytest.fixture(scope="module")
def ops():
    from diffuser_b200 import ops as _ops
    return _ops


def test_nf4_dequant_every_byte_every_scale_bit_exact(ops):
    packed = np.tile(np.arange(256, dtype=np.uint8), 32)          # 8192 bytes, 256 blocks
    rng = np.random.default_rng(0)
    absmax = np.concatenate([
        np.array([1.0, 1e-12, 0.02, 3.7, 123.456, 1e-30, 6.5e4, 1.0 + 2 ** -8], np.float32),
        (10.0 ** rng.uniform(-8, 4, 248)).astype(np.float32)])
    ref = R.nf4_dequantize_bf16_bits(packed, absmax)
    got = ops.ltx23_nf4_dequantize(torch.from_numpy(packed).cuda(), torch.from_numpy(absmax).cuda(),
                                   (128, 128))
    torch.cuda.synchronize()
    assert np.array_equal(to_bits(got).reshape(-1), ref)


@pytest.mark.parametrize("shape,std,seed", [((64, 128), 0.02, 321), ((12288 // 16, 3072), 0.02, 0),
                                            ((33, 192), 5.0, 3)])
def test_nf4_quantize_bit_exact_f32(ops, shape, std, seed):
    w = seeded_f32(shape, seed, std)
    w[0, :64] = 0.0
    pn, an = R.nf4_quantize(w.numpy())
    pg, ag = ops.ltx23_nf4_quantize(w.cuda())
    assert np.array_equal(pg.cpu().numpy(), pn)
    assert np.array_equal(ag.cpu().numpy(), an)


def test_nf4_quantize_bit_exact_bf16_input(ops):
    w = seeded_f32((96, 256), 11, 0.05).to(torch.bfloat16)
    pn, an = R.nf4_quantize(w.float().numpy())
    pg, ag = ops.ltx23_nf4_quantize(w.cuda())
    assert np.array_equal(pg.cpu().numpy(), pn)
    assert np.array_equal(ag.cpu().numpy(), an)


def test_nf4_golden_vectors(ops):
    g = np.load(GOLDEN)
    pg, ag = ops.ltx23_nf4_quantize(torch.from_numpy(g["nf4_w"]).cuda())
    assert np.array_equal(pg.cpu().numpy(), g["nf4_packed"])
    assert np.array_equal(ag.cpu().numpy(), g["nf4_absmax"])
    d = ops.ltx23_nf4_dequantize(pg, ag, (64, 128))
    assert np.array_equal(to_bits(d), g["nf4_deq_bf16"])
    pt, at = ops.ltx23_nf4_quantize(torch.from_numpy(g["nf4_tie_w"]).cuda())
    assert np.array_equal(pt.cpu().numpy(), g["nf4_tie_packed"])
    pz, az = ops.ltx23_nf4_quantize(torch.zeros(128, device="cuda"))
    assert np.array_equal(pz.cpu().numpy(), g["nf4_zero_packed"])
    assert np.array_equal(az.cpu().numpy(), g["nf4_zero_absmax"])


def test_reference_roundtrip_assertions_on_gpu(ops):
    # inst/tinytest/test_nf4_ltx23.R:17-37 through the GPU quantizer/dequantizer
    w = seeded_f32((64, 128), 321, 0.02)
    p, a = ops.ltx23_nf4_quantize(w.cuda())
    assert p.shape == (64 * 128 // 2,) and p.dtype == torch.uint8 and a.shape == (128,)
    w_rt = ops.ltx23_nf4_dequantize(p, a, (64, 128)).float().cpu()
    assert ((w_rt - w).abs().mean() / w.abs().mean()).item() < 0.1
    blocks = w_rt.reshape(-1, 64) / a.cpu().to(torch.bfloat16).float().unsqueeze(1)
    lv = torch.tensor(R.NF4_LEVELS_F64, dtype=torch.float32)
    d = (blocks.reshape(-1, 1) - lv.unsqueeze(0)).abs().min(dim=1).values
    assert d.max().item() < 2.0 ** -7  # bf16 rounding of level * absmax


def test_fp8_dequant_every_code_bit_exact(ops):
    codes = np.arange(256, dtype=np.uint8)
    codes = codes[(codes & 0x7F) != 0x7F]                        # drop the two NaN codes
    w8 = np.tile(codes, 8)
    for scale in (1.0, 0.02 / 448, 1e-12 / 448, 3.3e-5, 7.0):
        ref = R.fp8_dequantize_bf16_bits(w8, np.float32(scale))
        got = ops.fp8_dequantize(torch.from_numpy(w8).cuda().view(torch.float8_e4m3fn), np.float32(scale))
        assert np.array_equal(to_bits(got), ref), scale


@pytest.mark.parametrize("shape,std,seed", [((48, 96), 0.02, 7), ((3072, 4096), 0.02, 1), ((5, 7), 2.0, 2)])
def test_fp8_quantize_bit_exact(ops, shape, std, seed):
    w = seeded_f32(shape, seed, std)
    w8n, sn = R.fp8_quantize(w.numpy())
    w8g, sg = ops.fp8_quantize(w.cuda())
    assert sg.item() == float(sn)
    assert np.array_equal(w8g.view(torch.uint8).cpu().numpy(), w8n)
    wb = w.to(torch.bfloat16)
    w8n2, sn2 = R.fp8_quantize(wb.float().numpy())
    w8g2, sg2 = ops.fp8_quantize(wb.cuda())
    assert sg2.item() == float(sn2)
    assert np.array_equal(w8g2.view(torch.uint8).cpu().numpy(), w8n2)


def test_fp8_golden_vectors(ops):
    g = np.load(GOLDEN)
    w8, s = ops.fp8_quantize(torch.from_numpy(g["fp8_w"]).cuda())
    assert np.array_equal(w8.view(torch.uint8).cpu().numpy(), g["fp8_w8"])
    assert np.float32(s.item()) == g["fp8_scale"]
    d = ops.fp8_dequantize(w8, s.item())
    assert np.array_equal(to_bits(d), g["fp8_deq_bf16"])


def test_fp8_dequant_ragged_length(ops):
    w8 = np.random.default_rng(3).integers(0, 256, 1000 + 13, dtype=np.uint8)
    w8[(w8 & 0x7F) == 0x7F] = 0
    ref = R.fp8_dequantize_bf16_bits(w8, np.float32(0.01))
    got = ops.fp8_dequantize(torch.from_numpy(w8).cuda().view(torch.float8_e4m3fn), 0.01)
    assert np.array_equal(to_bits(got), ref)


def test_no_kernel_error_recorded(ops):
    assert ops.device_error() == 0
