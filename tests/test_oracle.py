"""CPU tests: pin the oracle against the reference's own known answers and
test assertions, and against the libtorch transcription of the R code."""
import os

import numpy as np
import pytest
import torch

from oracle import numpy_ref as R
from oracle import torch_ref as T

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quant_linear_golden.npz")


def test_byte_lut_known_answers():
    # inst/tinytest/test_jit_ltx23.R:243-251
    lut = R.nf4_byte_lut_f32()
    tl = T.ltx23_jit_table(torch.device("cpu"), torch.float32)
    assert lut.shape == (256, 2)
    assert np.array_equal(lut, tl.numpy())
    lv = R.NF4_LEVELS_F64
    for b in (0, 1, 15, 16, 137, 240, 255):
        assert np.allclose(lut[b], [lv[b // 16], lv[b % 16]], rtol=0, atol=1e-7)


def test_bf16_levels_single_vs_double_rounding():
    direct = torch.tensor(T.NF4_TABLE, dtype=torch.float64).to(torch.bfloat16)
    via_f32 = torch.tensor(T.NF4_TABLE, dtype=torch.float32).to(torch.bfloat16)
    assert torch.equal(direct, via_f32)
    ours = R.nf4_levels_bf16_bits()
    assert np.array_equal(ours, direct.view(torch.int16).numpy().view(np.uint16))


def test_reference_nf4_roundtrip_assertions():
    # inst/tinytest/test_nf4_ltx23.R:17-42 restated on the oracle
    g = torch.Generator().manual_seed(321)
    w = (torch.randn(64, 128, generator=g) * 0.02).numpy()
    packed, absmax = R.nf4_quantize(w)
    assert packed.shape == (64 * 128 // 2,) and packed.dtype == np.uint8
    assert absmax.shape == (64 * 128 // 64,)
    w_rt = R.nf4_dequantize_f32(packed, absmax).reshape(64, 128)
    rel = np.abs(w_rt - w).mean() / np.abs(w).mean()
    assert rel < 0.1
    blocks = w_rt.reshape(-1, 64) / absmax[:, None]
    d = np.abs(blocks.reshape(-1, 1) - R.NF4_LEVELS_F64[None, :]).min(axis=1)
    assert d.max() < 1e-5
    # chunked == single shot (the transcription's chunk loop)
    pt, at = torch.from_numpy(packed), torch.from_numpy(absmax)
    a = T.ltx23_nf4_dequantize(pt, at, (64, 128), dtype=torch.float32)
    b = T.ltx23_nf4_dequantize(pt, at, (64, 128), dtype=torch.float32, chunk_elements=512)
    assert torch.equal(a, b)
    assert np.array_equal(a.numpy().reshape(-1), R.nf4_dequantize_f32(packed, absmax))


def test_reference_nf4_linear_assertion():
    # inst/tinytest/test_nf4_ltx23.R:46-58: NF4 linear vs full linear, mean rel < 0.15
    g = torch.Generator().manual_seed(5)
    lin = torch.nn.Linear(128, 64)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(64, 128, generator=g) * 0.1)
        lin.bias.copy_(torch.randn(64, generator=g) * 0.1)
    packed, absmax = R.nf4_quantize(lin.weight.detach().numpy())
    x = torch.randn(5, 128, generator=g)
    y_ref = lin(x).detach().numpy()
    w = R.nf4_dequantize_f32(packed, absmax).reshape(64, 128)
    y = x.numpy() @ w.T + lin.bias.detach().numpy()
    assert np.abs(y - y_ref).mean() / np.abs(y_ref).mean() < 0.15


@pytest.mark.parametrize("seed,shape,std", [(0, (96, 256), 0.02), (1, (33, 64), 1.0),
                                            (2, (7, 192), 300.0), (3, (128, 128), 1e-30)])
def test_numpy_matches_libtorch_transcription_nf4(seed, shape, std):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(*shape, generator=g) * std
    if seed == 2:
        w[0, :64] = 0.0  # an all-zero block: absmax clamps to 1e-12
    pt, at = T.ltx23_nf4_quantize(w)
    pn, an = R.nf4_quantize(w.numpy())
    assert np.array_equal(pt.numpy(), pn)
    assert np.array_equal(at.numpy(), an)
    dt = T.ltx23_nf4_dequantize(pt, at, shape, dtype=torch.bfloat16)
    dn = R.nf4_dequantize_bf16_bits(pn, an)
    assert np.array_equal(dt.view(torch.int16).numpy().view(np.uint16).reshape(-1), dn)
    # the TorchScript nf4_lin gathers through embedding: same weights
    tbl = T.ltx23_jit_table(torch.device("cpu"), torch.bfloat16)
    vals = torch.embedding(tbl, pt.int()).reshape(-1, 64) * at.type_as(tbl).unsqueeze(1)
    assert torch.equal(vals.reshape(-1), dt.reshape(-1))


@pytest.mark.parametrize("seed,shape,std", [(0, (96, 256), 0.02), (1, (64, 48), 3.0), (2, (5, 7), 1e-3)])
def test_numpy_matches_libtorch_transcription_fp8(seed, shape, std):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(*shape, generator=g) * std
    w8t, st = T.fp8_quantize(w)
    w8n, sn = R.fp8_quantize(w.numpy())
    assert st.item() == float(sn)
    assert np.array_equal(w8t.view(torch.uint8).numpy(), w8n)
    wd = torch.empty(shape, dtype=torch.bfloat16)
    wd.copy_(w8t)
    wd.mul_(st.to(torch.bfloat16))
    assert np.array_equal(wd.view(torch.int16).numpy().view(np.uint16), R.fp8_dequantize_bf16_bits(w8n, sn))


def test_e4m3_encoder_matches_torch():
    vals = np.concatenate([np.linspace(-480, 480, 100001), [448, 449, 463.9, 464, 464.01, 500,
                                                             0.0, -0.0, 2.0 ** -9, 2.0 ** -10,
                                                             3 * 2.0 ** -11, 1e-30]]).astype(np.float32)
    t = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(t, R.f32_to_e4m3(vals))
    codes = np.arange(256, dtype=np.uint8)
    tv = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    ov = R.e4m3_to_f32(codes)
    assert np.array_equal(np.isnan(tv), np.isnan(ov))
    assert np.array_equal(tv[~np.isnan(tv)], ov[~np.isnan(ov)])


def test_golden_vectors_reproduced_by_oracle():
    g = np.load(GOLDEN)
    pn, an = R.nf4_quantize(g["nf4_w"])
    assert np.array_equal(pn, g["nf4_packed"]) and np.array_equal(an, g["nf4_absmax"])
    assert np.array_equal(R.nf4_dequantize_bf16_bits(pn, an), g["nf4_deq_bf16"].reshape(-1))
    assert np.array_equal(R.nf4_dequantize_f32(pn, an), g["nf4_deq_f32"].reshape(-1))
    y = R.nf4_linear_bf16(g["nf4_x"], pn, an, 64, 128, g["nf4_bias"])
    assert R.rel_err(y, g["nf4_y"]) <= 2.0 ** -8
    pt, at = R.nf4_quantize(g["nf4_tie_w"])
    assert np.array_equal(pt, g["nf4_tie_packed"]) and np.array_equal(at, g["nf4_tie_absmax"])
    pz, az = R.nf4_quantize(np.zeros(128, np.float32))
    assert np.array_equal(pz, g["nf4_zero_packed"]) and np.array_equal(az, g["nf4_zero_absmax"])
    w8, s = R.fp8_quantize(g["fp8_w"])
    assert np.array_equal(w8, g["fp8_w8"]) and np.float32(s) == g["fp8_scale"]
    assert np.array_equal(R.fp8_dequantize_bf16_bits(w8, s), g["fp8_deq_bf16"])
    y2 = R.fp8_linear_bf16(g["fp8_x"], w8, s, 48, 96, g["fp8_bias"])
    assert R.rel_err(y2, g["fp8_y"]) <= 2.0 ** -8


def test_midpoint_ties_take_lower_level():
    g = np.load(GOLDEN)
    codes = np.empty(64, np.uint8)
    codes[0::2] = g["nf4_tie_packed"] >> 4
    codes[1::2] = g["nf4_tie_packed"] & 15
    # value == midpoint(i, i+1) -> level i (bucketize right = FALSE)
    assert list(codes[1:16]) == list(range(15))
