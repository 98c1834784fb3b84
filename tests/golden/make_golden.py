"""Generate the committed golden vectors for the quantized-linear path.

Run from the repository root:  python tests/golden/make_golden.py

The vectors come from ``oracle.torch_ref``, the line-by-line libtorch
transcription of diffuseR's R functions (R/nf4_ltx23.R:35-115,
R/jit_ltx23.R:270-281, R/quantize_flux.R:406-409, R/fp8_ltx23.R:70-83); the R
interpreter itself is not available to run the package.  Inputs are seeded
(torch CPU generators) and small so the fixture stays a few tens of KB.
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import torch_ref as T  # noqa: E402


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    out = {}
    # test_nf4_ltx23.R:17-19: W = randn(64, 128) * 0.02 (seeded)
    g = torch.Generator().manual_seed(321)
    w = torch.randn(64, 128, generator=g) * 0.02
    packed, absmax = T.ltx23_nf4_quantize(w)
    deq = T.ltx23_nf4_dequantize(packed, absmax, (64, 128), dtype=torch.bfloat16)
    deq_f32 = T.ltx23_nf4_dequantize(packed, absmax, (64, 128), dtype=torch.float32)
    deq_chunk = T.ltx23_nf4_dequantize(packed, absmax, (64, 128), dtype=torch.bfloat16,
                                       chunk_elements=512)
    assert torch.equal(deq, deq_chunk)
    out["nf4_w"] = w.numpy()
    out["nf4_packed"] = packed.numpy()
    out["nf4_absmax"] = absmax.numpy()
    out["nf4_deq_bf16"] = bits(deq)
    out["nf4_deq_f32"] = deq_f32.numpy()
    # linear: x [5, 128] bf16, bias [64] bf16 (test_nf4_ltx23.R:46-58 shapes)
    x = (torch.randn(5, 128, generator=g)).to(torch.bfloat16)
    b = (torch.randn(64, generator=g) * 0.1).to(torch.bfloat16)
    y = torch.nn.functional.linear(x.double(), deq.double(), b.double()).float().to(torch.bfloat16)
    out["nf4_x"] = bits(x)
    out["nf4_bias"] = bits(b)
    out["nf4_y"] = bits(y)
    # a block whose value sits exactly on a midpoint (ties go to the lower level)
    tbl = torch.tensor(T.NF4_TABLE, dtype=torch.float32)
    mids = (tbl[:15] + tbl[1:]) / 2
    wt = torch.zeros(64)
    wt[0] = 1.0
    wt[1:16] = mids
    wt[16:31] = -mids.flip(0)
    pt, at = T.ltx23_nf4_quantize(wt)
    out["nf4_tie_w"] = wt.numpy()
    out["nf4_tie_packed"] = pt.numpy()
    out["nf4_tie_absmax"] = at.numpy()
    # zero block: absmax clamps to 1e-12
    pz, az = T.ltx23_nf4_quantize(torch.zeros(128))
    out["nf4_zero_packed"] = pz.numpy()
    out["nf4_zero_absmax"] = az.numpy()

    # fp8 per-tensor (R/quantize_flux.R:406-409)
    g2 = torch.Generator().manual_seed(7)
    w2 = torch.randn(48, 96, generator=g2) * 0.02
    w8, scale = T.fp8_quantize(w2)
    x2 = torch.randn(3, 96, generator=g2).to(torch.bfloat16)
    b2 = (torch.randn(48, generator=g2) * 0.1).to(torch.bfloat16)
    wd = torch.empty(48, 96, dtype=torch.bfloat16)
    wd.copy_(w8)
    wd.mul_(scale.to(torch.bfloat16))
    y2 = torch.nn.functional.linear(x2.double(), wd.double(), b2.double()).float().to(torch.bfloat16)
    out["fp8_w"] = w2.numpy()
    out["fp8_w8"] = w8.view(torch.uint8).numpy()
    out["fp8_scale"] = np.float32(scale.item())
    out["fp8_deq_bf16"] = bits(wd)
    out["fp8_x"] = bits(x2)
    out["fp8_bias"] = bits(b2)
    out["fp8_y"] = bits(y2)

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "quant_linear_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
