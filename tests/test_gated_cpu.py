"""Host side of the gated (SwiGLU / GeGLU) epilogue: the gated row order and
the oracle's gated activation (CPU, no GPU needed)."""
import numpy as np
import torch

from diffuser_b200 import ops
from oracle import numpy_ref as R
from oracle import torch_ref as T


def test_gated_row_order_pairs_each_gate_row_with_its_up_row():
    n = 96
    order = ops.gated_row_order(n)
    assert sorted(order.tolist()) == list(range(n))
    h = n // 2
    for b in range(n // 32):
        for i in range(16):
            assert order[32 * b + i] == 16 * b + i           # gate of feature 16b + i
            assert order[32 * b + 16 + i] == h + 16 * b + i  # its up row


def test_nf4_rows_reorder_as_whole_byte_ranges():
    n, k = 64, 128
    w = torch.randn(n, k) * 0.02
    p, a = T.ltx23_nf4_quantize(w)
    gp, ga = ops.to_gated_rows_nf4(p, a, n, k)
    order = ops.gated_row_order(n)
    got = T.ltx23_nf4_dequantize(gp, ga, (n, k))
    ref = T.ltx23_nf4_dequantize(p, a, (n, k))[order]
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    w8 = (w * 100).to(torch.float8_e4m3fn)
    assert torch.equal(ops.to_gated_rows(w8, n).view(torch.uint8), w8.view(torch.uint8)[order])


def test_oracle_gated_activation_matches_torch_chain():
    # the reference's chain on bf16 tensors: silu(first half) * second half
    y = (torch.randn(7, 64) * 3).to(torch.bfloat16)
    bits = y.view(torch.int16).numpy().view(np.uint16)
    got = R.gated_bf16(bits, "swiglu")
    ref = (torch.nn.functional.silu(y[:, :32]) * y[:, 32:]).view(torch.int16).numpy().view(np.uint16)
    # float32 exp in numpy vs torch's: the bf16 results agree except at rare ties
    assert (got != ref).mean() < 0.01
    assert R.rel_err(got, ref) < 1e-2
    g = R.gated_bf16(bits, "geglu_tanh")
    ref = (torch.nn.functional.gelu(y[:, :32], approximate="tanh") * y[:, 32:])
    assert R.rel_err(g, ref.view(torch.int16).numpy().view(np.uint16)) < 1e-2
