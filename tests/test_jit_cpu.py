"""The LTX-2.3 TorchScript block stack (diffuser_b200/jit.py) on the CPU:
the engine-bound unit compiles with the engine's operators registered, the
114-slot packer keeps the reference's layout (R/jit_ltx23.R:21-34), the same
source bound to the reference's own nf4_lin runs end to end (float32), and the
engine's operators refuse CPU tensors (no CPU fallback)."""
import pytest
import torch

from diffuser_b200 import jit
from oracle import torch_ref as T
from tests.ltx_jit_util import make_inputs, make_weights


def test_engine_stack_compiles_and_has_the_reference_entry_points():
    unit = jit.stack_unit()
    for fn in ("stack", "block", "attention", "feed_forward", "rms", "rotate"):
        assert hasattr(unit, fn)


def test_slot_layout():
    assert jit.SLOTS_PER_BLOCK == 114 and len(jit.ATTN_SLOTS) == 16
    assert jit.ATTN_SLOTS.index("out_absmax") == 12 and jit.ATTN_SLOTS.index("norm_k_w") == 15
    assert sorted(jit.ATTN_BASES.values()) == [0, 16, 32, 48, 64, 80]
    assert jit.FF_BASES == {"ff": 96, "audio_ff": 102}
    assert sorted(jit.TABLE_SLOTS.values()) == list(range(108, 114))
    attns = {n: {k: torch.zeros(1) for k in jit.ATTN_SLOTS} for n in jit.ATTN_BASES}
    ffs = {n: (torch.zeros(1),) * 6 for n in jit.FF_BASES}
    tables = {n: torch.full((1,), float(i)) for n, i in jit.TABLE_SLOTS.items()}
    slots = jit.pack_block(attns, ffs, tables)
    assert len(slots) == 114 and slots[110].item() == 110.0
    with pytest.raises(KeyError):
        jit.pack_block(attns, ffs, {})


def test_stack_source_runs_with_the_reference_linear_on_cpu():
    d = 128
    unit = torch.jit.CompilationUnit(jit.stack_source("REF_LIN", T.NF4_LIN_TS_SOURCE))
    ws = make_weights(1, d, T.ltx23_nf4_quantize, "cpu")
    inp = make_inputs(d, "cpu", tv=8, ta=4, te=4)
    table2 = T.ltx23_jit_table("cpu", torch.bfloat16)
    h, ah = unit.stack(*inp, ws, table2, 1, d // 64, d // 64)
    assert h.shape == (1, 8, d) and ah.shape == (1, 4, d)
    assert torch.isfinite(h.float()).all() and torch.isfinite(ah.float()).all()


def test_engine_operator_has_no_cpu_kernel():
    jit.register_ops()
    x = torch.zeros(2, 64, dtype=torch.bfloat16)
    with pytest.raises(Exception):
        torch.ops.diffuser_b200.nf4_lin(x, torch.zeros(64 * 32, dtype=torch.uint8),
                                        torch.ones(64, dtype=torch.float32),
                                        torch.zeros(64, dtype=torch.bfloat16),
                                        torch.zeros(256, 2, dtype=torch.bfloat16))


def test_oracle_nf4_lin_is_the_dequantize_then_linear():
    # R/jit_ltx23.R:40-50 against R/nf4_ltx23.R:77-115 + nnf_linear
    g = torch.Generator().manual_seed(2)
    w = torch.randn(96, 128, generator=g) * 0.02
    p, a = T.ltx23_nf4_quantize(w)
    x = torch.randn(5, 128, generator=g).to(torch.bfloat16)
    bias = torch.randn(96, generator=g).to(torch.bfloat16)
    y = T.nf4_lin(x, p, a, bias, T.ltx23_jit_table("cpu", torch.bfloat16))
    ref = torch.nn.functional.linear(x, T.ltx23_nf4_dequantize(p, a, (96, 128)), bias)
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
