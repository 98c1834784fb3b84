"""The LTX-2.3 TorchScript block stack on the GPU: the stack compiled with
the engine's operators (torch.ops.diffuser_b200.nf4_lin / nf4_lin_act) against
the same stack compiled with the reference's own nf4_lin (the byte-table
embedding gather times bf16 block scales, then linear; R/jit_ltx23.R:40-50),
two blocks on the same NF4 weights and inputs."""
import pytest
import torch

from diffuser_b200 import jit, ops
from oracle import torch_ref as T
from tests.ltx_jit_util import make_inputs, make_weights

pytestmark = pytest.mark.gpu


def test_engine_stack_matches_reference_stack():
    dev = torch.device("cuda", 0)
    d, n_blocks = 256, 2
    ws = make_weights(n_blocks, d, T.ltx23_nf4_quantize, dev, seed=3)
    inp = make_inputs(d, dev, tv=192, ta=64, te=32)
    table2 = T.ltx23_jit_table(dev, torch.bfloat16)
    engine = jit.stack_unit()
    ref = torch.jit.CompilationUnit(jit.stack_source("REF_LIN", T.NF4_LIN_TS_SOURCE))
    with torch.no_grad():
        h, ah = engine.stack(*inp, ws, table2, n_blocks, d // 64, d // 64)
        rh, rah = ref.stack(*inp, ws, table2, n_blocks, d // 64, d // 64)
    torch.cuda.synchronize()
    for a, b in ((h, rh), (ah, rah)):
        assert a.dtype == torch.bfloat16 and a.shape == b.shape
        err = ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()
        cos = torch.nn.functional.cosine_similarity(a.float().flatten(), b.float().flatten(), dim=0).item()
        assert err <= 1e-2 and cos >= 0.9999, (err, cos)
    assert ops.device_error() == 0


def test_engine_linear_operator_matches_reference_nf4_lin():
    dev = torch.device("cuda", 0)
    jit.register_ops()
    g = torch.Generator().manual_seed(8)
    w = torch.randn(384, 512, generator=g) * 0.02
    p, a = T.ltx23_nf4_quantize(w)
    p, a = p.to(dev), a.to(dev)
    bias = (torch.randn(384, generator=g) * 0.1).to(dev, torch.bfloat16)
    x = torch.randn(2, 70, 512, generator=g).to(dev, torch.bfloat16)
    table2 = T.ltx23_jit_table(dev, torch.bfloat16)
    y = torch.ops.diffuser_b200.nf4_lin(x, p, a, bias, table2)
    r = T.nf4_lin(x, p, a, bias, table2)
    yg = torch.ops.diffuser_b200.nf4_lin_act(x, p, a, bias, 1)
    rg = torch.nn.functional.gelu(r, approximate="tanh")
    torch.cuda.synchronize()
    assert y.shape == (2, 70, 384)
    assert ((y.float() - r.float()).abs().max() / r.float().abs().max()).item() <= 1e-2
    assert ((yg.float() - rg.float()).abs().max() / rg.float().abs().max()).item() <= 1e-2
