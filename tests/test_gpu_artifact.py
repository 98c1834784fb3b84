"""Artifacts on the GPU: a FLUX-shaped transformer written as an NF4 artifact
with the engine's quantizer, loaded into a fresh skeleton (the reference's
flux_load_transformer, R/quantize_flux.R:488-627), must produce the bits of
the same model quantized in memory (swap_quant_linears); with the block scales
repacked to bf16 at load time too.  A Gemma3-style gated MLP loaded from an
artifact runs gate_proj / up_proj as one NF4 linear with GELU-tanh fused."""
import copy

import pytest
import torch
from torch import nn

from diffuser_b200 import artifact, flux, modules, ops

pytestmark = pytest.mark.gpu

CFG = dict(in_channels=64, num_layers=1, num_single_layers=2, attention_head_dim=64,
           num_attention_heads=2, joint_attention_dim=128, pooled_projection_dim=64,
           axes_dims_rope=(16, 24, 24))


def _inputs(dev, s_img=256, s_txt=32):
    g = torch.Generator().manual_seed(4)
    x = torch.randn(1, s_img, 64, generator=g).to(dev, torch.bfloat16)
    text = torch.randn(1, s_txt, 128, generator=g).to(dev, torch.bfloat16)
    pooled = torch.randn(1, 64, generator=g).to(dev, torch.bfloat16)
    ids = torch.cat([torch.zeros(s_txt, 3), flux.prepare_latent_image_ids(16, 16)], dim=0)
    rope = flux.pos_embed(ids.to(dev), CFG["axes_dims_rope"])
    t = torch.ones(1, dtype=torch.float32, device=dev)
    return x, text, pooled, t, rope


@pytest.mark.parametrize("scales", ["f32", "bf16"])
def test_flux_artifact_loads_to_the_in_memory_quantized_model(tmp_path, scales):
    dev = torch.device("cuda", 0)
    with torch.device(dev):
        src = flux.FluxTransformer(**CFG).to(torch.bfloat16)
    flux.init_random_(src, seed=9)
    state = {k: v.detach().clone() for k, v in src.state_dict().items()}
    tensors, n_cast = artifact.quantize_state(state, modules.flux_is_quant_key, "nf4")
    artifact.write_artifact(str(tmp_path), tensors, "nf4", n_cast, config=CFG, shard_bytes=2e6)
    mem = copy.deepcopy(src)
    swapped = modules.swap_quant_linears(mem, modules.flux_is_quant_key, "nf4")
    with torch.device(dev):
        dst = flux.FluxTransformer(**CFG).to(torch.bfloat16)
    rep = artifact.load_quantized(dst, artifact.open_artifact(str(tmp_path)), scales=scales)
    assert sorted(rep["cast"]) == sorted(swapped) and not rep["missing"]
    inp = _inputs(dev)
    with torch.no_grad():
        a = mem.eval()(*inp)
        b = dst.eval()(*inp)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert ops.device_error() == 0


class _GemmaMlp(nn.Module):
    def __init__(self, hidden, inter):
        super().__init__()
        self.layers = nn.ModuleList([nn.Module()])
        mlp = nn.Module()
        mlp.gate_proj = nn.Linear(hidden, inter, bias=False)
        mlp.up_proj = nn.Linear(hidden, inter, bias=False)
        mlp.down_proj = nn.Linear(inter, hidden, bias=False)
        self.layers[0].mlp = mlp


def test_gemma3_gated_mlp_from_artifact(tmp_path):
    dev = torch.device("cuda", 0)
    hidden, inter, m = 512, 1536, 96
    torch.manual_seed(11)
    src = _GemmaMlp(hidden, inter).to(dev, torch.bfloat16)
    with torch.no_grad():
        for p in src.parameters():
            p.normal_(0, 0.02)
    state = {k: v.detach().clone() for k, v in src.state_dict().items()}
    tensors, n_cast = artifact.quantize_state(state, artifact.gemma3_is_quant_key, "nf4")
    assert n_cast == 3
    artifact.write_artifact(str(tmp_path), tensors, "nf4", n_cast, shard_prefix="gemma3",
                            extra={"model": "gemma3"})
    art = artifact.open_artifact(str(tmp_path))
    assert art.manifest["model"] == "gemma3"
    dst = _GemmaMlp(hidden, inter).to(dev, torch.bfloat16)
    artifact.load_quantized(dst, art)
    mlp = dst.layers[0].mlp
    x = torch.randn(m, hidden, device=dev).to(torch.bfloat16)
    ref = mlp.down_proj(torch.nn.functional.gelu(mlp.gate_proj(x), approximate="tanh") * mlp.up_proj(x))
    fused = modules.fuse_gated_pair(mlp.gate_proj, mlp.up_proj, "geglu_tanh")
    y = mlp.down_proj(fused(x))
    torch.cuda.synchronize()
    err = ((y.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
    assert err <= 1e-2, err
