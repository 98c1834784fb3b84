"""The on-disk artifact format (CPU, no GPU): written with the oracle's
quantizers, read back, and loaded into a module tree the way the reference's
loaders do (R/quantize_flux.R:366-444, :488-627; R/fp8_ltx23.R:230-265;
R/quantize_gemma3.R:29-215)."""
import json
import os

import pytest
import torch
from torch import nn

from diffuser_b200 import artifact, modules
from oracle import torch_ref as T


class Tiny(nn.Module):
    def __init__(self):
        super().__init__()
        self.proj_in = nn.Linear(128, 64)
        self.blocks = nn.ModuleList([nn.ModuleDict({"q_proj": nn.Linear(64, 128, bias=False),
                                                    "norm": nn.LayerNorm(64)}) for _ in range(2)])
        self.register_buffer("table", torch.arange(6, dtype=torch.float32))


def _is_quant(key):
    return key.endswith("q_proj.weight") or key == "proj_in.weight"


def _state(seed=0):
    torch.manual_seed(seed)
    m = Tiny()
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0, 0.02)
    return m, {k: v.detach().clone() for k, v in m.state_dict().items()}


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
def test_write_open_and_load_round_trip(tmp_path, fmt):
    src, state = _state()
    tensors, n_cast = artifact.quantize_state(state, _is_quant, fmt, quantize_nf4=T.ltx23_nf4_quantize,
                                              quantize_fp8=T.fp8_quantize)
    assert n_cast == 3
    man = artifact.write_artifact(str(tmp_path), tensors, fmt, n_cast, config={"dim": 64},
                                  shard_bytes=4096, shard_prefix="tiny")
    assert len(man["shards"]) > 1 and man["cast"] == 3 and man["format"] == fmt
    with open(os.path.join(tmp_path, "manifest.json")) as f:
        assert json.load(f)["config"] == {"dim": 64}
    art = artifact.open_artifact(str(tmp_path))
    assert sorted(art.cast_keys()) == sorted(k for k in state if _is_quant(k))
    if fmt == "nf4":
        assert art.get_tensor("proj_in.weight").dtype == torch.uint8
        assert art.get_tensor("proj_in.weight_absmax").dtype == torch.float32
    else:
        assert art.get_tensor("proj_in.weight").dtype == torch.float8_e4m3fn
        assert art.get_tensor("proj_in.weight_scale").shape == ()
    assert art.get_tensor("proj_in.bias").dtype == torch.bfloat16  # residents in bf16

    dst, _ = _state(seed=1)  # a skeleton with other values
    report = artifact.load_quantized(dst, art)
    cls = modules.Ltx23Nf4Linear if fmt == "nf4" else modules.Ltx23Fp8Linear
    assert isinstance(dst.proj_in, cls) and isinstance(dst.blocks[1]["q_proj"], cls)
    assert isinstance(dst.blocks[0]["norm"], nn.LayerNorm)
    assert "proj_in.bias" in report["residents"] and not report["missing"]
    assert torch.equal(dst.proj_in.bias.detach(), state["proj_in.bias"].to(torch.bfloat16).float())
    assert torch.equal(dst.table, state["table"])
    if fmt == "nf4":
        p, a = T.ltx23_nf4_quantize(state["proj_in.weight"])
        assert torch.equal(dst.proj_in.weight_nf4, p) and torch.equal(dst.proj_in.weight_absmax, a)
    else:
        w8, s = T.fp8_quantize(state["proj_in.weight"])
        assert torch.equal(dst.proj_in.weight_fp8.view(torch.uint8), w8.view(torch.uint8))


def test_bf16_scales_repack_is_the_forward_cast(tmp_path):
    _, state = _state()
    tensors, n_cast = artifact.quantize_state(state, _is_quant, "nf4", quantize_nf4=T.ltx23_nf4_quantize)
    artifact.write_artifact(str(tmp_path), tensors, "nf4", n_cast)
    dst, _ = _state(seed=2)
    artifact.load_quantized(dst, artifact.open_artifact(str(tmp_path)), scales="bf16")
    a16 = dst.blocks[0]["q_proj"].weight_absmax
    assert a16.dtype == torch.bfloat16
    assert torch.equal(a16, tensors["blocks.0.q_proj.weight_absmax"].to(torch.bfloat16))
    # the dequantized weight is unchanged (R/nf4_ltx23.R:97 casts absmax to bf16)
    p = dst.blocks[0]["q_proj"].weight_nf4
    w16 = T.ltx23_nf4_dequantize(p, a16.float(), (128, 64))
    w32 = T.ltx23_nf4_dequantize(p, tensors["blocks.0.q_proj.weight_absmax"], (128, 64))
    assert torch.equal(w16.view(torch.int16), w32.view(torch.int16))
    # a dtype move keeps the repacked scales
    assert dst.blocks[0]["q_proj"].to(torch.float32).weight_absmax.dtype == torch.bfloat16


def test_strict_loading_refuses_gaps_and_strays(tmp_path):
    _, state = _state()
    del state["blocks.1.norm.weight"]
    state["stray.weight"] = torch.zeros(3)
    tensors, n_cast = artifact.quantize_state(state, _is_quant, "nf4", quantize_nf4=T.ltx23_nf4_quantize)
    artifact.write_artifact(str(tmp_path), tensors, "nf4", n_cast)
    dst, _ = _state()
    with pytest.raises(KeyError):
        artifact.load_quantized(dst, artifact.open_artifact(str(tmp_path)))
    dst, _ = _state()
    rep = artifact.load_quantized(dst, artifact.open_artifact(str(tmp_path)), strict=False)
    assert rep["unknown"] == ["stray.weight"] and "blocks.1.norm.weight" in rep["missing"]
    with pytest.raises(FileNotFoundError):
        artifact.open_artifact(str(tmp_path / "nowhere"))


def test_gemma3_selector_and_key_normalization():
    # R/quantize_gemma3.R:91-95 and :126-130
    assert artifact.gemma3_normalize_key("language_model.model.layers.3.mlp.up_proj.weight") == \
        "layers.3.mlp.up_proj.weight"
    assert artifact.gemma3_normalize_key("vision_tower.encoder.weight") is None
    assert artifact.gemma3_normalize_key("lm_head.weight") is None
    for k in ("layers.0.self_attn.q_proj.weight", "layers.47.self_attn.o_proj.weight",
              "layers.1.mlp.gate_proj.weight", "layers.1.mlp.down_proj.weight"):
        assert artifact.gemma3_is_quant_key(k)
    for k in ("layers.0.self_attn.q_norm.weight", "embed_tokens.weight", "layers.0.mlp.up_proj.bias",
              "norm.weight", "layers.0.input_layernorm.weight"):
        assert not artifact.gemma3_is_quant_key(k)


def test_gated_pair_fusion_concatenates_rows_in_gated_order():
    torch.manual_seed(3)
    g, u = modules.Ltx23Nf4Linear(64, 128, bias=False), modules.Ltx23Nf4Linear(64, 128, bias=False)
    for m in (g, u):
        m.set_nf4_weight(*T.ltx23_nf4_quantize(torch.randn(64, 128) * 0.02))
    f = modules.fuse_gated_pair(g, u, "geglu_tanh")
    assert f.gated_act == "geglu_tanh" and f.out_features == 128
    w = T.ltx23_nf4_dequantize(f.weight_nf4, f.weight_absmax, (128, 128))
    wg = T.ltx23_nf4_dequantize(g.weight_nf4, g.weight_absmax, (64, 128))
    wu = T.ltx23_nf4_dequantize(u.weight_nf4, u.weight_absmax, (64, 128))
    assert torch.equal(w[0:16], wg[0:16]) and torch.equal(w[16:32], wu[0:16])
    assert torch.equal(w[32:48], wg[16:32]) and torch.equal(w[112:128], wu[48:64])
