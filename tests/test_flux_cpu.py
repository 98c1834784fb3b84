"""The FLUX DiT port against the reference's own fixtures (CPU, float32):
the tiny transformer's output, the rotary tables, the rotary application and
the latent packing.  The fixtures are the reference's test vectors
(inst/tinytest/fixtures/flux_model.safetensors and rope_flux.safetensors),
committed as tests/golden/flux_reference_fixtures.safetensors by
tests/golden/extract_flux_fixtures.py; DIFFUSER_REF_FIXTURES may name the
reference's fixture directory to read the originals instead."""
import os

import pytest
import torch

from diffuser_b200 import flux

FIXTURES = os.environ.get("DIFFUSER_REF_FIXTURES")
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                      "flux_reference_fixtures.safetensors")


def _load(name):
    from safetensors.torch import load_file
    if FIXTURES:
        path = os.path.join(FIXTURES, name)
        if not os.path.exists(path):
            pytest.skip(f"reference fixture {name} not available")
        return load_file(path)
    stem = name[:-len(".safetensors")]
    return {k[len(stem) + 1:]: v for k, v in load_file(GOLDEN).items() if k.startswith(stem + "/")}


def _max_abs(a, b):
    return (a.float() - b.float()).abs().max().item()


def test_tiny_transformer_matches_reference_fixture():
    # R/dit_flux.R + inst/tinytest/test_flux_transformer.R: 1 double + 1 single block
    fx = _load("flux_model.safetensors")
    model = flux.FluxTransformer(in_channels=4, num_layers=1, num_single_layers=1,
                                 attention_head_dim=8, num_attention_heads=2,
                                 joint_attention_dim=16, pooled_projection_dim=12,
                                 axes_dims_rope=(2, 2, 4)).eval()
    state = {k[len("model."):]: v for k, v in fx.items() if k.startswith("model.")}
    model.load_state_dict(state, strict=True)  # every key lands, every parameter fills
    ids = torch.cat([fx["txt_ids"], fx["img_ids"]], dim=0)
    rope = flux.pos_embed(ids, (2, 2, 4))
    with torch.no_grad():
        out = model(fx["hidden"], fx["encoder"], fx["pooled"], fx["timestep"], rope)
    assert out.shape == fx["out"].shape
    assert _max_abs(out, fx["out"]) < 1e-4


def test_rotary_tables_match_reference_fixture():
    fx = _load("rope_flux.safetensors")
    cos, sin = flux.pos_embed(fx["ids"], (16, 56, 56))
    assert _max_abs(cos, fx["pos_full_cos"]) < 1e-6 and _max_abs(sin, fx["pos_full_sin"]) < 1e-6
    cos, sin = flux.pos_embed(fx["ids"], (2, 2, 4))
    assert _max_abs(cos, fx["pos_tiny_cos"]) < 1e-6 and _max_abs(sin, fx["pos_tiny_sin"]) < 1e-6
    img_ids = flux.prepare_latent_image_ids(8, 12)
    assert torch.equal(img_ids, fx["img_ids"])


def test_rotary_application_matches_reference_fixture():
    fx = _load("rope_flux.safetensors")
    freqs = (fx["pos_tiny_cos"], fx["pos_tiny_sin"])
    assert _max_abs(flux.apply_rotary_emb(fx["rot_x"], freqs), fx["rot_out"]) < 1e-5
    out16 = flux.apply_rotary_emb(fx["rot_x_f16"], freqs)
    assert out16.dtype == torch.float16
    assert _max_abs(out16, fx["rot_out_f16"]) < 1e-2


def test_latent_pack_roundtrip_matches_reference_fixture():
    fx = _load("rope_flux.safetensors")
    packed = flux.pack_latents(fx["pack_in"])
    assert torch.equal(packed, fx["pack_out"])
    assert torch.equal(flux.unpack_latents(fx["pack_out"], 8, 12, 16), fx["unpack_out"])


def test_euler_step_is_the_flowmatch_update():
    v = torch.randn(2, 5, 4, dtype=torch.bfloat16)
    x = torch.randn(2, 5, 4, dtype=torch.bfloat16)
    out = flux.euler_step(v, 0.75, 0.5, x)
    ref = (x.float() + (0.5 - 0.75) * v).to(torch.bfloat16)
    assert torch.equal(out, ref)


def test_cast_set_has_494_weights_at_full_size():
    # R/checkpoint_flux.R:21-42: the FLUX.1 quantization cast set
    from diffuser_b200 import modules
    with torch.device("meta"):
        model = flux.FluxTransformer()
    keys = [n for n, _ in model.named_parameters() if modules.flux_is_quant_key(n)]
    assert len(keys) == 494


def test_concat_nf4_linears_concatenates_rows():
    # NF4 rows are contiguous byte ranges: the concatenated module's buffers
    # decode to the stacked weights of the parts, biases follow (a missing
    # bias reads as zeros), and mixed input widths are refused
    from diffuser_b200 import flux, modules
    from oracle import torch_ref as T
    torch.manual_seed(0)
    parts = []
    for n, with_bias in ((64, True), (128, False), (192, True)):
        m = modules.Ltx23Nf4Linear(n, 256, bias=with_bias)
        p, a = T.ltx23_nf4_quantize(torch.randn(n, 256) * 0.02)
        m.set_nf4_weight(p, a)
        if with_bias:
            with torch.no_grad():
                m.bias.copy_(torch.randn(n))
        parts.append(m.to(torch.bfloat16))
    fused = flux.concat_nf4_linears(parts)
    assert fused.out_features == 384 and fused.in_features == 256
    w = T.ltx23_nf4_dequantize(fused.weight_nf4, fused.weight_absmax, (384, 256))
    ref = torch.cat([T.ltx23_nf4_dequantize(m.weight_nf4, m.weight_absmax, (m.out_features, 256))
                     for m in parts])
    assert torch.equal(w.view(torch.int16), ref.view(torch.int16))
    assert torch.equal(fused.bias[:64], parts[0].bias) and not fused.bias[64:192].any()
    assert torch.equal(fused.bias[192:], parts[2].bias)
    assert flux.concat_nf4_linears([parts[0], modules.Ltx23Nf4Linear(8, 128)]) is None
