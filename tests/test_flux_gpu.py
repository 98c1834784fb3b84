"""FLUX.1 1024x1024 DiT with NF4 cast linears on the fused engine versus the
same model on the reference's linear (dequantize into a bf16 buffer, then
F.linear; R/nf4_ltx23.R:235-246), over the 4-step Euler flow-match schedule
sigmas {1, .75, .5, .25}: final latents must agree to cosine >= 0.999."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(device):
    from diffuser_b200 import flux
    g = torch.Generator().manual_seed(2)
    latents = torch.randn(1, 16, 128, 128, generator=g)
    g1 = torch.Generator().manual_seed(3)
    text = torch.randn(1, 512, 4096, generator=g1)
    pooled = torch.randn(1, 768, generator=g1)
    x = flux.pack_latents(latents).to(device, torch.bfloat16)
    ids = torch.cat([torch.zeros(512, 3), flux.prepare_latent_image_ids(64, 64)], dim=0)
    rope = flux.pos_embed(ids.to(device), (16, 56, 56))
    return x, text.to(device, torch.bfloat16), pooled.to(device, torch.bfloat16), rope


class _ReferenceBackend:
    """Swap every fused NF4 linear's forward for the oracle's restatement of
    the reference's op sequence, with one bf16 weight buffer per shape."""

    def __init__(self, model):
        from diffuser_b200 import modules
        from oracle import torch_ref as T
        self.saved = []
        buffers = {}
        for m in model.modules():
            if isinstance(m, modules.Ltx23Nf4Linear):
                key = (m.out_features, m.in_features)
                if key not in buffers:
                    buffers[key] = torch.empty(key, dtype=torch.bfloat16, device=m.weight_nf4.device)
                buf = buffers[key]

                def fwd(x, m=m, buf=buf):
                    return T.nf4_linear_forward(x, m.weight_nf4, m.weight_absmax, m.out_features,
                                                m.in_features, m.bias, w_buffer=buf)
                self.saved.append((m, m.forward))
                m.forward = fwd

    def restore(self):
        for m, f in self.saved:
            m.forward = f


def test_flux_dit_fused_matches_reference_backend():
    from diffuser_b200 import flux, ops
    dev = torch.device("cuda", 0)
    model = flux.build_flux_nf4(dev, seed=0)
    x, text, pooled, rope = _inputs(dev)
    sigmas = [1.0, 0.75, 0.5, 0.25]
    with torch.no_grad():
        out = flux.sample(model, x, text, pooled, rope, sigmas)
        ref_backend = _ReferenceBackend(model)
        try:
            ref = flux.sample(model, x, text, pooled, rope, sigmas)
        finally:
            ref_backend.restore()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.isfinite(out.float()).all()
    cos = torch.nn.functional.cosine_similarity(out.float().flatten(), ref.float().flatten(), dim=0)
    assert cos.item() >= 0.999, cos.item()
