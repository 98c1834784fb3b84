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

                def fwd(x, act=None, m=m, buf=buf):
                    y = T.nf4_linear_forward(x, m.weight_nf4, m.weight_absmax, m.out_features,
                                             m.in_features, m.bias, w_buffer=buf)
                    # the reference applies nnf_gelu(approximate = "tanh") after the linear
                    return torch.nn.functional.gelu(y, approximate="tanh") if act else y
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
        # the reference calls q, k and v separately and concatenates with torch.cat
        flux.FUSED_QKV = flux.FUSED_CONCAT = False
        try:
            ref = flux.sample(model, x, text, pooled, rope, sigmas)
        finally:
            ref_backend.restore()
            flux.FUSED_QKV = flux.FUSED_CONCAT = True
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.isfinite(out.float()).all()
    cos = torch.nn.functional.cosine_similarity(out.float().flatten(), ref.float().flatten(), dim=0)
    assert cos.item() >= 0.999, cos.item()


def test_concatenated_qkv_projection_matches_separate_linears():
    # one NF4 linear over the concatenated q/k/v rows gives the three
    # projections' outputs (text stream: 512 tokens, image: 4096)
    from diffuser_b200 import flux
    from oracle import numpy_ref as R
    from tests.gpu_util import to_bits
    dev = torch.device("cuda", 0)
    model = flux.build_flux_nf4(dev, seed=3, num_layers=1, num_single_layers=1)
    attn = model.transformer_blocks[0].attn
    for fused, parts, m in ((attn.to_qkv, (attn.to_q, attn.to_k, attn.to_v), 4096),
                            (attn.add_qkv, (attn.add_q_proj, attn.add_k_proj, attn.add_v_proj), 512)):
        x = torch.randn(1, m, 3072, device=dev).to(torch.bfloat16)
        with torch.no_grad():
            y = fused(x)
            ref = torch.cat([p(x) for p in parts], dim=-1)
        assert y.shape == ref.shape
        assert R.rel_err(to_bits(y.reshape(m, -1)), to_bits(ref.reshape(m, -1))) <= 1e-2
        assert (y != ref).float().mean().item() < 0.01


def test_flux_step_captures_in_a_cuda_graph():
    # the engine's launches (ctypes on the current stream, cluster launches,
    # cached workspaces) capture; replay reproduces the eager step bit for bit
    from diffuser_b200 import flux, ops
    dev = torch.device("cuda", 0)
    model = flux.build_flux_nf4(dev, seed=1, num_layers=2, num_single_layers=2)
    x, text, pooled, rope = _inputs(dev)
    t = torch.ones(1, dtype=torch.float32, device=dev)

    def step():
        with torch.no_grad():
            return flux.euler_step(model(x, text, pooled, t, rope), 1.0, 0.75, x)

    eager = step()
    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = step()
    g.replay()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.equal(out, eager)


def test_fused_attention_glue_wide_and_scalar_accesses_agree():
    # the kernels move aligned rows with 16/8/4-byte accesses and fall back to
    # element accesses for unaligned views (odd row stride or offset): both
    # give the same bits
    from diffuser_b200 import flux
    torch.manual_seed(1)
    dev = torch.device("cuda", 0)
    for (B, S_img, S_txt, H, D) in ((2, 21, 5, 3, 128), (1, 9, 4, 2, 64), (1, 7, 2, 2, 192),
                                    (1, 6, 3, 1, 256)):
        wide_i = torch.randn(B, S_img, H * D + 1, device=dev).to(torch.bfloat16)
        wide_t = torch.randn(B, S_txt, H * D + 1, device=dev).to(torch.bfloat16)
        img_u, txt_u = wide_i[..., 1:], wide_t[..., 1:]          # unaligned views
        img_a, txt_a = img_u.contiguous(), txt_u.contiguous()    # aligned copies
        w_img = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
        w_txt = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
        pos = torch.randint(0, 64, (S_txt + S_img, 3), device=dev).float()
        axes = {64: (16, 24, 24), 128: (16, 56, 56), 192: (32, 80, 80), 256: (32, 112, 112)}[D]
        rope = flux.pos_embed(pos, axes)
        with torch.no_grad():
            a = flux.qk_norm_rope(img_a, txt_a, H, w_img, w_txt, rope)
            u = flux.qk_norm_rope(img_u, txt_u, H, w_img, w_txt, rope)
            assert torch.equal(a, u)
            assert torch.equal(flux.qk_norm_rope(img_a, txt_a, H), flux.qk_norm_rope(img_u, txt_u, H))
            t_out, i_out = flux.heads_to_tokens(a, S_txt)
            # an unaligned source for the inverse layout: offset by one element
            buf = torch.empty(a.numel() + 1, dtype=torch.bfloat16, device=dev)
            a_u = buf[1:].view(a.shape)
            a_u.copy_(a)
            t_u, i_u = flux.heads_to_tokens(a_u, S_txt)
            assert torch.equal(t_out, t_u) and torch.equal(i_out, i_u)
            # image tokens into the first columns of a wider buffer
            wide = torch.full((B, S_img, H * D + 64), 3.0, dtype=torch.bfloat16, device=dev)
            _, i_w = flux.heads_to_tokens(a, S_txt, wide[..., :H * D])
            assert torch.equal(i_w, i_out) and (wide[..., H * D:] == 3.0).all()


def test_qkv_glue_in_one_launch_matches_one_call_per_part():
    # dq_qkv_norm_rope (q, k, v of one attention in one launch) gives the bits
    # of three dq_qk_norm_rope calls: column views of one concatenated
    # projection (aligned and unaligned rows), with and without text tokens
    from diffuser_b200 import flux
    torch.manual_seed(3)
    dev = torch.device("cuda", 0)
    for (B, S_img, S_txt, H, D, off) in ((2, 37, 9, 24, 128, 0), (1, 64, 0, 3, 64, 0),
                                         (1, 5, 3, 2, 256, 0), (1, 11, 4, 5, 128, 1)):
        hd = H * D
        qkv_i = torch.randn(B, S_img, 3 * hd + off, device=dev).to(torch.bfloat16)[..., off:]
        qkv_t = torch.randn(B, S_txt, 3 * hd + off, device=dev).to(torch.bfloat16)[..., off:] \
            if S_txt else None
        parts_i = [qkv_i[..., j * hd:(j + 1) * hd] for j in range(3)]
        parts_t = [None if qkv_t is None else qkv_t[..., j * hd:(j + 1) * hd] for j in range(3)]
        wq_i, wk_i, wq_t, wk_t = [(1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
                                  for _ in range(4)]
        if not S_txt:
            wq_t = wk_t = None
        pos = torch.randint(0, 64, (S_txt + S_img, 3), device=dev).float()
        axes = {64: (16, 24, 24), 128: (16, 56, 56), 256: (32, 112, 112)}[D]
        rope = flux.pos_embed(pos, axes)
        with torch.no_grad():
            q, k, v = flux.qkv_norm_rope(parts_i, parts_t, H, (wq_i, wk_i, None), (wq_t, wk_t, None),
                                         (True, True, False), rope, 1e-6)
            assert torch.equal(q, flux.qk_norm_rope(parts_i[0], parts_t[0], H, wq_i, wq_t, rope))
            assert torch.equal(k, flux.qk_norm_rope(parts_i[1], parts_t[1], H, wk_i, wk_t, rope))
            assert torch.equal(v, flux.qk_norm_rope(parts_i[2], parts_t[2], H))
            # two parts, no rotary table
            q2, v2 = flux.qkv_norm_rope(parts_i[0::2], parts_t[0::2], H, (wq_i, None), (wq_t, None),
                                        (False, False), None, 1e-6)
            assert torch.equal(q2, flux.qk_norm_rope(parts_i[0], parts_t[0], H, wq_i, wq_t))
            assert torch.equal(v2, v)


def test_adaln_glue_matches_tensor_ops():
    # AdaLN modulation and gated residual kernels vs the blocks' tensor-op
    # chains (R/dit_flux_modules.R:26-42, 54-70, 280-321): the residual is
    # the same bits; the modulation's LayerNorm statistics are summed in
    # another order, so its normalized value can sit one bf16 step away
    from diffuser_b200 import flux
    torch.manual_seed(2)
    dev = torch.device("cuda", 0)
    # the residual uses 16-byte runs when rows allow
    for (B, S, D) in ((2, 37, 256), (1, 65, 3072), (3, 5, 1028), (1, 3, 8192), (2, 9, 4096),
                      (1, 7, 1000)):
        x = (torch.randn(B, S, D, device=dev) * 3 + 0.5).to(torch.bfloat16)
        mods = (torch.randn(B, 6 * D, device=dev) * 0.5).to(torch.bfloat16)
        p = mods.chunk(6, dim=1)                                  # strided [B, D] views
        norm = torch.nn.LayerNorm(D, eps=1e-6, elementwise_affine=False)
        with torch.no_grad():
            ref = norm(x) * (p[1][:, None] + 1) + p[0][:, None]
            got = flux.adaln_modulate(x, p[1], p[0], 1e-6)
            assert got.shape == ref.shape and got.dtype == torch.bfloat16
            # one bf16 step of the normalized value, carried through the scale
            n = norm(x).float()
            tol = (n.abs() * 2.0 ** -7 + 1e-6) * (p[1][:, None].float() + 1).abs() \
                + ref.float().abs() * 2.0 ** -7
            assert ((got.float() - ref.float()).abs() <= tol + 1e-6).all()
            assert (got != ref).float().mean().item() < 0.02
            y = torch.randn(B, S, D, device=dev).to(torch.bfloat16)
            assert torch.equal(flux.gated_residual(x, p[2], y), x + p[2][:, None] * y)
            # a non-contiguous y (every other token row)
            y2 = torch.randn(B, 2 * S, D, device=dev).to(torch.bfloat16)[:, ::2]
            assert torch.equal(flux.gated_residual(x, p[5], y2), x + p[5][:, None] * y2)


def test_fused_attention_glue_matches_tensor_ops():
    # one kernel for norm + [text; image] + transpose + rotary vs the tensor-op
    # chain of the harness (R/dit_flux_modules.R:161-190, R/rope_flux.R:96-110)
    from diffuser_b200 import flux
    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    for (B, S_img, S_txt, H, D) in ((2, 37, 9, 3, 128), (1, 64, 0, 2, 64), (1, 5, 3, 2, 256)):
        img = torch.randn(B, S_img, H * D, device=dev).to(torch.bfloat16)
        txt = torch.randn(B, S_txt, H * D, device=dev).to(torch.bfloat16) if S_txt else None
        w_img = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
        w_txt = (1 + 0.1 * torch.randn(D, device=dev)).to(torch.bfloat16)
        pos = torch.randint(0, 64, (S_txt + S_img, 3), device=dev).float()
        axes = {64: (16, 24, 24), 128: (16, 56, 56), 256: (32, 112, 112)}[D]
        rope = flux.pos_embed(pos, axes)
        norm_i, norm_t = flux.RMSNorm(D).to(dev, torch.bfloat16), flux.RMSNorm(D).to(dev, torch.bfloat16)
        with torch.no_grad():
            norm_i.weight.copy_(w_img)
            norm_t.weight.copy_(w_txt)
            parts = [norm_i(img.unflatten(-1, (H, -1)))]
            if S_txt:
                parts.insert(0, norm_t(txt.unflatten(-1, (H, -1))))
            ref = flux.apply_rotary_emb(torch.cat(parts, dim=1).transpose(1, 2), rope)
            got = flux.qk_norm_rope(img, txt, H, w_img, w_txt if S_txt else None, rope)
            # the mean is summed in another order: at most one bf16 step apart
            step = ref.float().abs().clamp(min=1e-30) * 2.0 ** -7
            assert ((got.float() - ref.float()).abs() <= step + 1e-30).all()
            assert (got != ref).float().mean().item() < 0.02
            vparts = [img.unflatten(-1, (H, -1))]
            if S_txt:
                vparts.insert(0, txt.unflatten(-1, (H, -1)))
            vref = torch.cat(vparts, dim=1).transpose(1, 2)
            assert torch.equal(flux.qk_norm_rope(img, txt, H), vref)
            t_out, i_out = flux.heads_to_tokens(vref.contiguous(), S_txt)
            assert torch.equal(i_out, img)
            if S_txt:
                assert torch.equal(t_out, txt)
