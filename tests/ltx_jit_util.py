"""Synthetic LTX-2.3 block-stack weights and inputs for the TorchScript stack
tests (all widths D, heads of 64, feed-forward 4 D)."""
import torch

from diffuser_b200 import jit


def make_weights(n_blocks, d, quantize, device, seed=0):
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape, std=0.02):
        return (torch.randn(*shape, generator=g) * std)

    def q_lin(n, k):
        p, a = quantize(rnd(n, k))
        return p.to(device), a.to(device), (rnd(n, std=0.1)).to(device, torch.bfloat16)

    heads = d // 64
    ws = []
    for _ in range(n_blocks):
        attns = {}
        for name in jit.ATTN_BASES:
            e = {"gate_w": rnd(heads, d).to(device, torch.bfloat16),
                 "gate_b": rnd(heads, std=0.1).to(device, torch.bfloat16),
                 "norm_q_w": (1 + rnd(d, std=0.1)).to(device, torch.bfloat16),
                 "norm_k_w": (1 + rnd(d, std=0.1)).to(device, torch.bfloat16)}
            for proj in ("q", "k", "v", "out"):
                e[proj + "_packed"], e[proj + "_absmax"], e[proj + "_bias"] = q_lin(d, d)
            attns[name] = e
        ffs = {name: q_lin(4 * d, d) + q_lin(d, 4 * d) for name in jit.FF_BASES}
        rows = {"scale_shift_table": 9, "audio_scale_shift_table": 9, "prompt_scale_shift_table": 2,
                "audio_prompt_scale_shift_table": 2, "video_a2v_cross_attn_scale_shift_table": 5,
                "audio_a2v_cross_attn_scale_shift_table": 5}
        tables = {name: rnd(r, d, std=0.1).to(device, torch.bfloat16) for name, r in rows.items()}
        ws += jit.pack_block(attns, ffs, tables)
    return ws


def make_inputs(d, device, tv=64, ta=32, te=16, seed=1):
    g = torch.Generator().manual_seed(seed)

    def bf(*shape, std=1.0):
        return (torch.randn(*shape, generator=g) * std).to(device, torch.bfloat16)

    def rope(t):
        ang = torch.randn(1, t, d // 2, generator=g)
        return torch.cos(ang).to(device), torch.sin(ang).to(device)

    v_cos, v_sin = rope(tv)
    a_cos, a_sin = rope(ta)
    cav_cos, cav_sin = rope(tv)
    caa_cos, caa_sin = rope(ta)
    return [bf(1, tv, d), bf(1, ta, d), bf(1, te, d), bf(1, te, d),
            bf(1, 1, 9 * d, std=0.1), bf(1, 1, 9 * d, std=0.1), bf(1, 1, 4 * d, std=0.1),
            bf(1, 1, 4 * d, std=0.1), bf(1, 1, d, std=0.1), bf(1, 1, d, std=0.1),
            bf(1, 1, 2 * d, std=0.1), bf(1, 1, 2 * d, std=0.1),
            v_cos, v_sin, a_cos, a_sin, cav_cos, cav_sin, caa_cos, caa_sin,
            None, None, None]
