"""The LTX-2.3 TorchScript block stack on the engine.

The reference compiles its 48-block NF4 LTX-2.3 transformer step into one
TorchScript unit (R/jit_ltx23.R:40-195) so that a whole step is a single
R -> libtorch crossing; inside it every quantized linear is ``nf4_lin``, a
byte-table embedding gather times the bf16 block scales followed by
``torch.linear`` (:40-50).  Here the same stack (written for the Python
TorchScript frontend, which spells the aten ops ``torch.nn.functional.*``)
calls the engine instead,
through two operators registered with the PyTorch dispatcher, which
TorchScript resolves like any builtin:

* ``torch.ops.diffuser_b200.nf4_lin(x, packed, absmax, bias, table2)`` --
  the drop-in for ``nf4_lin`` (same arguments; ``table2``, the reference's
  byte LUT, is accepted and unused: the kernels carry their own);
* ``torch.ops.diffuser_b200.nf4_lin_act(x, packed, absmax, bias, act)`` --
  the same with an epilogue activation (1 = GELU-tanh, the feed-forward's
  up-projection, R/jit_ltx23.R:97-99).

Both run only on CUDA tensors (there is no CPU kernel).  ``stack_unit()``
compiles the block stack with them; its weights are the reference's flat
``List[Tensor]`` with 114 slots per block (the per-attention and per-block
layout at R/jit_ltx23.R:21-34, kept identical so that a packer written for
the reference fills it), built here by ``pack_block``.
"""
from __future__ import annotations

import torch

from . import ops

_LIB = None

SLOTS_PER_BLOCK = 114
# per-attention slot offsets (R/jit_ltx23.R:21-25)
ATTN_SLOTS = ("gate_w", "gate_b", "q_packed", "q_absmax", "q_bias", "k_packed", "k_absmax", "k_bias",
              "v_packed", "v_absmax", "v_bias", "out_packed", "out_absmax", "out_bias",
              "norm_q_w", "norm_k_w")
# attention bases within a block (R/jit_ltx23.R:26-28)
ATTN_BASES = {"attn1": 0, "audio_attn1": 16, "attn2": 32, "audio_attn2": 48,
              "audio_to_video_attn": 64, "video_to_audio_attn": 80}
FF_BASES = {"ff": 96, "audio_ff": 102}  # proj (packed, absmax, bias), net2 (packed, absmax, bias)
TABLE_SLOTS = {"scale_shift_table": 108, "audio_scale_shift_table": 109,
               "prompt_scale_shift_table": 110, "audio_prompt_scale_shift_table": 111,
               "video_a2v_cross_attn_scale_shift_table": 112,
               "audio_a2v_cross_attn_scale_shift_table": 113}


def _nf4_lin(x, packed, absmax, bias, table2):
    return ops.nf4_linear(x, packed, absmax, bias.size(0), bias)


def _nf4_lin_act(x, packed, absmax, bias, act):
    return ops.nf4_linear(x, packed, absmax, bias.size(0), bias,
                          act={0: None, 1: "gelu_tanh"}[int(act)])


def register_ops():
    """Register the two operators (idempotent)."""
    global _LIB
    if _LIB is not None:
        return
    lib = torch.library.Library("diffuser_b200", "DEF")
    lib.define("nf4_lin(Tensor x, Tensor packed, Tensor absmax, Tensor bias, Tensor table2) -> Tensor")
    lib.define("nf4_lin_act(Tensor x, Tensor packed, Tensor absmax, Tensor bias, int act) -> Tensor")
    lib.impl("nf4_lin", _nf4_lin, "CUDA")
    lib.impl("nf4_lin_act", _nf4_lin_act, "CUDA")
    _LIB = lib


# The block stack, TorchScript source.  LIN / LIN_GELU name the quantized
# linear and the linear followed by GELU-tanh; stack_unit() binds them to the
# engine's operators.
_STACK_SOURCE = '''
def rms(x: Tensor) -> Tensor:
    ms = x.float().pow(2).mean(-1, keepdim=True)
    return (x * torch.rsqrt(ms + 1e-6)).type_as(x)

def rms_scaled(x: Tensor, w: Tensor) -> Tensor:
    ms = x.float().pow(2).mean(-1, keepdim=True)
    return (x * torch.rsqrt(ms + 1e-6)).type_as(w) * w

def rotate(x: Tensor, c: Tensor, s: Tensor) -> Tensor:
    # split-half rotary embedding, over the whole width ([B, T, r] tables) or
    # per head ([B, H, T, r] tables)
    if c.dim() == 4:
        b = c.size(0)
        nh = c.size(1)
        t = c.size(2)
        xh = x.reshape([b, t, nh, -1]).transpose(1, 2)
        half = xh.size(-1) // 2
        a = xh.narrow(-1, 0, half).float()
        z = xh.narrow(-1, half, half).float()
        r = torch.cat([a * c - z * s, z * c + a * s], -1)
        return r.transpose(1, 2).reshape([b, t, -1]).type_as(x)
    half = x.size(-1) // 2
    a = x.narrow(-1, 0, half).float()
    z = x.narrow(-1, half, half).float()
    return torch.cat([a * c - z * s, z * c + a * s], -1).type_as(x)

def modulation(table: Tensor, emb: Tensor, n: int) -> Tensor:
    return table.unsqueeze(0).unsqueeze(0) + emb.reshape([emb.size(0), emb.size(1), n, -1])

def mod_at(m: Tensor, j: int, idx: Optional[Tensor]) -> Tensor:
    v = m.select(2, j)
    if idx is None:
        return v
    return v.index_select(1, idx)

def attention(x: Tensor, ctx: Tensor, ws: List[Tensor], o: int, table2: Tensor, heads: int,
              qc: Optional[Tensor], qs: Optional[Tensor], kc: Optional[Tensor], ks: Optional[Tensor],
              mask: Optional[Tensor]) -> Tensor:
    gate = torch.nn.functional.linear(x, ws[o], ws[o + 1])
    q = rms_scaled(LIN(x, ws[o + 2], ws[o + 3], ws[o + 4], table2), ws[o + 14])
    k = rms_scaled(LIN(ctx, ws[o + 5], ws[o + 6], ws[o + 7], table2), ws[o + 15])
    v = LIN(ctx, ws[o + 8], ws[o + 9], ws[o + 10], table2)
    if qc is not None and qs is not None:
        q = rotate(q, qc, qs)
    if kc is not None and ks is not None:
        k = rotate(k, kc, ks)
    a = torch.nn.functional.scaled_dot_product_attention(q.unflatten(-1, [heads, -1]).transpose(1, 2),
                                                         k.unflatten(-1, [heads, -1]).transpose(1, 2),
                                                         v.unflatten(-1, [heads, -1]).transpose(1, 2),
                                                         attn_mask=mask)
    a = a.transpose(1, 2).flatten(2).type_as(x)
    a = (a.unflatten(-1, [heads, -1]) * (torch.sigmoid(gate) * 2.0).unsqueeze(-1)).flatten(2)
    return LIN(a, ws[o + 11], ws[o + 12], ws[o + 13], table2)

def feed_forward(x: Tensor, ws: List[Tensor], o: int, table2: Tensor) -> Tensor:
    return LIN(LIN_GELU(x, ws[o], ws[o + 1], ws[o + 2], table2), ws[o + 3], ws[o + 4], ws[o + 5], table2)

def block(h: Tensor, ah: Tensor, enc: Tensor, aenc: Tensor, temb: Tensor, temb_a: Tensor,
          tcss: Tensor, tcass: Tensor, tcg: Tensor, tcag: Tensor, tp: Tensor, tpa: Tensor,
          v_cos: Tensor, v_sin: Tensor, a_cos: Tensor, a_sin: Tensor,
          cav_cos: Tensor, cav_sin: Tensor, caa_cos: Tensor, caa_sin: Tensor,
          enc_mask: Optional[Tensor], aenc_mask: Optional[Tensor], cond_idx: Optional[Tensor],
          ws: List[Tensor], o: int, table2: Tensor, heads: int, aheads: int) -> Tuple[Tensor, Tensor]:
    vm = modulation(ws[o + 108], temb, 9)
    am = modulation(ws[o + 109], temb_a, 9)
    # self-attention, video then audio
    x = rms(h) * (mod_at(vm, 1, cond_idx) + 1.0) + mod_at(vm, 0, cond_idx)
    h = h + attention(x, x, ws, o, table2, heads, v_cos, v_sin, v_cos, v_sin, None) * mod_at(vm, 2, cond_idx)
    xa = rms(ah) * (am.select(2, 1) + 1.0) + am.select(2, 0)
    ah = ah + attention(xa, xa, ws, o + 16, table2, aheads, a_cos, a_sin, a_cos, a_sin, None) * am.select(2, 2)
    # cross-attention to the prompts
    pm = modulation(ws[o + 110], tp, 2)
    apm = modulation(ws[o + 111], tpa, 2)
    x = rms(h) * (mod_at(vm, 7, cond_idx) + 1.0) + mod_at(vm, 6, cond_idx)
    e = enc * (pm.select(2, 1) + 1.0) + pm.select(2, 0)
    h = h + attention(x, e, ws, o + 32, table2, heads, None, None, None, None, enc_mask) * mod_at(vm, 8, cond_idx)
    xa = rms(ah) * (am.select(2, 7) + 1.0) + am.select(2, 6)
    ea = aenc * (apm.select(2, 1) + 1.0) + apm.select(2, 0)
    ah = ah + attention(xa, ea, ws, o + 48, table2, aheads, None, None, None, None, aenc_mask) * am.select(2, 8)
    # audio <-> video cross-attention
    hn = rms(h)
    an = rms(ah)
    vc = modulation(ws[o + 112].narrow(0, 0, 4), tcss, 4)
    vg = modulation(ws[o + 112].narrow(0, 4, 1), tcg, 1)
    ac = modulation(ws[o + 113].narrow(0, 0, 4), tcass, 4)
    ag = modulation(ws[o + 113].narrow(0, 4, 1), tcag, 1)
    xv = hn * (vc.select(2, 0) + 1.0) + vc.select(2, 1)
    xa = an * (ac.select(2, 0) + 1.0) + ac.select(2, 1)
    h = h + vg.select(2, 0) * attention(xv, xa, ws, o + 64, table2, aheads, cav_cos, cav_sin, caa_cos, caa_sin, None)
    xv = hn * (vc.select(2, 2) + 1.0) + vc.select(2, 3)
    xa = an * (ac.select(2, 2) + 1.0) + ac.select(2, 3)
    ah = ah + ag.select(2, 0) * attention(xa, xv, ws, o + 80, table2, aheads, caa_cos, caa_sin, cav_cos, cav_sin, None)
    # feed-forward, video then audio
    x = rms(h) * (mod_at(vm, 4, cond_idx) + 1.0) + mod_at(vm, 3, cond_idx)
    h = h + feed_forward(x, ws, o + 96, table2) * mod_at(vm, 5, cond_idx)
    xa = rms(ah) * (am.select(2, 4) + 1.0) + am.select(2, 3)
    ah = ah + feed_forward(xa, ws, o + 102, table2) * am.select(2, 5)
    return (h, ah)

def stack(h: Tensor, ah: Tensor, enc: Tensor, aenc: Tensor, temb: Tensor, temb_a: Tensor,
          tcss: Tensor, tcass: Tensor, tcg: Tensor, tcag: Tensor, tp: Tensor, tpa: Tensor,
          v_cos: Tensor, v_sin: Tensor, a_cos: Tensor, a_sin: Tensor,
          cav_cos: Tensor, cav_sin: Tensor, caa_cos: Tensor, caa_sin: Tensor,
          enc_mask: Optional[Tensor], aenc_mask: Optional[Tensor], cond_idx: Optional[Tensor],
          ws: List[Tensor], table2: Tensor, n_blocks: int, heads: int, aheads: int) -> Tuple[Tensor, Tensor]:
    for i in range(n_blocks):
        h, ah = block(h, ah, enc, aenc, temb, temb_a, tcss, tcass, tcg, tcag, tp, tpa,
                      v_cos, v_sin, a_cos, a_sin, cav_cos, cav_sin, caa_cos, caa_sin,
                      enc_mask, aenc_mask, cond_idx, ws, i * 114, table2, heads, aheads)
    return (h, ah)
'''


def stack_source(lin: str, lin_gelu_prefix: str = "") -> str:
    """The stack's TorchScript source with LIN bound to `lin` and LIN_GELU to
    a function defined in `lin_gelu_prefix` (a caller may bind other linears,
    e.g. a restatement of the reference's own nf4_lin for comparison)."""
    return lin_gelu_prefix + _STACK_SOURCE.replace("LIN_GELU(", "LIN_GELU_FN(").replace("LIN(", lin + "(")


_ENGINE_PREFIX = '''
def LIN_GELU_FN(x: Tensor, packed: Tensor, absmax: Tensor, bias: Tensor, table2: Tensor) -> Tensor:
    return torch.ops.diffuser_b200.nf4_lin_act(x, packed, absmax, bias, 1)
'''


def stack_unit() -> torch.jit.CompilationUnit:
    """The block stack compiled with the engine's operators (``.stack``,
    ``.block``, ``.attention``, ``.feed_forward``)."""
    register_ops()
    return torch.jit.CompilationUnit(stack_source("torch.ops.diffuser_b200.nf4_lin", _ENGINE_PREFIX))


def pack_block(attns: dict, ffs: dict, tables: dict) -> list:
    """One block's 114 slots: attns[name] = dict of ATTN_SLOTS tensors for
    each of ATTN_BASES, ffs[name] = (proj_packed, proj_absmax, proj_bias,
    net2_packed, net2_absmax, net2_bias), tables[name] = the modulation tables
    of TABLE_SLOTS."""
    slots = [None] * SLOTS_PER_BLOCK
    for name, base in ATTN_BASES.items():
        for i, key in enumerate(ATTN_SLOTS):
            slots[base + i] = attns[name][key]
    for name, base in FF_BASES.items():
        for i, t in enumerate(ffs[name]):
            slots[base + i] = t
    for name, i in TABLE_SLOTS.items():
        slots[i] = tables[name]
    missing = [i for i, t in enumerate(slots) if t is None]
    if missing:
        raise ValueError(f"block slots left empty: {missing}")
    return slots
