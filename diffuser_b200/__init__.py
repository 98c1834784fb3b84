"""diffuser_b200 -- a B200-native (sm_100a) quantized weight-only linear engine
for diffuseR's NF4 and fp8-e4m3 DiT linears.

Public surface (mirrors the reference's R API names):
  ops.ltx23_nf4_quantize / ops.ltx23_nf4_dequantize / ops.fp8_quantize /
  ops.fp8_dequantize / ops.nf4_linear / ops.fp8_linear
  modules.ltx23_nf4_linear / modules.ltx23_fp8_linear / modules.swap_quant_linears
  tp.ColumnParallelQuantLinear (column-parallel over NCCL)
The compute path is the C-ABI library built from ``csrc/`` (see build.py);
there is no CPU fallback.
"""
from . import build  # noqa: F401

__all__ = ["build", "ops", "modules"]


def __getattr__(name):
    if name in ("ops", "modules", "tp"):
        import importlib
        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)
