"""ctypes binding of the C ABI in ``include/dq_linear.h``.

The shared library must have been built (``diffuser_b200.build.build()``);
there is no fallback: loading fails loudly when it is missing.
"""
from __future__ import annotations

import ctypes
import os

from .build import LIB_PATH

_c_i64 = ctypes.c_int64
_c_p = ctypes.c_void_p
_c_sz = ctypes.c_size_t

# name -> (restype, argtypes); every symbol the header declares.
SIGNATURES = {
    "dq_version": (ctypes.c_char_p, []),
    "dq_abi_version": (ctypes.c_int, []),
    "dq_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "dq_quantize_nf4": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_p, _c_p, _c_p]),
    "dq_quantize_fp8": (ctypes.c_int, [_c_p, ctypes.c_int, _c_i64, _c_p, _c_p, _c_p]),
    "dq_dequant_nf4": (ctypes.c_int, [_c_p, _c_p, _c_i64, _c_p, _c_p]),
    "dq_dequant_fp8": (ctypes.c_int, [_c_p, ctypes.c_float, _c_i64, _c_p, _c_p]),
    "dq_workspace_size": (_c_sz, [_c_i64, _c_i64, _c_i64, ctypes.c_int]),
    "dq_linear_nf4": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_i64, _c_p,
                                     _c_p, _c_sz, _c_p]),
    "dq_linear_fp8": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_p, ctypes.c_float, _c_p, _c_i64,
                                     _c_p, _c_p, _c_sz, _c_p]),
    "dq_linear_nf4_noalloc": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_i64,
                                             _c_p, _c_p]),
    "dq_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), _c_p]),
    "dq_set_tile_override": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    "dq_set_pair_mode": (ctypes.c_int, [ctypes.c_int]),
    "dq_tp_buffer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "dq_tp_buffer_free": (ctypes.c_int, [ctypes.c_void_p]),
    "dq_ipc_handle": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "dq_ipc_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "dq_ipc_close": (ctypes.c_int, [ctypes.c_void_p]),
    "dq_tp_linear_nf4": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, _c_i64, ctypes.c_int, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                        ctypes.c_void_p, ctypes.c_uint, ctypes.c_void_p]),
    "dq_tp_linear_fp8": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p, ctypes.c_float,
                                        ctypes.c_void_p, _c_i64, ctypes.c_int, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                        ctypes.c_void_p, ctypes.c_uint, ctypes.c_void_p]),
    "dq_tp_linear_nf4_ws": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p, _c_i64, ctypes.c_int, ctypes.c_int,
                                           ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                           ctypes.c_void_p, ctypes.c_uint, ctypes.c_void_p, _c_sz,
                                           ctypes.c_void_p]),
    "dq_tp_linear_fp8_ws": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p, ctypes.c_float,
                                           ctypes.c_void_p, _c_i64, ctypes.c_int, ctypes.c_int,
                                           ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                           ctypes.c_void_p, ctypes.c_uint, ctypes.c_void_p, _c_sz,
                                           ctypes.c_void_p]),
    "dq_tp_linear_nf4_mc_ws": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_void_p, _c_i64, ctypes.c_int,
                                              ctypes.c_int, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p,
                                              ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_uint,
                                              ctypes.c_void_p, _c_sz, ctypes.c_void_p]),
    "dq_tp_linear_fp8_mc_ws": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p,
                                              ctypes.c_float, ctypes.c_void_p, _c_i64, ctypes.c_int,
                                              ctypes.c_int, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p,
                                              ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_uint,
                                              ctypes.c_void_p, _c_sz, ctypes.c_void_p]),
    "dq_qk_norm_rope": (ctypes.c_int, [ctypes.c_void_p, _c_i64, ctypes.c_void_p, _c_i64, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]),
    "dq_qkv_norm_rope": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                        ctypes.POINTER(_c_i64), ctypes.POINTER(ctypes.c_void_p),
                                        ctypes.POINTER(_c_i64), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                        ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_int),
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float,
                                        ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]),
    "dq_heads_to_tokens": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_void_p]),
    "dq_linear_nf4_ld": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, _c_i64, ctypes.c_int, ctypes.c_void_p, _c_i64,
                                        ctypes.c_void_p, _c_sz, ctypes.c_void_p]),
    "dq_linear_fp8_ld": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p, ctypes.c_float,
                                        ctypes.c_void_p, _c_i64, ctypes.c_int, ctypes.c_void_p, _c_i64,
                                        ctypes.c_void_p, _c_sz, ctypes.c_void_p]),
    "dq_heads_to_tokens_ld": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, ctypes.c_int, ctypes.c_void_p, _c_i64,
                                             ctypes.c_void_p, _c_i64, ctypes.c_void_p]),
    "dq_adaln_modulate": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_void_p, ctypes.c_void_p, _c_i64, ctypes.c_float,
                                         ctypes.c_void_p, _c_i64, ctypes.c_void_p]),
    "dq_gated_residual": (ctypes.c_int, [ctypes.c_void_p, _c_i64, ctypes.c_void_p, _c_i64, ctypes.c_void_p,
                                         _c_i64, _c_i64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, _c_i64,
                                         ctypes.c_void_p]),
    "dq_linear_nf4_ex": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, _c_i64, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_void_p, _c_sz, ctypes.c_void_p]),
    "dq_linear_fp8_ex": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p, ctypes.c_float,
                                        ctypes.c_void_p, _c_i64, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_void_p, _c_sz, ctypes.c_void_p]),
    "dq_linear_nf4_scaled": (ctypes.c_int, [ctypes.c_void_p, _c_i64, _c_i64, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, _c_i64,
                                            ctypes.c_int, ctypes.c_void_p, _c_i64, ctypes.c_void_p,
                                            _c_sz, ctypes.c_void_p]),
    "dq_dequant_nf4_scaled": (ctypes.c_int, [_c_p, _c_p, ctypes.c_int, _c_i64, _c_p, _c_p]),
    "dq_plan_info": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, ctypes.c_int] + [ctypes.POINTER(ctypes.c_int)] * 4),
}

DQ_OK = 0
DQ_ERR_TIMEOUT = 5
DQ_ERR_SCRATCH_LIMIT = 9
DQ_NOALLOC_SCRATCH_BYTES = 8 << 20
DQ_IPC_HANDLE_BYTES = 64
DQ_ACT_NONE, DQ_ACT_GELU_TANH, DQ_ACT_SWIGLU, DQ_ACT_GEGLU_TANH = 0, 1, 2, 3
DQ_FMT_NF4, DQ_FMT_FP8 = 0, 1
DQ_DTYPE_F32, DQ_DTYPE_BF16 = 0, 1

_LIB = None


class DqError(RuntimeError):
    """A non-zero dq_status returned by the engine."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed: status {status} ({status_string(status)})")


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"engine library {LIB_PATH} is missing: build it with "
                "`python -m diffuser_b200.build` (no CPU fallback exists)")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = h
    return _LIB


def status_string(status: int) -> str:
    return lib().dq_status_string(int(status)).decode()


def check(fn: str, status: int) -> None:
    if status != DQ_OK:
        raise DqError(fn, status)


def version() -> str:
    return lib().dq_version().decode()
