"""CPU tests of the C-ABI library: it builds for sm_100a, loads without a GPU,
exports every symbol the header declares, and rejects bad arguments on the
host before touching a device."""
import ctypes
import os
import re

import pytest

from diffuser_b200 import _lib
from diffuser_b200 import build as B

INCLUDE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
HEADER = os.path.join(INCLUDE, "dq_linear.h")


def _header_functions():
    names = set()
    for h in sorted(os.listdir(INCLUDE)):
        if h.endswith(".h"):
            src = re.sub(r"/\*.*?\*/", "", open(os.path.join(INCLUDE, h)).read(), flags=re.S)
            names.update(re.findall(r"\b(dq_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    B.build()
    return _lib.lib()


def test_header_declares_expected_entry_points():
    names = _header_functions()
    for must in ("dq_linear_nf4", "dq_linear_fp8", "dq_dequant_nf4", "dq_dequant_fp8",
                 "dq_quantize_nf4", "dq_quantize_fp8", "dq_workspace_size", "dq_version"):
        assert must in names


def test_library_exports_every_header_symbol(lib):
    for name in _header_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"binding missing for {name}"


def test_version_and_status_strings(lib):
    assert "sm_100a" in _lib.version()
    assert lib.dq_abi_version() == 2
    assert _lib.status_string(0) == "ok"
    assert "shape" in _lib.status_string(1)


def test_shape_errors_rejected_on_host(lib):
    p = ctypes.c_void_p(16)
    # K not a multiple of 64
    assert lib.dq_linear_nf4(p, 4, 100, p, p, None, 8, p, None, 0, None) == 1
    assert lib.dq_linear_fp8(p, 4, 100, p, ctypes.c_float(1.0), None, 8, p, None, 0, None) == 1
    # non-positive N / K
    assert lib.dq_linear_nf4(p, 4, 64, p, p, None, 0, p, None, 0, None) == 1
    assert lib.dq_linear_nf4(p, 4, -64, p, p, None, 8, p, None, 0, None) == 1
    # lengths not a multiple of 64
    assert lib.dq_dequant_nf4(p, p, 100, p, None) == 1
    assert lib.dq_quantize_nf4(p, 0, 100, p, p, None) == 1


def test_null_and_alignment_errors_rejected_on_host(lib):
    p = ctypes.c_void_p(4096)
    odd = ctypes.c_void_p(4096 + 8)
    assert lib.dq_linear_nf4(None, 4, 64, p, p, None, 8, p, None, 0, None) == 7
    assert lib.dq_linear_nf4(p, 4, 64, p, None, None, 8, p, None, 0, None) == 7
    assert lib.dq_linear_nf4(odd, 4, 64, p, p, None, 8, p, None, 0, None) == 2
    assert lib.dq_linear_fp8(p, 4, 64, odd, ctypes.c_float(1.0), None, 8, p, None, 0, None) == 2
    assert lib.dq_dequant_nf4(odd, p, 64, p, None) == 2
    assert lib.dq_quantize_nf4(p, 5, 64, p, p, None) == 7
    assert lib.dq_set_tile_override(48, 0) == 7
    assert lib.dq_set_tile_override(0, 0) == 0


def test_empty_batch_is_a_noop(lib):
    p = ctypes.c_void_p(4096)
    assert lib.dq_linear_nf4(p, 0, 64, p, p, None, 8, p, None, 0, None) == 0
    assert lib.dq_dequant_nf4(p, p, 0, p, None) == 0


def test_product_path_refuses_cpu_tensors():
    import torch
    from diffuser_b200 import ops
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.nf4_linear(torch.zeros(2, 64, dtype=torch.bfloat16),
                       torch.zeros(64 * 8 // 2, dtype=torch.uint8), torch.ones(8), 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.ltx23_nf4_quantize(torch.zeros(64))


def test_plan_info_rejects_bad_arguments_on_host(lib):
    v = [ctypes.c_int(0) for _ in range(4)]
    refs = [ctypes.byref(x) for x in v]
    assert lib.dq_plan_info(4, 8, 100, 0, *refs) == 1      # NF4 needs K % 64 == 0
    assert lib.dq_plan_info(0, 8, 64, 0, *refs) == 1       # empty batch has no plan
    assert lib.dq_plan_info(4, 8, 64, 5, *refs) == 1       # unknown format
    assert lib.dq_plan_info(4, 8, 64, 0, None, *refs[1:]) == 7


def test_strided_and_glue_entry_points_reject_bad_arguments_on_host(lib):
    # validation happens before any CUDA call, so no GPU is needed to see it
    p = ctypes.c_void_p(0x1000)
    # y row stride below N
    assert lib.dq_linear_nf4_ld(p, 4, 64, p, p, None, 64, 0, p, 32, None, 0, None) == 1
    assert lib.dq_linear_fp8_ld(p, 4, 64, p, ctypes.c_float(1.0), None, 64, 0, p, 63, None, 0,
                                None) == 1
    # heads_to_tokens: output rows narrower than H * D
    assert lib.dq_heads_to_tokens_ld(p, 1, 2, 0, 4, 64, None, 128, p, 100, None) == 1
    # AdaLN modulation: D % 4, D above 8192, T not a multiple of S, NULL scale
    assert lib.dq_adaln_modulate(p, 6, 4, 2, 6, p, p, 6, ctypes.c_float(1e-6), p, 6, None) == 1
    assert lib.dq_adaln_modulate(p, 8196, 4, 2, 8196, p, p, 8196, ctypes.c_float(1e-6), p, 8196,
                                 None) == 1
    assert lib.dq_adaln_modulate(p, 8, 5, 2, 8, p, p, 8, ctypes.c_float(1e-6), p, 8, None) == 1
    assert lib.dq_adaln_modulate(p, 8, 4, 2, 8, None, p, 8, ctypes.c_float(1e-6), p, 8, None) == 7
    # q/k/v glue: no parts, a part with a row stride below H * D, rope without a table
    P3 = ctypes.c_void_p * 3
    L3 = ctypes.c_int64 * 3
    I3 = ctypes.c_int * 3
    ptrs, nul = P3(p, p, p), P3(None, None, None)
    assert lib.dq_qkv_norm_rope(0, ptrs, L3(384, 384, 384), None, None, 1, 4, 0, 3, 128, nul, nul,
                                I3(0, 0, 0), None, None, ctypes.c_float(1e-6), ptrs, None) == 7
    assert lib.dq_qkv_norm_rope(3, ptrs, L3(384, 100, 384), None, None, 1, 4, 0, 3, 128, nul, nul,
                                I3(0, 0, 0), None, None, ctypes.c_float(1e-6), ptrs, None) == 1
    assert lib.dq_qkv_norm_rope(3, ptrs, L3(384, 384, 384), None, None, 1, 4, 0, 3, 128, nul, nul,
                                I3(1, 0, 0), None, None, ctypes.c_float(1e-6), ptrs, None) == 7
    # gated residual: row stride below D, misaligned rows
    assert lib.dq_gated_residual(p, 4, p, 8, p, 8, 4, 2, 8, p, 8, None) == 1
    assert lib.dq_gated_residual(ctypes.c_void_p(0x1002), 8, p, 8, p, 8, 4, 2, 8, p, 8, None) == 2


def test_linear_out_argument_is_validated_on_host():
    # out= must be a bf16 CUDA view with unit feature stride and evenly spaced
    # rows; the checks run before any launch
    import torch
    from diffuser_b200 import ops
    with pytest.raises(TypeError):
        ops._out_rows(torch.empty(4, 8, dtype=torch.float32), 4, 8)
    if torch.cuda.is_available():
        return
    # on a host without CUDA the device check is the first to refuse
    with pytest.raises(TypeError):
        ops._out_rows(torch.empty(4, 8, dtype=torch.bfloat16), 4, 8)
