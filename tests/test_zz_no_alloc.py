"""dq_linear_nf4_noalloc: the NF4 linear for callers that cannot allocate device
memory (an embedder whose memory belongs to another allocator and who has no
workspace to lend, or code that must not allocate while it runs).  Its split-K
scratch is an 8 MiB array built into the library.

The test drives it through the C ABI (ctypes) and checks two consecutive calls
against the workspace-taking dq_linear_nf4, within the linear tolerance used
by the other parity tests.  This file sorts last so that a run stopping at the
first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from diffuser_b200 import _lib, ops
from oracle import numpy_ref as R
from tests.gpu_util import seeded_bf16, seeded_f32, to_bits

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _weights(n, k, seed):
    w = seeded_f32((n, k), seed, 0.02)
    p, a = R.nf4_quantize(w.numpy())
    return torch.from_numpy(p).cuda(), torch.from_numpy(a).cuda()


def _noalloc(x, packed, absmax, bias, n):
    m, k = x.shape
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    rc = _lib.lib().dq_linear_nf4_noalloc(
        _p(x), m, k, _p(packed), _p(absmax), _p(bias), n, _p(y),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, y


@pytest.mark.parametrize("m,n,k,splits", [(64, 1024, 4096, 4), (16, 3072, 3072, 0),
                                          (5, 200, 1088, 3), (300, 640, 512, 0)])
def test_noalloc_matches_workspace_entry_point_twice(m, n, k, splits):
    packed, absmax = _weights(n, k, 7 + n)
    bias = seeded_bf16((n,), 11, 0.5).cuda()
    ops.set_tile_override(0, splits)
    try:
        for call, seed in enumerate((100 + m, 200 + m)):  # two calls in a row, new inputs
            x = seeded_bf16((m, k), seed).cuda()
            ref = ops.nf4_linear(x, packed, absmax, n, bias)
            rc, y = _noalloc(x, packed, absmax, bias, n)
            torch.cuda.synchronize()
            assert rc == 0, _lib.status_string(rc)
            err = R.rel_err(to_bits(y), to_bits(ref))
            assert err <= TOL, (call, err)
    finally:
        ops.set_tile_override(0, 0)
    assert ops.device_error() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    # 64 x 8192 outputs split 16 ways need 32 MiB of partial sums > 8 MiB
    n, k, m = 8192, 4096, 64
    packed, absmax = _weights(n, k, 3)
    x = seeded_bf16((m, k), 5).cuda()
    ops.set_tile_override(0, 16)
    try:
        rc, _ = _noalloc(x, packed, absmax, None, n)
    finally:
        ops.set_tile_override(0, 0)
    assert rc == _lib.DQ_ERR_SCRATCH_LIMIT
    assert "scratch" in _lib.status_string(rc)
