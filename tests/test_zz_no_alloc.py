"""dq_linear_nf4_noalloc: the NF4 linear for callers that cannot allocate device
memory (an embedder whose memory belongs to another allocator and who has no
workspace to lend, or code that must not allocate while it runs).  Its split-K
scratch is an 8 MiB array built into the library.

The test drives it through the C ABI (ctypes) and checks two consecutive calls
against the oracle (within the linear tolerance used by the other parity
tests) and against the workspace-taking dq_linear_nf4: bit for bit where both
run the same plan, within the tolerance where the built-in array's size makes
the allocation-free call split less.  This file sorts last so that a run stopping at the
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


def _same_plan_as_workspace_entry_point(m, n, k, splits):
    """True when dq_linear_nf4 picks the plan the allocation-free entry point
    picks: no two-phase plan (M < 1024) and split-K partial sums that fit the
    built-in array (a forced split count always gives both the same plan)."""
    if m >= 1024:
        return False
    return splits > 0 or ops.workspace_size(m, n, k, 0) <= _lib.DQ_NOALLOC_SCRATCH_BYTES


@pytest.mark.parametrize("m,n,k,splits", [
    (64, 1024, 4096, 4), (16, 3072, 3072, 0), (5, 200, 1088, 3), (300, 640, 512, 0),
    (96, 3072, 3072, 0),     # automatic split (6 ways, 7.1 MiB) just under the array's size
    (128, 3072, 3072, 0),    # automatic split would need 9.4 MiB: capped at 5 ways (7.9 MiB)
    (512, 3072, 12288, 0),   # long-K split would need 12.6 MiB: runs unsplit
])
def test_noalloc_matches_workspace_entry_point_twice(m, n, k, splits):
    w = seeded_f32((n, k), 7 + n, 0.02)
    pn, an = R.nf4_quantize(w.numpy())
    packed, absmax = torch.from_numpy(pn).cuda(), torch.from_numpy(an).cuda()
    bias = seeded_bf16((n,), 11, 0.5)
    bias_d = bias.cuda()
    same_plan = _same_plan_as_workspace_entry_point(m, n, k, splits)
    ops.set_tile_override(0, splits)
    try:
        for call, seed in enumerate((100 + m, 200 + m)):  # two calls in a row, new inputs
            x = seeded_bf16((m, k), seed)
            xd = x.cuda()
            ref = ops.nf4_linear(xd, packed, absmax, n, bias_d)
            rc, y = _noalloc(xd, packed, absmax, bias_d, n)
            torch.cuda.synchronize()
            assert rc == 0, _lib.status_string(rc)
            # against the oracle (the reference's dequantize-then-linear, float64)
            oracle = R.nf4_linear_bf16(to_bits(x), pn, an, n, k, to_bits(bias))
            err = R.rel_err(to_bits(y), oracle)
            assert err <= TOL, (call, "oracle", err)
            # against the workspace-taking entry point: the same bits when both
            # run the same plan (a mix-up in the scratch would show here), else
            # within the linear tolerance
            if same_plan:
                assert np.array_equal(to_bits(y), to_bits(ref)), (call, "bits differ")
            else:
                err = R.rel_err(to_bits(y), to_bits(ref))
                assert err <= TOL, (call, "dq_linear_nf4", err)
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
    # sizes are validated before the scratch: an oversized M is a shape error
    rc = _lib.lib().dq_linear_nf4_noalloc(_p(x), 1 << 31, k, _p(packed), _p(absmax), None, n,
                                          _p(x), None)
    assert rc == 1, _lib.status_string(rc)  # DQ_ERR_SHAPE
