"""GPU parity of the fused NF4 / fp8 linear against the oracle.

Tolerance (the contract stated for the GEMM): max|y - y_ref| / max|y_ref| <= 1e-2,
where y_ref is the oracle's dequantize-then-matmul in float64 on the
bit-identical bf16 weights, rounded once to bf16.
"""
import numpy as np
import pytest
import torch

from oracle import numpy_ref as R
from tests.gpu_util import from_bits, seeded_bf16, seeded_f32, to_bits

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.fixture(scope="module")
def ops():
    from diffuser_b200 import ops as _ops
    yield _ops
    _ops.set_tile_override(0, 0)
    _ops.set_pair_mode(0)


def _case(m, n, k, seed, fmt, with_bias):
    x = seeded_bf16((m, k), seed)
    w = seeded_f32((n, k), seed + 1000, 0.02)
    bias = seeded_bf16((n,), seed + 2000, 0.5) if with_bias else None
    xb = to_bits(x)
    bb = to_bits(bias) if with_bias else None
    if fmt == "nf4":
        p, a = R.nf4_quantize(w.numpy())
        ref = R.nf4_linear_bf16(xb, p, a, n, k, bb)
        return x, (torch.from_numpy(p).cuda(), torch.from_numpy(a).cuda()), bias, ref
    w8, s = R.fp8_quantize(w.numpy())
    ref = R.fp8_linear_bf16(xb, w8, s, n, k, bb)
    return x, (torch.from_numpy(w8).cuda().view(torch.float8_e4m3fn), float(s)), bias, ref


def _run(ops, fmt, x, w, bias, n):
    xc = x.cuda()
    bc = bias.cuda() if bias is not None else None
    if fmt == "nf4":
        return ops.nf4_linear(xc, w[0], w[1], n, bc)
    return ops.fp8_linear(xc, w[0], w[1], bc)


SHAPES = [(1, 64, 64), (5, 64, 128), (7, 200, 192), (16, 128, 256), (65, 130, 256),
          (128, 128, 128), (200, 384, 640), (257, 1000, 1024), (600, 512, 3072)]


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_linear_matches_oracle(ops, fmt, m, n, k):
    x, w, bias, ref = _case(m, n, k, m * 7 + n, fmt, with_bias=(m % 2 == 1))
    y = _run(ops, fmt, x, w, bias, n)
    torch.cuda.synchronize()
    assert y.shape == (m, n) and y.dtype == torch.bfloat16
    err = R.rel_err(to_bits(y), ref)
    assert err <= TOL, err


@pytest.mark.parametrize("m,n,k", [(3, 48, 96), (70, 200, 80), (130, 136, 1040)])
def test_fp8_ragged_k(ops, m, n, k):
    # fp8 has no block structure: K need only keep 16-byte row strides
    x, w, bias, ref = _case(m, n, k, 31 + k, "fp8", with_bias=True)
    y = _run(ops, "fp8", x, w, bias, n)
    assert R.rel_err(to_bits(y), ref) <= TOL


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("bm", [16, 32, 64, 128, 192, 256])
def test_every_tile_height(ops, fmt, bm):
    m, n, k = 300, 640, 512
    x, w, bias, ref = _case(m, n, k, bm, fmt, with_bias=True)
    ops.set_tile_override(bm, 0)
    try:
        y = _run(ops, fmt, x, w, bias, n)
        torch.cuda.synchronize()
    finally:
        ops.set_tile_override(0, 0)
    assert R.rel_err(to_bits(y), ref) <= TOL


@pytest.mark.parametrize("mode", [3, 4])
@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("bm", [64, 128, 192, 256])
@pytest.mark.parametrize("m,n,k", [(300, 640, 512), (1000, 136, 1088), (70, 264, 3072)])
def test_two_phase(ops, mode, fmt, bm, m, n, k):
    # dequantize once into bf16 scratch, then the bf16 CTA-pair GEMM: inside
    # the GEMM launch (mode 3) or as a launch of its own (mode 4)
    x, w, bias, ref = _case(m, n, k, 3 * bm + n, fmt, with_bias=True)
    ops.set_pair_mode(mode)
    ops.set_tile_override(bm, 0)
    try:
        assert ops.plan_info(m, n, k, 0 if fmt == "nf4" else 1)["twophase"]
        y = _run(ops, fmt, x, w, bias, n)
        torch.cuda.synchronize()
    finally:
        ops.set_tile_override(0, 0)
        ops.set_pair_mode(0)
    assert R.rel_err(to_bits(y), ref) <= TOL


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("m,n,k", [(4608, 6000, 128), (2048, 12800, 64), (1100, 300, 4096)])
def test_two_phase_weight_groups(ops, fmt, m, n, k):
    # the in-launch decode walks the weight in groups of the tile order (a
    # narrow first group, then 16 weight tiles): several groups, a ragged
    # last weight tile, and a single group
    x, w, bias, ref = _case(m, n, k, 11 + n, fmt, with_bias=True)
    y = _run(ops, fmt, x, w, bias, n)
    torch.cuda.synchronize()
    assert ops.plan_info(m, n, k, 0 if fmt == "nf4" else 1)["twophase"]
    assert R.rel_err(to_bits(y), ref) <= TOL
    y2 = _run(ops, fmt, x, w, bias, n)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("bm", [64, 128, 192, 256])
@pytest.mark.parametrize("m,n,k", [(300, 640, 512), (1000, 136, 1088)])
def test_cta_pair_tiles(ops, fmt, bm, m, n, k):
    # two-SM kernel: 256 weight rows per CTA pair, bm tokens split across the pair
    x, w, bias, ref = _case(m, n, k, bm + n, fmt, with_bias=True)
    ops.set_pair_mode(2)
    ops.set_tile_override(bm, 0)
    try:
        y = _run(ops, fmt, x, w, bias, n)
        torch.cuda.synchronize()
    finally:
        ops.set_tile_override(0, 0)
        ops.set_pair_mode(0)
    assert R.rel_err(to_bits(y), ref) <= TOL


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("m,n,k,splits", [(1, 1024, 4096, 0), (16, 3072, 3072, 0),
                                          (64, 2304, 3072, 5), (3, 200, 1088, 3)])
def test_split_k(ops, fmt, m, n, k, splits):
    # the fused one-CTA kernel with K split across CTAs (automatic count when
    # splits == 0) and the f32 reduce kernel
    x, w, bias, ref = _case(m, n, k, 17 + m, fmt, with_bias=True)
    ops.set_pair_mode(1)
    ops.set_tile_override(0, splits)
    try:
        assert ops.plan_info(m, n, k, 0 if fmt == "nf4" else 1)["splits"] > 1
        y = _run(ops, fmt, x, w, bias, n)
        torch.cuda.synchronize()
    finally:
        ops.set_tile_override(0, 0)
        ops.set_pair_mode(0)
    assert R.rel_err(to_bits(y), ref) <= TOL


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("m,n,k,with_bias", [(1, 64, 128, True), (3, 200, 384, False),
                                             (8, 3072, 3072, True), (9, 136, 1024, True),
                                             (16, 1000, 1152, False), (16, 18432, 3072, True),
                                             (2, 3072, 15360, True), (5, 9000, 256, True),
                                             (1, 18432, 512, False)])
@pytest.mark.parametrize("mode", [5, 6])
def test_small_m_kernel(ops, fmt, m, n, k, with_bias, mode):
    # decode-sized token counts: weights decoded straight into warp-MMA
    # registers (one and two 8-token tiles; one, two and four 16-row groups
    # per CTA; ragged N; long K), the weight streamed through the TMA ring
    # (mode 5, where K allows) or loaded into registers (mode 6)
    x, w, bias, ref = _case(m, n, k, 23 + m + n, fmt, with_bias=with_bias)
    ops.set_pair_mode(mode)
    try:
        plan = ops.plan_info(m, n, k, 0 if fmt == "nf4" else 1)
        assert plan["smallm"] and plan["splits"] == 1
        assert plan["ring"] == (mode == 5 and m <= 16 and k % (256 if fmt == "nf4" else 128) == 0)
        y = _run(ops, fmt, x, w, bias, n)
        y2 = _run(ops, fmt, x, w, bias, n)
        torch.cuda.synchronize()
    finally:
        ops.set_pair_mode(0)
    assert R.rel_err(to_bits(y), ref) <= TOL
    assert torch.equal(y, y2)
    assert ops.device_error() == 0


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("m,n,k", [(1, 18432, 3072), (8, 3072, 3072), (4, 9216, 3072),
                                   (1, 12288, 4096), (3, 1000, 15360), (2, 200, 256),
                                   (16, 18432, 3072), (12, 3072, 4096), (9, 1000, 15360)])
def test_small_m_ring_and_register_kernels_agree(ops, fmt, m, n, k):
    # the two small-M kernels decode the same weights into the same MMA
    # fragments in the same k order; the ring kernel alternates two
    # accumulators, so the sums differ only by f32 rounding
    x, w, bias, ref = _case(m, n, k, 5 + m + n, fmt, with_bias=True)
    outs = {}
    for mode in (5, 6):
        ops.set_pair_mode(mode)
        try:
            outs[mode] = _run(ops, fmt, x, w, bias, n)
            torch.cuda.synchronize()
        finally:
            ops.set_pair_mode(0)
        assert R.rel_err(to_bits(outs[mode]), ref) <= TOL, mode
    assert R.rel_err(to_bits(outs[5]), to_bits(outs[6])) <= TOL


def test_small_m_ring_falls_back_on_unaligned_scales(ops):
    # the ring kernel copies NF4 block scales by TMA (16-byte aligned rows);
    # a 4-byte aligned absmax view takes the register-stream kernel instead
    m, n, k = 4, 4096, 3072
    x, (p, a), bias, ref = _case(m, n, k, 77, "nf4", with_bias=True)
    buf = torch.empty(a.numel() + 1, dtype=torch.float32, device="cuda")
    buf[1:].copy_(a)
    shifted = buf[1:]
    assert shifted.data_ptr() % 16 != 0
    ops.set_pair_mode(5)
    try:
        assert ops.plan_info(m, n, k, 0)["ring"]
        y = ops.nf4_linear(x.cuda(), p, shifted, n, bias.cuda())
        torch.cuda.synchronize()
    finally:
        ops.set_pair_mode(0)
    assert R.rel_err(to_bits(y), ref) <= TOL
    assert ops.device_error() == 0


def test_leading_dims_and_noncontiguous_input(ops):
    m, n, k = 24, 192, 256
    x, w, bias, ref = _case(m, n, k, 5, "nf4", with_bias=True)
    x3 = x.reshape(2, 12, k).cuda()
    y = ops.nf4_linear(x3, w[0], w[1], n, bias.cuda())
    assert y.shape == (2, 12, n)
    assert R.rel_err(to_bits(y.reshape(m, n)), ref) <= TOL
    xt = x.cuda().t().contiguous().t()  # same values, column-major storage
    y2 = ops.nf4_linear(xt, w[0], w[1], n, bias.cuda())
    assert torch.equal(y2, y.reshape(m, n))


def test_deterministic_repeat(ops):
    m, n, k = 333, 1280, 1024
    x, w, bias, _ = _case(m, n, k, 9, "nf4", with_bias=True)
    a = _run(ops, "nf4", x, w, bias, n)
    b = _run(ops, "nf4", x, w, bias, n)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def _full_size_check(ops, fmt):
    # The NF4 / fp8 linear at the benchmarked shape: x [4608, 3072], W [12288, 3072].
    m, n, k = 4608, 12288, 3072
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    g0 = torch.Generator(device="cuda").manual_seed(0)
    w = torch.randn(n, k, generator=g0, device="cuda") * 0.02
    if fmt == "nf4":
        p, a = ops.ltx23_nf4_quantize(w)
        y = ops.nf4_linear(x, p, a, n)
        wd = ops.ltx23_nf4_dequantize(p, a, (n, k))
    else:
        w8, s = ops.fp8_quantize(w)
        y = ops.fp8_linear(x, w8, s.item())
        wd = ops.fp8_dequantize(w8, s.item())
    # cuBLAS on the bit-exact dequantized weight = the reference's GPU algorithm
    ref = (x.float() @ wd.float().t()).to(torch.bfloat16)
    err = ((y.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
    assert err <= TOL, err
    # exact oracle on a sample of rows
    rows = torch.arange(0, m, 97, device="cuda")
    yb = to_bits(y[rows])
    ref_rows = R.linear_bf16(to_bits(x[rows]), to_bits(wd), None)
    assert R.rel_err(yb, ref_rows) <= TOL
    return y


def test_full_size_nf4(ops):
    _full_size_check(ops, "nf4")


def test_full_size_fp8(ops):
    _full_size_check(ops, "fp8")


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("mode,bm", [(1, 128), (1, 192), (1, 256), (2, 192), (2, 256),
                                     (3, 128), (3, 256), (4, 256)])
def test_full_size_every_plan(ops, fmt, mode, bm):
    # every tile plan at the benchmarked shape, twice: a pipeline race shows
    # up as a large or run-to-run varying error here
    ops.set_pair_mode(mode)
    ops.set_tile_override(bm, 0)
    try:
        y1 = _full_size_check(ops, fmt)
        y2 = _full_size_check(ops, fmt)
    finally:
        ops.set_tile_override(0, 0)
        ops.set_pair_mode(0)
    assert torch.equal(y1, y2)


def test_golden_linear(ops):
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_linear_golden.npz"))
    y = ops.nf4_linear(from_bits(g["nf4_x"]), torch.from_numpy(g["nf4_packed"]).cuda(),
                       torch.from_numpy(g["nf4_absmax"]).cuda(), 64, from_bits(g["nf4_bias"]))
    assert R.rel_err(to_bits(y), g["nf4_y"]) <= TOL
    y2 = ops.fp8_linear(from_bits(g["fp8_x"]),
                        torch.from_numpy(g["fp8_w8"]).cuda().view(torch.float8_e4m3fn),
                        float(g["fp8_scale"]), from_bits(g["fp8_bias"]))
    assert R.rel_err(to_bits(y2), g["fp8_y"]) <= TOL


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("mode,bm,splits,m,n,k", [(1, 128, 0, 300, 640, 512),   # fused one-CTA
                                                  (2, 192, 0, 300, 640, 512),   # fused pair
                                                  (3, 256, 0, 300, 640, 512),   # two-phase
                                                  (4, 256, 0, 300, 640, 512),   # two launches
                                                  (1, 0, 3, 16, 640, 1088),     # split-K reduce
                                                  (5, 0, 0, 12, 640, 1024),     # small-M, TMA ring
                                                  (6, 0, 0, 12, 640, 1024)])    # small-M, registers
def test_gelu_tanh_epilogue(ops, fmt, mode, bm, splits, m, n, k):
    # y = bf16(gelu_tanh(bf16(x W^T + b))) in the epilogue equals the linear
    # followed by torch's GELU-tanh on its bf16 output (the reference's
    # gelu_proj), up to the last bit of the activation arithmetic
    x, w, bias, ref = _case(m, n, k, 97 + m, fmt, with_bias=True)
    ops.set_pair_mode(mode)
    ops.set_tile_override(bm, splits)
    try:
        y_plain = _run(ops, fmt, x, w, bias, n)
        xc, bc = x.cuda(), bias.cuda()
        if fmt == "nf4":
            y_act = ops.nf4_linear(xc, w[0], w[1], n, bc, act="gelu_tanh")
        else:
            y_act = ops.fp8_linear(xc, w[0], w[1], bc, act="gelu_tanh")
        torch.cuda.synchronize()
    finally:
        ops.set_tile_override(0, 0)
        ops.set_pair_mode(0)
    ref_act = torch.nn.functional.gelu(y_plain, approximate="tanh")
    step = ref_act.float().abs() * 2.0 ** -7 + 1e-6
    assert ((y_act.float() - ref_act.float()).abs() <= step).all()
    assert (y_act != ref_act).float().mean().item() < 0.01
    # and against the oracle's linear through the same activation
    gelu_oracle = torch.nn.functional.gelu(
        torch.from_numpy(ref.view(np.int16)).view(torch.bfloat16).float(), approximate="tanh")
    err = (y_act.float().cpu() - gelu_oracle).abs().max() / gelu_oracle.abs().max()
    assert err.item() <= TOL


def test_plan_choice(ops):
    # large token batches dequantize once and run the bf16 pair GEMM,
    # mid-sized ones the fused kernels, decode-sized ones one-CTA tiles
    big = ops.plan_info(4608, 12288, 3072)
    assert big["twophase"] and big["bm"] == 256 and big["splits"] == 1
    # the bf16 weight, then 256 bytes of weight-group counters
    assert ops.workspace_size(4608, 12288, 3072) == 12288 * 3072 * 2 + 256
    mid = ops.plan_info(512, 12288, 3072)
    assert not mid["twophase"]
    # decode-sized batches: the small-M kernel (one 8-token tile always, two
    # only with two 16-row groups per CTA), else fused one-CTA tiles
    assert ops.plan_info(1, 18432, 3072)["smallm"] and ops.plan_info(1, 18432, 3072)["ring"]
    assert ops.plan_info(8, 3072, 3072)["bm"] == 8
    assert not ops.plan_info(4, 3072, 3200)["ring"]  # NF4 K % 256 != 0: register-stream kernel
    assert ops.plan_info(4, 3072, 3200, 1)["ring"]
    assert not ops.plan_info(8, 18432, 3072)["ring"]  # from 5 tokens: register-stream kernel
    assert ops.plan_info(16, 18432, 3072)["smallm"]
    # two token tiles take the ring kernel where its 64-row grid fills the SMs
    assert ops.plan_info(16, 18432, 3072)["ring"] and ops.plan_info(12, 12288, 4096)["ring"]
    assert not ops.plan_info(16, 9216, 3072)["ring"]
    small = ops.plan_info(16, 3072, 3072)
    assert not small["smallm"] and not small["pair"] and small["bm"] == 16 and small["splits"] > 1
    assert not ops.plan_info(4, 3072, 3008)["smallm"]  # K % 128 != 0: fused kernel
    assert ops.workspace_size(4, 3072, 3072) == 0


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
def test_long_k_split_plan(ops, fmt):
    # long K on a partial wave: two K halves of one-CTA tiles fill the SMs once
    f = 0 if fmt == "nf4" else 1
    plan = ops.plan_info(512, 3072, 12288, f)
    assert not plan["pair"] and not plan["twophase"] and plan["bm"] == 192 and plan["splits"] == 2
    m, n, k = 300, 3072, 8192
    plan = ops.plan_info(m, n, k, f)
    assert not plan["pair"] and plan["splits"] == 2
    x, w, bias, ref = _case(m, n, k, 5 + m, fmt, with_bias=True)
    y = _run(ops, fmt, x, w, bias, n)
    torch.cuda.synchronize()
    assert R.rel_err(to_bits(y), ref) <= TOL


def test_no_kernel_error_recorded(ops):
    assert ops.device_error() == 0


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("mode,splits,m", [(0, 0, 4),      # small-M kernel (TMA ring)
                                           (6, 0, 4),      # small-M kernel (registers)
                                           (1, 0, 300),    # fused one-CTA tiles
                                           (2, 0, 300),    # fused CTA pairs
                                           (1, 3, 16),     # split-K + reduce
                                           (3, 0, 1100)])  # two-phase
def test_output_into_column_range(ops, fmt, mode, splits, m):
    # dq_linear_*_ld: y lands in columns [c0, c0 + N) of a wider row-major
    # buffer, bit-identical to the plain call, with the other columns untouched
    n, k, c0, width = 640, 1024, 256, 1280
    x, w, bias, _ = _case(m, n, k, 41 + m, fmt, with_bias=True)
    xc, bc = x.cuda(), bias.cuda()
    ops.set_pair_mode(mode)
    ops.set_tile_override(0, splits)
    try:
        buf = torch.full((m, width), 7.0, dtype=torch.bfloat16, device="cuda")
        if fmt == "nf4":
            plain = ops.nf4_linear(xc, w[0], w[1], n, bc, act="gelu_tanh")
            ops.nf4_linear(xc, w[0], w[1], n, bc, act="gelu_tanh", out=buf[:, c0:c0 + n])
        else:
            plain = ops.fp8_linear(xc, w[0], w[1], bc, act="gelu_tanh")
            ops.fp8_linear(xc, w[0], w[1], bc, act="gelu_tanh", out=buf[:, c0:c0 + n])
        torch.cuda.synchronize()
    finally:
        ops.set_tile_override(0, 0)
        ops.set_pair_mode(0)
    assert torch.equal(buf[:, c0:c0 + n], plain)
    assert (buf[:, :c0] == 7.0).all() and (buf[:, c0 + n:] == 7.0).all()


@pytest.mark.parametrize("mode,bm,splits,m", [(1, 128, 0, 300), (2, 192, 0, 300), (3, 256, 0, 1100),
                                              (4, 256, 0, 300), (1, 0, 3, 16), (5, 0, 0, 4),
                                              (6, 0, 0, 12)])
def test_bf16_block_scales_give_the_same_bits(ops, mode, bm, splits, m):
    # scales repacked to bf16 at load time (dq_linear_nf4_scaled): the forward
    # casts absmax to bf16 anyway, so every plan returns the same bits
    n, k = 640, 1024
    x, (p, a), bias, ref = _case(m, n, k, 61 + m, "nf4", with_bias=True)
    a16 = a.to(torch.bfloat16)
    xc, bc = x.cuda(), bias.cuda()
    ops.set_pair_mode(mode)
    ops.set_tile_override(bm, splits)
    try:
        y32 = ops.nf4_linear(xc, p, a, n, bc)
        y16 = ops.nf4_linear(xc, p, a16, n, bc)
        torch.cuda.synchronize()
    finally:
        ops.set_tile_override(0, 0)
        ops.set_pair_mode(0)
    assert torch.equal(y32, y16)
    assert R.rel_err(to_bits(y16), ref) <= TOL
    w32 = ops.ltx23_nf4_dequantize(p, a, (n, k))
    w16 = ops.ltx23_nf4_dequantize(p, a16, (n, k))
    assert torch.equal(w32, w16)
    assert ops.device_error() == 0
