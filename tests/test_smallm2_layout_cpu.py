"""Host-side check of the TMA-ring small-M kernel's stage layout
(csrc/dq_smallm2.cuh), no GPU needed.

A stage holds, per weight box, a tile of 16 * R16 rows x 128 bytes copied by
TMA with the 128-byte swizzle (16-byte chunk c of row r lands at chunk
c ^ (r % 8) of that row), and for NF4 a [16 * R16, 2 * (8 / R16)] tile of f32
block scales.  This test emulates those copies (zero fill past K and N), then
reads the stage back with exactly the addresses each consumer thread computes
and checks that every thread gets the packed bytes and scales of its own
32-weight runs (rows g4 and g4 + 8 of its row group, k 32*tig.. of its
k-group), that every k-group of every row is read exactly once, and that the
shared-memory regions of the configuration do not overlap and fit the
planned resident CTAs per SM.  It also restates the planner's choice of row
groups and CTAs per SM.
"""
import numpy as np
import pytest


def cfg(fmt, mt, r16, cps=2):
    c = {}
    c["rows"] = 16 * r16
    c["kg_per_box"] = 2 if fmt == "nf4" else 1
    c["kg_per_stage"] = 8 // r16
    c["boxes"] = c["kg_per_stage"] // c["kg_per_box"]
    c["box_bytes"] = 128 * c["rows"]
    c["w_stage"] = c["boxes"] * c["box_bytes"]
    c["abs_per_row"] = 2 * c["kg_per_stage"] if fmt == "nf4" else 0
    c["a_stage"] = c["abs_per_row"] * 4 * c["rows"]
    # two token tiles: x staged as 16-row x 64-k boxes, two per k-group
    c["x_box"] = 16 * 128
    c["x_stage"] = 2 * c["kg_per_stage"] * c["x_box"] if mt == 2 else 0
    c["off_x"] = c["w_stage"] + c["a_stage"]
    c["stage"] = c["w_stage"] + c["a_stage"] + c["x_stage"]
    if mt == 2:
        c["stages"] = 4
    elif cps == 2:
        c["stages"] = 8 if fmt == "nf4" else 6
    else:
        c["stages"] = 4
    c["lut"] = 256 * 32 * 4 if fmt == "nf4" else 0
    c["red"] = 8 * mt * 128 * 4
    c["off_lut"] = c["stages"] * c["stage"]
    c["off_red"] = c["off_lut"] + c["lut"]
    c["off_bar"] = c["off_red"] + c["red"]
    c["off_flag"] = c["off_bar"] + 2 * c["stages"] * 8
    c["smem"] = c["off_flag"] + 16 + 1024
    return c


def tma_box_swizzled(src, c0, r0, rows):
    """2-D TMA tile of `rows` x 128 bytes at (byte c0, row r0), 128-byte swizzle."""
    out = np.zeros(rows * 128, dtype=np.uint8)
    for r in range(rows):
        for b in range(128):
            gr, gc = r0 + r, c0 + b
            v = src[gr, gc] if gr < src.shape[0] and gc < src.shape[1] else 0
            out[r * 128 + (((b // 16) ^ (r % 8)) * 16) + b % 16] = v
    return out


def tma_box_plain(src, c0, r0, rows, cols):
    out = np.zeros((rows, cols), dtype=src.dtype)
    for r in range(rows):
        for b in range(cols):
            gr, gc = r0 + r, c0 + b
            if gr < src.shape[0] and gc < src.shape[1]:
                out[r, b] = src[gr, gc]
    return out.reshape(-1)


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("r16", [1, 2, 4])
@pytest.mark.parametrize("mt", [1, 2])
@pytest.mark.parametrize("cps", [2, 3])
def test_smem_regions_fit_the_resident_ctas(fmt, r16, mt, cps):
    if mt == 2 and (r16, cps) != (4, 2):
        pytest.skip("two token tiles run 64-row CTAs, two per SM")
    c = cfg(fmt, mt, r16, cps)
    assert c["off_x"] % 1024 == 0
    assert c["stage"] % 1024 == 0 and c["box_bytes"] % 1024 == 0
    assert c["boxes"] * c["kg_per_box"] == c["kg_per_stage"]
    assert c["off_lut"] + c["lut"] <= c["off_red"] <= c["off_bar"] < c["off_flag"]
    assert cps * (c["smem"] + 1024) <= 228 * 1024
    if fmt == "nf4":  # the scale box's inner extent is whole 16-byte units
        assert (c["abs_per_row"] * 4) % 16 == 0


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("r16", [1, 2, 4])
def test_every_thread_reads_its_runs(fmt, r16):
    rng = np.random.default_rng(r16)
    c = cfg(fmt, 1, r16)
    n, k = c["rows"] + 5, 3 * 128 * c["kg_per_stage"] - 128  # ragged N, ragged last stage
    if fmt == "nf4":
        k = max(256, (k // 256) * 256)
    row_bytes = k // 2 if fmt == "nf4" else k
    w = rng.integers(0, 256, size=(n, row_bytes), dtype=np.uint8)
    absmax = rng.random((n, k // 64)).astype(np.float32) + 1.0
    kg_total = k // 128
    stages = -(-kg_total // c["kg_per_stage"])
    seen = np.zeros((n, kg_total), dtype=int)
    for blk in range(-(-n // c["rows"])):
        row0 = blk * c["rows"]
        for s in range(stages):
            stage = np.zeros(c["stage"], dtype=np.uint8)
            for b in range(c["boxes"]):
                stage[b * c["box_bytes"]:(b + 1) * c["box_bytes"]] = tma_box_swizzled(
                    w, (s * c["boxes"] + b) * 128, row0, c["rows"])
            if fmt == "nf4":
                a = tma_box_plain(absmax, s * c["abs_per_row"], row0, c["rows"], c["abs_per_row"])
                stage[c["w_stage"]:] = a.view(np.uint8)
            for warp in range(8):
                rg, kgl = warp % r16, warp // r16
                bx, kk = kgl // c["kg_per_box"], kgl % c["kg_per_box"]
                g = s * c["kg_per_stage"] + kgl
                if g >= kg_total:
                    continue
                for lane in range(32):
                    g4, tig = lane >> 2, lane & 3
                    r_lo = 16 * rg + g4
                    box = bx * c["box_bytes"]
                    for r in (r_lo, r_lo + 8):
                        base = box + r * 128
                        if fmt == "nf4":
                            ch = ((4 * kk + tig) ^ g4) * 16
                            got = stage[base + ch:base + ch + 16]
                            want_lo = g * 64 + 16 * tig
                            want = w[row0 + r, want_lo:want_lo + 16] if row0 + r < n else np.zeros(16, np.uint8)
                            sc_off = c["w_stage"] + 4 * (r * c["abs_per_row"] + 2 * kgl + (tig >> 1))
                            sc = stage[sc_off:sc_off + 4].view(np.float32)[0]
                            want_sc = absmax[row0 + r, (g * 128 + 32 * tig) // 64] if row0 + r < n else 0.0
                            assert sc == want_sc
                        else:
                            c0, c1 = ((2 * tig) ^ g4) * 16, ((2 * tig + 1) ^ g4) * 16
                            got = np.concatenate([stage[base + c0:base + c0 + 16], stage[base + c1:base + c1 + 16]])
                            want_lo = g * 128 + 32 * tig
                            want = w[row0 + r, want_lo:want_lo + 32] if row0 + r < n else np.zeros(32, np.uint8)
                        np.testing.assert_array_equal(got, want)
                        if row0 + r < n and tig == 0:
                            seen[row0 + r, g] += 1
    assert (seen == 1).all()


@pytest.mark.parametrize("r16", [1, 2, 4])
@pytest.mark.parametrize("mt", [1, 2])
def test_partial_sums_meet_once_per_warp(r16, mt):
    # output o of row group orow sums the warps q * R16 + orow, q < 8 / R16
    kgs = 8 // r16
    hits = np.zeros((8, mt, 128), dtype=int)
    for o in range(r16 * mt * 128):
        row, tok, rm = o & 15, (o >> 4) & 7, o >> 7
        orow, m = rm // mt, rm % mt
        for q in range(kgs):
            w = q * r16 + orow
            assert w % r16 == orow and w // r16 == q
            hits[w, m, tok * 16 + row] += 1
    assert (hits == 1).all()


def smallm2_config(n, sms):
    """The planner's choice (dq_capi.cu smallm2_config): the (R16, CPS) whose
    one-wave grid fills the largest share of CPS * SMs resident slots."""
    best, out = -1.0, (4, 3)
    for cps in (3, 2):
        for r16 in (4, 2, 1):
            grid = -(-n // (16 * r16))
            if grid > cps * sms:
                continue
            fill = grid / (cps * sms)
            if fill > best + 1e-9:
                best, out = fill, (r16, cps)
    return out


def test_planner_fills_one_wave_on_148_sms():
    # measured choices on B200 (148 SMs)
    assert smallm2_config(18432, 148) == (4, 2)
    assert smallm2_config(12288, 148) == (2, 3)
    assert smallm2_config(9216, 148) == (2, 2)
    assert smallm2_config(6144, 148) == (1, 3)
    assert smallm2_config(3072, 148) == (1, 2)
    for n in (64, 1000, 3072, 9000, 18432, 21504, 28416):
        r16, cps = smallm2_config(n, 148)
        assert -(-n // (16 * r16)) <= cps * 148
    assert smallm2_config(40000, 148) == (4, 3)  # beyond one wave


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
@pytest.mark.parametrize("m", [9, 13, 16])
def test_two_token_tiles_read_x_from_the_stage(fmt, m):
    """Emulate the x boxes of a stage (TMA 128-byte swizzle, rows past M
    zero-filled) and read them back with the consumer threads' addresses:
    thread (g4, tig) of warp w gets x[t, 128 g + 32 tig .. + 31] for tokens
    t = g4 and 8 + g4, zeros for t >= M."""
    rng = np.random.default_rng(m)
    c = cfg(fmt, 2, 4, 2)
    k = 3 * 128 * c["kg_per_stage"]
    x = rng.integers(0, 1 << 16, size=(m, k), dtype=np.uint16)
    xb = x.view(np.uint8).reshape(m, 2 * k)  # bf16 rows as bytes
    stages = k // (128 * c["kg_per_stage"])
    for s in range(stages):
        xs = np.zeros(c["x_stage"], dtype=np.uint8)
        for b in range(2 * c["kg_per_stage"]):
            k0 = (s * 2 * c["kg_per_stage"] + b) * 64
            box = np.zeros(16 * 128, dtype=np.uint8)
            for r in range(min(m, 16)):
                for byte in range(128):
                    box[r * 128 + ((byte // 16) ^ (r % 8)) * 16 + byte % 16] = xb[r, 2 * k0 + byte]
            xs[b * c["x_box"]:(b + 1) * c["x_box"]] = box
        for warp in range(8):
            kgl = warp // 4
            g = s * c["kg_per_stage"] + kgl
            for lane in range(32):
                g4, tig = lane >> 2, lane & 3
                xbox = (2 * kgl + (tig >> 1)) * c["x_box"]
                for mt in range(2):
                    t = 8 * mt + g4
                    chunks = []
                    for q in range(4):
                        off = xbox + t * 128 + ((4 * (tig & 1) + q) ^ (t & 7)) * 16
                        chunks.append(xs[off:off + 16])
                    got = np.concatenate(chunks).view(np.uint16)
                    k_run = 128 * g + 32 * tig
                    want = x[t, k_run:k_run + 32] if t < m else np.zeros(32, np.uint16)
                    np.testing.assert_array_equal(got, want)
