"""Host-side check of the small-M kernel's operand layout (csrc/dq_smallm.cuh).

The kernel hands each warp-level m16n8k16 MMA a permuted slice of K: thread
(g4, tig) owns weights k0 + 32*tig .. +31 of rows g4 and g4 + 8 of a 16-row
group, and MMA j takes elements 4j, 4j+1 (k-slots 2*tig, 2*tig+1) and
4j+2, 4j+3 (slots 2*tig+8, 2*tig+9) of that run for both A (weights) and B
(tokens).  This test emulates the MMA fragment layout (PTX ISA, m16n8k16 with
.bf16 A row-major / B column-major / f32 D) with numpy, feeds it exactly the
way the kernel does, and checks the sum equals W[16, 128] . x[8, 128]^T for
every k-group.  No GPU needed.
"""
import numpy as np


def mma_m16n8k16(a_frag, b_frag, d):
    """One warp MMA from per-lane fragments.

    a_frag[lane] = 8 A values (a0..a7), b_frag[lane] = 4 B values (b0..b3),
    d = [16, 8] accumulator, updated and returned.
    """
    A = np.zeros((16, 16))
    B = np.zeros((16, 8))
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        a = a_frag[lane]
        A[g, 2 * t], A[g, 2 * t + 1] = a[0], a[1]
        A[g + 8, 2 * t], A[g + 8, 2 * t + 1] = a[2], a[3]
        A[g, 2 * t + 8], A[g, 2 * t + 9] = a[4], a[5]
        A[g + 8, 2 * t + 8], A[g + 8, 2 * t + 9] = a[6], a[7]
        b = b_frag[lane]
        B[2 * t, g], B[2 * t + 1, g] = b[0], b[1]
        B[2 * t + 8, g], B[2 * t + 9, g] = b[2], b[3]
    return d + A @ B


def kernel_order_sum(w, x):
    """w [16, 128] (one row group, one k-group), x [8, 128]: the sum the
    kernel forms with its eight MMAs and the permuted k order."""
    d = np.zeros((16, 8))
    for j in range(8):
        a_frag, b_frag = [], []
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            run0 = w[g, 32 * t:32 * t + 32]        # row g4, this thread's run
            run1 = w[g + 8, 32 * t:32 * t + 32]    # row g4 + 8
            xr = x[g, 32 * t:32 * t + 32]          # token g4, same k
            # w0[2j] = run elements 4j, 4j+1; w0[2j+1] = 4j+2, 4j+3
            a_frag.append([run0[4 * j], run0[4 * j + 1], run1[4 * j], run1[4 * j + 1],
                           run0[4 * j + 2], run0[4 * j + 3], run1[4 * j + 2], run1[4 * j + 3]])
            b_frag.append([xr[4 * j], xr[4 * j + 1], xr[4 * j + 2], xr[4 * j + 3]])
        d = mma_m16n8k16(a_frag, b_frag, d)
    return d


def test_k_permutation_reproduces_the_product():
    rng = np.random.default_rng(7)
    for _ in range(3):
        w = rng.standard_normal((16, 128))
        x = rng.standard_normal((8, 128))
        np.testing.assert_allclose(kernel_order_sum(w, x), w @ x.T, rtol=1e-12, atol=1e-12)


def test_every_k_is_used_once_per_row_and_token():
    # indicator weights: D[r, n] counts how often (row r, token n) met each k
    w = np.ones((16, 128))
    for k in range(128):
        x = np.zeros((8, 128))
        x[:, k] = 1.0
        np.testing.assert_array_equal(kernel_order_sum(w, x), np.ones((16, 8)))
