"""CPU check of the planes GEMV's operand layout (csrc/w8a16_planes.cuh,
``w8a16_pgemv_kernel``): the per-lane K permutation gives the plain dot product.

The kernel never shuffles: lane (g, q) of warp w feeds its own 16 weight bytes of
rows g and g + 8 (K [64w + 16q, +16) of a stage) into the A registers of two
m16n8k32 MMAs, and its own 16 plane bytes at the same K into the B registers.
Here every lane's registers are placed into the MMA's 16 x 32 A and 32 x 8 B
matrices by the PTX fragment layout of ``mma.sync.m16n8k32`` with 8-bit
operands (A: register j holds row g + 8 (j & 1), k 4q + i + 16 (j >> 1); B:
register j holds k 4q + i + 16 j, column g; D: element i is row g + 8 (i >> 1),
column 2q + (i & 1)), the products are formed, the D fragments are read back
the way the kernel stores them into its reduction array, and the result must be
W @ planes^T exactly (integer codes stand in for the e4m3 values).
"""
import numpy as np

ROWS, WARPS, STAGE_K = 32, 8, 512


def _lane_regs(W, Pl, k0, g, q, rg, kk, ng):
    """The kernel's A and B registers of lane (g, q) for row group rg, MMA kk,
    column group ng, as 4-byte groups of physical K indices' values."""
    lo = W[16 * rg + g, k0 + 16 * q:k0 + 16 * q + 16]        # wv[2 rg]
    hi = W[16 * rg + g + 8, k0 + 16 * q:k0 + 16 * q + 16]    # wv[2 rg + 1]
    pa = Pl[8 * ng + g, k0 + 16 * q:k0 + 16 * q + 16]
    b = 8 * kk
    a = [lo[b:b + 4], hi[b:b + 4], lo[b + 4:b + 8], hi[b + 4:b + 8]]
    bb = [pa[b:b + 4], pa[b + 4:b + 8]]
    return a, bb


def _emulate(W, Pl, K, NG):
    acc = np.zeros((WARPS, NG * 8, ROWS), dtype=np.int64)   # red[warp][col][row]
    nst = -(-K // STAGE_K)
    for w in range(WARPS):
        for st in range(nst):
            k0 = st * STAGE_K + 64 * w
            if k0 >= K:
                continue
            for rg in range(2):
                for ng in range(NG):
                    for kk in range(2):
                        A = np.full((16, 32), -10**9, dtype=np.int64)
                        B = np.full((32, 8), -10**9, dtype=np.int64)
                        for lane in range(32):
                            g, q = lane >> 2, lane & 3
                            a, bb = _lane_regs(W, Pl, k0, g, q, rg, kk, ng)
                            for j in range(4):
                                for i in range(4):
                                    A[g + 8 * (j & 1), 4 * q + i + 16 * (j >> 1)] = a[j][i]
                            for j in range(2):
                                for i in range(4):
                                    B[4 * q + i + 16 * j, g] = bb[j][i]
                        assert (A > -10**9).all() and (B > -10**9).all()  # every slot written once
                        D = A @ B
                        for lane in range(32):
                            g, q = lane >> 2, lane & 3
                            for i in range(4):
                                r, c = g + 8 * (i >> 1), 2 * q + (i & 1)
                                acc[w, 8 * ng + c, 16 * rg + r] += D[r, c]
    return acc.sum(axis=0)   # [col][row]


def test_pgemv_lane_permutation_is_the_dot_product():
    rng = np.random.default_rng(3)
    for K, NG in ((1040, 1), (2048, 2)):     # a K tail (K % 512 != 0) and two column groups
        Kp = -(-K // STAGE_K) * STAGE_K
        W = np.zeros((ROWS, Kp), dtype=np.int64)
        Pl = np.zeros((NG * 8, Kp), dtype=np.int64)
        W[:, :K] = rng.integers(-120, 121, size=(ROWS, K))   # zero fill past K, as TMA does
        Pl[:, :K] = rng.integers(-120, 121, size=(NG * 8, K))
        got = _emulate(W, Pl, K, NG)
        want = Pl[:, :K] @ W[:, :K].T
        assert np.array_equal(got, want)
