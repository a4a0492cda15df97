"""CPU check of the GEMV kernels' operand layouts: the per-lane K permutations
of the planes GEMV (csrc/w8a16_planes.cuh, ``w8a16_pgemv_kernel``) and of the
decode-in-kernel GEMV (csrc/w8a16.cuh, ``w8a16_gemv_kernel``) give the plain
dot product.

Neither kernel shuffles.  In the planes GEMV lane (g, q) of warp w feeds its own
16 weight bytes of rows g and g + 8 (K [64w + 16q, +16) of a stage) into the A
registers of two m16n8k32 MMAs, and its own 16 plane bytes at the same K into
the B registers (the decode-in-kernel GEMV's m16n8k16 mapping is described at
``_emulate_gemv``).
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


def _emulate_gemv(W, X, K, MT):
    """w8a16_gemv_kernel<MT>: lane (g, q) of warp w holds the 16 weight bytes of
    row 8 gr + g at K [k0 + 16q, +16) and the activations of tokens 16 mt + 8 h + g
    at K [k0 + 16q + 8p, +8); MMA t (m16n8k16) takes weight bytes 4t .. 4t + 3
    (b0 = bytes 4t, 4t + 1 at logical k 2q, 2q + 1; b1 = bytes 4t + 2, 4t + 3 at
    2q + 8, 2q + 9) and the activation pairs at the same K positions (a0/a1 rows g
    and g + 8 at logical k 2q, 2q + 1; a2/a3 at 2q + 8, 2q + 9)."""
    acc = np.zeros((WARPS, MT * 16, ROWS), dtype=np.int64)   # red[warp][token][row]
    nst = -(-K // STAGE_K)
    for w in range(WARPS):
        for st in range(nst):
            k0 = st * STAGE_K + 64 * w
            if k0 >= K:
                continue
            for t in range(4):
                for gr in range(4):
                    for mt in range(MT):
                        A = np.full((16, 16), -10**9, dtype=np.int64)
                        B = np.full((16, 8), -10**9, dtype=np.int64)
                        for lane in range(32):
                            g, q = lane >> 2, lane & 3
                            kb = k0 + 16 * q + 4 * t
                            for j in range(2):
                                A[g, 2 * q + j] = X[16 * mt + g, kb + j]
                                A[g + 8, 2 * q + j] = X[16 * mt + 8 + g, kb + j]
                                A[g, 2 * q + 8 + j] = X[16 * mt + g, kb + 2 + j]
                                A[g + 8, 2 * q + 8 + j] = X[16 * mt + 8 + g, kb + 2 + j]
                                B[2 * q + j, g] = W[8 * gr + g, kb + j]
                                B[2 * q + 8 + j, g] = W[8 * gr + g, kb + 2 + j]
                        assert (A > -10**9).all() and (B > -10**9).all()
                        D = A @ B
                        for lane in range(32):
                            g, q = lane >> 2, lane & 3
                            for i in range(4):
                                r, c = g + 8 * (i >> 1), 2 * q + (i & 1)
                                acc[w, 16 * mt + r, 8 * gr + c] += D[r, c]
    return acc.sum(axis=0)   # [token][row]


def test_gemv_lane_permutation_is_the_dot_product():
    rng = np.random.default_rng(4)
    for K, MT in ((1040, 1), (1536, 2)):
        Kp = -(-K // STAGE_K) * STAGE_K
        W = np.zeros((ROWS, Kp), dtype=np.int64)
        X = np.zeros((MT * 16, Kp), dtype=np.int64)
        W[:, :K] = rng.integers(-120, 121, size=(ROWS, K))
        X[:, :K] = rng.integers(-1000, 1001, size=(MT * 16, K))
        got = _emulate_gemv(W, X, K, MT)
        assert np.array_equal(got, X[:, :K] @ W[:, :K].T)
