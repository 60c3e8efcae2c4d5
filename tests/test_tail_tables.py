"""The iSTFT basis tables the tail kernels build on the host, and the shapes the kernels rely on.

`tail.cu` computes the inverse real-DFT basis exactly as the reference graph's constants are made
(cos / sin of 2*pi*k*n/16 in double, rounded to fp32, times the one-sided weight, divided by 16 in
fp32) and checks, before the first launch on a device, two facts the kernels' arithmetic assumes
(`tail_math.cuh`): the sine table is exactly zero at k = 0 and at n = 0 and nowhere else, the
cosine table nowhere; and the tables are mirror-symmetric, bc[k][16 - n] = bc[k][n] and
bs[k][16 - n] = -bs[k][n], up to entries below 1e-15 that stand for exact zeros.  The library makes
the check on the GPU box with the host's libm; this test restates the table construction in numpy
(IEEE fp32 operations, the same order) and checks both facts on the CPU, so a libm whose results
broke them would show here first.
"""
import numpy as np


def basis_tables():
    bc = np.zeros((9, 16), np.float32)
    bs = np.zeros((9, 16), np.float32)
    for k in range(9):
        wk = np.float32(1.0 if k in (0, 8) else 2.0)
        for n in range(16):
            ang = 2.0 * np.pi * float(k) * float(n) / 16.0
            c, s = np.float32(np.cos(ang)), np.float32(np.sin(ang))
            bc[k, n] = np.float32(np.float32(wk * c) / np.float32(16.0))
            bs[k, n] = np.float32(np.float32(-wk * s) / np.float32(16.0))
    return bc, bs


def test_zero_pattern_the_kernels_skip():
    bc, bs = basis_tables()
    assert (bc != 0).all()
    for k in range(9):
        for n in range(16):
            assert (bs[k, n] == 0) == (k == 0 or n == 0), (k, n, bs[k, n])


def test_mirror_symmetry_up_to_stand_in_zeros():
    bc, bs = basis_tables()
    for k in range(9):
        for n in range(9, 16):
            assert abs(float(bc[k, n]) - float(bc[k, 16 - n])) <= 1e-15, (k, n)
            assert abs(float(bs[k, n]) + float(bs[k, 16 - n])) <= 1e-15, (k, n)
    # every entry that is not a stand-in zero is exactly symmetric
    big = np.abs(bc[:, 9:]) > 1e-15
    assert (bc[:, 9:][big] == bc[:, 7:0:-1][big]).all()
    big = np.abs(bs[:, 9:]) > 1e-15
    assert (bs[:, 9:][big] == -bs[:, 7:0:-1][big]).all()


def test_symmetric_sums_equal_the_full_contraction_in_exact_arithmetic():
    """Columns n and 16 - n from one pair of sums (er +- ei) reproduce the full 9 -> 16 contraction
    up to the stand-in zeros' contribution (here: below 1e-14 of the spectrum's scale)."""
    bc, bs = basis_tables()
    rng = np.random.default_rng(5)
    re, im = rng.standard_normal((2, 1000, 9))
    full = re @ bc.astype(np.float64) + im @ bs.astype(np.float64)
    er = re @ bc[:, :9].astype(np.float64)
    ei = im @ bs[:, :9].astype(np.float64)
    sym = np.concatenate([er + ei, (er - ei)[:, 7:0:-1]], axis=1)
    assert np.abs(sym - full).max() <= 1e-14 * np.abs(full).max()
