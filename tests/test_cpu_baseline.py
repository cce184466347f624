"""The restated CPU MLIRBackend (the timed CPU baseline) computes the same
results as the checkers, and keeps the reference's CPU launch rule that the
ndrange must be a multiple of the workgroup (ext/KernelAbstractionsExt.jl:256-258)."""
import ctypes as C

import numpy as np
import pytest

import oracle

L = oracle.lib()


def p(a):
    return a.ctypes.data


def test_vadd_matches_and_requires_multiple_of_w():
    r = np.random.Generator(np.random.Philox(3))
    a = r.random(4096, dtype=np.float32); b = r.random(4096, dtype=np.float32)
    c = np.empty_like(a)
    assert L.mlirb_vadd_f32(p(c), p(a), p(b), 4096, 256) == 0
    np.testing.assert_array_equal(c, a + b)
    assert L.mlirb_vadd_f32(p(c), p(a), p(b), 4000, 256) == -1


def test_sum_sq_materialised_tree_close_to_fp64():
    r = np.random.Generator(np.random.Philox(4))
    n = 1 << 20
    x = (r.random(n, dtype=np.float32) * 2 - 1).astype(np.float32)
    tmp = np.empty(n + n // 512 + 2, dtype=np.float32)
    got = L.mlirb_sum_sq_f32(p(x), n, 256, p(tmp))
    assert got == pytest.approx(oracle.sum_sq(x), rel=1e-5)


def test_gather_and_hist_exact():
    r = np.random.Generator(np.random.Philox(5))
    n = 1 << 16
    a = r.random(n, dtype=np.float32)
    idx = r.integers(1, n + 1, size=n, dtype=np.int32)
    c = np.empty(n, dtype=np.float32)
    assert L.mlirb_gather_f32(p(c), p(a), n, p(idx), n, 256) == 0
    np.testing.assert_array_equal(c, oracle.gather(a, idx)[0])
    keys = r.integers(1, 4097, size=n, dtype=np.int32)
    counts = np.zeros(4096, dtype=np.uint32)
    assert L.mlirb_hist_u32(p(counts), 4096, p(keys), n, 256) == 0
    np.testing.assert_array_equal(counts, oracle.hist(keys, 4096)[0])


def test_mm_tiled16_bitexact_with_checker():
    r = np.random.Generator(np.random.Philox(6))
    M, N, K = 64, 48, 40
    A = np.asfortranarray(r.standard_normal((M, K), dtype=np.float32))
    B = np.asfortranarray(r.standard_normal((K, N), dtype=np.float32))
    Cm = np.zeros((M, N), dtype=np.float32, order="F")
    assert L.mlirb_mm_tiled16_f32(p(Cm), p(A), p(B), M, N, K, M, K, M, 0, N) == 0
    np.testing.assert_array_equal(Cm, oracle.mm_tiled16_f32(A, B))


@pytest.mark.parametrize("find_max", [1, 0])
def test_mlirb_findext_matches_checker(find_max):
    """The OpenMP findmax/findmin baseline agrees with the sequential checker:
    first index among ties, NaN wins both, +0.0 above -0.0 (chunk borders included)."""
    import ctypes as C
    r = np.random.Generator(np.random.Philox(21))
    for n in (1, 2, 7, 1000, 100_003):
        x = r.standard_normal(n, dtype=np.float32)
        x[n // 3] = x[n // 2] = x.max() if find_max else x.min()
        for case in range(3):
            y = x.copy()
            if case == 1 and n > 10:
                y[n // 5] = y[(4 * n) // 5] = np.nan
            if case == 2:
                y[:] = -0.0
                y[n // 2:] = 0.0
            v = C.c_double()
            got = oracle.lib().mlirb_findext_f32(C.byref(v), y.ctypes.data, n, find_max)
            assert got == oracle.findext(y, bool(find_max))[1]

