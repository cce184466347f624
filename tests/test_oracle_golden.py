"""Pin the CPU oracle against the reference's known-answer tests
(tests/golden/*.npz, restated from the reference test suite by make_golden.py)."""
import numpy as np
import pytest

import oracle
from conftest import golden


@pytest.mark.parametrize("name", ["vadd_4096", "vadd_tail_1000", "vadd_tail_257"])
def test_vadd_exact(name):
    g = golden(name)
    np.testing.assert_array_equal(oracle.vadd(g["a"], g["b"]), g["c"])


@pytest.mark.parametrize("name", ["hist_ka_4096_256", "hist_mod_4096_8", "hist_one_65536"])
def test_hist_exact(name):
    g = golden(name)
    counts, rc = oracle.hist(g["keys"], int(g["nbins"]))
    assert rc == 0
    np.testing.assert_array_equal(counts, g["counts"])


def test_hist_accumulates_and_wraps():
    start = np.array([0xFFFFFFFF, 7], dtype=np.uint32)
    counts, rc = oracle.hist(np.array([1, 2, 2], dtype=np.int32), 2, start)
    assert rc == 0
    np.testing.assert_array_equal(counts, np.array([0, 9], dtype=np.uint32))


def test_hist_bad_key_reported_and_skipped():
    counts, rc = oracle.hist(np.array([0, 1, 3, -5], dtype=np.int32), 2)
    assert rc == -5
    np.testing.assert_array_equal(counts, np.array([1, 0], dtype=np.uint32))


def test_reduce_sum_1_to_1024():
    g = golden("reduce_1_1024")
    assert oracle.mapreduce(g["x"]) == g["sum"]


def test_gpuarrays_reductions():
    g = golden("gpuarrays_1024")
    a, p = g["a"], g["p"]
    assert oracle.mapreduce(a) == pytest.approx(float(g["sum"]), rel=1e-14)
    assert oracle.mapreduce(a, "identity", "max", -np.inf) == g["maximum"]
    assert oracle.mapreduce(a, "identity", "min", np.inf) == g["minimum"]
    assert oracle.sum_sq(a) == pytest.approx(float(g["sum_abs2"]), rel=1e-14)
    assert oracle.mapreduce(p, "identity", "mul", 1.0) == pytest.approx(float(g["prod"]), rel=1e-12)
    assert oracle.mapreduce(g["s"], "gt0", "add") == g["count_s_gt0"]


def test_max_min_julia_nan_and_zero_semantics():
    x = np.array([1.0, np.nan, 3.0], dtype=np.float32)
    assert np.isnan(oracle.mapreduce(x, "identity", "max", -np.inf))
    z = np.array([-0.0, 0.0], dtype=np.float32)
    assert np.signbit(oracle.mapreduce(z, "identity", "max", -np.inf)) == False  # noqa: E712
    assert np.signbit(oracle.mapreduce(z, "identity", "min", np.inf)) == True  # noqa: E712


def test_gather_permutation_exact():
    g = golden("gather_perm_4096")
    c, rc = oracle.gather(g["a"], g["idx"])
    assert rc == 0
    np.testing.assert_array_equal(c, g["c"])


def test_gather_out_of_range():
    a = np.arange(1, 5, dtype=np.float32)
    c, rc = oracle.gather(a, np.array([1, 0, 5, 4], dtype=np.int32))
    assert rc == -5
    np.testing.assert_array_equal(c, np.array([1, 0, 0, 4], dtype=np.float32))


def test_matmul_f64_vs_golden():
    g = golden("mm_tiled_256")
    np.testing.assert_allclose(oracle.matmul_f64(g["A"], g["B"]), g["C"], rtol=1e-12, atol=1e-9)


def test_mm_tiled16_close_to_fp64_and_ignores_k_remainder():
    g = golden("mm_tiled_256")
    C32 = oracle.mm_tiled16_f32(g["A"], g["B"])
    np.testing.assert_allclose(C32, g["C"], rtol=1e-5)
    # K % 16 is ignored by the reference tiled kernel (examples/tiled_matmul.jl:34)
    A = np.asfortranarray(g["A"][:40, :40])
    B = np.asfortranarray(g["B"][:40, :24])
    ref = A[:, :32].astype(np.float64) @ B[:32, :].astype(np.float64)
    np.testing.assert_allclose(oracle.matmul_f64(A, B), ref, rtol=1e-12)
    np.testing.assert_allclose(oracle.mm_tiled16_f32(A, B), ref, rtol=1e-5)


def test_matmul_properties_agree():
    r = np.random.Generator(np.random.Philox(5))
    A = np.asfortranarray(r.standard_normal((64, 48), dtype=np.float32))
    B = np.asfortranarray(r.standard_normal((48, 80), dtype=np.float32))
    C64 = oracle.matmul_f64(A, B)
    v = r.standard_normal(80)
    np.testing.assert_allclose(oracle.matvec_chain_f64(A, B, v), C64 @ v, rtol=1e-10, atol=1e-9)
    ii = np.array([0, 63, 5]); jj = np.array([0, 79, 40])
    np.testing.assert_allclose(oracle.matmul_entries_f64(A, B, ii, jj), C64[ii, jj], rtol=1e-12)


def test_findext_follows_julia_isless_rules():
    # Base._rf_findmax keeps the current candidate unless isless(current, new);
    # _rf_findmin uses isgreater, under which NaN is the smallest value.
    x = np.float32([1, 3, 3, np.nan, 2, np.nan])
    assert oracle.findext(x, True)[1] == 4 and oracle.findext(x, False)[1] == 4
    z = np.float32([-0.0, 0.0, -0.0])
    assert oracle.findext(z, True)[1] == 2      # +0.0 above -0.0
    assert oracle.findext(np.float32([0.0, -0.0]), False)[1] == 2
    r = np.random.Generator(np.random.Philox(2000)).random(2000, dtype=np.float32)
    assert oracle.findext(r, True) == (float(r.max()), int(np.argmax(r)) + 1)
    assert oracle.findext(r, False) == (float(r.min()), int(np.argmin(r)) + 1)


def test_dims_and_scan_oracles_agree_with_numpy():
    # independent restatements (numpy fp64) of mapreducedim!(dims) and accumulate!
    r = np.random.Generator(np.random.Philox(17))
    m3 = np.asfortranarray(r.random((8, 4, 3), dtype=np.float32))
    for d in (1, 2, 3):
        np.testing.assert_allclose(oracle.mapreduce_dim(m3, d), m3.astype(np.float64).sum(d - 1, keepdims=True),
                                   rtol=1e-13)
        np.testing.assert_array_equal(oracle.mapreduce_dim(m3, d, "identity", "max", -np.inf),
                                      m3.max(d - 1, keepdims=True).astype(np.float64))
    x = r.random(1000, dtype=np.float32)
    np.testing.assert_allclose(oracle.accumulate(x), np.cumsum(x.astype(np.float64)), rtol=1e-13)
    ex = oracle.accumulate(x, "add", 1.5, exclusive=True)
    assert ex[0] == 1.5
    np.testing.assert_allclose(ex[1:], 1.5 + np.cumsum(x.astype(np.float64))[:-1], rtol=1e-13)
    np.testing.assert_array_equal(oracle.accumulate(x, "max", -np.inf), np.maximum.accumulate(x).astype(np.float64))
    # cumsum(1:1024) (test/test_downstream_ka.jl:39-42)
    np.testing.assert_array_equal(oracle.accumulate(np.arange(1, 1025, dtype=np.float32)),
                                  np.cumsum(np.arange(1, 1025)).astype(np.float64))
