"""Parity of the CUDA kernels with the CPU oracle, called through the C ABI
(libkernels.so via ctypes) on seeded inputs and the golden known-answer
fixtures.  Bars: bit-exact for vadd, gather, histogram and the SIMT tiled
matmul; rel 1e-5 (vs fp64) for the reductions."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
from conftest import golden
from cutilecpu_b200 import _lib

pytestmark = pytest.mark.gpu

RTOL_REDUCE = 1e-5


@pytest.fixture(scope="module")
def L(cuda):
    lib = _lib.lib()
    assert lib.mk_init(0) == 0, _lib.last_error()
    return lib


def dev(a: np.ndarray) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(
        np.int32 if a.dtype == np.uint32 else a.dtype))
    return t.to("cuda")


def host(t: torch.Tensor, dtype=None) -> np.ndarray:
    torch.cuda.synchronize()
    h = t.cpu().numpy()
    return h.view(dtype) if dtype is not None else h


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def poll(L) -> int:
    return L.mk_error_poll(stream())


# ---------------------------------------------------------------- vadd -----

@pytest.mark.parametrize("name", ["vadd_4096", "vadd_tail_1000", "vadd_tail_257"])
def test_vadd_golden(L, name):
    g = golden(name)
    a, b = dev(g["a"]), dev(g["b"])
    c = torch.zeros_like(a)
    assert L.mk_vadd_f32(c.data_ptr(), a.data_ptr(), b.data_ptr(), a.numel(), stream()) == 0
    np.testing.assert_array_equal(host(c), g["c"])


@pytest.mark.parametrize("n", [1, 3, 4, 5, 255, 256, 257, 1 << 20, (1 << 22) + 3])
@pytest.mark.parametrize("offset", [0, 1, 3])
def test_vadd_sizes_and_misaligned_views(L, n, offset):
    r = np.random.Generator(np.random.Philox(n * 7 + offset))
    a_h = r.random(n + 4, dtype=np.float32); b_h = r.random(n + 4, dtype=np.float32)
    a, b = dev(a_h), dev(b_h)
    c = torch.full((n + 4,), -1.0, device="cuda")
    o = offset
    assert L.mk_vadd_f32(c.data_ptr() + 4 * o, a.data_ptr() + 4 * o, b.data_ptr() + 4 * o, n, stream()) == 0
    got = host(c)
    np.testing.assert_array_equal(got[o:o + n], oracle.vadd(a_h[o:o + n], b_h[o:o + n]))
    assert (got[:o] == -1).all() and (got[o + n:] == -1).all()


def test_vadd_chain_with_dependent_launch_in_a_graph(L):
    # mk_vadd_f32 uses programmatic dependent launch: a kernel may start while
    # its predecessor drains, but must not read before the predecessor's writes
    # land.  A chain c1 = a + b, c2 = c1 + b, ... where each vadd reads the
    # previous output, launched eagerly and as a CUDA graph, must equal the
    # oracle's chain exactly.
    n = (1 << 20) + 8
    r = np.random.Generator(np.random.Philox(31))
    a_h, b_h = r.random(n, dtype=np.float32), r.random(n, dtype=np.float32)
    want = [a_h]
    for _ in range(12):
        want.append(oracle.vadd(want[-1], b_h))
    b = dev(b_h)
    for use_graph in (False, True):
        bufs = [dev(a_h)] + [torch.full((n,), -1.0, device="cuda") for _ in range(12)]

        def chain():
            for k in range(12):
                assert L.mk_vadd_f32(bufs[k + 1].data_ptr(), bufs[k].data_ptr(), b.data_ptr(), n, stream()) == 0

        if use_graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                chain()
            g.replay()
        else:
            chain()
        torch.cuda.synchronize()
        for k in range(13):
            np.testing.assert_array_equal(host(bufs[k]), want[k])


def test_vadd_empty_and_invalid(L):
    assert L.mk_vadd_f32(0, 0, 0, 0, stream()) == 0
    assert L.mk_vadd_f32(0, 0, 0, -1, stream()) == _lib.MK_ERR_INVALID
    assert b"n must be" in L.mk_last_error()


# ----------------------------------------------------------- mapreduce -----

def reduce_dev(L, x: torch.Tensor, f="identity", op="add", init=0.0, n=None, off=0):
    out = torch.empty(1, dtype=torch.float64, device="cuda")
    rc = L.mk_mapreduce_f32(out.data_ptr(), x.data_ptr() + 4 * off, x.numel() - off if n is None else n,
                            _lib.MK_F[f], _lib.MK_OP[op], float(init), stream())
    assert rc == 0, _lib.last_error()
    return host(out)[0]


def test_reduce_sum_1_to_1024(L):
    g = golden("reduce_1_1024")
    assert reduce_dev(L, dev(g["x"])) == g["sum"]


def test_reduce_gpuarrays_golden(L):
    g = golden("gpuarrays_1024")
    a, p, s = dev(g["a"]), dev(g["p"]), dev(g["s"])
    assert reduce_dev(L, a) == pytest.approx(float(g["sum"]), rel=RTOL_REDUCE)
    assert reduce_dev(L, a, op="max", init=-np.inf) == g["maximum"]
    assert reduce_dev(L, a, op="min", init=np.inf) == g["minimum"]
    assert reduce_dev(L, a, f="abs2") == pytest.approx(float(g["sum_abs2"]), rel=RTOL_REDUCE)
    assert reduce_dev(L, p, op="mul", init=1.0) == pytest.approx(float(g["prod"]), rel=RTOL_REDUCE)
    assert reduce_dev(L, s, f="gt0") == g["count_s_gt0"]


@pytest.mark.parametrize("n", [1, 2, 3, 5, 17, 1000, 4096, 65537, (1 << 22) + 1])
@pytest.mark.parametrize("off", [0, 1, 2, 3])
def test_reduce_sum_sq_sizes(L, n, off):
    r = np.random.Generator(np.random.Philox(n + 31 * off))
    x_h = (r.random(n + off, dtype=np.float32) * 2 - 1).astype(np.float32)
    got = reduce_dev(L, dev(x_h), f="abs2", off=off)
    assert got == pytest.approx(oracle.sum_sq(x_h[off:]), rel=RTOL_REDUCE)


@pytest.mark.parametrize("f,op,init", [("identity", "add", 0.0), ("abs", "add", 0.0), ("identity", "max", -np.inf),
                                       ("identity", "min", np.inf), ("abs2", "add", 2.5), ("gt0", "add", 0.0),
                                       ("abs", "max", -np.inf)])
def test_reduce_ops_vs_oracle(L, f, op, init):
    r = np.random.Generator(np.random.Philox(99))
    x_h = (r.random(300_001, dtype=np.float32) * 2 - 1).astype(np.float32)
    got = reduce_dev(L, dev(x_h), f, op, init)
    want = oracle.mapreduce(x_h, f, op, init)
    if op in ("max", "min") or f == "gt0":
        assert got == want
    else:
        assert got == pytest.approx(want, rel=RTOL_REDUCE)


def test_reduce_empty_gives_init(L):
    out = torch.zeros(1, dtype=torch.float64, device="cuda")
    x = torch.zeros(4, device="cuda")
    assert L.mk_mapreduce_f32(out.data_ptr(), x.data_ptr(), 0, 0, 0, 3.5, stream()) == 0
    assert host(out)[0] == 3.5


def test_reduce_nan_propagates_in_max(L):
    x = dev(np.array([1, np.nan, 2, 3, 4], dtype=np.float32))
    assert np.isnan(reduce_dev(L, x, op="max", init=-np.inf))


def test_reduce_deterministic_and_reusable(L):
    r = np.random.Generator(np.random.Philox(5))
    x = dev((r.random(1 << 24, dtype=np.float32) * 2 - 1).astype(np.float32))
    vals = {reduce_dev(L, x, f="abs2") for _ in range(5)}
    assert len(vals) == 1


def test_reduce_two_streams(L):
    """Scratch is per (device, stream): interleaved reductions on two streams agree."""
    r = np.random.Generator(np.random.Philox(6))
    xh = (r.random(1 << 22, dtype=np.float32)).astype(np.float32)
    x = dev(xh)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    outs = [torch.empty(1, dtype=torch.float64, device="cuda") for _ in range(8)]
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        s = s1 if i % 2 == 0 else s2
        assert L.mk_mapreduce_f32(o.data_ptr(), x.data_ptr(), x.numel(), 1, 0, 0.0, s.cuda_stream) == 0
    torch.cuda.synchronize()
    vals = [o.item() for o in outs]
    assert len(set(vals)) == 1
    assert vals[0] == pytest.approx(oracle.sum_sq(xh), rel=RTOL_REDUCE)


def test_reduce_first_use_of_fresh_nonblocking_streams(L):
    """A stream's reduce scratch is zeroed in that stream's own order: first use
    of fresh non-blocking streams while the legacy default stream is busy."""
    rt = pytest.importorskip("cuda.bindings.runtime")
    r = np.random.Generator(np.random.Philox(13))
    xh = r.random(1 << 22, dtype=np.float32)
    x = dev(xh)
    want = oracle.sum_sq(xh)
    big = torch.empty(1 << 28, device="cuda")
    handles = []
    try:
        for _ in range(6):
            err, h = rt.cudaStreamCreateWithFlags(rt.cudaStreamNonBlocking)
            assert err == rt.cudaError_t.cudaSuccess
            handles.append(h)
        outs = [torch.full((1,), np.nan, dtype=torch.float64, device="cuda") for _ in handles]
        torch.cuda.synchronize()
        big.fill_(1.0)                        # queued on the legacy default stream
        big.mul_(2.0)
        for o, h in zip(outs, handles):
            assert L.mk_mapreduce_f32(o.data_ptr(), x.data_ptr(), x.numel(), 1, 0, 0.0, int(h)) == 0
        for h in handles:
            rt.cudaStreamSynchronize(h)
        torch.cuda.synchronize()
        for o in outs:
            assert o.item() == pytest.approx(want, rel=RTOL_REDUCE)
    finally:
        torch.cuda.synchronize()
        for h in handles:
            rt.cudaStreamDestroy(h)


# -------------------------------------------------------------- gather -----

def gather_dev(L, a_h, idx_h, off=0):
    a, idx = dev(a_h), dev(idx_h)
    n = idx_h.size - off
    c = torch.full((idx_h.size,), -7.0, device="cuda")
    assert L.mk_gather_f32(c.data_ptr() + 4 * off, a.data_ptr(), a_h.size, idx.data_ptr() + 4 * off, n,
                           stream()) == 0
    return host(c)[off:]


def test_gather_golden(L):
    g = golden("gather_perm_4096")
    np.testing.assert_array_equal(gather_dev(L, g["a"], g["idx"]), g["c"])
    assert poll(L) == 0


@pytest.mark.parametrize("n", [1, 3, 4, 7, 1000, 65536, (1 << 21) + 5])
@pytest.mark.parametrize("off", [0, 1])
def test_gather_random_vs_oracle(L, n, off):
    r = np.random.Generator(np.random.Philox(n + off))
    na = max(1, n // 2)
    a_h = r.random(na, dtype=np.float32)
    idx_h = r.integers(1, na + 1, size=n + off, dtype=np.int32)
    got = gather_dev(L, a_h, idx_h, off)
    want, rc = oracle.gather(a_h, idx_h[off:])
    assert rc == 0
    np.testing.assert_array_equal(got, want)
    assert poll(L) == 0


def test_gather_out_of_range_flags_fault(L):
    a_h = np.arange(1, 9, dtype=np.float32)
    idx_h = np.array([1, 0, 9, 8, -3, 2, 2, 2], dtype=np.int32)
    got = gather_dev(L, a_h, idx_h)
    want, rc = oracle.gather(a_h, idx_h)
    np.testing.assert_array_equal(got, want)
    assert rc == -5
    assert poll(L) == _lib.MK_ERR_DEVICE_FAULT
    assert b"gather index" in L.mk_last_error()
    assert poll(L) == 0  # the word is cleared by the poll


# ----------------------------------------------------------- histogram -----

def hist_dev(L, keys_h, nbins, start=None, off=0):
    keys = dev(keys_h)
    counts = dev(np.zeros(nbins, dtype=np.uint32) if start is None else start)
    assert L.mk_hist_u32(counts.data_ptr(), nbins, keys.data_ptr() + 4 * off, keys_h.size - off,
                         stream()) == 0
    return host(counts, np.uint32)


@pytest.mark.parametrize("name", ["hist_ka_4096_256", "hist_mod_4096_8", "hist_one_65536"])
def test_hist_golden(L, name):
    g = golden(name)
    np.testing.assert_array_equal(hist_dev(L, g["keys"], int(g["nbins"])), g["counts"])
    assert poll(L) == 0


@pytest.mark.parametrize("nbins", [1, 7, 256, 4096, 20000, 100_000])
@pytest.mark.parametrize("off", [0, 3])
def test_hist_random_vs_oracle(L, nbins, off):
    r = np.random.Generator(np.random.Philox(nbins + off))
    n = 300_007
    keys = r.integers(1, nbins + 1, size=n, dtype=np.int32)
    got = hist_dev(L, keys, nbins, off=off)
    np.testing.assert_array_equal(got, oracle.hist(keys[off:], nbins)[0])


def test_hist_zipf_vs_oracle(L):
    from cutilecpu_b200 import workloads
    keys = workloads.zipf_keys(1 << 22, 4096, 1.1, seed=3)
    np.testing.assert_array_equal(hist_dev(L, keys, 4096), oracle.hist(keys, 4096)[0])


def test_hist_zipf_full_config_vs_oracle(L):
    # BASELINE configs[3] at its full size: 2^26 Zipf(1.1) keys over 4096 bins,
    # exact counts (the reference pins its KA histogram exactly,
    # test/test_gpu_simt.jl:353-359)
    from cutilecpu_b200 import workloads
    keys = workloads.zipf_keys(1 << 26, 4096, 1.1, stream=30)
    got = hist_dev(L, keys, 4096)
    want = oracle.hist(keys, 4096)[0]
    np.testing.assert_array_equal(got, want)
    assert int(got.sum(dtype=np.int64)) == 1 << 26


def test_hist_accumulates_and_wraps(L):
    start = np.zeros(16, dtype=np.uint32)
    start[0] = 0xFFFFFFFF
    start[5] = 10
    keys = np.array([1, 1, 6, 16], dtype=np.int32)
    want = oracle.hist(keys, 16, start)[0]
    np.testing.assert_array_equal(hist_dev(L, keys, 16, start), want)


def test_hist_bad_keys_flag_fault(L):
    keys = np.array([0, 1, 2, 17, -1, 16] * 100, dtype=np.int32)
    got = hist_dev(L, keys, 16)
    np.testing.assert_array_equal(got, oracle.hist(keys, 16)[0])
    assert poll(L) == _lib.MK_ERR_DEVICE_FAULT
    assert b"histogram key" in L.mk_last_error()


def test_hist_empty_and_invalid(L):
    c = torch.zeros(4, dtype=torch.int32, device="cuda")
    assert L.mk_hist_u32(c.data_ptr(), 4, 0, 0, stream()) == 0
    assert L.mk_hist_u32(c.data_ptr(), 0, 0, 1, stream()) == _lib.MK_ERR_INVALID


# -------------------------------------------------- SIMT tiled matmul -----

@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (100, 70, 40), (16, 16, 15), (33, 1, 48)])
def test_tiled16_bitexact(L, M, N, K):
    r = np.random.Generator(np.random.Philox(M * N + K))
    A_h = np.asfortranarray(r.standard_normal((M, K), dtype=np.float32))
    B_h = np.asfortranarray(r.standard_normal((K, N), dtype=np.float32))
    A, B = dev(A_h.ravel(order="F")), dev(B_h.ravel(order="F"))
    Cd = torch.full((M * N,), -1.0, device="cuda")
    assert L.mk_matmul_tiled16_f32(Cd.data_ptr(), A.data_ptr(), B.data_ptr(), M, N, K, M, K, M, stream()) == 0
    got = host(Cd).reshape((M, N), order="F")
    np.testing.assert_array_equal(got, oracle.mm_tiled16_f32(A_h, B_h))


def test_tiled16_golden(L):
    g = golden("mm_tiled_256")
    A, B = dev(g["A"].ravel(order="F")), dev(g["B"].ravel(order="F"))
    Cd = torch.empty(256 * 256, device="cuda")
    assert L.mk_matmul_tiled16_f32(Cd.data_ptr(), A.data_ptr(), B.data_ptr(), 256, 256, 256, 256, 256, 256,
                                   stream()) == 0
    np.testing.assert_allclose(host(Cd).reshape((256, 256), order="F"), g["C"], rtol=1e-5)


# large sources: mixed valid/invalid indices into a 128-256 MiB `a`, and the
# full benchmark configuration (2^27 into 2^27)
@pytest.mark.parametrize("n,na", [((1 << 22) + 3, (1 << 25) + 7), (1 << 23, 1 << 26)])
def test_gather_large_vs_oracle(L, n, na):
    r = np.random.Generator(np.random.Philox(n ^ na))
    a_h = r.random(na, dtype=np.float32)
    idx_h = r.integers(1, na + 1, size=n, dtype=np.int32)
    idx_h[::100_003] = 0          # a few out-of-range indices
    idx_h[7::200_003] = na + 1
    got = gather_dev(L, a_h, idx_h)
    want, rc = oracle.gather(a_h, idx_h)
    assert rc == -5
    np.testing.assert_array_equal(got, want)
    assert poll(L) == _lib.MK_ERR_DEVICE_FAULT


def test_gather_full_size(L):
    from cutilecpu_b200 import workloads
    n = na = 1 << 27
    a_h = workloads.uniform01(na, stream=20)
    idx_h = workloads.indices1(n, na, stream=21)
    got = gather_dev(L, a_h, idx_h)
    np.testing.assert_array_equal(got, a_h[idx_h.astype(np.int64) - 1])
    assert poll(L) == 0


# the reference's other histogram forms: Int keys / Int bins (KA example,
# test/test_gpu_simt.jl:353-359) and Float32 bins (test/test_ka_cpu.jl:67-79)
def test_hist_ka_example_int64_keys_and_bins(L):
    import cutilecpu_b200 as mk
    g = golden("hist_ka_4096_256")
    keys = mk.MLIRArray(g["keys"].astype(np.int64))
    bins = mk.zeros(mk.MLIRCUDABackend(), "Int64", 256)
    mk.histogram(mk.MLIRCUDABackend(), (256,))(bins, keys, ndrange=4096)
    mk.synchronize(mk.MLIRCUDABackend())
    np.testing.assert_array_equal(mk.Array(bins), g["counts"].astype(np.int64))


@pytest.mark.parametrize("name", ["hist_mod_4096_8", "hist_one_65536"])
def test_hist_float32_bins(L, name):
    import cutilecpu_b200 as mk
    g = golden(name)
    bins = mk.zeros(mk.MLIRCUDABackend(), "Float32", int(g["nbins"]))
    mk.histogram(mk.MLIRCUDABackend(), 16)(bins, mk.MLIRArray(g["keys"]), ndrange=g["keys"].size)
    np.testing.assert_array_equal(mk.Array(bins), g["counts"].astype(np.float32))


@pytest.mark.parametrize("bin_type,np_t", [(1, np.int64), (2, np.float32)])
@pytest.mark.parametrize("key_type,key_t", [(0, np.int32), (1, np.int64)])
@pytest.mark.parametrize("nbins", [7, 4096, 100_000])
def test_hist_types_vs_oracle(L, bin_type, np_t, key_type, key_t, nbins):
    r = np.random.Generator(np.random.Philox(nbins + 3 * bin_type + key_type))
    keys = r.integers(1, nbins + 1, size=200_003, dtype=np.int32)
    keys[::50_001] = nbins + 2  # out of range
    kd = torch.from_numpy(keys.astype(key_t)).cuda()
    start = np.arange(nbins, dtype=np_t) % 5
    bd = torch.from_numpy(start.copy()).cuda()
    assert L.mk_hist(bd.data_ptr(), bin_type, nbins, kd.data_ptr() + kd.element_size(), key_type,
                     keys.size - 1, stream()) == 0
    want = oracle.hist(keys[1:], nbins)[0].astype(np_t) + start
    np.testing.assert_array_equal(host(bd), want)
    assert poll(L) == _lib.MK_ERR_DEVICE_FAULT


# ------------------------------------------------------- findmax/findmin -----

def findext_dev(L, x_h, find_max, off=0):
    xd = dev(np.concatenate([np.zeros(off, np.float32), x_h]))
    v = torch.empty(1, dtype=torch.float64, device="cuda")
    i = torch.empty(1, dtype=torch.int64, device="cuda")
    assert L.mk_findext_f32(v.data_ptr(), i.data_ptr(), xd.data_ptr() + 4 * off, x_h.size, int(find_max),
                            stream()) == 0, _lib.last_error()
    return host(v)[0], int(host(i)[0])


@pytest.mark.parametrize("n", [1, 3, 2000, 100_003, (1 << 24) + 1])
@pytest.mark.parametrize("find_max", [True, False])
@pytest.mark.parametrize("off", [0, 1])
def test_findext_vs_oracle(L, n, find_max, off):
    r = np.random.Generator(np.random.Philox(n))
    x = r.random(n, dtype=np.float32)
    x[n // 3] = x[n // 7] = x.max() if find_max else x.min()  # ties: the first index wins
    gv, gi = findext_dev(L, x, find_max, off)
    wv, wi = oracle.findext(x, find_max)
    assert (gv, gi) == (wv, wi)


def test_findext_nan_and_signed_zero(L):
    x = np.float32([1, 5, np.nan, 5, np.nan])
    assert findext_dev(L, x, True)[1] == 3 and findext_dev(L, x, False)[1] == 3
    z = np.float32([-0.0, 0.0, -0.0, 0.0])
    assert findext_dev(L, z, True)[1] == 2
    assert findext_dev(L, np.float32([0.0, -0.0]), False)[1] == 2
    assert L.mk_findext_f32(0, 0, 0, 0, 1, stream()) == _lib.MK_ERR_INVALID


def test_findext_large_ties_nan_zero(L):
    # the vectorised main loop keeps one candidate per vector lane: ties,
    # NaNs and signed zeros must still resolve to Julia's first-index answer
    n = (1 << 22) + 5
    x = np.full(n, 7.0, np.float32)
    for fm in (True, False):
        assert findext_dev(L, x, fm) == (7.0, 1)
    x[3_000_001] = 9.0
    x[2_000_003] = 9.0
    assert findext_dev(L, x, True) == (9.0, 2_000_004)
    x[1_500_002] = np.nan
    x[1_000_001] = np.nan
    for fm in (True, False):
        v, i = findext_dev(L, x, fm)
        assert np.isnan(v) and i == 1_000_002
    z = np.full(n, -0.0, np.float32)
    z[2_222_223] = 0.0
    z[3_333_334] = 0.0
    v, i = findext_dev(L, z, True)
    assert i == 2_222_224 and v == 0.0 and not np.signbit(v)
    assert findext_dev(L, z, False)[1] == 1
    z[:] = 0.0
    z[1_234_567] = -0.0
    assert findext_dev(L, z, False)[1] == 1_234_568
    assert findext_dev(L, z, True)[1] == 1


def test_reduce_large_max_min_nan_and_signed_zero(L):
    n = (1 << 22) + 7
    z = np.full(n, -0.0, np.float32)
    z[3_000_001] = 0.0
    got = reduce_dev(L, dev(z), op="max", init=-np.inf)
    assert got == 0.0 and not np.signbit(got)
    z[:] = 0.0
    z[2_000_003] = -0.0
    got = reduce_dev(L, dev(z), op="min", init=np.inf)
    assert got == 0.0 and np.signbit(got)
    r = np.random.Generator(np.random.Philox(12))
    x = r.standard_normal(n, dtype=np.float32)
    assert reduce_dev(L, dev(x), op="max", init=-np.inf) == float(x.max())
    assert reduce_dev(L, dev(x), op="min", init=np.inf) == float(x.min())
    assert reduce_dev(L, dev(x), f="abs", op="max", init=-np.inf) == float(np.abs(x).max())
    x[1_111_111] = np.nan
    assert np.isnan(reduce_dev(L, dev(x), op="max", init=-np.inf))
    assert np.isnan(reduce_dev(L, dev(x), op="min", init=np.inf))


def test_findmax_surface(L):
    import cutilecpu_b200 as mk
    r = np.random.Generator(np.random.Philox(2000))
    fx = r.random(2000, dtype=np.float32)
    a = mk.MLIRArray(fx)
    assert mk.findmax(a) == (float(fx.max()), int(np.argmax(fx)) + 1)
    assert mk.findmin(a) == (float(fx.min()), int(np.argmin(fx)) + 1)
    assert mk.argmax(a) == int(np.argmax(fx)) + 1 and mk.argmin(a) == int(np.argmin(fx)) + 1
    assert mk.extrema(a) == (float(fx.min()), float(fx.max()))
    s = mk.MLIRArray(fx - np.float32(0.5))
    assert mk.any_(mk.positive, s) and not mk.all_(mk.positive, s)


# ------------------------------------------------------ measurement probes -----

def _mix32(h: np.ndarray) -> np.ndarray:
    h = h.astype(np.uint64)
    h ^= h >> np.uint64(16)
    h = (h * np.uint64(0x85EBCA6B)) & np.uint64(0xFFFFFFFF)
    h ^= h >> np.uint64(13)
    h = (h * np.uint64(0xC2B2AE35)) & np.uint64(0xFFFFFFFF)
    h ^= h >> np.uint64(16)
    return h


@pytest.mark.parametrize("n,na", [(1000, 777), ((1 << 20) + 5, 1 << 20)])
def test_random_read_probe_reads_the_hashed_positions(L, n, na):
    # the XOR of all per-block words equals the XOR of a[hash(i) * na >> 32]
    r = np.random.Generator(np.random.Philox(na))
    a_h = r.random(na, dtype=np.float32)
    a = dev(a_h)
    sums = torch.zeros(torch.cuda.get_device_properties(0).multi_processor_count * 8, dtype=torch.int32,
                       device="cuda")
    assert L.mk_probe_random_read_f32(sums.data_ptr(), sums.numel(), a.data_ptr(), na, n, 11, stream()) == 0
    pos = (_mix32(np.arange(n, dtype=np.uint32) ^ np.uint32(11)) * np.uint64(na)) >> np.uint64(32)
    want = np.bitwise_xor.reduce(a_h.view(np.uint32)[pos])
    assert np.bitwise_xor.reduce(host(sums).view(np.uint32)) == want
    assert L.mk_probe_random_read_f32(sums.data_ptr(), 4, a.data_ptr(), na, n, 0, stream()) == _lib.MK_ERR_INVALID


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_vadd_probe_modes(L, mode):
    n = 1 << 20
    r = np.random.Generator(np.random.Philox(mode))
    a_h, b_h = r.random(n, dtype=np.float32), r.random(n, dtype=np.float32)
    a, b = dev(a_h), dev(b_h)
    c = torch.zeros(n, device="cuda")
    st = torch.tensor([-1, 0], dtype=torch.int64, device="cuda")
    assert L.mk_probe_vadd_f32(mode, c.data_ptr(), a.data_ptr(), b.data_ptr(), n, st.data_ptr(), stream()) == 0
    t = host(st).view(np.uint64)
    assert t[0] != np.uint64(0xFFFFFFFFFFFFFFFF) and t[1] >= t[0]  # both stamps written, in order
    if mode in (2, 3):
        np.testing.assert_array_equal(host(c), oracle.vadd(a_h, b_h))
