"""The KernelAbstractions surface on the GPU, mirroring the reference's own
tests: test/test_gpu_simt.jl (vadd, masked tails, histogram, tiled matmul),
test/test_downstream_ka.jl (AK.reduce/sum/mapreduce/count, views) and
test/test_gpuarrays.jl (Base reductions, copyto!)."""
import operator

import numpy as np
import pytest

import cutilecpu_b200 as mk
import oracle
from conftest import golden

pytestmark = pytest.mark.gpu


@pytest.fixture
def be(cuda):
    return mk.MLIRCUDABackend()


def test_vadd_via_get_backend(be):
    # test/test_gpu_simt.jl:322-328
    g = golden("vadd_4096")
    a1, b1 = mk.MLIRArray(g["a"]), mk.MLIRArray(g["b"])
    c1 = mk.zeros(be, "Float32", 4096)
    backend = mk.get_backend(a1)
    assert isinstance(backend, mk.MLIRCUDABackend)
    mk.vadd(backend, 256)(c1, a1, b1, ndrange=4096)
    mk.synchronize(backend)
    np.testing.assert_array_equal(mk.Array(c1), g["c"])


@pytest.mark.parametrize("name", ["vadd_tail_1000", "vadd_tail_257"])
def test_vadd_masked_tail(be, name):
    # test/test_gpu_simt.jl:441-446: ndrange not a multiple of the workgroup
    g = golden(name)
    n = g["a"].size
    c = mk.zeros(be, "Float32", n)
    mk.vadd(be, 256)(c, mk.MLIRArray(g["a"]), mk.MLIRArray(g["b"]), ndrange=n)
    np.testing.assert_array_equal(mk.Array(c), g["c"])


def test_histogram_ka(be):
    # test/test_gpu_simt.jl:353-359 with UInt32 bins
    g = golden("hist_ka_4096_256")
    out = mk.zeros(be, "UInt32", 256)
    mk.histogram(be, (256,))(out, mk.MLIRArray(g["keys"]), ndrange=4096)
    np.testing.assert_array_equal(mk.Array(out), g["counts"])


@pytest.mark.parametrize("nm", [256, 512])
def test_tiled_matmul(be, nm):
    # test/test_gpu_simt.jl:407-413 (reference bar rtol 1e-2; here rel Frobenius 1e-5)
    r = np.random.Generator(np.random.Philox(nm))
    A, B = (np.asfortranarray(r.random((nm, nm), dtype=np.float32)) for _ in range(2))
    Cm = mk.zeros(be, "Float32", (nm, nm))
    mk.mm_tiled(be, (16, 16))(Cm, mk.MLIRArray(A), mk.MLIRArray(B), ndrange=(nm, nm))
    C64 = oracle.matmul_f64(A, B)
    assert np.linalg.norm(mk.Array(Cm) - C64) / np.linalg.norm(C64) <= 1e-5
    Cs = mk.zeros(be, "Float32", (nm, nm))
    mk.mm_tiled_simt(be, (16, 16))(Cs, mk.MLIRArray(A), mk.MLIRArray(B), ndrange=(nm, nm))
    np.testing.assert_array_equal(mk.Array(Cs), oracle.mm_tiled16_f32(A, B))


def test_ak_reductions(be):
    # test/test_downstream_ka.jl:26-35
    src = mk.MLIRArray(np.arange(1, 1025, dtype=np.float32))
    assert mk.reduce(operator.add, src, init=0.0) == 524800.0
    assert mk.sum(src) == 524800.0
    assert mk.mapreduce(mk.identity, operator.add, src, init=0.0) == 524800.0
    assert mk.count(mk.positive, src) == 1024
    assert mk.maximum(src) == 1024.0 and mk.minimum(src) == 1.0


def test_gpuarrays_reductions(be):
    # test/test_gpuarrays.jl:83-91
    g = golden("gpuarrays_1024")
    a, p = mk.MLIRArray(g["a"]), mk.MLIRArray(g["p"])
    assert mk.sum(a) == pytest.approx(float(g["sum"]), rel=1e-5)
    assert mk.maximum(a) == g["maximum"] and mk.minimum(a) == g["minimum"]
    assert mk.sum(mk.abs2, a) == pytest.approx(float(g["sum_abs2"]), rel=1e-5)
    assert mk.prod(p) == pytest.approx(float(g["prod"]), rel=1e-5)
    assert mk.count(mk.positive, mk.MLIRArray(g["s"])) == g["count_s_gt0"]
    # sum(x.^2) as a fused broadcast: mapreducedim! into a 1-element result
    R = mk.zeros(be, "Float32", 1)
    mk.mapreducedim(mk.identity, operator.add, R, mk.Broadcasted(mk.abs2, a))
    assert float(mk.Array(R)[0]) == pytest.approx(float(g["sum_abs2"]), rel=1e-6)


def test_views_and_copyto(be):
    # test/test_downstream_ka.jl:60-66 (contiguous views share storage)
    seq = mk.MLIRArray(np.arange(1, 1025, dtype=np.float32))
    np.testing.assert_array_equal(mk.Array(seq.view(3, 7)), np.float32([3, 4, 5, 6, 7]))
    v = seq.view(2, 1001)  # an odd offset: kernels take their scalar paths
    out = mk.zeros(be, "Float32", 1000)
    mk.vadd(be, 256)(out, v, v, ndrange=1000)
    np.testing.assert_array_equal(mk.Array(out), 2 * np.arange(2, 1002, dtype=np.float32))
    assert mk.sum(v) == float(np.arange(2, 1002).sum())
    c = mk.zeros(be, "Float32", 1024)
    mk.copyto(be, c, seq)
    np.testing.assert_array_equal(mk.Array(c), mk.Array(seq))


def test_out_of_range_gather_raises_kernel_exception(be):
    # device throw -> KernelException at synchronize (test/test_gpu_simt.jl:497-565)
    a = mk.MLIRArray(np.arange(1, 9, dtype=np.float32))
    idx = mk.MLIRArray(np.array([1, 2, 9, 3], dtype=np.int32))
    c = mk.zeros(be, "Float32", 4)
    mk.gather(be, 256)(c, a, idx, ndrange=4)
    with pytest.raises(mk.KernelException, match="gather index"):
        mk.synchronize(be)
    mk.synchronize(be)  # cleared
    np.testing.assert_array_equal(mk.Array(c), np.float32([1, 2, 0, 3]))


def test_launch_errors_on_gpu(be):
    c = mk.zeros(be, "Float32", 8)
    with pytest.raises(mk.MLIRKernelsError, match="element type"):
        mk.vadd(be, 8)(c, mk.MLIRArray(np.ones(8, np.int32)), c, ndrange=8)
    with pytest.raises(mk.MLIRKernelsError, match="ndrange needs"):
        mk.vadd(be, 8)(c, c, c, ndrange=16)


@pytest.mark.skipif(__import__("torch").cuda.device_count() < 2, reason="needs two GPUs")
def test_launch_follows_the_arrays_device(be):
    import torch
    with torch.cuda.device(1):
        a = mk.MLIRArray(np.arange(8, dtype=np.float32))
        c = mk.zeros(be, "Float32", 8)
    assert a.device == 1 and torch.cuda.current_device() == 0
    mk.vadd(be, 8)(c, a, a, ndrange=8)  # launched on device 1, its current stream
    assert mk.sum(a) == 28.0
    np.testing.assert_array_equal(mk.Array(c), 2 * np.arange(8, dtype=np.float32))
    with pytest.raises(mk.MLIRKernelsError, match="different devices"):
        mk.vadd(be, 8)(c, a, mk.zeros(be, "Float32", 8), ndrange=8)


def test_threads_share_the_library(be):
    """Launches from several host threads (per-device state is created once,
    scratch is per stream)."""
    import threading
    import torch
    r = np.random.Generator(np.random.Philox(12))
    xs = [r.random(1 << 20, dtype=np.float32) for _ in range(4)]
    res = [None] * 4

    def work(i):
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            x = mk.MLIRArray(xs[i])
            res[i] = mk.sum(mk.abs2, x)

    ts = [threading.Thread(target=work, args=(i,)) for i in range(4)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    for i in range(4):
        assert res[i] == pytest.approx(oracle.sum_sq(xs[i]), rel=1e-5)


def test_ak_map_and_broadcasts(be):
    # AK.map!(x -> 2f0 * x, dst, src) (test/test_downstream_ka.jl:18-20);
    # 2f0 .* a and a .+ b (test/test_gpuarrays.jl:31-32): bit-exact
    r = np.random.Generator(np.random.Philox(31))
    src_h, b_h = r.random(1027, dtype=np.float32), r.random(1027, dtype=np.float32)
    src, b = mk.MLIRArray(src_h), mk.MLIRArray(b_h)
    dst = mk.zeros(be, "Float32", 1027)
    mk.map_(mk.Scale(2.0), dst, src)
    np.testing.assert_array_equal(mk.Array(dst), np.float32(2) * src_h)
    mk.axpby(dst, 1.0, src, 1.0, b)
    np.testing.assert_array_equal(mk.Array(dst), src_h + b_h)
    mk.axpby(dst, 3.0, src, -0.5, b)
    np.testing.assert_array_equal(mk.Array(dst), np.float32(3) * src_h + np.float32(-0.5) * b_h)
    v = src.view(2, 1001)  # misaligned view: scalar path
    out = mk.zeros(be, "Float32", 1000)
    mk.axpby(out, 2.0, v)
    np.testing.assert_array_equal(mk.Array(out), np.float32(2) * src_h[1:1001])
    with pytest.raises(mk.MLIRKernelsError, match="no kernel"):
        mk.map_(lambda x: x + 1, dst, src)
