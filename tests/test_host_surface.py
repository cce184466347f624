"""Host-side logic of the KA launch surface that needs no GPU: launch-geometry
resolution and its errors (ext/MLIRCUDAExt.jl:477-538), launch_config
(:154-161), sharding helpers, and the reduce selector mapping."""
import operator

import pytest

import cutilecpu_b200 as mk
from cutilecpu_b200 import _lib, distributed
from cutilecpu_b200.reductions import _f_name, _op_name


def test_get_backend_rejects_non_mlirarray():
    with pytest.raises(TypeError):
        mk.get_backend([1, 2, 3])


def test_default_workgroup_is_min_256_ndrange():
    k = mk.vadd(mk.MLIRCUDABackend())
    assert k.launch_setup(ndrange=4096) == ((4096,), (256,))
    assert k.launch_setup(ndrange=100) == ((100,), (100,))


def test_static_workgroup_conflict_errors():
    k = mk.vadd(mk.MLIRCUDABackend(), 256)
    assert k.launch_setup(ndrange=1000) == ((1000,), (256,))
    with pytest.raises(_lib.MLIRKernelsError, match="conflicts with the kernel's static workgroupsize"):
        k.launch_setup(ndrange=1000, workgroupsize=512)


def test_missing_ndrange_errors():
    with pytest.raises(_lib.MLIRKernelsError, match="ndrange must be specified"):
        mk.vadd(mk.MLIRCUDABackend(), 256).launch_setup()
    assert mk.vadd(mk.MLIRCUDABackend(), 256, 512).launch_setup() == ((512,), (256,))


def test_rank_mismatch_errors():
    with pytest.raises(_lib.MLIRKernelsError, match="same number of dimensions"):
        mk.vadd(mk.MLIRCUDABackend(), (16, 16)).launch_setup(ndrange=1024)
    with pytest.raises(_lib.MLIRKernelsError, match="indexes a 1-D ndrange"):
        mk.vadd(mk.MLIRCUDABackend(), (16, 16)).launch_setup(ndrange=(64, 64))


def test_matmul_requires_16x16_workgroup():
    k = mk.mm_tiled_simt(mk.MLIRCUDABackend(), (16, 16))
    assert k.launch_setup(ndrange=(256, 256)) == ((256, 256), (16, 16))
    with pytest.raises(_lib.MLIRKernelsError, match="written for workgroupsize"):
        mk.mm_tiled_simt(mk.MLIRCUDABackend(), (8, 8)).launch_setup(ndrange=(256, 256))


def test_workgroup_too_large():
    with pytest.raises(_lib.MLIRKernelsError, match="invalid workgroupsize"):
        mk.vadd(mk.MLIRCUDABackend(), 2048).launch_setup(ndrange=4096)


def test_launch_config_defaults():
    assert mk.launch_config(None, 1000, None) == ((1000,), (256,), None, None)
    assert mk.launch_config(None, (8, 4), None) == ((8, 4), (8, 1), None, None)
    assert mk.launch_config(None, 10, 2) == ((10,), (2,), None, None)


def test_backend_requires_mlircudabackend():
    with pytest.raises(TypeError):
        mk.vadd("cpu", 256)


def test_reduce_selectors():
    assert _f_name(mk.identity) == "identity" and _f_name(mk.abs2) == "abs2"
    assert _op_name(operator.add) == "add" and _op_name(max) == "max"
    with pytest.raises(_lib.MLIRKernelsError, match="no kernel for f"):
        _f_name(lambda x: x + 1)
    with pytest.raises(_lib.MLIRKernelsError, match="no kernel for op"):
        _op_name(operator.sub)


@pytest.mark.parametrize("n,w", [(0, 1), (1, 1), (10, 3), (2**28, 8), (7, 8), (1 << 20, 3)])
def test_shard_range_partitions(n, w):
    spans = [distributed.shard_range(n, r, w) for r in range(w)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a, b), (c, _) in zip(spans, spans[1:]):
        assert b == c
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_row_block_aligned():
    spans = [distributed.row_block(8192, r, 8) for r in range(8)]
    assert spans == [(r * 1024, (r + 1) * 1024) for r in range(8)]
    spans = [distributed.row_block(1000, r, 3) for r in range(3)]
    assert spans[0][0] == 0 and spans[-1][1] == 1000
    assert all(lo % 128 == 0 for lo, _ in spans)


def test_world_without_process_group():
    assert distributed.world() == (0, 1)


@pytest.mark.parametrize("bad,msg", [(0, "positive"), (-8, "positive"), (24, "power of two"), (4, "multiple of sizeof")])
def test_aligned_array_rejects_bad_alignment(bad, msg):
    # src/allocator.jl:52-61 checks, raised before any allocation
    with pytest.raises(ValueError, match=msg):
        mk.aligned_array("Float32", 16, alignment=bad)


def test_c_abi_alignment_checks_without_gpu():
    import ctypes as C
    L = _lib.lib()
    p = C.c_void_p()
    assert L.mk_host_alloc_aligned(C.byref(p), 64, 24) == _lib.MK_ERR_INVALID
    assert b"power of two" in L.mk_last_error()
    assert L.mk_host_alloc_aligned(C.byref(p), 64, 0) == _lib.MK_ERR_INVALID
