"""Device and pinned memory pools (mk_pool_* / mk_host_*): pool-backed
MLIRArrays run every kernel zero-copy, freed blocks are reused, and pinned
host arrays honour the aligned_array contract (src/allocator.jl:32-71)."""
import gc
import operator

import numpy as np
import pytest
import torch

import cutilecpu_b200 as mk
import oracle

pytestmark = pytest.mark.gpu


def test_pool_array_is_zero_copy_and_runs_kernels(cuda):
    be = mk.MLIRCUDABackend()
    r = np.random.Generator(np.random.Philox(1))
    a_h, b_h = r.random(10_001, dtype=np.float32), r.random(10_001, dtype=np.float32)
    a, b, c = (mk.pool_allocate("Float32", 10_001) for _ in range(3))
    mk.copyto(be, a, a_h)
    mk.copyto(be, b, b_h)
    mk.vadd(be, 256)(c, a, b, ndrange=10_001)
    mk.synchronize(be)
    np.testing.assert_array_equal(mk.Array(c), oracle.vadd(a_h, b_h))
    assert mk.sum(mk.abs2, a) == pytest.approx(oracle.sum_sq(a_h), rel=1e-5)
    keys = mk.pool_allocate("Int32", 5000)
    mk.copyto(be, keys, r.integers(1, 33, 5000, dtype=np.int32))
    counts = mk.pool_allocate("UInt32", 32)
    counts.storage.zero_()
    mk.histogram(be)(counts, keys, ndrange=5000)
    assert int(mk.Array(counts).sum()) == 5000


def test_pool_reuses_freed_blocks(cuda):
    torch.cuda.synchronize()
    x = mk.pool_allocate("Float32", 1 << 24)
    used = mk.pool_stats()["device_used"]
    assert used >= 4 << 24
    ptr = x.pointer()
    del x
    gc.collect()
    torch.cuda.synchronize()
    reserved = mk.pool_stats()["device_reserved"]
    y = mk.pool_allocate("Float32", 1 << 24)
    assert mk.pool_stats()["device_reserved"] == reserved   # served from the cache
    assert y.pointer() == ptr


def test_aligned_pinned_array(cuda):
    h = mk.aligned_array("Float32", (64, 3), alignment=128)
    assert h.shape == (64, 3) and mk.pointer_aligned(h, 128)
    t = torch.from_numpy(h.reshape(-1, order="F"))
    assert t.is_pinned()
    h[:] = 2.5
    d = mk.pool_allocate("Float32", (64, 3))
    mk.copyto(mk.MLIRCUDABackend(), d, t)
    assert mk.sum(d) == pytest.approx(2.5 * 192)
    stats = mk.pool_stats()
    assert stats["pinned_live"] >= 4096


def test_pool_trim(cuda):
    mk.pool_trim()
    s = mk.pool_stats()
    assert s["pinned_cached"] == 0
