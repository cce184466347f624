"""Single-dimension reductions (mk_mapreduce_dim_f32) against the fp64
oracle: the dims form of GPUArrays.mapreducedim! (test/test_gpuarrays.jl:98-107
reduces a 32x17 matrix over dims 1 and 2 and an 8x4x3 array over each dim).
Bar: rel 1e-5 for sums/products (fp64 accumulation, one Float32 rounding),
exact for max/min."""
import operator

import numpy as np
import pytest
import torch

import cutilecpu_b200 as mk
import oracle
from cutilecpu_b200 import _lib

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def run_dim(x: np.ndarray, dim: int, f="identity", op="add", init=0.0) -> np.ndarray:
    xf = np.asfortranarray(x, dtype=np.float32)
    shape = xf.shape
    pre = int(np.prod(shape[:dim - 1])); ln = shape[dim - 1]; post = int(np.prod(shape[dim:]))
    xd = torch.from_numpy(xf.ravel(order="F").copy()).cuda()
    out = torch.full((pre * post,), np.nan, dtype=torch.float32, device="cuda")
    rc = _lib.lib().mk_mapreduce_dim_f32(out.data_ptr(), xd.data_ptr(), pre, ln, post, _lib.MK_F[f],
                                         _lib.MK_OP[op], float(init), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    return out.cpu().numpy().reshape(shape[:dim - 1] + (1,) + shape[dim:], order="F")


def check(got, want, exact):
    if exact:
        np.testing.assert_array_equal(got, want.astype(np.float32))
    else:
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=1e-30)


@pytest.mark.parametrize("shape", [(32, 17), (8, 4, 3), (1, 5), (5, 1), (4096, 300), (300, 4096),
                                   (1 << 22, 2), (2, 1 << 22), (7, 100_003, 3), (4097, 33), (1023, 257)])
@pytest.mark.parametrize("f,op,init", [("identity", "add", 0.0), ("abs2", "add", 0.0),
                                       ("identity", "max", -np.inf), ("identity", "min", np.inf)])
def test_dims_vs_oracle(cuda, shape, f, op, init):
    r = np.random.Generator(np.random.Philox(sum(shape)))
    x = np.asfortranarray(r.random(shape, dtype=np.float32))
    for dim in range(1, len(shape) + 1):
        got = run_dim(x, dim, f, op, init)
        check(got, oracle.mapreduce_dim(x, dim, f, op, init), exact=op in ("max", "min"))


def test_dims_prod_and_count(cuda):
    r = np.random.Generator(np.random.Philox(3))
    p = np.asfortranarray((r.random((64, 9), dtype=np.float32) + 0.5).astype(np.float32))
    check(run_dim(p, 1, "identity", "mul", 1.0), oracle.mapreduce_dim(p, 1, "identity", "mul", 1.0), False)
    s = np.asfortranarray((r.random((100, 50), dtype=np.float32) - 0.5).astype(np.float32))
    check(run_dim(s, 2, "gt0", "add"), oracle.mapreduce_dim(s, 2, "gt0", "add"), True)


def test_dims_empty_reduced_dimension_gives_init(cuda):
    x = np.zeros((4, 0, 3), dtype=np.float32)
    got = run_dim(x, 2, "identity", "add", 2.5)
    assert got.shape == (4, 1, 3) and (got == 2.5).all()


def test_surface_sum_dims_and_mapreducedim(cuda):
    r = np.random.Generator(np.random.Philox(4))
    m = np.asfortranarray(r.random((32, 17), dtype=np.float32))
    M = mk.MLIRArray(m)
    np.testing.assert_allclose(mk.Array(mk.sum(M, dims=1)), m.astype(np.float64).sum(0, keepdims=True), rtol=RTOL)
    np.testing.assert_allclose(mk.Array(mk.sum(mk.abs2, M, dims=2)),
                               (m.astype(np.float64) ** 2).sum(1, keepdims=True), rtol=RTOL)
    np.testing.assert_array_equal(mk.Array(mk.maximum(M, dims=2)), m.max(1, keepdims=True))
    np.testing.assert_array_equal(mk.Array(mk.minimum(M, dims=1)), m.min(0, keepdims=True))
    R = mk.zeros(mk.get_backend(M), "Float32", (1, 17))
    mk.mapreducedim(mk.identity, operator.add, R, M)
    np.testing.assert_allclose(mk.Array(R), m.astype(np.float64).sum(0, keepdims=True), rtol=RTOL)
    with pytest.raises(mk.MLIRKernelsError, match="single-dim"):
        mk.mapreducedim(mk.identity, operator.add, mk.zeros(mk.get_backend(M), "Float32", (1, 1, 3)),
                        mk.MLIRArray(np.ones((2, 2, 3), dtype=np.float32)))
