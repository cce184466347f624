"""The allocation-free reduction entry point, mk_mapreduce_f32_noalloc.

It serves callers that cannot let a library call cudaMalloc: hosts whose
device memory belongs to their own pool allocator (CUDA.jl's, torch's caching
allocator) or to a fixed budget set at start-up.  Its scratch is a static
device array inside libkernels.so.  This file is named to be collected last,
so a run that stops at the first failure has already run every other test; it
also passes when run alone in a fresh process.
"""
import numpy as np
import pytest
import torch

from cutilecpu_b200 import _lib

pytestmark = pytest.mark.gpu

RTOL = 1e-5  # the reductions' tolerance against fp64


def _call(fn, x: torch.Tensor, f: str, op: str, init: float) -> float:
    out = torch.full((1,), np.nan, dtype=torch.float64, device="cuda")
    rc = fn(out.data_ptr(), x.data_ptr(), x.numel(), _lib.MK_F[f], _lib.MK_OP[op], init,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    return out.item()


@pytest.mark.parametrize("n,f,op,init", [
    ((1 << 24) + 3, "abs2", "add", 0.0),
    (1 << 28, "abs2", "add", 0.0),
    (1000, "identity", "max", -np.inf),
    (65537, "identity", "add", 1.5),
])
def test_noalloc_matches_allocating_entry_point_twice(cuda, n, f, op, init):
    L = _lib.lib()
    r = np.random.Generator(np.random.Philox(n))
    x = torch.from_numpy((r.random(n, dtype=np.float32) * 2 - 1).astype(np.float32)).to(cuda)
    want = _call(L.mk_mapreduce_f32, x, f, op, init)
    # two calls in a row: the second starts from what the first left in the array
    first = _call(L.mk_mapreduce_f32_noalloc, x, f, op, init)
    second = _call(L.mk_mapreduce_f32_noalloc, x, f, op, init)
    # same kernel, same grid, same fold order: the results agree bit for bit
    assert first == second == want
    xs = x.cpu().numpy().astype(np.float64)
    ref = {"abs2": xs * xs, "identity": xs}[f]
    exact = init + ref.sum() if op == "add" else max(init, ref.max())
    assert want == pytest.approx(exact, rel=RTOL)


def test_noalloc_rejects_bad_arguments(cuda):
    L = _lib.lib()
    out = torch.zeros(1, dtype=torch.float64, device=cuda)
    x = torch.zeros(8, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    assert L.mk_mapreduce_f32_noalloc(out.data_ptr(), x.data_ptr(), -1, 0, 0, 0.0, s) == _lib.MK_ERR_INVALID
    assert L.mk_mapreduce_f32_noalloc(out.data_ptr(), x.data_ptr(), 8, 9, 0, 0.0, s) == _lib.MK_ERR_INVALID
    assert L.mk_mapreduce_f32_noalloc(out.data_ptr(), x.data_ptr() + 2, 4, 0, 0, 0.0, s) == _lib.MK_ERR_INVALID
    assert b"4-byte aligned" in L.mk_last_error()
