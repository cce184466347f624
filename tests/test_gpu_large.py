"""Inputs past 2^31 elements (8-17 GiB per tensor): every entry point takes
int64 lengths while the reference's device index is Int32
(src/lower.jl:991), so these cases check the 64-bit index arithmetic of each
kernel.  Inputs are made on the device with torch and checked exactly
(integer-valued data, or against torch's own fp32 elementwise results) or, for
the GEMM, against fp64 dot products at sampled entries."""
import numpy as np
import pytest
import torch

from cutilecpu_b200 import _lib

pytestmark = pytest.mark.gpu

BIG = (1 << 31) + 37  # elements; not a multiple of any tile or vector width


@pytest.fixture(scope="module")
def L(cuda):
    lib = _lib.lib()
    assert lib.mk_init(0) == 0, _lib.last_error()
    free, _ = torch.cuda.mem_get_info()
    if free < 40 << 30:
        pytest.skip(f"needs 40 GiB of free device memory, {free >> 30} GiB free")
    return lib


@pytest.fixture(autouse=True)
def _release():
    yield
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def ok(rc: int) -> None:
    assert rc == 0, _lib.last_error()


def scalar_f64(L, x, n, f, op, init=0.0) -> float:
    out = torch.empty(1, dtype=torch.float64, device="cuda")
    ok(L.mk_mapreduce_f32(out.data_ptr(), x.data_ptr(), n, f, op, init, stream()))
    return float(out.item())


def test_vadd_big(L):
    g = torch.Generator(device="cuda").manual_seed(1)
    a = torch.rand(BIG, device="cuda", generator=g)
    b = torch.rand(BIG, device="cuda", generator=g)
    c = torch.empty_like(a)
    ok(L.mk_vadd_f32(c.data_ptr(), a.data_ptr(), b.data_ptr(), BIG, stream()))
    torch.add(a, b, out=a)
    assert torch.equal(c, a)


def test_mapreduce_big(L):
    x = torch.ones(BIG, device="cuda")
    assert scalar_f64(L, x, BIG, 0, 0) == float(BIG)          # sum: exact in fp64
    x.fill_(2.0)
    assert scalar_f64(L, x, BIG, 1, 0) == 4.0 * BIG           # sum(abs2)
    x[BIG - 1] = 7.5
    assert scalar_f64(L, x, BIG, 0, 1, -np.inf) == 7.5        # maximum, last element
    x[BIG - 1] = 2.0
    x[(1 << 31) + 1] = -3.0
    assert scalar_f64(L, x, BIG, 0, 2, np.inf) == -3.0        # minimum past 2^31


@pytest.mark.parametrize("find_max", [1, 0])
def test_findext_big(L, find_max):
    x = torch.zeros(BIG, device="cuda")
    at = (1 << 31) + 10
    x[at] = 5.0 if find_max else -5.0
    x[at + 7] = x[at]  # a later tie: the first index wins
    val = torch.empty(1, dtype=torch.float64, device="cuda")
    idx = torch.empty(1, dtype=torch.int64, device="cuda")
    ok(L.mk_findext_f32(val.data_ptr(), idx.data_ptr(), x.data_ptr(), BIG, find_max, stream()))
    assert float(val.item()) == (5.0 if find_max else -5.0)
    assert int(idx.item()) == at + 1


def test_accumulate_big(L):
    x = torch.zeros(BIG, device="cuda")
    marks = [5, (1 << 31) - 1, (1 << 31) + 3, BIG - 1]
    for p in marks:
        x[p] = 1.0
    out = torch.empty_like(x)
    ok(L.mk_accumulate_f32(out.data_ptr(), x.data_ptr(), BIG, 0, 0.0, 0, stream()))
    want = torch.zeros_like(x)
    for p in marks:
        want[p:] += 1.0
    assert torch.equal(out, want)
    del want
    # exclusive: out[i] = sum(x[0:i])
    ok(L.mk_accumulate_f32(out.data_ptr(), x.data_ptr(), BIG, 0, 0.0, 1, stream()))
    for k, p in enumerate(marks):
        assert float(out[p].item()) == k          # x[p] itself not yet included
        if p + 1 < BIG:
            assert float(out[p + 1].item()) == k + 1
    assert float(out[0].item()) == 0.0


def test_gather_big(L):
    na = (1 << 20) + 3
    g = torch.Generator(device="cuda").manual_seed(2)
    a = torch.rand(na, device="cuda", generator=g)
    idx = torch.randint(1, na + 1, (BIG,), dtype=torch.int32, device="cuda", generator=g)
    c = torch.empty(BIG, device="cuda")
    ok(L.mk_gather_f32(c.data_ptr(), a.data_ptr(), na, idx.data_ptr(), BIG, stream()))
    assert L.mk_error_poll(stream()) == 0
    step = 1 << 28
    for s in range(0, BIG, step):
        e = min(BIG, s + step)
        assert torch.equal(c[s:e], a[(idx[s:e] - 1).long()])


def test_hist_big(L):
    nbins = 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    keys = torch.randint(1, nbins + 1, (BIG,), dtype=torch.int32, device="cuda", generator=g)
    counts = torch.zeros(nbins, dtype=torch.int32, device="cuda")
    ok(L.mk_hist_u32(counts.data_ptr(), nbins, keys.data_ptr(), BIG, stream()))
    assert L.mk_error_poll(stream()) == 0
    want = torch.zeros(nbins + 1, dtype=torch.int64, device="cuda")
    step = 1 << 28
    for s in range(0, BIG, step):
        want += torch.bincount(keys[s:s + step], minlength=nbins + 1)
    assert torch.equal(counts.long(), want[1:])
    assert int(want.sum().item()) == BIG


@pytest.mark.parametrize("dims", [1, 2])
def test_mapreduce_dim_big(L, dims):
    rows, cols = 1 << 16, (1 << 15) + 1   # column-major rows x cols, 2^31 + 2^16 elements
    x = torch.ones(rows * cols, device="cuda")
    if dims == 1:   # sum over rows: pre=1, len=rows, post=cols
        out = torch.empty(cols, device="cuda")
        ok(L.mk_mapreduce_dim_f32(out.data_ptr(), x.data_ptr(), 1, rows, cols, 0, 0, 0.0, stream()))
        assert torch.equal(out, torch.full_like(out, float(rows)))
    else:           # sum over columns: pre=rows, len=cols, post=1
        out = torch.empty(rows, device="cuda")
        ok(L.mk_mapreduce_dim_f32(out.data_ptr(), x.data_ptr(), rows, cols, 1, 0, 0, 0.0, stream()))
        assert torch.equal(out, torch.full_like(out, float(cols)))


def test_sgemm_big_c(L):
    # C has 65636 x 32801 = 2.15e9 entries; ragged in both M and N
    M, N, K = (1 << 16) + 100, (1 << 15) + 33, 16
    g = torch.Generator(device="cuda").manual_seed(4)
    A = torch.randn(K, M, device="cuda", generator=g)   # column-major M x K = row-major K x M
    B = torch.randn(N, K, device="cuda", generator=g)   # column-major K x N
    Cm = torch.empty(N, M, device="cuda")               # column-major M x N
    ok(L.mk_sgemm_3xtf32(Cm.data_ptr(), A.data_ptr(), B.data_ptr(), M, N, K, M, K, M, stream()))
    rng = np.random.default_rng(5)
    ii = np.concatenate([rng.integers(0, M, 64), [0, M - 1, M - 1]])
    jj = np.concatenate([rng.integers(0, N, 64), [0, N - 1, 0]])
    Ah, Bh = A.double().cpu().numpy(), B.double().cpu().numpy()
    want = np.einsum("kp,pk->p", Ah[:, ii], Bh[jj, :])
    got = Cm[torch.as_tensor(jj), torch.as_tensor(ii)].double().cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
    # the last column block, whole, past element 2^31 of C
    tail = Cm[N - 1].double().cpu().numpy()
    np.testing.assert_allclose(tail, Ah.T @ Bh[N - 1], rtol=1e-5, atol=1e-5)
