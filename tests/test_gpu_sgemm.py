"""Parity of the tcgen05 3xTF32 GEMM (mk_sgemm_3xtf32) with the fp64 oracle.

Bar: relative Frobenius error <= 1e-5 against an fp64 product with the
reference tiled kernel's K rule (only 16*floor(K/16) terms,
examples/tiled_matmul.jl:34); at the full 8192^3 size through size-independent
properties (C*v == A*(B*v) in fp64, and sampled entries)."""
import numpy as np
import pytest
import torch

import oracle
from conftest import golden
from cutilecpu_b200 import _lib

pytestmark = pytest.mark.gpu

RTOL_FRO = 1e-5


def frob_rel(got, want):
    return float(np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a.ravel(order="F"))).to("cuda")


def sgemm(A_h, B_h, lda=None, ldb=None, ldc=None):
    M, K = A_h.shape
    N = B_h.shape[1]
    L = _lib.lib()
    lda = lda or M
    ldb = ldb or K
    ldc = ldc or M
    Ap = np.zeros((lda, K), dtype=np.float32, order="F"); Ap[:M] = A_h
    Bp = np.zeros((ldb, N), dtype=np.float32, order="F"); Bp[:K] = B_h
    A, B = dev(Ap), dev(Bp)
    Cd = torch.full((ldc * N,), -3.0, device="cuda")
    rc = L.mk_sgemm_3xtf32(Cd.data_ptr(), A.data_ptr(), B.data_ptr(), M, N, K, lda, ldb, ldc,
                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    assert L.mk_error_poll(torch.cuda.current_stream().cuda_stream) == 0, _lib.last_error()
    Cf = Cd.cpu().numpy().reshape((ldc, N), order="F")
    assert (Cf[M:] == -3.0).all(), "wrote outside C"
    return Cf[:M]


@pytest.mark.parametrize("M,N,K", [(128, 256, 16), (128, 256, 256), (256, 512, 1024), (100, 70, 40),
                                   (1, 1, 16), (300, 500, 1000), (129, 257, 33), (640, 384, 4096)])
def test_sgemm_vs_fp64(cuda, M, N, K):
    r = np.random.Generator(np.random.Philox(M * 7 + N * 3 + K))
    A = np.asfortranarray(r.standard_normal((M, K), dtype=np.float32))
    B = np.asfortranarray(r.standard_normal((K, N), dtype=np.float32))
    got = sgemm(A, B)
    want = oracle.matmul_f64(A, B)
    assert frob_rel(got, want) <= RTOL_FRO


def test_sgemm_golden_tiled_256(cuda):
    g = golden("mm_tiled_256")
    got = sgemm(g["A"], g["B"])
    assert frob_rel(got, g["C"]) <= RTOL_FRO
    np.testing.assert_allclose(got, g["C"], rtol=1e-5, atol=1e-5)


def test_sgemm_leading_dimensions(cuda):
    r = np.random.Generator(np.random.Philox(77))
    A = np.asfortranarray(r.standard_normal((200, 96), dtype=np.float32))
    B = np.asfortranarray(r.standard_normal((96, 300), dtype=np.float32))
    got = sgemm(A, B, lda=203, ldb=100, ldc=210)
    assert frob_rel(got, oracle.matmul_f64(A, B)) <= RTOL_FRO


def test_sgemm_k_below_16_gives_zero(cuda):
    A = np.ones((64, 15), dtype=np.float32, order="F")
    B = np.ones((15, 32), dtype=np.float32, order="F")
    assert (sgemm(A, B) == 0).all()


def test_sgemm_keeps_bits_tf32_would_drop(cuda):
    # All-positive operands whose low mantissa bits TF32 alone would drop
    # (plain TF32 errs by ~2^-11 = 5e-4 here).  Every product has the same sign,
    # the worst case for the tensor core's biased in-chunk accumulation.
    r = np.random.Generator(np.random.Philox(78))
    A = np.asfortranarray((1 + r.random((256, 512), dtype=np.float32) * 2**-12).astype(np.float32))
    B = np.asfortranarray((1 + r.random((512, 256), dtype=np.float32) * 2**-12).astype(np.float32))
    got = sgemm(A, B)
    want = oracle.matmul_f64(A, B)
    assert np.max(np.abs(got - want) / np.abs(want)) < RTOL_FRO


def test_sgemm_full_size_properties(cuda):
    from cutilecpu_b200 import workloads
    n = 8192
    A = workloads.normal((n, n), stream=40)
    B = workloads.normal((n, n), stream=41)
    Ad, Bd = dev(A), dev(B)
    Cd = torch.empty(n * n, device="cuda")
    L = _lib.lib()
    s = torch.cuda.current_stream().cuda_stream
    assert L.mk_sgemm_3xtf32(Cd.data_ptr(), Ad.data_ptr(), Bd.data_ptr(), n, n, n, n, n, n, s) == 0
    assert L.mk_error_poll(s) == 0
    C = Cd.cpu().numpy().reshape((n, n), order="F")
    v = np.random.Generator(np.random.Philox(9)).standard_normal(n)
    want = oracle.matvec_chain_f64(A, B, v)
    got = oracle.matvec_f64(C, v)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= RTOL_FRO
    ii = np.array([0, 1, 127, 128, 4095, 8191, 8191]); jj = np.array([0, 255, 256, 17, 4000, 0, 8191])
    np.testing.assert_allclose(C[ii, jj], oracle.matmul_entries_f64(A, B, ii, jj), rtol=1e-4, atol=2e-4)


def sgemm_full(A_h, B_h):
    M, K = A_h.shape
    N = B_h.shape[1]
    A, B = dev(A_h), dev(B_h)
    Cd = torch.empty(M * N, device="cuda")
    rc = _lib.lib().mk_sgemm_f32(Cd.data_ptr(), A.data_ptr(), B.data_ptr(), M, N, K, M, K, M,
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    return Cd.cpu().numpy().reshape((M, N), order="F")


@pytest.mark.parametrize("M,N,K", [(64, 32, 1), (100, 70, 15), (129, 257, 17), (256, 256, 33), (300, 200, 1000)])
def test_sgemm_full_k_vs_fp64(cuda, M, N, K):
    r = np.random.Generator(np.random.Philox(M + N + K))
    A = np.asfortranarray(r.standard_normal((M, K), dtype=np.float32))
    B = np.asfortranarray(r.standard_normal((K, N), dtype=np.float32))
    want = A.astype(np.float64) @ B.astype(np.float64)
    assert frob_rel(sgemm_full(A, B), want) <= RTOL_FRO


def test_mul_and_mm_naive_surface(cuda):
    import cutilecpu_b200 as mk
    r = np.random.Generator(np.random.Philox(5))
    A = np.asfortranarray(r.standard_normal((8, 4), dtype=np.float32))
    B = np.asfortranarray(r.standard_normal((4, 6), dtype=np.float32))
    Am, Bm = mk.MLIRArray(A), mk.MLIRArray(B)
    Cm = mk.zeros(mk.get_backend(Am), "Float32", (8, 6))
    mk.mul(Cm, Am, Bm)
    want = A.astype(np.float64) @ B.astype(np.float64)
    assert np.max(np.abs(mk.Array(Cm) - want)) < 1e-5      # test/test_gpu_simt.jl:335 uses < 1f-3
    C2 = mk.zeros(mk.get_backend(Am), "Float32", (8, 6))
    mk.mm_naive(mk.get_backend(Am), (4, 2))(C2, Am, Bm, ndrange=(8, 6))
    np.testing.assert_array_equal(mk.Array(C2), mk.Array(Cm))


@pytest.mark.parametrize("mode", ["0", "1"])
def test_sgemm_shapes_with_each_kernel(cuda, mode):
    """The shape tests again with the kernel forced: MK_SGEMM_PAIR=1 runs every
    shape (ragged, split-K, K % 16) on CTA pairs, =0 on single CTAs; the
    automatic choice picks one of the two by problem size."""
    import os
    import subprocess
    import sys
    env = dict(os.environ, MK_SGEMM_PAIR=mode)
    r = subprocess.run([sys.executable, "-m", "pytest", __file__, "-m", "gpu", "-q", "-x", "-p", "no:cacheprovider",
                        "-k", "vs_fp64 or leading or golden or below_16 or keeps_bits"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]

