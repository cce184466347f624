// tiled16.cu — the reference's own matmul algorithm on CUDA cores, kept as the
// SIMT comparison point: mm_tiled! of examples/tiled_matmul.jl:28-48.
// Block (16,16), one output per thread, two 16x16 fp32 shared tiles, two
// barriers per k-tile, the per-tile partial `out` added to `acc` after the
// inner loop (:40-44), and the K % 16 remainder ignored (nkt = K ÷ 16, :34).
// Column-major operands with leading dimensions.  Out-of-range rows/columns of
// a ragged edge load 0 and skip the store (the reference masks tail threads).
#include "mk_common.cuh"

namespace {

constexpr int T = 16;

__global__ void __launch_bounds__(T * T)
mm_tiled16(float* __restrict__ C, const float* __restrict__ A, const float* __restrict__ B, int64_t M,
           int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc) {
  __shared__ float tA[T][T + 1];  // [ii][jj], padded against bank conflicts
  __shared__ float tB[T][T + 1];
  const int ii = threadIdx.x, jj = threadIdx.y;  // Julia's (ii, jj), ii fastest
  const int64_t I = (int64_t)blockIdx.x * T + ii;
  const int64_t J = (int64_t)blockIdx.y * T + jj;
  float acc = 0.0f;
  const int64_t nkt = K / T;
  for (int64_t kt = 0; kt < nkt; ++kt) {
    const int64_t kb = kt * T;
    tA[ii][jj] = (I < M) ? A[I + (kb + jj) * lda] : 0.0f;
    tB[ii][jj] = (J < N) ? B[(kb + ii) + J * ldb] : 0.0f;
    __syncthreads();
    float out = 0.0f;
#pragma unroll
    for (int kk = 0; kk < T; ++kk) out = __fmaf_rn(tA[ii][kk], tB[kk][jj], out);
    acc = __fadd_rn(acc, out);
    __syncthreads();
  }
  if (I < M && J < N) C[I + J * ldc] = acc;
}

}  // namespace

extern "C" int mk_matmul_tiled16_f32(float* C, const float* A, const float* B, int64_t M, int64_t N,
                                     int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  MK_ENTRY_DEVICE(dev);
  (void)dev;
  if (M < 0 || N < 0 || K < 0) return mk::fail(MK_ERR_INVALID, "mk_matmul_tiled16_f32: negative size");
  if (M == 0 || N == 0) return MK_OK;
  if (lda < M || ldb < K || ldc < M || lda < 1 || ldb < 1)
    return mk::fail(MK_ERR_INVALID, "mk_matmul_tiled16_f32: leading dimension too small");
  if (!C || ((K / T) > 0 && (!A || !B))) return mk::fail(MK_ERR_INVALID, "mk_matmul_tiled16_f32: null pointer");
  if (mk::cdiv(N, T) > 65535) return mk::fail(MK_ERR_INVALID, "mk_matmul_tiled16_f32: N too large");
  dim3 grid((unsigned)mk::cdiv(M, T), (unsigned)mk::cdiv(N, T));
  mm_tiled16<<<grid, dim3(T, T), 0, mk::as_stream(stream)>>>(C, A, B, M, N, K, lda, ldb, ldc);
  return mk::check_launch("mk_matmul_tiled16_f32: launch");
}
