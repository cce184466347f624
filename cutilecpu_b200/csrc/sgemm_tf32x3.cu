// sgemm_tf32x3.cu — C = A*B in fp32 on the 5th-generation tensor cores
// (tcgen05, TMEM accumulators, TMA), with 3xTF32 split precision.
//
// Replaces the reference's 16x16 @localmem SIMT kernel mm_tiled!
// (examples/tiled_matmul.jl:28-48): same operands (column-major, Julia
// layout) and the same K rule (only 16*floor(K/16) terms, :34), computed as
//     C = Ahi*Bhi + Ahi*Blo + Alo*Bhi            (Alo*Blo dropped)
// with x = hi + lo, hi = rna_tf32(x), lo = rna_tf32(x - hi): every operand
// the tensor core sees is an exact TF32 value, products are exact and the
// accumulation is fp32 in TMEM, so the result is within ~1e-6 relative of an
// fp64 GEMM (the split method of Ootomo & Yokota, 2022).
//
// Two launches per call:
//  1. split: A and B are re-laid out K-major into a per-stream workspace with
//     each 16-wide k-block stored as [hi(16) | lo(16)], i.e. one 128-byte row
//     segment per (row, k-block).  A is transposed on the way (column-major A
//     is M-major); B is already K-major.
//  2. gemm: one CTA per 128x256 tile of C, 10 warps:
//       warp 0     TMA producer: per k-block one 128x32 box of A2 and one
//                  256x32 box of B2 (128B swizzle) into a 4-stage ring;
//       warp 1     MMA issuer: per stage 6 x tcgen05.mma.kind::tf32 (M=128,
//                  N=256, K=8): hi.hi, hi.lo, lo.hi over the two k-halves,
//                  addressed by offsetting the descriptor start inside the
//                  swizzle atom; tcgen05.commit frees the stage;
//       warps 2-9  epilogue: the tensor core accumulates each chunk of 256 k
//                  (16 k-blocks) afresh into one of two 256-column TMEM buffers;
//                  the epilogue warps (each a 32-lane quarter x 128 columns)
//                  drain a finished chunk with tcgen05.ld 32x32b and add it into
//                  fp32 registers with round-to-nearest, while the MMAs of the
//                  next chunk run into the other buffer.  The tensor core's
//                  internal fp32 accumulation is biased (it does not round to
//                  nearest); bounding it to 256 terms keeps the K=8192 result
//                  within 1e-5 of fp64.  Finally coalesced column-major stores.
// sgemm_tf32x3_pair (below) runs the same pipeline on CTA pairs with 256x256
// tiles; it is used whenever those tiles fill every SM pair (see pair_mode).
// Every mbarrier wait is bounded (mk::wait_limit_cycles); a timeout raises
// ERRBIT_TIMEOUT in the device error word, stops the other roles, drains the
// producer's in-flight copies (bounded), frees TMEM and returns.
// No TMA multicast is used anywhere.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "mbarrier.cuh"
#include "mk_common.cuh"

#ifndef MK_SGEMM_CHUNK_KB
#define MK_SGEMM_CHUNK_KB 16
#endif

namespace {

using namespace mk::tma;

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int KB = 16;                       // k per block (per split pair)
constexpr int ROWF = 2 * KB;                 // floats per row segment: hi(16) | lo(16)
constexpr int STAGES = 4;
constexpr int A_STAGE = BM * ROWF * 4;       // 16 KiB
constexpr int B_STAGE = BN * ROWF * 4;       // 32 KiB
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int EPI_WARPS = 8;
constexpr int kThreads = 32 * (2 + EPI_WARPS);  // producer, MMA, 8 epilogue warps
constexpr int CHUNK_KB = MK_SGEMM_CHUNK_KB;                      // k-blocks per TMEM accumulation chunk (256 k)
constexpr uint32_t TMEM_COLS = 2 * BN;           // two 256-column accumulators
constexpr int GROUP_M = 16;                      // tile-rows per raster group
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;

// kind::tf32 instruction descriptor: D f32, A/B tf32, both K-major, M=128, N=256.
constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

// ---------------------------------------------------------------- PTX ------

// Shared-memory matrix descriptor: K-major, 128B swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: thread i gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t u;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
  return __uint_as_float(u);
}

// ------------------------------------------------------------- split -------

__device__ __forceinline__ float4 hi4(float4 x) {
  return make_float4(tf32_rna(x.x), tf32_rna(x.y), tf32_rna(x.z), tf32_rna(x.w));
}
__device__ __forceinline__ float4 lo4(float4 x, float4 h) {
  return make_float4(tf32_rna(x.x - h.x), tf32_rna(x.y - h.y), tf32_rna(x.z - h.z), tf32_rna(x.w - h.w));
}

// Output segment layout: each (row, k-block) owns 8 float4 = one 128-byte
// line: float4 i < 4 holds hi of source float4 i, float4 4 + i its lo.  Eight
// consecutive lanes build one segment, one float4 each, so every warp store
// covers four whole lines.
__device__ __forceinline__ float4 segment_part(float4 x, int i) {
  const float4 h = hi4(x);
  return i < 4 ? h : lo4(x, h);
}

// A (M x K column-major, lda) -> A2 (M rows x 2Kt, row-major).  One block per
// 128 rows x 2 k-blocks: the 32 source columns are read coalesced into shared
// memory (the transpose), then written as whole 128-byte segments.
constexpr int SA_ROWS = 128;
constexpr int SA_KBS = 2;
__global__ void __launch_bounds__(256) split_a(float* __restrict__ A2, const float* __restrict__ A, int64_t M,
                                               int64_t lda, int nkb, int64_t kvalid) {
  __shared__ float t[SA_KBS * KB][SA_ROWS + 1];
  const int64_t m0 = (int64_t)blockIdx.x * SA_ROWS;
  const int kb0 = blockIdx.y * SA_KBS;
  const int nk = min(SA_KBS, nkb - kb0) * KB;
  // 16-byte loads along m (A is column-major) when A, lda and the block's
  // rows allow them: all of the block's loads are then issued before any is
  // used; otherwise one 4-byte load per element
  const bool vec = ((reinterpret_cast<uintptr_t>(A) & 15u) == 0) && (lda & 3) == 0 && m0 + SA_ROWS <= M;
  if (vec) {
    constexpr int kV = SA_KBS * KB * SA_ROWS / 4 / 256;  // float4 per thread
    float4 q[kV];
#pragma unroll
    for (int u = 0; u < kV; ++u) {
      const int e = u * 256 + threadIdx.x;
      const int kk = e / (SA_ROWS / 4), m4 = e % (SA_ROWS / 4);
      const int64_t k = (int64_t)kb0 * KB + kk;  // columns at or past kvalid are zero padding
      q[u] = (kk < nk && k < kvalid) ? __ldcs(reinterpret_cast<const float4*>(A + m0 + 4 * m4 + k * lda))
                                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int u = 0; u < kV; ++u) {
      const int e = u * 256 + threadIdx.x;
      const int kk = e / (SA_ROWS / 4), m4 = e % (SA_ROWS / 4);
      t[kk][4 * m4] = q[u].x;
      t[kk][4 * m4 + 1] = q[u].y;
      t[kk][4 * m4 + 2] = q[u].z;
      t[kk][4 * m4 + 3] = q[u].w;
    }
  } else {
    for (int e = threadIdx.x; e < SA_KBS * KB * SA_ROWS; e += 256) {
      const int kk = e / SA_ROWS, mm = e % SA_ROWS;
      const int64_t m = m0 + mm;
      const int64_t k = (int64_t)kb0 * KB + kk;  // columns at or past kvalid are zero padding
      t[kk][mm] = (kk < nk && m < M && k < kvalid) ? A[m + k * lda] : 0.0f;
    }
  }
  __syncthreads();
  const int64_t row_len = (int64_t)nkb * ROWF;
#pragma unroll
  for (int it = 0; it < SA_ROWS * SA_KBS * 8 / 256; ++it) {
    const int f = it * 256 + threadIdx.x;
    const int seg = f >> 3, i = f & 7;
    const int j = seg % SA_KBS, mm = seg / SA_KBS;  // consecutive segments: adjacent k-blocks of a row
    const int64_t m = m0 + mm;
    if (m < M && j * KB < nk) {
      const int k = j * KB + 4 * (i & 3);
      const float4 x = make_float4(t[k][mm], t[k + 1][mm], t[k + 2][mm], t[k + 3][mm]);
      reinterpret_cast<float4*>(A2 + m * row_len + (int64_t)(kb0 + j) * ROWF)[i] = segment_part(x, i);
    }
  }
}

// B (K x N column-major, ldb) -> B2 (N rows x 2Kt): already K-major, so B2 is
// written linearly.  A thread takes one source float4 (4 consecutive k of one
// column n) per step and writes its hi part into float4 q and its lo part into
// float4 4 + q of the (n, k-block) segment; two steps are in flight per
// thread.  VEC: B and ldb allow 16-byte loads.
template <bool VEC>
__device__ __forceinline__ float4 load_b4(const float* __restrict__ B, int64_t ldb, int nkb, int64_t kvalid,
                                          int64_t src, int64_t& seg, int& q) {
  seg = src >> 2;
  q = (int)(src & 3);
  const int64_t n = seg / nkb;
  const int kb = (int)(seg - n * nkb);
  const int64_t k = (int64_t)kb * KB + 4 * q;
  const float* p = B + n * ldb + k;
  if (VEC && k + 4 <= kvalid) return *reinterpret_cast<const float4*>(p);
  // unaligned B, or the zero-padded K remainder
  return make_float4(k < kvalid ? p[0] : 0.0f, k + 1 < kvalid ? p[1] : 0.0f, k + 2 < kvalid ? p[2] : 0.0f,
                     k + 3 < kvalid ? p[3] : 0.0f);
}

template <bool VEC>
__global__ void __launch_bounds__(256) split_b(float* __restrict__ B2, const float* __restrict__ B, int64_t N,
                                               int64_t ldb, int nkb, int64_t kvalid) {
  const int64_t total = N * (int64_t)nkb * 4;  // source float4s
  const int64_t stride = (int64_t)gridDim.x * 256;
  float4* out = reinterpret_cast<float4*>(B2);
  int64_t t = (int64_t)blockIdx.x * 256 + threadIdx.x;
  for (; t + stride < total; t += 2 * stride) {
    int64_t s0, s1;
    int q0, q1;
    const float4 x0 = load_b4<VEC>(B, ldb, nkb, kvalid, t, s0, q0);
    const float4 x1 = load_b4<VEC>(B, ldb, nkb, kvalid, t + stride, s1, q1);
    const float4 h0 = hi4(x0), h1 = hi4(x1);
    out[s0 * 8 + q0] = h0;
    out[s0 * 8 + 4 + q0] = lo4(x0, h0);
    out[s1 * 8 + q1] = h1;
    out[s1 * 8 + 4 + q1] = lo4(x1, h1);
  }
  for (; t < total; t += stride) {
    int64_t s0;
    int q0;
    const float4 x0 = load_b4<VEC>(B, ldb, nkb, kvalid, t, s0, q0);
    const float4 h0 = hi4(x0);
    out[s0 * 8 + q0] = h0;
    out[s0 * 8 + 4 + q0] = lo4(x0, h0);
  }
}

// -------------------------------------------------------------- gemm -------

__global__ void __launch_bounds__(kThreads, 1)
sgemm_tf32x3(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
             float* __restrict__ C, int64_t M, int64_t N, int64_t ldc, int nkb_total, int kb_per_split, int tiles,
             int64_t split_stride, unsigned long long limit, unsigned* __restrict__ err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars: [0,S) full, [S,2S) empty, 2S+{0,1} acc_full, 2S+{2,3} acc_empty, 2S+4 done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Grouped raster: consecutive CTAs walk GROUP_M tile-rows column by column,
  // so a wave of ~148 CTAs shares ~16 A panels and ~9 B panels in L2.
  // Split-K (small problems): CTA blockIdx.x handles tile (blockIdx.x % tiles)
  // over k-blocks [split * kb_per_split, +kb_per_split) and writes its own
  // partial C at C + split * split_stride (summed in order by split_reduce).
  const int split = blockIdx.x / tiles;
  const int kb0 = split * kb_per_split;
  const int nkb = min(nkb_total - kb0, kb_per_split);
  C += (int64_t)split * split_stride;
  int64_t m0, n0;
  {
    const int nM = (int)((M + BM - 1) / BM), nN = (int)((N + BN - 1) / BN);
    const int t = blockIdx.x % tiles;
    const int per_group = GROUP_M * nN;
    const int first_m = (t / per_group) * GROUP_M;
    const int gsize = min(GROUP_M, nM - first_m);
    const int r = t % per_group;
    m0 = (int64_t)(first_m + r % gsize) * BM;
    n0 = (int64_t)(r / gsize) * BN;
  }
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * STAGES), acce0 = smem_u32(bars + 2 * STAGES + 2);
  const uint32_t done = smem_u32(bars + 2 * STAGES + 4);
  const int nchunks = (nkb + CHUNK_KB - 1) / CHUNK_KB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, EPI_WARPS);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer
      const uint32_t smem0 = smem_u32(smem);
      int issued = 0;
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        if (kb >= STAGES && !wait_bounded(empty0 + 8 * s, ((kb / STAGES) - 1) & 1, limit, abort_flag)) {
          ok = false;
          break;
        }
        mbar_expect_tx(full0 + 8 * s, STAGE_BYTES);
        const uint32_t dst = smem0 + s * STAGE_BYTES;
        tma_load_2d(dst, &tmA, (kb0 + kb) * ROWF, (int)m0, full0 + 8 * s);
        tma_load_2d(dst + A_STAGE, &tmB, (kb0 + kb) * ROWF, (int)n0, full0 + 8 * s);
        ++issued;
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, mk::ERRBIT_TIMEOUT);
      }
      // Drain, whether or not anything aborted: the last (up to STAGES) copies
      // may still be landing in shared memory if the MMA stopped consuming.
      // Every earlier stage was consumed (its slot was freed before reuse), so
      // only this window can be in flight.  On the normal path each of these
      // phases has completed and the waits return at once.
      volatile int no_abort = 0;
      for (int kb = issued - 1; kb >= 0 && kb >= issued - STAGES; --kb)
        wait_bounded(full0 + 8 * (kb % STAGES), (kb / STAGES) & 1, kDrainCycles, &no_abort);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: chunk c accumulates afresh into TMEM buffer c & 1
      const uint32_t smem0 = smem_u32(smem);
      bool ok = true;
      for (int c = 0; c < nchunks && ok; ++c) {
        const int b = c & 1;
        if (c >= 2 && !wait_bounded(acce0 + 8 * b, ((c >> 1) - 1) & 1, limit, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BN);
        const int kb_end = min(nkb, (c + 1) * CHUNK_KB);
        for (int kb = c * CHUNK_KB; kb < kb_end; ++kb) {
          const int s = kb % STAGES;
          if (!wait_bounded(full0 + 8 * s, (kb / STAGES) & 1, limit, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem0 + s * STAGE_BYTES, bb = a + A_STAGE;
          // (A offset, B offset) in bytes inside the 128-byte row: k-halves
          // at +0/+32 (hi) and +64/+96 (lo).
          mma_tf32(d, smem_desc(a + 0), smem_desc(bb + 0), kb > c * CHUNK_KB ? 1u : 0u);
          mma_tf32(d, smem_desc(a + 32), smem_desc(bb + 32), 1u);
          mma_tf32(d, smem_desc(a + 0), smem_desc(bb + 64), 1u);
          mma_tf32(d, smem_desc(a + 32), smem_desc(bb + 96), 1u);
          mma_tf32(d, smem_desc(a + 64), smem_desc(bb + 0), 1u);
          mma_tf32(d, smem_desc(a + 96), smem_desc(bb + 32), 1u);
          mma_commit(empty0 + 8 * s);
        }
        if (ok) mma_commit(accf0 + 8 * b);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, mk::ERRBIT_TIMEOUT);
      }
      // "done" completes once every MMA issued so far has finished
      mma_commit(done);
    }
  } else {
    // ---- epilogue: 8 warps; TMEM lane quarter q = warp % 4, column half h.
    // Each chunk's TMEM partial is added into fp32 registers with
    // round-to-nearest, so the tensor core's internal accumulation only ever
    // spans CHUNK_KB*16 terms.
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    float acc[BN / 2];
#pragma unroll
    for (int j = 0; j < BN / 2; ++j) acc[j] = 0.0f;
    bool ok = true;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    for (int c = 0; c < nchunks; ++c) {
      const int b = c & 1;
      bool w = wait_bounded(accf0 + 8 * b, (c >> 1) & 1, limit, abort_flag);
      w = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
      if (!w) {
        ok = false;
        if (lane == 0) *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t0 = tmem + lane_base + (uint32_t)(b * BN + h * (BN / 2));
#pragma unroll
      for (int i = 0; i < BN / 64; ++i) {
        uint32_t r[32];
        tmem_ld32(t0 + i * 32, r);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[i * 32 + j] = __fadd_rn(acc[i * 32 + j], __uint_as_float(r[j]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * b);
    }
    if (ok) {
      const int64_t row = m0 + q * 32 + lane;
      if (row < M) {
        const int64_t nb = n0 + h * (BN / 2);
        float* dst = C + row + nb * ldc;
#pragma unroll
        for (int j = 0; j < BN / 2; ++j)
          if (nb + j < N) __stcs(dst + (int64_t)j * ldc, acc[j]);
      }
    } else {
      atomicOr(err, mk::ERRBIT_TIMEOUT);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    // every issued MMA has completed before the columns are released
    volatile int no_abort = 0;
    wait_bounded(done, 0, kDrainCycles, &no_abort);
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------- gemm, 2-SM ----
//
// The same product on CTA pairs (cluster of 2): one tcgen05.mma.cta_group::2
// computes a 256x256 tile per pair.  Each CTA stages its own 128 rows of A2
// and its own 128 rows of B2 (half the tile's N), so every SM reads 128+128
// operand rows per k-step instead of 128+256: a third less shared-memory
// traffic into the tensor core for the same FLOPs, and 6 pipeline stages fit.
//   * both CTAs: TMA producer (warp 0) with .cta_group::2 loads that complete
//     on the leader's (rank 0) full barrier; epilogue (warps 2-9) over its own
//     128 TMEM lanes; TMEM is allocated and freed by warp 2 of both CTAs;
//   * leader only: the MMA issuer; its commits arrive on both CTAs' barriers
//     (tcgen05.commit multicast), and it waits on its accumulator-empty
//     barrier, which both CTAs' epilogue warps arrive on.
// Loads carry no cluster multicast: every CTA loads only its own tiles.

constexpr int P_BM = 128;                     // A rows per CTA (pair tile M = 256)
constexpr int P_BNH = 128;                    // B rows per CTA (pair tile N = 256)
constexpr int P_STAGES = 6;
constexpr int P_A_STAGE = P_BM * ROWF * 4;    // 16 KiB
constexpr int P_B_STAGE = P_BNH * ROWF * 4;   // 16 KiB
constexpr int P_STAGE_BYTES = P_A_STAGE + P_B_STAGE;
constexpr int P_GROUP_M = 8;                  // pair tile-rows per raster group
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256;
// kind::tf32, D f32, A/B tf32 K-major, M=256 (pair), N=256.
constexpr uint32_t P_IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(256 >> 3) << 17) |
                             ((uint32_t)(256 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n barrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(dst),
      "l"(map), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(P_IDESC), "r"(acc)
      : "memory");
}

// Arrive on the barrier at offset `bar` in both CTAs of the pair once every
// previously issued tcgen05 operation of this thread has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
sgemm_tf32x3_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  float* __restrict__ C, int64_t M, int64_t N, int64_t ldc, int nkb_total, int kb_per_split,
                  int tiles, int64_t split_stride, unsigned long long limit, unsigned* __restrict__ err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P_STAGES * P_STAGE_BYTES);
  // bars: [0,S) full (leader), [S,2S) empty, 2S+{0,1} acc_full, 2S+{2,3} acc_empty (leader), 2S+4 done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // stages whose copies each producer issued: [0] this CTA's (written by the
  // leader's producer), [1] the partner's (written by the partner's producer
  // into the leader's shared memory); read by the leader's drain
  volatile int* issued_slot = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int split = pair / tiles;
  const int kb0 = split * kb_per_split;
  const int nkb = min(nkb_total - kb0, kb_per_split);
  C += (int64_t)split * split_stride;
  int64_t m0, n0;  // the pair's tile origin
  {
    const int nM = (int)((M + 255) / 256), nN = (int)((N + 255) / 256);
    const int t = pair % tiles;
    const int per_group = P_GROUP_M * nN;
    const int first_m = (t / per_group) * P_GROUP_M;
    const int gsize = min(P_GROUP_M, nM - first_m);
    const int r = t % per_group;
    m0 = (int64_t)(first_m + r % gsize) * 256;
    n0 = (int64_t)(r / gsize) * 256;
  }
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + P_STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * P_STAGES), acce0 = smem_u32(bars + 2 * P_STAGES + 2);
  const uint32_t done = smem_u32(bars + 2 * P_STAGES + 4);
  const int nchunks = (nkb + CHUNK_KB - 1) / CHUNK_KB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 2 * EPI_WARPS);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs): own A rows and own half of the B rows
      const uint32_t smem0 = smem_u32(smem);
      const int a_row = (int)(m0 + rank * P_BM), b_row = (int)(n0 + rank * P_BNH);
      bool ok = true;
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % P_STAGES;
        if (kb >= P_STAGES && !wait_bounded(empty0 + 8 * s, ((kb / P_STAGES) - 1) & 1, limit, abort_flag)) {
          ok = false;
          break;
        }
        if (leader) mbar_expect_tx(full0 + 8 * s, 2 * P_STAGE_BYTES);
        const uint32_t bar = map_rank(full0 + 8 * s, 0);
        const uint32_t dst = smem0 + s * P_STAGE_BYTES;
        tma_load_2d_pair(dst, &tmA, (kb0 + kb) * ROWF, a_row, bar);
        tma_load_2d_pair(dst + P_A_STAGE, &tmB, (kb0 + kb) * ROWF, b_row, bar);
        ++issued;
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, mk::ERRBIT_TIMEOUT);
      }
      if (leader) {
        issued_slot[0] = issued;
      } else {
        const uint32_t remote = map_rank(smem_u32((const void*)(issued_slot + 1)), 0);
        asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(remote), "r"(issued) : "memory");
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---- MMA issuer (leader): chunk c accumulates afresh into TMEM buffer c & 1
      const uint32_t smem0 = smem_u32(smem);
      bool ok = true;
      for (int c = 0; c < nchunks && ok; ++c) {
        const int b = c & 1;
        if (c >= 2 && !wait_bounded(acce0 + 8 * b, ((c >> 1) - 1) & 1, limit, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BN);
        const int kb_end = min(nkb, (c + 1) * CHUNK_KB);
        for (int kb = c * CHUNK_KB; kb < kb_end; ++kb) {
          const int s = kb % P_STAGES;
          if (!wait_bounded(full0 + 8 * s, (kb / P_STAGES) & 1, limit, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem0 + s * P_STAGE_BYTES, bb = a + P_A_STAGE;
          mma_tf32_pair(d, smem_desc(a + 0), smem_desc(bb + 0), kb > c * CHUNK_KB ? 1u : 0u);
          mma_tf32_pair(d, smem_desc(a + 32), smem_desc(bb + 32), 1u);
          mma_tf32_pair(d, smem_desc(a + 0), smem_desc(bb + 64), 1u);
          mma_tf32_pair(d, smem_desc(a + 32), smem_desc(bb + 96), 1u);
          mma_tf32_pair(d, smem_desc(a + 64), smem_desc(bb + 0), 1u);
          mma_tf32_pair(d, smem_desc(a + 96), smem_desc(bb + 32), 1u);
          mma_commit_pair(empty0 + 8 * s);
        }
        if (ok) mma_commit_pair(accf0 + 8 * b);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, mk::ERRBIT_TIMEOUT);
      }
      mma_commit_pair(done);
    }
  } else {
    // ---- epilogue (both CTAs): 8 warps over this CTA's 128 TMEM lanes x 256 columns
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    float acc[BN / 2];
#pragma unroll
    for (int j = 0; j < BN / 2; ++j) acc[j] = 0.0f;
    bool ok = true;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    for (int c = 0; c < nchunks; ++c) {
      const int b = c & 1;
      bool w = wait_bounded(accf0 + 8 * b, (c >> 1) & 1, limit, abort_flag);
      w = __shfl_sync(0xffffffffu, w ? 1 : 0, 0) != 0;
      if (!w) {
        ok = false;
        if (lane == 0) *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t t0 = tmem + lane_base + (uint32_t)(b * BN + h * (BN / 2));
#pragma unroll
      for (int i = 0; i < BN / 64; ++i) {
        uint32_t r[32];
        tmem_ld32(t0 + i * 32, r);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[i * 32 + j] = __fadd_rn(acc[i * 32 + j], __uint_as_float(r[j]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_rank(acce0 + 8 * b, 0));
    }
    if (ok) {
      const int64_t row = m0 + rank * P_BM + q * 32 + lane;
      if (row < M) {
        const int64_t nb = n0 + h * (BN / 2);
        float* dst = C + row + nb * ldc;
#pragma unroll
        for (int j = 0; j < BN / 2; ++j)
          if (nb + j < N) __stcs(dst + (int64_t)j * ldc, acc[j]);
      }
    } else {
      atomicOr(err, mk::ERRBIT_TIMEOUT);
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // every role of both CTAs has finished with the peer's barriers and TMEM
  if (leader && warp == 0 && lane == 0) {
    // Drain before either CTA exits: both CTAs' copies complete on the
    // leader's full barriers (expect_tx counts both halves), so only the
    // leader can see them land.  Every stage below the larger issued count
    // minus P_STAGES was consumed, so only that window can be in flight.  A
    // phase that one producer never issued gets its missing half completed
    // here (and, if the leader never issued it, the leader's arrival), so the
    // phase completes exactly when the copies that were issued have landed.
    // On the normal path both counts equal nkb and every wait returns at once.
    const int iL = issued_slot[0], iN = issued_slot[1];
    const int hi = max(iL, iN);
    volatile int no_abort = 0;
    for (int kb = max(0, hi - P_STAGES); kb < hi; ++kb) {
      const uint32_t bar = full0 + 8 * (kb % P_STAGES);
      if (kb >= iL) mbar_expect_tx(bar, P_STAGE_BYTES);     // only the partner's half is coming
      if (kb >= iN) mbar_complete_tx(bar, P_STAGE_BYTES);   // the partner's half never comes
      wait_bounded(bar, (kb / P_STAGES) & 1, kDrainCycles, &no_abort);
    }
  }
  if (warp == 2) {
    volatile int no_abort = 0;
    wait_bounded(done, 0, kDrainCycles, &no_abort);  // every MMA writing this CTA's TMEM has completed
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
  __syncwarp();
  cluster_sync_all();
}

// Sum of the split-K partials in split order (deterministic): column-major
// partials with leading dimension M, result into C with ldc.
__global__ void __launch_bounds__(256) split_reduce(float* __restrict__ C, const float* __restrict__ P, int64_t M,
                                                    int64_t N, int64_t ldc, int splits) {
  const int64_t total = M * N, stride = (int64_t)gridDim.x * 256;
  for (int64_t e = (int64_t)blockIdx.x * 256 + threadIdx.x; e < total; e += stride) {
    float acc = __ldcs(P + e);
    for (int sp = 1; sp < splits; ++sp) acc = __fadd_rn(acc, __ldcs(P + (int64_t)sp * total + e));
    const int64_t j = e / M, i = e - j * M;
    C[i + j * ldc] = acc;
  }
}

// ------------------------------------------------------------- host --------

// Row-major (rows x cols) fp32 panel, boxes of box_rows x 32 with 128B swizzle.
int make_map(CUtensorMap* map, const float* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  return mk::encode_rows_f32(map, base, cols, rows, (uint32_t)ROWF, box_rows, "mk_sgemm_3xtf32");
}

}  // namespace

namespace {

// Kernel choice: CTA pairs (256x256 tiles) when their tiles fill every SM
// pair at least once, else one CTA per 128x256 tile (smaller tiles fill a
// small problem better).  MK_SGEMM_PAIR=1 forces pairs, MK_SGEMM_PAIR=0 forbids them.
int pair_mode() {
  static const int mode = [] {
    const char* e = getenv("MK_SGEMM_PAIR");
    if (e && e[0] == '0') return 0;
    if (e && e[0] == '1') return 1;
    return -1;
  }();
  return mode;
}

// full_k: every K term (LinearAlgebra.mul!); otherwise 16*floor(K/16) terms
// (mm_tiled!).  The remainder of a full-K product is zero-padded by the split.
int sgemm_impl(const char* name, bool full_k, float* C, const float* A, const float* B, int64_t M, int64_t N,
               int64_t K, int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  mk::Device* dev = mk::current_device();
  if (!dev) return MK_ERR_CUDA;
  const std::string who(name);
  if (M < 0 || N < 0 || K < 0) return mk::fail(MK_ERR_INVALID, who + ": negative size");
  if (M == 0 || N == 0) return MK_OK;
  if (lda < M || ldb < K || ldc < M || lda < 1 || ldb < 1)
    return mk::fail(MK_ERR_INVALID, who + ": leading dimension too small");
  const int64_t Kt = full_k ? mk::cdiv(K, KB) * KB : (K / KB) * KB;  // padded / truncated K
  const int64_t kvalid = full_k ? K : Kt;
  if (!C || (Kt > 0 && (!A || !B))) return mk::fail(MK_ERR_INVALID, who + ": null pointer");
  if (mk::cdiv(M, BM) * mk::cdiv(N, BN) > INT32_MAX || M > INT32_MAX || N > INT32_MAX || mk::cdiv(Kt / KB, SA_KBS) > 65535)
    return mk::fail(MK_ERR_INVALID, who + ": problem too large");
  cudaStream_t s = mk::as_stream(stream);
  if (Kt == 0) {
    cudaError_t e = cudaMemset2DAsync(C, (size_t)ldc * 4, 0, (size_t)M * 4, (size_t)N, s);
    return e == cudaSuccess ? MK_OK : mk::fail_cuda(e, "sgemm: zero fill");
  }
  const int nkb = (int)(Kt / KB);
  const uint64_t cols = (uint64_t)nkb * ROWF;
  const size_t a_bytes = (((size_t)M * cols * 4) + 1023) & ~(size_t)1023;
  const size_t b_bytes = (size_t)N * cols * 4;
  void* ws = nullptr;
  int rc = mk::stream_workspace(dev, s, a_bytes + b_bytes, &ws, mk::WS_GEMM);
  if (rc != MK_OK) return rc;
  float* A2 = static_cast<float*>(ws);
  float* B2 = reinterpret_cast<float*>(static_cast<char*>(ws) + a_bytes);

  split_a<<<dim3((unsigned)mk::cdiv(M, SA_ROWS), (unsigned)mk::cdiv(nkb, SA_KBS)), 256, 0, s>>>(A2, A, M, lda, nkb, kvalid);
  {
    const int64_t total = N * (int64_t)nkb * 4;
    int64_t blocks = mk::cdiv(total, 256);
    const int64_t cap = (int64_t)dev->sms * 8;
    if (blocks > cap) blocks = cap;
    if (mk::aligned16(B) && ldb % 4 == 0)
      split_b<true><<<(unsigned)blocks, 256, 0, s>>>(B2, B, N, ldb, nkb, kvalid);
    else
      split_b<false><<<(unsigned)blocks, 256, 0, s>>>(B2, B, N, ldb, nkb, kvalid);
  }
  const int mode = pair_mode();
  const bool pair = mode == 1 || (mode < 0 && mk::cdiv(N, 256) * mk::cdiv(M, 256) >= dev->sms / 2);
  CUtensorMap mapA, mapB;
  if ((rc = make_map(&mapA, A2, cols, (uint64_t)M, BM)) != MK_OK) return rc;
  if ((rc = make_map(&mapB, B2, cols, (uint64_t)N, pair ? P_BNH : BN)) != MK_OK) return rc;
  const void* kfn = pair ? reinterpret_cast<const void*>(sgemm_tf32x3_pair) : reinterpret_cast<const void*>(sgemm_tf32x3);
  const int smem_bytes = pair ? P_SMEM_BYTES : SMEM_BYTES;
  if ((rc = mk::allow_dynamic_smem(kfn, smem_bytes)) != MK_OK) return rc;
  // tiles of C: 128x256 per CTA, or 256x256 per CTA pair
  const int64_t tiles = pair ? mk::cdiv(N, 256) * mk::cdiv(M, 256) : mk::cdiv(N, BN) * mk::cdiv(M, BM);
  const int64_t slots = pair ? dev->sms / 2 : dev->sms;  // tiles that run at once
  // Split K when the tiles cannot fill the GPU: each split keeps >= 1 chunk.
  int splits = 1;
  if (tiles < slots) {
    splits = (int)(slots / tiles);
    const int max_by_k = nkb / CHUNK_KB;
    if (splits > max_by_k) splits = max_by_k;
    if (splits > 8) splits = 8;
    if (splits < 1) splits = 1;
  }
  const int kb_per_split = (int)mk::cdiv(nkb, splits);
  splits = (int)mk::cdiv(nkb, kb_per_split);
  float* target = C;
  int64_t target_ld = ldc, split_stride = 0;
  if (splits > 1) {
    void* pw = nullptr;
    if ((rc = mk::stream_workspace(dev, s, (size_t)splits * M * N * 4, &pw, mk::WS_GEMM_SPLIT)) != MK_OK) return rc;
    target = static_cast<float*>(pw);
    target_ld = M;
    split_stride = M * N;
  }
  if (pair) {
    dim3 grid((unsigned)(2 * tiles * splits));
    sgemm_tf32x3_pair<<<grid, kThreads, P_SMEM_BYTES, s>>>(mapA, mapB, target, M, N, target_ld, nkb, kb_per_split,
                                                           (int)tiles, split_stride, mk::wait_limit_cycles(),
                                                           dev->err_word);
  } else {
    dim3 grid((unsigned)(tiles * splits));
    sgemm_tf32x3<<<grid, kThreads, SMEM_BYTES, s>>>(mapA, mapB, target, M, N, target_ld, nkb, kb_per_split,
                                                     (int)tiles, split_stride, mk::wait_limit_cycles(), dev->err_word);
  }
  if (splits > 1) {
    int64_t blocks = mk::cdiv(M * N, 256);
    if (blocks > (int64_t)dev->sms * 8) blocks = (int64_t)dev->sms * 8;
    split_reduce<<<(unsigned)blocks, 256, 0, s>>>(C, target, M, N, ldc, splits);
  }
  return mk::check_launch("mk_sgemm_3xtf32: launch");
}

}  // namespace

extern "C" int mk_sgemm_3xtf32(float* C, const float* A, const float* B, int64_t M, int64_t N, int64_t K,
                               int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  mk::clear_error();
  return sgemm_impl("mk_sgemm_3xtf32", false, C, A, B, M, N, K, lda, ldb, ldc, stream);
}

extern "C" int mk_sgemm_f32(float* C, const float* A, const float* B, int64_t M, int64_t N, int64_t K,
                            int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  mk::clear_error();
  return sgemm_impl("mk_sgemm_f32", true, C, A, B, M, N, K, lda, ldb, ldc, stream);
}
