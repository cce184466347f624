// histogram.cu — counts[key-1] += 1 over 1-based Int32 keys with u32
// wrap-around, accumulating into the caller's counts: the `@atomic` histogram of
// the reference (simple form test/test_ka_cpu.jl:16-19; KA's shared-memory form
// test/test_gpu_simt.jl:49-73; atomic kind `addi` src/lower.jl:3600-3623).
//
// Design (HBM-bound on the key stream, 4 B/key; contention-bound on hot bins):
//   * persistent grid (2 x 1024 threads per SM); every block privatises the
//     whole histogram in shared memory (optionally several replicas, warp w
//     using copy w % replicas); keys arrive as 16-byte int4 vectors, several
//     in flight per thread;
//   * one shared atomic per key.  Warp aggregation with match.any measured 7x
//     slower (instruction-issue bound) even on Zipf(1.1) keys, where one bin
//     holds 16 % of the keys: same-address shared atomics do not serialise
//     enough to matter;
//   * flush: one global atomicAdd per non-zero bin per block (sum of replicas).
// nbins too large for shared memory falls back to per-key global atomics.
// Keys outside [1, nbins] are skipped and raise ERRBIT_HIST_KEY.
#include <stdlib.h>

#include "mk_common.cuh"

namespace {

constexpr int kThreads = 1024;

struct Tune {
  int blocks_per_sm = 2;
  int replicas = 1;
  int unroll = 2;
};

const Tune& tune() {
  static Tune t = [] {
    Tune v;
    if (const char* e = getenv("MK_TUNE_HIST_BLOCKS_PER_SM")) v.blocks_per_sm = atoi(e);
    if (const char* e = getenv("MK_TUNE_HIST_REPLICAS")) v.replicas = atoi(e);
    if (const char* e = getenv("MK_TUNE_HIST_UNROLL")) v.unroll = atoi(e);
    if (v.blocks_per_sm < 1 || v.blocks_per_sm > 2) v.blocks_per_sm = 2;
    if (v.replicas < 1 || v.replicas > 32) v.replicas = 1;
    return v;
  }();
  return t;
}

__device__ __forceinline__ void add_key(unsigned* __restrict__ rep, uint32_t nbins, int32_t key, unsigned& bad) {
  const uint32_t u = (uint32_t)key - 1u;  // 1-based -> 0-based; key < 1 wraps to huge
  if (u < nbins) atomicAdd(rep + u, 1u);
  else bad = 1u;
}

__device__ __forceinline__ void add_key4(unsigned* __restrict__ rep, uint32_t nbins, int4 k, unsigned& bad) {
  add_key(rep, nbins, k.x, bad);
  add_key(rep, nbins, k.y, bad);
  add_key(rep, nbins, k.z, bad);
  add_key(rep, nbins, k.w, bad);
}

// UNR int4 key vectors in flight per thread.
template <int UNR>
__global__ void __launch_bounds__(kThreads)
hist_smem(unsigned* __restrict__ counts, uint32_t nbins, const int32_t* __restrict__ keys, int64_t n,
          int head, int replicas, unsigned* __restrict__ err) {
  extern __shared__ unsigned sh[];
  // replica r lives at r * (nbins + 1): the extra word moves the same bin of
  // neighbouring replicas into different banks
  const uint32_t rstride = nbins + 1;
  const uint32_t total = rstride * (uint32_t)replicas;
  for (uint32_t b = threadIdx.x; b < total; b += kThreads) sh[b] = 0u;
  __syncthreads();
  // lanes of one warp spread over the replicas, so a hot bin hit by several
  // lanes of the same instruction is split across copies
  unsigned* rep = sh + (uint32_t)((threadIdx.x & 31) % replicas) * rstride;
  unsigned bad = 0u;

  const int64_t tid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  const int4* k4 = reinterpret_cast<const int4*>(keys + head);
  const int64_t n4 = (n - head) / 4;
  int64_t i = tid;
  for (; i + (UNR - 1) * stride < n4; i += UNR * stride) {
    int4 k[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) k[u] = __ldcs(k4 + i + u * stride);
#pragma unroll
    for (int u = 0; u < UNR; ++u) add_key4(rep, nbins, k[u], bad);
  }
  for (; i < n4; i += stride) add_key4(rep, nbins, __ldcs(k4 + i), bad);
  const int64_t tail_start = head + n4 * 4;
  if (tid < head) add_key(rep, nbins, keys[tid], bad);
  if (tid < n - tail_start) add_key(rep, nbins, keys[tail_start + tid], bad);
  __syncthreads();

  for (uint32_t b = threadIdx.x; b < nbins; b += kThreads) {
    unsigned sum = 0;
    for (int r = 0; r < replicas; ++r) sum += sh[(uint32_t)r * rstride + b];
    if (sum) atomicAdd(counts + b, sum);
  }
  if (bad) atomicOr(err, mk::ERRBIT_HIST_KEY);
}

__global__ void __launch_bounds__(256)
hist_global(unsigned* __restrict__ counts, uint32_t nbins, const int32_t* __restrict__ keys, int64_t n,
            unsigned* __restrict__ err) {
  unsigned bad = 0u;
  const int64_t stride = (int64_t)gridDim.x * 256;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += stride)
    add_key(counts, nbins, keys[i], bad);
  if (bad) atomicOr(err, mk::ERRBIT_HIST_KEY);
}

template <int UNR>
int launch_smem(int64_t blocks, int64_t smem, cudaStream_t s, uint32_t* counts, int32_t nbins, const int32_t* keys,
                int64_t n, int head, int replicas, unsigned* err) {
  int rc = mk::allow_dynamic_smem(reinterpret_cast<const void*>(hist_smem<UNR>), (size_t)smem);
  if (rc != MK_OK) return rc;
  hist_smem<UNR><<<(unsigned)blocks, kThreads, (size_t)smem, s>>>(counts, (uint32_t)nbins, keys, n, head, replicas,
                                                                  err);
  return mk::check_launch("mk_hist_u32: launch");
}

}  // namespace

extern "C" int mk_hist_u32(uint32_t* counts, int32_t nbins, const int32_t* keys1, int64_t n, void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n < 0) return mk::fail(MK_ERR_INVALID, "mk_hist_u32: n must be >= 0");
  if (nbins < 1) return mk::fail(MK_ERR_INVALID, "mk_hist_u32: nbins must be >= 1");
  if (n == 0) return MK_OK;
  if (!counts || !keys1) return mk::fail(MK_ERR_INVALID, "mk_hist_u32: null pointer");
  if ((reinterpret_cast<uintptr_t>(keys1) & 3u) != 0)
    return mk::fail(MK_ERR_INVALID, "mk_hist_u32: keys must be 4-byte aligned");
  cudaStream_t s = mk::as_stream(stream);
  const Tune& t = tune();
  int replicas = t.replicas;
  const int64_t smem_cap = dev->max_smem_optin / t.blocks_per_sm - 1024;
  while (replicas > 1 && (int64_t)replicas * (nbins + 1) * 4 > smem_cap) --replicas;
  const int64_t smem = (int64_t)replicas * (nbins + 1) * 4;
  if (smem > smem_cap) {
    int64_t blocks = mk::cdiv(n, 256);
    const int64_t cap = (int64_t)dev->sms * 8;
    if (blocks > cap) blocks = cap;
    hist_global<<<(unsigned)blocks, 256, 0, s>>>(counts, (uint32_t)nbins, keys1, n, dev->err_word);
    return mk::check_launch("mk_hist_u32: launch (global)");
  }
  // Keys before the first 16-byte boundary are handled as scalars.
  int64_t head = (int64_t)(((16u - (reinterpret_cast<uintptr_t>(keys1) & 15u)) & 15u) / 4u);
  if (head > n) head = n;
  int64_t blocks = mk::cdiv(n, (int64_t)kThreads * 16);
  const int64_t cap = (int64_t)dev->sms * t.blocks_per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  switch (t.unroll) {
    case 1: return launch_smem<1>(blocks, smem, s, counts, nbins, keys1, n, (int)head, replicas, dev->err_word);
    case 4: return launch_smem<4>(blocks, smem, s, counts, nbins, keys1, n, (int)head, replicas, dev->err_word);
    case 8: return launch_smem<8>(blocks, smem, s, counts, nbins, keys1, n, (int)head, replicas, dev->err_word);
    default: return launch_smem<2>(blocks, smem, s, counts, nbins, keys1, n, (int)head, replicas, dev->err_word);
  }
}
