// histogram.cu — counts[key-1] += 1 over 1-based Int32 keys with u32
// wrap-around, accumulating into the caller's counts: the `@atomic` histogram of
// the reference (simple form test/test_ka_cpu.jl:16-19; KA's shared-memory form
// test/test_gpu_simt.jl:49-73; atomic kind `addi` src/lower.jl:3600-3623).
//
// Design (HBM-bound on the key stream, 4 B/key; contention-bound on hot bins):
//   * persistent grid; every block privatises the whole histogram in shared
//     memory, kReplicas copies so that warps spread their atomics (warp w uses
//     copy w % replicas); keys arrive as 16-byte int4 vectors;
//   * optional warp aggregation: lanes holding the same key elect a leader
//     (match.any) that adds the population count once — this is what keeps
//     Zipf-skewed input (one bin can hold 16 % of all keys) from serialising;
//   * flush: one global atomicAdd per non-zero bin per block (sum of replicas).
// nbins too large for shared memory falls back to per-key global atomics.
// Keys outside [1, nbins] are skipped and raise ERRBIT_HIST_KEY.
#include <stdlib.h>

#include "mk_common.cuh"

namespace {

constexpr int kThreads = 1024;

struct Tune {
  int blocks_per_sm = 2;
  int replicas = 2;
  int aggregate = 0;
};

const Tune& tune() {
  static Tune t = [] {
    Tune v;
    if (const char* e = getenv("MK_TUNE_HIST_BLOCKS_PER_SM")) v.blocks_per_sm = atoi(e);
    if (const char* e = getenv("MK_TUNE_HIST_REPLICAS")) v.replicas = atoi(e);
    if (const char* e = getenv("MK_TUNE_HIST_AGGREGATE")) v.aggregate = atoi(e);
    if (v.blocks_per_sm < 1 || v.blocks_per_sm > 2) v.blocks_per_sm = 2;
    if (v.replicas < 1 || v.replicas > 32) v.replicas = 2;
    return v;
  }();
  return t;
}

template <bool AGG>
__device__ __forceinline__ void add_key(unsigned* __restrict__ rep, uint32_t nbins, int32_t key, bool& bad) {
  const uint32_t u = (uint32_t)key - 1u;  // 1-based -> 0-based; key < 1 wraps to huge
  const bool ok = u < nbins;
  if (!ok) bad = true;
  if (AGG) {
    const unsigned active = __activemask();
    const unsigned peers = __match_any_sync(active, ok ? u : 0xffffffffu);
    const int leader = __ffs(peers) - 1;
    if (ok && (int)(threadIdx.x & 31) == leader) atomicAdd(rep + u, (unsigned)__popc(peers));
  } else {
    if (ok) atomicAdd(rep + u, 1u);
  }
}

template <bool AGG>
__global__ void __launch_bounds__(kThreads)
hist_smem(unsigned* __restrict__ counts, uint32_t nbins, const int32_t* __restrict__ keys, int64_t n,
          int head, int replicas, unsigned* __restrict__ err) {
  extern __shared__ unsigned sh[];
  const uint32_t total = nbins * (uint32_t)replicas;
  for (uint32_t b = threadIdx.x; b < total; b += kThreads) sh[b] = 0u;
  __syncthreads();
  unsigned* rep = sh + (uint32_t)((threadIdx.x >> 5) % replicas) * nbins;
  bool bad = false;

  const int64_t tid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  const int4* k4 = reinterpret_cast<const int4*>(keys + head);
  const int64_t n4 = (n - head) / 4;
  // Two int4 key vectors in flight per thread; uniform trip count per warp
  // keeps match.any's participants whole in the aggregating form.
  int64_t base = (int64_t)blockIdx.x * kThreads;
  for (; base + stride < n4; base += 2 * stride) {
    const int64_t i = base + threadIdx.x;
    const bool second = i + stride < n4;
    const int4 k0 = __ldcs(k4 + i);
    int4 k1 = make_int4(1, 1, 1, 1);
    if (second) k1 = __ldcs(k4 + i + stride);
    add_key<AGG>(rep, nbins, k0.x, bad);
    add_key<AGG>(rep, nbins, k0.y, bad);
    add_key<AGG>(rep, nbins, k0.z, bad);
    add_key<AGG>(rep, nbins, k0.w, bad);
    if (second) {
      add_key<AGG>(rep, nbins, k1.x, bad);
      add_key<AGG>(rep, nbins, k1.y, bad);
      add_key<AGG>(rep, nbins, k1.z, bad);
      add_key<AGG>(rep, nbins, k1.w, bad);
    }
  }
  for (; base < n4; base += stride) {
    const int64_t i = base + threadIdx.x;
    if (i < n4) {
      const int4 k = __ldcs(k4 + i);
      add_key<AGG>(rep, nbins, k.x, bad);
      add_key<AGG>(rep, nbins, k.y, bad);
      add_key<AGG>(rep, nbins, k.z, bad);
      add_key<AGG>(rep, nbins, k.w, bad);
    }
  }
  const int64_t tail_start = head + n4 * 4;
  if (tid < head) add_key<false>(rep, nbins, keys[tid], bad);
  if (tid < n - tail_start) add_key<false>(rep, nbins, keys[tail_start + tid], bad);
  __syncthreads();

  for (uint32_t b = threadIdx.x; b < nbins; b += kThreads) {
    unsigned sum = 0;
    for (int r = 0; r < replicas; ++r) sum += sh[(uint32_t)r * nbins + b];
    if (sum) atomicAdd(counts + b, sum);
  }
  if (bad) atomicOr(err, mk::ERRBIT_HIST_KEY);
}

__global__ void __launch_bounds__(256)
hist_global(unsigned* __restrict__ counts, uint32_t nbins, const int32_t* __restrict__ keys, int64_t n,
            unsigned* __restrict__ err) {
  bool bad = false;
  const int64_t stride = (int64_t)gridDim.x * 256;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += stride)
    add_key<false>(counts, nbins, keys[i], bad);
  if (bad) atomicOr(err, mk::ERRBIT_HIST_KEY);
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
  while (replicas > 1 && (int64_t)replicas * nbins * 4 > smem_cap) --replicas;
  const int64_t smem = (int64_t)replicas * nbins * 4;
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
  cudaError_t e;
  if (t.aggregate) {
    e = cudaFuncSetAttribute(hist_smem<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return mk::fail_cuda(e, "mk_hist_u32: cudaFuncSetAttribute");
    hist_smem<true><<<(unsigned)blocks, kThreads, (size_t)smem, s>>>(counts, (uint32_t)nbins, keys1, n, (int)head,
                                                                    replicas, dev->err_word);
  } else {
    e = cudaFuncSetAttribute(hist_smem<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return mk::fail_cuda(e, "mk_hist_u32: cudaFuncSetAttribute");
    hist_smem<false><<<(unsigned)blocks, kThreads, (size_t)smem, s>>>(counts, (uint32_t)nbins, keys1, n, (int)head,
                                                                     replicas, dev->err_word);
  }
  return mk::check_launch("mk_hist_u32: launch");
}
