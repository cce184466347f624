// histogram.cu — bins[key-1] += 1 over 1-based keys, accumulating into the
// caller's bins: the `@atomic` histogram of the reference in its forms
//   * test/test_ka_cpu.jl:16-19 (Int32 keys, Float32 bins, `+= 1f0`),
//   * test/test_gpu_simt.jl:49-73 (KA's example: Int keys, Int bins),
//   * BASELINE configs[3] (Int32 keys, UInt32 bins),
// atomic kind `addi`/`addf` (src/lower.jl:3600-3623).
//
// Design (HBM-bound on the key stream; 4 or 8 bytes per key):
//   * persistent grid (2 x 1024 threads per SM); every block privatises the
//     whole histogram in shared memory as u32 counters; keys arrive as 16-byte
//     vectors, two vectors in flight per thread;
//   * one shared atomic per key.  Warp aggregation with match.any measured 7x
//     slower (instruction-issue bound) even on Zipf(1.1) keys, where one bin
//     holds 16 % of the keys, and lane-spread replicas measured no faster:
//     same-address shared atomics do not serialise enough to matter;
//   * flush: one global atomic per non-zero bin per block, in the bin type:
//     u32 (wraps mod 2^32; Int32 bins use the same bits), 64-bit integer
//     (Int64 bins, two's complement), or fp32 (Float32 bins: the block's count
//     is added as one float, exact while a bin stays below 2^24, where adding
//     1f0 one at a time would also be exact).
// Bins that do not fit in shared memory use per-key global atomics.
// Keys outside [1, nbins] are skipped and raise ERRBIT_HIST_KEY.
#include "mk_common.cuh"

namespace {

constexpr int kThreads = 1024;
constexpr int kBlocksPerSM = 2;
constexpr int kUnroll = 2;

template <typename K>
struct KeyVec;
template <>
struct KeyVec<int32_t> {
  using V = int4;
  static constexpr int N = 4;
  __device__ static int64_t at(const int4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
};
template <>
struct KeyVec<int64_t> {
  using V = longlong2;
  static constexpr int N = 2;
  __device__ static int64_t at(const longlong2& v, int i) { return i == 0 ? v.x : v.y; }
};

__device__ __forceinline__ void add_key(unsigned* __restrict__ h, uint64_t nbins, int64_t key, unsigned& bad) {
  const uint64_t u = (uint64_t)key - 1u;  // 1-based -> 0-based; key < 1 wraps to huge
  if (u < nbins) atomicAdd(h + u, 1u);
  else bad = 1u;
}

template <int BT>
__device__ __forceinline__ void flush_add(void* bins, uint32_t b, unsigned cnt) {
  if (BT == MK_BIN_U32) atomicAdd(static_cast<unsigned*>(bins) + b, cnt);
  else if (BT == MK_BIN_I64) atomicAdd(static_cast<unsigned long long*>(bins) + b, (unsigned long long)cnt);
  else atomicAdd(static_cast<float*>(bins) + b, (float)cnt);
}

template <typename K, int BT>
__global__ void __launch_bounds__(kThreads)
hist_smem(void* __restrict__ bins, uint32_t nbins, const K* __restrict__ keys, int64_t n, int head,
          unsigned* __restrict__ err) {
  using KV = KeyVec<K>;
  using V = typename KV::V;
  extern __shared__ unsigned sh[];
  for (uint32_t b = threadIdx.x; b < nbins; b += kThreads) sh[b] = 0u;
  __syncthreads();
  unsigned bad = 0u;

  const int64_t tid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  const V* kv = reinterpret_cast<const V*>(keys + head);
  const int64_t nv = (n - head) / KV::N;
  int64_t i = tid;
  for (; i + (kUnroll - 1) * stride < nv; i += kUnroll * stride) {
    V k[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) k[u] = __ldcs(kv + i + u * stride);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int e = 0; e < KV::N; ++e) add_key(sh, nbins, KV::at(k[u], e), bad);
  }
  for (; i < nv; i += stride) {
    const V k = __ldcs(kv + i);
#pragma unroll
    for (int e = 0; e < KV::N; ++e) add_key(sh, nbins, KV::at(k, e), bad);
  }
  const int64_t tail_start = head + nv * KV::N;
  if (tid < head) add_key(sh, nbins, keys[tid], bad);
  if (tid < n - tail_start) add_key(sh, nbins, keys[tail_start + tid], bad);
  __syncthreads();

  for (uint32_t b = threadIdx.x; b < nbins; b += kThreads)
    if (sh[b]) flush_add<BT>(bins, b, sh[b]);
  if (bad) atomicOr(err, mk::ERRBIT_HIST_KEY);
}

template <typename K, int BT>
__global__ void __launch_bounds__(256)
hist_global(void* __restrict__ bins, uint64_t nbins, const K* __restrict__ keys, int64_t n,
            unsigned* __restrict__ err) {
  unsigned bad = 0u;
  const int64_t stride = (int64_t)gridDim.x * 256;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += stride) {
    const uint64_t u = (uint64_t)(int64_t)keys[i] - 1u;
    if (u < nbins) flush_add<BT>(bins, (uint32_t)u, 1u);
    else bad = 1u;
  }
  if (bad) atomicOr(err, mk::ERRBIT_HIST_KEY);
}

template <typename K, int BT>
int run(mk::Device* dev, cudaStream_t s, void* bins, int32_t nbins, const K* keys, int64_t n) {
  const int64_t smem = (int64_t)nbins * 4;
  const int64_t smem_cap = dev->max_smem_optin / kBlocksPerSM - 1024;
  if (smem > smem_cap) {
    int64_t blocks = mk::cdiv(n, 256);
    if (blocks > (int64_t)dev->sms * 8) blocks = (int64_t)dev->sms * 8;
    hist_global<K, BT><<<(unsigned)blocks, 256, 0, s>>>(bins, (uint64_t)nbins, keys, n, dev->err_word);
    return mk::check_launch("mk_hist: launch (global)");
  }
  // keys before the first 16-byte boundary are folded as scalars
  int64_t head = (int64_t)(((16u - (reinterpret_cast<uintptr_t>(keys) & 15u)) & 15u) / sizeof(K));
  if (head > n) head = n;
  int64_t blocks = mk::cdiv(n, (int64_t)kThreads * 16);
  if (blocks > (int64_t)dev->sms * kBlocksPerSM) blocks = (int64_t)dev->sms * kBlocksPerSM;
  if (blocks < 1) blocks = 1;
  int rc = mk::allow_dynamic_smem(reinterpret_cast<const void*>(hist_smem<K, BT>), (size_t)smem);
  if (rc != MK_OK) return rc;
  hist_smem<K, BT><<<(unsigned)blocks, kThreads, (size_t)smem, s>>>(bins, (uint32_t)nbins, keys, n, (int)head,
                                                                    dev->err_word);
  return mk::check_launch("mk_hist: launch");
}

template <typename K>
int run_bins(mk::Device* dev, cudaStream_t s, void* bins, int bin_type, int32_t nbins, const K* keys, int64_t n) {
  switch (bin_type) {
    case MK_BIN_U32: return run<K, MK_BIN_U32>(dev, s, bins, nbins, keys, n);
    case MK_BIN_I64: return run<K, MK_BIN_I64>(dev, s, bins, nbins, keys, n);
    default: return run<K, MK_BIN_F32>(dev, s, bins, nbins, keys, n);
  }
}

}  // namespace

extern "C" int mk_hist(void* bins, int bin_type, int32_t nbins, const void* keys1, int key_type, int64_t n,
                       void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n < 0) return mk::fail(MK_ERR_INVALID, "mk_hist: n must be >= 0");
  if (nbins < 1) return mk::fail(MK_ERR_INVALID, "mk_hist: nbins must be >= 1");
  if (bin_type < MK_BIN_U32 || bin_type > MK_BIN_F32) return mk::fail(MK_ERR_INVALID, "mk_hist: unknown bin type");
  if (key_type != MK_KEY_I32 && key_type != MK_KEY_I64) return mk::fail(MK_ERR_INVALID, "mk_hist: unknown key type");
  if (n == 0) return MK_OK;
  if (!bins || !keys1) return mk::fail(MK_ERR_INVALID, "mk_hist: null pointer");
  const unsigned ksize = key_type == MK_KEY_I32 ? 4u : 8u;
  const unsigned bsize = bin_type == MK_BIN_I64 ? 8u : 4u;
  if ((reinterpret_cast<uintptr_t>(keys1) % ksize) != 0) return mk::fail(MK_ERR_INVALID, "mk_hist: misaligned keys");
  if ((reinterpret_cast<uintptr_t>(bins) % bsize) != 0) return mk::fail(MK_ERR_INVALID, "mk_hist: misaligned bins");
  cudaStream_t s = mk::as_stream(stream);
  if (key_type == MK_KEY_I32)
    return run_bins<int32_t>(dev, s, bins, bin_type, nbins, static_cast<const int32_t*>(keys1), n);
  return run_bins<int64_t>(dev, s, bins, bin_type, nbins, static_cast<const int64_t*>(keys1), n);
}

extern "C" int mk_hist_u32(uint32_t* counts, int32_t nbins, const int32_t* keys1, int64_t n, void* stream) {
  return mk_hist(counts, MK_BIN_U32, nbins, keys1, MK_KEY_I32, n, stream);
}
