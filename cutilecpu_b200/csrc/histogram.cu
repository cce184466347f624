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
//     vectors, three vectors in flight per thread;
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
//
// Multi-GPU (mk_hist_u32_allreduce[_async]): the same kernel ends with the
// exchange of the rank's counts over NVLink peer memory, in place of an NCCL
// all-reduce launch: the last block to finish (atomic ticket) writes every
// count, tagged with the epoch, into every rank's mailbox, and a pending
// pipelined result is folded by the first block to finish (see peer.cuh).
#include "mk_common.cuh"
#include "peer.cuh"

namespace {

constexpr int kThreads = 1024;
constexpr int kBlocksPerSM = 2;
// Key vectors in flight per thread: 3 x 16 B x 2048 threads = 96 KiB per SM
// within the 32 registers that two 1024-thread blocks allow.  2^26 Zipf keys:
// 2 -> 3 took a graph step from 45.6 to 43.6 us (0.84 -> 0.87 of HBM); 768-
// thread blocks with 4 in flight measured the same, 5 or 6 in flight slower.
constexpr int kUnroll = 3;

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

// ---- exchange of u32 counts through the mailbox's histogram region --------

__device__ __forceinline__ unsigned long long* hist_region(unsigned long long* mailbox) {
  return reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(mailbox) + mk::kHistRegionOffset);
}

// Whole block: write this rank's counts of epoch e into every rank's
// mailbox, one tagged 8-byte word per bin and peer, no fence.
__device__ void hist_publish(const mk::PeerArgs& peer, unsigned long long e, const unsigned* counts,
                             uint32_t nbins) {
  const unsigned long long tag = (e & 0xffffffffull) << 32;
  const size_t row = ((size_t)(e % mk::kMailboxRing) * MK_MAX_PEERS + peer.rank) * mk::kHistMaxBins;
  for (uint32_t b = threadIdx.x; b < nbins; b += blockDim.x) {
    const unsigned long long w = tag | __ldcg(counts + b);
    for (int p = 0; p < peer.world; ++p)
      asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(hist_region(peer.slots[p]) + row + b), "l"(w)
                   : "memory");
  }
}

// Whole block: out[b] = sum over ranks (u32, wrapping) of rank q's count of
// `epoch`, waiting (bounded) for each word's tag.  A rank that never arrives
// is left out and sets ERRBIT_TIMEOUT.
__device__ void hist_fold(const mk::PeerArgs& peer, unsigned long long epoch, unsigned* out, uint32_t nbins,
                          unsigned* err) {
  const unsigned want = (unsigned)(epoch & 0xffffffffull);
  const unsigned long long* mine =
      hist_region(peer.slots[peer.rank]) + (size_t)(epoch % mk::kMailboxRing) * MK_MAX_PEERS * mk::kHistMaxBins;
  const long long t0 = clock64();
  bool late = false;
  for (uint32_t b = threadIdx.x; b < nbins; b += blockDim.x) {
    unsigned long long w[MK_MAX_PEERS];
#pragma unroll
    for (int q = 0; q < MK_MAX_PEERS; ++q)
      if (q < peer.world)
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[q]) : "l"(mine + (size_t)q * mk::kHistMaxBins + b)
                     : "memory");
    unsigned sum = 0u;
#pragma unroll
    for (int q = 0; q < MK_MAX_PEERS; ++q) {
      if (q >= peer.world) break;
      while ((unsigned)(w[q] >> 32) != want) {
        if ((unsigned long long)(clock64() - t0) > peer.limit) break;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[q]) : "l"(mine + (size_t)q * mk::kHistMaxBins + b)
                     : "memory");
      }
      if ((unsigned)(w[q] >> 32) == want) sum += (unsigned)w[q];
      else late = true;
    }
    out[b] = sum;
  }
  if (late) atomicOr(err, mk::ERRBIT_TIMEOUT);
}

// Whole block: if epoch e's histogram result is pending (pipelined), fold it
// into its output and clear the record.
__device__ void hist_complete_pending(const mk::PeerArgs& peer, unsigned long long e, unsigned* err) {
  if (e == 0) return;
  mk::PendingResult& r = peer.st->pend[e & 1];
  __shared__ unsigned long long s_re;
  __syncthreads();
  if (threadIdx.x == 0)
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(s_re) : "l"(&r.epoch) : "memory");
  __syncthreads();
  if (s_re != e) return;  // nothing pending (blocking call, or already written)
  hist_fold(peer, e, static_cast<unsigned*>(r.out), (uint32_t)r.op, err);
  __syncthreads();
  if (threadIdx.x == 0) r.epoch = 0;
}

// Finishes the pending pipelined histogram result (one block).
__global__ void __launch_bounds__(kThreads) hist_complete_kernel(const mk::PeerArgs peer, unsigned* __restrict__ err) {
  __shared__ unsigned long long s_e;
  if (threadIdx.x == 0) s_e = mk::peerdev::read_epoch(peer);
  __syncthreads();
  hist_complete_pending(peer, s_e, err);
}

// Int32 keys: two 1024-thread blocks per SM (32 registers a thread); the
// exchange code of the EXCH form would otherwise raise the count and halve
// the residency.  Int64 keys need more registers and are left unconstrained.
template <typename K, int BT, bool EXCH = false>
__global__ void __launch_bounds__(kThreads, sizeof(K) == 4 ? kBlocksPerSM : 1)
hist_smem(void* __restrict__ bins, uint32_t nbins, const K* __restrict__ keys, int64_t n, int head,
          unsigned* __restrict__ err, const mk::PeerArgs peer = mk::PeerArgs(), unsigned* __restrict__ ticket = nullptr,
          unsigned* __restrict__ global_out = nullptr) {
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
  if (EXCH) {
    // every block's flush is complete before its ticket is taken
    __threadfence();
    __syncthreads();
    __shared__ unsigned tk;
    __shared__ unsigned long long s_e;  // the channel's last published epoch E
    if (threadIdx.x == 0) {
      s_e = mk::peerdev::read_epoch(peer);  // before the ticket (see read_epoch)
      __threadfence();
      tk = atomicAdd(ticket, 1u);
    }
    __syncthreads();
    const bool fold_early = gridDim.x > 1;
    if (fold_early && tk == 0) hist_complete_pending(peer, s_e, err);
    if (tk == gridDim.x - 1) {
      __threadfence();
      if (threadIdx.x == 0) *ticket = 0u;  // re-arm for the next launch on this stream
      const unsigned long long e1 = s_e + 1;
      hist_publish(peer, e1, static_cast<const unsigned*>(bins), nbins);
      if (!fold_early) hist_complete_pending(peer, s_e, err);
      if (peer.mode == mk::XMODE_BLOCKING) hist_fold(peer, e1, global_out, nbins, err);
      __syncthreads();
      if (threadIdx.x == 0) mk::peerdev::finish_epoch(peer, e1);
    }
  }
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

namespace {

int hist_allreduce(bool blocking, uint32_t* global_out, uint32_t* counts, int32_t nbins, const int32_t* keys1,
                   int64_t n, void* stream) {
  MK_ENTRY_DEVICE(dev);
  const char* who = blocking ? "mk_hist_u32_allreduce" : "mk_hist_u32_allreduce_async";
  // argument errors before an epoch is taken, so a rejected call leaves the
  // ranks' epoch counters in step
  if (n < 0) return mk::fail(MK_ERR_INVALID, std::string(who) + ": n must be >= 0");
  if (nbins < 1 || nbins > mk::kHistMaxBins)
    return mk::fail(MK_ERR_INVALID, std::string(who) + ": need 1 <= nbins <= " + std::to_string(mk::kHistMaxBins));
  if (!global_out || !counts || (n > 0 && !keys1)) return mk::fail(MK_ERR_INVALID, std::string(who) + ": null pointer");
  if ((reinterpret_cast<uintptr_t>(keys1) & 3u) != 0 || (reinterpret_cast<uintptr_t>(counts) & 3u) != 0)
    return mk::fail(MK_ERR_INVALID, std::string(who) + ": misaligned keys or counts");
  const int64_t smem = (int64_t)nbins * 4;
  if (smem > dev->max_smem_optin / kBlocksPerSM - 1024)
    return mk::fail(MK_ERR_INVALID, std::string(who) + ": too many bins for the shared-memory kernel");
  cudaStream_t s = mk::as_stream(stream);
  mk::ReduceScratch rs;
  int rc = mk::reduce_scratch(dev, s, &rs);
  if (rc != MK_OK) return rc;
  rc = mk::allow_dynamic_smem(reinterpret_cast<const void*>(hist_smem<int32_t, MK_BIN_U32, true>), (size_t)smem);
  if (rc != MK_OK) return rc;
  mk::PeerArgs peer;
  rc = mk::peer_args(dev, mk::CH_HIST, blocking ? mk::XMODE_BLOCKING : mk::XMODE_PIPELINED, global_out, nbins, 0.0,
                     &peer);
  if (rc != MK_OK) return rc;
  int64_t head = n > 0 ? (int64_t)(((16u - (reinterpret_cast<uintptr_t>(keys1) & 15u)) & 15u) / 4u) : 0;
  if (head > n) head = n;
  int64_t blocks = mk::cdiv(n, (int64_t)kThreads * 16);
  if (blocks > (int64_t)dev->sms * kBlocksPerSM) blocks = (int64_t)dev->sms * kBlocksPerSM;
  if (blocks < 1) blocks = 1;
  hist_smem<int32_t, MK_BIN_U32, true><<<(unsigned)blocks, kThreads, (size_t)smem, s>>>(
      counts, (uint32_t)nbins, keys1, n, (int)head, dev->err_word, peer, rs.ticket, global_out);
  return mk::check_launch(who);
}

}  // namespace

extern "C" int mk_hist_u32_allreduce(uint32_t* global_out, uint32_t* counts, int32_t nbins, const int32_t* keys1,
                                     int64_t n, void* stream) {
  return hist_allreduce(true, global_out, counts, nbins, keys1, n, stream);
}

extern "C" int mk_hist_u32_allreduce_async(uint32_t* global_out, uint32_t* counts, int32_t nbins,
                                           const int32_t* keys1, int64_t n, void* stream) {
  return hist_allreduce(false, global_out, counts, nbins, keys1, n, stream);
}

extern "C" int mk_hist_allreduce_complete(void* stream) {
  MK_ENTRY_DEVICE(dev);
  mk::PeerArgs peer;
  int rc = mk::peer_args(dev, mk::CH_HIST, mk::XMODE_COMPLETE, nullptr, 0, 0.0, &peer);
  if (rc != MK_OK) return rc;
  hist_complete_kernel<<<1, kThreads, 0, mk::as_stream(stream)>>>(peer, dev->err_word);
  return mk::check_launch("mk_hist_allreduce_complete: launch");
}
