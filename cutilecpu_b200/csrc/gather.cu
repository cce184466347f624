// gather.cu — c[i] = a[idx[i]] with 1-based Int32 indices: the indirect load
// the reference lowers to two scalar loads per thread on the GPU
// (src/lower.jl:4110-4115) and to `vector.gather` on the CPU (:4134-4140), with
// the 1-based -> 0-based shift of :4064-4077.
//
// Design: the index and output streams are read/written as 16-byte vectors with
// streaming hints; the data loads are independent 4-byte loads cached in L2
// only (no reuse across a random stream), kUnroll x 4 of them in flight per
// thread so enough 32-byte sectors are outstanding to cover HBM latency.
// Algorithmic traffic 12 B/element; the device moves >= 40 B/element (a whole
// 32-byte sector per random 4-byte read) unless `a` is L2-resident.
// Out-of-range indices (reference: BoundsError -> KernelException) write 0 and
// raise bit ERRBIT_GATHER_INDEX of the device error word.
#include "mk_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;  // int4 index vectors per thread per iteration

// The random reads of `a` bypass L1 (no reuse) and are cached in L2 only
// (.cg).  Measured against .nc.L1::no_allocate, plain, .cs and an .L2::64B
// prefetch hint: .cg and plain were fastest (2.64 vs 2.77 ms at 2^27).
template <int LD>
__device__ __forceinline__ float load_rand(const float* p) {
  return __ldcg(p);
}

template <int LD>
__device__ __forceinline__ float fetch(const float* __restrict__ a, uint64_t na, int32_t k1, bool& bad) {
  const uint64_t k = (uint64_t)(int64_t)k1 - 1u;  // 1-based -> 0-based; <1 wraps to huge
  if (k < na) return load_rand<LD>(a + k);
  bad = true;
  return 0.0f;
}

template <int LD>
__global__ void __launch_bounds__(kThreads)
gather_f32_vec4(float4* __restrict__ c, const float* __restrict__ a, uint64_t na,
                const int4* __restrict__ idx, int64_t n4, unsigned* __restrict__ err) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  bool bad = false;
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    int4 k[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) k[u] = __ldcs(idx + i + u * stride);
    float4 r[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      r[u].x = fetch<LD>(a, na, k[u].x, bad);
      r[u].y = fetch<LD>(a, na, k[u].y, bad);
      r[u].z = fetch<LD>(a, na, k[u].z, bad);
      r[u].w = fetch<LD>(a, na, k[u].w, bad);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) __stcs(c + i + u * stride, r[u]);
  }
  for (; i < n4; i += stride) {
    int4 k = __ldcs(idx + i);
    float4 r;
    r.x = fetch<LD>(a, na, k.x, bad);
    r.y = fetch<LD>(a, na, k.y, bad);
    r.z = fetch<LD>(a, na, k.z, bad);
    r.w = fetch<LD>(a, na, k.w, bad);
    __stcs(c + i, r);
  }
  if (bad) atomicOr(err, mk::ERRBIT_GATHER_INDEX);
}

template <int LD>
__global__ void __launch_bounds__(kThreads)
gather_f32_scalar(float* __restrict__ c, const float* __restrict__ a, uint64_t na,
                  const int32_t* __restrict__ idx, int64_t n, unsigned* __restrict__ err) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  bool bad = false;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride)
    c[i] = fetch<LD>(a, na, idx[i], bad);
  if (bad) atomicOr(err, mk::ERRBIT_GATHER_INDEX);
}

template <int LD>
void launch_vec4(unsigned blocks, cudaStream_t s, float* c, const float* a, int64_t na, const int32_t* idx1,
                 int64_t n4, unsigned* err) {
  gather_f32_vec4<LD><<<blocks, kThreads, 0, s>>>(reinterpret_cast<float4*>(c), a, (uint64_t)na,
                                                  reinterpret_cast<const int4*>(idx1), n4, err);
}

}  // namespace

extern "C" int mk_gather_f32(float* c, const float* a, int64_t na, const int32_t* idx1, int64_t n,
                             void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n < 0 || na < 0) return mk::fail(MK_ERR_INVALID, "mk_gather_f32: sizes must be >= 0");
  if (n == 0) return MK_OK;
  if (!c || !idx1 || (na > 0 && !a)) return mk::fail(MK_ERR_INVALID, "mk_gather_f32: null pointer");
  cudaStream_t s = mk::as_stream(stream);
  const int64_t max_blocks = (int64_t)dev->sms * (2048 / kThreads);
  if (mk::aligned16(c) && mk::aligned16(idx1)) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      int64_t blocks = mk::cdiv(n4, kThreads);
      if (blocks > max_blocks) blocks = max_blocks;
      launch_vec4<1>((unsigned)blocks, s, c, a, na, idx1, n4, dev->err_word);
    }
    const int64_t done = n4 * 4;
    if (done < n)
      gather_f32_scalar<0><<<1, kThreads, 0, s>>>(c + done, a, (uint64_t)na, idx1 + done, n - done,
                                               dev->err_word);
  } else {
    int64_t blocks = mk::cdiv(n, kThreads);
    if (blocks > max_blocks) blocks = max_blocks;
    gather_f32_scalar<0><<<(unsigned)blocks, kThreads, 0, s>>>(c, a, (uint64_t)na, idx1, n, dev->err_word);
  }
  return mk::check_launch("mk_gather_f32: launch");
}

// ---------------------------------------------------------------------------
// Random-read probe: the device's ceiling for the gather's dominant cost.
// n independent 4-byte reads of a[h(i) mod na] with h a 32-bit integer hash of
// the element number, the same loads (.cg, 8 in flight per thread) and grid as
// gather_f32_vec4, but no index stream and no output stream: what is left is
// the random-read rate of this GPU's memory system for an array of na floats.
// Each block writes one u32 (XOR of the bits it read) so no load is dead code.
// ---------------------------------------------------------------------------
namespace {

// Integer finaliser of MurmurHash3 (Appleby, public domain): a bijection of
// u32 with full avalanche, so consecutive i land on unrelated lines.
__device__ __forceinline__ uint32_t mix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x85ebca6bu;
  h ^= h >> 13;
  h *= 0xc2b2ae35u;
  h ^= h >> 16;
  return h;
}

__global__ void __launch_bounds__(kThreads)
random_read_probe(unsigned* __restrict__ sums, const float* __restrict__ a, uint64_t na, int64_t n, uint32_t seed) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  constexpr int kInFlight = 4 * kUnroll;
  unsigned acc = 0;
  for (; i + (kInFlight - 1) * stride < n; i += kInFlight * stride) {
    float v[kInFlight];
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const uint32_t h = mix32((uint32_t)(i + u * stride) ^ seed);
      v[u] = __ldcg(a + (uint64_t)(((uint64_t)h * na) >> 32));
    }
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) acc ^= __float_as_uint(v[u]);
  }
  for (; i < n; i += stride) acc ^= __float_as_uint(__ldcg(a + (((uint64_t)mix32((uint32_t)i ^ seed) * na) >> 32)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ unsigned part[kThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned r = 0;
    for (int w = 0; w < kThreads / 32; ++w) r ^= part[w];
    sums[blockIdx.x] = r;
  }
}

}  // namespace

extern "C" int mk_probe_random_read_f32(unsigned* sums, int64_t sums_len, const float* a, int64_t na, int64_t n,
                                        unsigned seed, void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n < 0 || na <= 0 || na > (int64_t)UINT32_MAX)
    return mk::fail(MK_ERR_INVALID, "mk_probe_random_read_f32: need n >= 0 and 0 < na < 2^32");
  if (!sums || !a) return mk::fail(MK_ERR_INVALID, "mk_probe_random_read_f32: null pointer");
  const int64_t blocks = (int64_t)dev->sms * (2048 / kThreads);
  if (sums_len < blocks)
    return mk::fail(MK_ERR_INVALID, "mk_probe_random_read_f32: sums must hold " + std::to_string(blocks) +
                                        " values (SMs x 8)");
  if (n == 0) return MK_OK;
  random_read_probe<<<(unsigned)blocks, kThreads, 0, mk::as_stream(stream)>>>(sums, a, (uint64_t)na, n, seed);
  return mk::check_launch("mk_probe_random_read_f32: launch");
}
