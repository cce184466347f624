// gather.cu — c[i] = a[idx[i]] with 1-based Int32 indices: the indirect load
// the reference lowers to two scalar loads per thread on the GPU
// (src/lower.jl:4110-4115) and to `vector.gather` on the CPU (:4134-4140), with
// the 1-based -> 0-based shift of :4064-4077.
//
// Design: the index and output streams are read/written as 16-byte vectors with
// streaming hints; the data loads are independent 4-byte read-only loads that
// skip L1 (no reuse across a random stream), kUnroll x 4 of them in flight per
// thread so enough 32-byte sectors are outstanding to cover HBM latency.
// Algorithmic traffic 12 B/element; the device moves >= 40 B/element (a whole
// 32-byte sector per random 4-byte read) unless `a` is L2-resident.
// Out-of-range indices (reference: BoundsError -> KernelException) write 0 and
// raise bit ERRBIT_GATHER_INDEX of the device error word.
#include <stdlib.h>

#include "mk_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;  // int4 index vectors per thread per iteration

// Load flavours for the random reads of `a` (tuning knob MK_TUNE_GATHER_LOAD).
template <int LD>
__device__ __forceinline__ float load_rand(const float* p) {
  float v;
  if (LD == 0) {
    asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
  } else if (LD == 1) {
    v = __ldcg(p);
  } else if (LD == 2) {
    asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
  } else if (LD == 3) {
    v = __ldcs(p);
  } else {
    asm volatile("ld.global.cg.L2::64B.f32 %0, [%1];" : "=f"(v) : "l"(p));
  }
  return v;
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

int load_flavour() {
  static int v = [] {
    const char* e = getenv("MK_TUNE_GATHER_LOAD");
    int b = e ? atoi(e) : 0;
    return (b >= 0 && b <= 4) ? b : 0;
  }();
  return v;
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
  static int l2_fetch_done = [] {
    const char* e = getenv("MK_TUNE_L2_FETCH");
    if (e) cudaDeviceSetLimit(cudaLimitMaxL2FetchGranularity, (size_t)atoi(e));
    return 1;
  }();
  (void)l2_fetch_done;
  const int64_t max_blocks = (int64_t)dev->sms * (2048 / kThreads);
  if (mk::aligned16(c) && mk::aligned16(idx1)) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      int64_t blocks = mk::cdiv(n4, kThreads);
      if (blocks > max_blocks) blocks = max_blocks;
      switch (load_flavour()) {
        case 1: launch_vec4<1>((unsigned)blocks, s, c, a, na, idx1, n4, dev->err_word); break;
        case 2: launch_vec4<2>((unsigned)blocks, s, c, a, na, idx1, n4, dev->err_word); break;
        case 3: launch_vec4<3>((unsigned)blocks, s, c, a, na, idx1, n4, dev->err_word); break;
        case 4: launch_vec4<4>((unsigned)blocks, s, c, a, na, idx1, n4, dev->err_word); break;
        default: launch_vec4<0>((unsigned)blocks, s, c, a, na, idx1, n4, dev->err_word); break;
      }
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
