// findext.cu — findmax / findmin (and argmax / argmin) of a Float32 vector:
// the (value, index) reductions of GPUArrays on an MLIRArray
// (test/test_gpuarrays.jl:124-128), in one launch.
//
// Julia's order is used: findmax treats NaN as greater than every other value,
// findmin treats NaN as smaller than every other value, +0.0 ranks above -0.0,
// and among equal candidates the first (lowest) index wins.  Each thread keeps
// its best (value, index) over a grid-stride sweep with 16-byte loads, warps
// and blocks combine with the same rule, and the last block (atomic ticket)
// folds the block candidates in block order.  The returned index is 1-based.
#include "mk_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kVec = 8;  // float4 loads in flight per thread
// Minimum resident blocks per SM the register budget is fitted to: 4 leaves
// 62 registers, so the eight vectors, the four candidate chains and their
// 64-bit indices stay in registers.  At 6 (40 registers) the chains spilled
// and findmax over 2^28 ran 0.191 ms (0.88 of HBM); at 4, 0.183 ms (0.92);
// 5 measured 0.185 ms, six vectors at 6 per SM 0.194 ms.
constexpr int kMinBlocks = 4;

struct Cand {
  float v;
  int64_t i;
};

// Is a strictly better than b (as the candidate to keep)?
template <bool MAX>
__device__ __forceinline__ bool better(float a, int64_t ia, float b, int64_t ib) {
  const bool na = a != a, nb = b != b;
  if (na || nb) {
    if (na && nb) return ia < ib;
    return na;  // NaN wins for both findmax and findmin
  }
  if (a == b) {
    const bool sa = signbit(a), sb = signbit(b);
    if (sa != sb) return MAX ? !sa : sa;  // +0.0 above -0.0
    return ia < ib;
  }
  return MAX ? a > b : a < b;
}

// Julia's order as an unsigned key, larger = preferred: the float bits made
// monotone (negative values complemented, so -0 ranks below +0), complemented
// again for findmin, and every NaN mapped to the largest key (NaN wins both).
// No value maps to 0.
template <bool MAX>
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  if (!MAX) k = ~k;
  return v != v ? 0xFFFFFFFFu : k;
}

// The value a key came from (every NaN comes back as the canonical NaN).
template <bool MAX>
__device__ __forceinline__ float key_value(uint32_t k) {
  if (k == 0xFFFFFFFFu) return __uint_as_float(0x7FC00000u);
  if (!MAX) k = ~k;
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

template <bool MAX>
__device__ __forceinline__ void keep(Cand& c, float v, int64_t i) {
  if (better<MAX>(v, i, c.v, c.i)) c = {v, i};
}

template <bool MAX>
__device__ __forceinline__ Cand warp_best(Cand c) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, c.v, o);
    const int64_t i = __shfl_xor_sync(0xffffffffu, c.i, o);
    keep<MAX>(c, v, i);
  }
  return c;
}

template <bool MAX>
__device__ Cand block_best(Cand c, Cand* sm) {
  c = warp_best<MAX>(c);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sm[warp] = c;
  __syncthreads();
  if (warp == 0) {
    c = lane < kThreads / 32 ? sm[lane] : Cand{MAX ? -INFINITY : INFINITY, INT64_MAX};
    c = warp_best<MAX>(c);
  }
  __syncthreads();
  return c;  // valid in thread 0
}

template <bool MAX>
__global__ void __launch_bounds__(kThreads, kMinBlocks)
findext_kernel(const float* __restrict__ x, int64_t n, int head, float* __restrict__ pv, int64_t* __restrict__ pi,
               unsigned* __restrict__ ticket, double* __restrict__ val_out, int64_t* __restrict__ idx_out) {
  __shared__ Cand sm[kThreads / 32];
  __shared__ bool is_last;
  const int64_t tid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  // start from the worst possible candidate: an index past every real one
  Cand c{MAX ? -INFINITY : INFINITY, INT64_MAX};
  const float4* x4 = reinterpret_cast<const float4*>(x + head);
  const int64_t n4 = (n - head) / 4;
  {
    // One candidate per vector lane, kVec vectors in flight.  Each value is
    // ranked by an unsigned key in Julia's order (see order_key), so a step is
    // one compare; a chain visits increasing indices, so the strict compare
    // keeps the first index among equals.  Chains and threads then combine
    // with the same rule (greater key, else lower index).
    uint32_t bk[4] = {0u, 0u, 0u, 0u};  // 0: no candidate (no value maps to 0)
    int64_t bi[4] = {INT64_MAX, INT64_MAX, INT64_MAX, INT64_MAX};
    auto step = [&](int l, float v, int64_t e) {
      const uint32_t k = order_key<MAX>(v);
      if (k > bk[l]) {
        bk[l] = k;
        bi[l] = e;
      }
    };
    int64_t i = tid;
    for (; i + (kVec - 1) * stride < n4; i += kVec * stride) {
      float4 q[kVec];
#pragma unroll
      for (int u = 0; u < kVec; ++u) q[u] = __ldcs(x4 + i + u * stride);
#pragma unroll
      for (int u = 0; u < kVec; ++u) {
        const int64_t e = head + 4 * (i + u * stride);
        step(0, q[u].x, e);
        step(1, q[u].y, e + 1);
        step(2, q[u].z, e + 2);
        step(3, q[u].w, e + 3);
      }
    }
    for (; i < n4; i += stride) {
      const float4 q = __ldcs(x4 + i);
      const int64_t e = head + 4 * i;
      step(0, q.x, e);
      step(1, q.y, e + 1);
      step(2, q.z, e + 2);
      step(3, q.w, e + 3);
    }
#pragma unroll
    for (int l = 0; l < 4; ++l)
      if (bk[l] != 0u) keep<MAX>(c, key_value<MAX>(bk[l]), bi[l]);
  }
  const int64_t tail = head + 4 * n4;
  if (tid < head) keep<MAX>(c, x[tid], tid);
  if (tid < n - tail) keep<MAX>(c, x[tail + tid], tail + tid);
  c = block_best<MAX>(c, sm);
  if (threadIdx.x == 0) {
    pv[blockIdx.x] = c.v;
    pi[blockIdx.x] = c.i;
    __threadfence();
    is_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  Cand b{MAX ? -INFINITY : INFINITY, INT64_MAX};
  for (int k = threadIdx.x; k < (int)gridDim.x; k += kThreads) keep<MAX>(b, __ldcg(pv + k), __ldcg(pi + k));
  b = block_best<MAX>(b, sm);
  if (threadIdx.x == 0) {
    val_out[0] = (double)b.v;
    idx_out[0] = b.i + 1;
    *ticket = 0u;
  }
}

template <typename Kernel>
int resident_per_sm(Kernel k) {
  int b = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k, kThreads, 0) != cudaSuccess || b < 1) b = 1;
  return b;
}

}  // namespace

extern "C" int mk_findext_f32(double* val_out, int64_t* idx_out, const float* x, int64_t n, int find_max,
                              void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n <= 0) return mk::fail(MK_ERR_INVALID, "mk_findext_f32: collection must be non-empty");
  if (!val_out || !idx_out || !x) return mk::fail(MK_ERR_INVALID, "mk_findext_f32: null pointer");
  if ((reinterpret_cast<uintptr_t>(x) & 3u) != 0) return mk::fail(MK_ERR_INVALID, "mk_findext_f32: misaligned x");
  cudaStream_t s = mk::as_stream(stream);
  constexpr int kMaxBlocks = 2048;
  void* ws = nullptr;
  // [ticket (256 B) | values | indices]; the ticket is re-armed by every call
  int rc = mk::stream_workspace(dev, s, 256 + kMaxBlocks * 12 + 256, &ws, mk::WS_FIND);
  if (rc != MK_OK) return rc;
  char* b = static_cast<char*>(ws);
  unsigned* ticket = reinterpret_cast<unsigned*>(b);
  int64_t* pi = reinterpret_cast<int64_t*>(b + 256);
  float* pv = reinterpret_cast<float*>(b + 256 + kMaxBlocks * 8);
  cudaError_t e = cudaMemsetAsync(ticket, 0, 4, s);
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_findext_f32: ticket");
  int64_t head = (int64_t)(((16u - (reinterpret_cast<uintptr_t>(x) & 15u)) & 15u) / 4u);
  if (head > n) head = n;
  // persistent grid: as many blocks as are resident at once (one wave)
  static const int per_sm[2] = {resident_per_sm(findext_kernel<false>), resident_per_sm(findext_kernel<true>)};
  int64_t blocks = mk::cdiv(n, (int64_t)kThreads * 16);
  int64_t cap = (int64_t)dev->sms * per_sm[find_max ? 1 : 0];
  if (cap > kMaxBlocks) cap = kMaxBlocks;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (find_max)
    findext_kernel<true><<<(unsigned)blocks, kThreads, 0, s>>>(x, n, (int)head, pv, pi, ticket, val_out, idx_out);
  else
    findext_kernel<false><<<(unsigned)blocks, kThreads, 0, s>>>(x, n, (int)head, pv, pi, ticket, val_out, idx_out);
  return mk::check_launch("mk_findext_f32: launch");
}
