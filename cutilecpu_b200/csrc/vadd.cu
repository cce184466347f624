// vadd.cu — c[i] = a[i] + b[i] (fp32), the elementwise map of the reference's
// vadd kernel (test/test_gpu_simt.jl:13-16, examples/reflection_and_perf.jl:11-14).
//
// The reference lowers it to one scalar 4-byte load/store per thread with a
// masked tail (src/lower.jl:4110-4115, 4170-4174, valid_index :1895-1915).
// Here: 16-byte vector loads/stores, two float4 pairs in flight per thread,
// streaming (evict-first) cache hints, grid sized to fill every SM once and
// grid-striding beyond that.  Pure HBM traffic: 12 bytes per element.
#include "mk_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;  // float4 per operand in flight per thread

__global__ void __launch_bounds__(kThreads)
vadd_f32_vec4(float4* __restrict__ c, const float4* __restrict__ a,
              const float4* __restrict__ b, int64_t n4) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  // Main body: kUnroll independent loads per operand before any store.
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    float4 va[kUnroll], vb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      va[u] = __ldcs(a + i + u * stride);
      vb[u] = __ldcs(b + i + u * stride);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float4 r;
      r.x = __fadd_rn(va[u].x, vb[u].x);
      r.y = __fadd_rn(va[u].y, vb[u].y);
      r.z = __fadd_rn(va[u].z, vb[u].z);
      r.w = __fadd_rn(va[u].w, vb[u].w);
      __stcs(c + i + u * stride, r);
    }
  }
  for (; i < n4; i += stride) {
    float4 va = __ldcs(a + i), vb = __ldcs(b + i), r;
    r.x = __fadd_rn(va.x, vb.x);
    r.y = __fadd_rn(va.y, vb.y);
    r.z = __fadd_rn(va.z, vb.z);
    r.w = __fadd_rn(va.w, vb.w);
    __stcs(c + i, r);
  }
}

// Scalar form: the <4-element tail of the vector path, and any call whose
// three pointers are not all 16-byte aligned (e.g. views at odd offsets).
__global__ void __launch_bounds__(kThreads)
vadd_f32_scalar(float* __restrict__ c, const float* __restrict__ a,
                const float* __restrict__ b, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride)
    c[i] = __fadd_rn(a[i], b[i]);
}

}  // namespace

extern "C" int mk_vadd_f32(float* c, const float* a, const float* b, int64_t n, void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n < 0) return mk::fail(MK_ERR_INVALID, "mk_vadd_f32: n must be >= 0");
  if (n == 0) return MK_OK;
  if (!c || !a || !b) return mk::fail(MK_ERR_INVALID, "mk_vadd_f32: null pointer");
  cudaStream_t s = mk::as_stream(stream);
  const int64_t max_blocks = (int64_t)dev->sms * (2048 / kThreads);
  if (mk::aligned16(a) && mk::aligned16(b) && mk::aligned16(c)) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      int64_t blocks = mk::cdiv(n4, kThreads);
      if (blocks > max_blocks) blocks = max_blocks;
      vadd_f32_vec4<<<(unsigned)blocks, kThreads, 0, s>>>(
          reinterpret_cast<float4*>(c), reinterpret_cast<const float4*>(a),
          reinterpret_cast<const float4*>(b), n4);
    }
    const int64_t done = n4 * 4;
    if (done < n) vadd_f32_scalar<<<1, kThreads, 0, s>>>(c + done, a + done, b + done, n - done);
  } else {
    int64_t blocks = mk::cdiv(n, kThreads);
    if (blocks > max_blocks) blocks = max_blocks;
    vadd_f32_scalar<<<(unsigned)blocks, kThreads, 0, s>>>(c, a, b, n);
  }
  return mk::check_launch("mk_vadd_f32: launch");
}
