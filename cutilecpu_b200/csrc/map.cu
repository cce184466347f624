// map.cu — elementwise maps beyond vadd: out = alpha*x + beta*y (fp32), the
// closures of AK.map!(x -> 2f0 * x, dst, src) (test/test_downstream_ka.jl:18-20)
// and of GPUArrays broadcasts such as 2f0 .* a and a .+ b
// (test/test_gpuarrays.jl:31-32).  Computed in Julia's order without FMA
// contraction, fl(fl(alpha*x) + fl(beta*y)), so it is bit-exact with the
// reference; with y == NULL the result is fl(alpha*x).  Same memory design as
// vadd: 16-byte vectors, streaming hints, a grid that fills every SM once.
#include "mk_common.cuh"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float ax_by(float a, float x, float b, float y, bool has_y) {
  const float ax = __fmul_rn(a, x);
  return has_y ? __fadd_rn(ax, __fmul_rn(b, y)) : ax;
}

template <bool HAS_Y>
__global__ void __launch_bounds__(kThreads)
axpby_vec4(float4* __restrict__ out, float a, const float4* __restrict__ x, float b, const float4* __restrict__ y,
           int64_t n4) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n4; i += stride) {
    const float4 u = __ldcs(x + i);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (HAS_Y) v = __ldcs(y + i);
    __stcs(out + i, make_float4(ax_by(a, u.x, b, v.x, HAS_Y), ax_by(a, u.y, b, v.y, HAS_Y),
                                ax_by(a, u.z, b, v.z, HAS_Y), ax_by(a, u.w, b, v.w, HAS_Y)));
  }
}

__global__ void __launch_bounds__(kThreads)
axpby_scalar(float* __restrict__ out, float a, const float* __restrict__ x, float b, const float* __restrict__ y,
             int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride)
    out[i] = ax_by(a, x[i], b, y ? y[i] : 0.0f, y != nullptr);
}

}  // namespace

extern "C" int mk_axpby_f32(float* out, float alpha, const float* x, float beta, const float* y, int64_t n,
                            void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n < 0) return mk::fail(MK_ERR_INVALID, "mk_axpby_f32: n must be >= 0");
  if (n == 0) return MK_OK;
  if (!out || !x) return mk::fail(MK_ERR_INVALID, "mk_axpby_f32: null pointer");
  cudaStream_t s = mk::as_stream(stream);
  const int64_t max_blocks = (int64_t)dev->sms * (2048 / kThreads);
  if (mk::aligned16(out) && mk::aligned16(x) && (!y || mk::aligned16(y))) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      int64_t blocks = mk::cdiv(n4, kThreads);
      if (blocks > max_blocks) blocks = max_blocks;
      auto* o4 = reinterpret_cast<float4*>(out);
      auto* x4 = reinterpret_cast<const float4*>(x);
      if (y)
        axpby_vec4<true><<<(unsigned)blocks, kThreads, 0, s>>>(o4, alpha, x4, beta, reinterpret_cast<const float4*>(y), n4);
      else
        axpby_vec4<false><<<(unsigned)blocks, kThreads, 0, s>>>(o4, alpha, x4, beta, nullptr, n4);
    }
    const int64_t done = n4 * 4;
    if (done < n)
      axpby_scalar<<<1, kThreads, 0, s>>>(out + done, alpha, x + done, beta, y ? y + done : nullptr, n - done);
  } else {
    int64_t blocks = mk::cdiv(n, kThreads);
    if (blocks > max_blocks) blocks = max_blocks;
    axpby_scalar<<<(unsigned)blocks, kThreads, 0, s>>>(out, alpha, x, beta, y, n);
  }
  return mk::check_launch("mk_axpby_f32: launch");
}
