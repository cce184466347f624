// reduce_ops.cuh — the element maps and reduction operators shared by the
// full reduction (mapreduce.cu) and the single-dimension reduction
// (mapreduce_dims.cu).  Julia semantics: max/min propagate NaN and order
// -0.0 < +0.0 (Base.max/min on Float32, what `maximum`/`minimum` use).
#pragma once

#include <math.h>

#include "mk_common.cuh"

namespace mk {
namespace rops {

__device__ __forceinline__ float mapf(int f, float v) {
  switch (f) {
    case MK_F_ABS2: return __fmul_rn(v, v);
    case MK_F_ABS: return fabsf(v);
    case MK_F_GT0: return v > 0.0f ? 1.0f : 0.0f;
    default: return v;
  }
}

__device__ __forceinline__ double jl_max(double a, double b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
__device__ __forceinline__ double jl_min(double a, double b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}

template <int OP>
__device__ __forceinline__ double combine(double a, double b) {
  if (OP == MK_OP_ADD) return a + b;
  if (OP == MK_OP_MUL) return a * b;
  if (OP == MK_OP_MAX) return jl_max(a, b);
  return jl_min(a, b);
}

template <int OP>
__device__ __forceinline__ double neutral() {
  if (OP == MK_OP_ADD) return 0.0;
  if (OP == MK_OP_MUL) return 1.0;
  if (OP == MK_OP_MAX) return -INFINITY;
  return INFINITY;
}

// fp32 forms (same semantics) for kernels that combine Float32 values.
__device__ __forceinline__ float jl_max32(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
__device__ __forceinline__ float jl_min32(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}

template <int OP>
__device__ __forceinline__ float combine32(float a, float b) {
  if (OP == MK_OP_ADD) return __fadd_rn(a, b);
  if (OP == MK_OP_MUL) return __fmul_rn(a, b);
  if (OP == MK_OP_MAX) return jl_max32(a, b);
  return jl_min32(a, b);
}

template <int OP>
__device__ __forceinline__ float neutral32() {
  if (OP == MK_OP_ADD) return 0.0f;
  if (OP == MK_OP_MUL) return 1.0f;
  if (OP == MK_OP_MAX) return -INFINITY;
  return INFINITY;
}

}  // namespace rops
}  // namespace mk
