// mapreduce_dims.cu — reduction of ONE dimension of a column-major Float32
// array: the dims form of GPUArrays.mapreducedim! (ext/MLIRCUDAExt.jl:114-119,
// `sum(m; dims=d)`, `maximum(m; dims=d)`, test/test_gpuarrays.jl:98-107).
//
// The array is viewed as (pre, len, post) with the reduced dimension in the
// middle (pre = product of the dims before it, post = after it):
//     out[p + q*pre] = op(init, op_k f(x[p + k*pre + q*pre*len]))
// Two shapes of parallelism, both accumulating in fp64 (max/min exact) and
// rounding once to Float32:
//   * pre == 1 (dims=1): each output is a contiguous segment; a warp (or, for
//     few long segments, a 256-thread block) strides it with coalesced 16-byte
//     loads, four in flight per thread;
//   * pre > 1: one thread per p walks k with loads coalesced across p, four
//     k-steps in flight.  When
//     pre*post threads cannot fill the GPU, k is cut into chunks whose fp64
//     partials go to a per-stream workspace and are folded in chunk order by
//     a second launch, so results stay deterministic.
#include "mk_common.cuh"
#include "reduce_ops.cuh"

namespace {

using namespace mk::rops;

template <int F, int OP>
__device__ __forceinline__ double fold(double acc, float v) {
  return combine<OP>(acc, (double)mapf(F, v));
}

template <int OP>
__device__ __forceinline__ double warp_reduce(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = combine<OP>(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Fold of one contiguous segment by `nt` cooperating threads (index i): the
// scalar head up to the first 16-byte boundary, then float4 vectors with four
// in flight per thread into four accumulators (a fixed order, so the result
// is deterministic), then the scalar tail.  Returns this thread's partial.
template <int F, int OP>
__device__ __forceinline__ double fold_segment(const float* __restrict__ seg, int64_t len, int i, int nt) {
  double a0 = neutral<OP>(), a1 = neutral<OP>(), a2 = neutral<OP>(), a3 = neutral<OP>();
  int64_t h = (int64_t)(((16u - (reinterpret_cast<uintptr_t>(seg) & 15u)) & 15u) / 4u);
  if (h > len) h = len;
  if (i < h) a0 = fold<F, OP>(a0, __ldcs(seg + i));
  const float4* v = reinterpret_cast<const float4*>(seg + h);
  const int64_t n4 = (len - h) / 4;
  auto fold4 = [](double a, float4 q) {
    a = fold<F, OP>(a, q.x);
    a = fold<F, OP>(a, q.y);
    a = fold<F, OP>(a, q.z);
    return fold<F, OP>(a, q.w);
  };
  int64_t j = i;
  for (; j + 3 * nt < n4; j += 4 * nt) {
    const float4 q0 = __ldcs(v + j), q1 = __ldcs(v + j + nt), q2 = __ldcs(v + j + 2 * nt),
                 q3 = __ldcs(v + j + 3 * nt);
    a0 = fold4(a0, q0);
    a1 = fold4(a1, q1);
    a2 = fold4(a2, q2);
    a3 = fold4(a3, q3);
  }
  for (; j < n4; j += nt) a0 = fold4(a0, __ldcs(v + j));
  const int64_t tail = h + 4 * n4;
  for (int64_t k = tail + i; k < len; k += nt) a1 = fold<F, OP>(a1, __ldcs(seg + k));
  return combine<OP>(combine<OP>(a0, a1), combine<OP>(a2, a3));
}

// pre == 1, a warp per segment.
template <int F, int OP>
__global__ void __launch_bounds__(256) seg_warp(float* __restrict__ out, const float* __restrict__ x, int64_t len,
                                                int64_t post, double init) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * 8;
  for (int64_t q = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); q < post; q += warps) {
    double acc = fold_segment<F, OP>(x + q * len, len, lane, 32);
    acc = warp_reduce<OP>(acc);
    if (lane == 0) out[q] = (float)combine<OP>(init, acc);
  }
}

// pre == 1, a 256-thread block per segment (few, long segments).
template <int F, int OP>
__global__ void __launch_bounds__(256) seg_block(float* __restrict__ out, const float* __restrict__ x, int64_t len,
                                                 int64_t post, double init) {
  __shared__ double sm[8];
  for (int64_t q = blockIdx.x; q < post; q += gridDim.x) {
    double acc = fold_segment<F, OP>(x + q * len, len, threadIdx.x, 256);
    acc = warp_reduce<OP>(acc);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
      double v = threadIdx.x < 8 ? sm[threadIdx.x] : neutral<OP>();
      v = warp_reduce<OP>(v);
      if (threadIdx.x == 0) out[q] = (float)combine<OP>(init, v);
    }
    __syncthreads();
  }
}

// pre > 1: thread per (p, q) and k-chunk `blockIdx.y`; writes the finished
// value when there is one chunk, else an fp64 partial.
template <int F, int OP>
__global__ void __launch_bounds__(256) strided(float* __restrict__ out, double* __restrict__ partial,
                                               const float* __restrict__ x, int64_t pre, int64_t len, int64_t post,
                                               int64_t chunk, double init) {
  const int64_t total = pre * post;
  const int64_t k0 = (int64_t)blockIdx.y * chunk;
  const int64_t k1 = min(len, k0 + chunk);
  const int64_t stride = (int64_t)gridDim.x * 256;
  for (int64_t o = (int64_t)blockIdx.x * 256 + threadIdx.x; o < total; o += stride) {
    const int64_t q = o / pre, p = o - q * pre;
    const float* base = x + p + q * pre * len;
    // four independent k-chains (k mod 4), combined in a fixed order
    double a0 = neutral<OP>(), a1 = neutral<OP>(), a2 = neutral<OP>(), a3 = neutral<OP>();
    int64_t k = k0;
    for (; k + 3 < k1; k += 4) {
      const float v0 = __ldcs(base + k * pre), v1 = __ldcs(base + (k + 1) * pre), v2 = __ldcs(base + (k + 2) * pre),
                  v3 = __ldcs(base + (k + 3) * pre);
      a0 = fold<F, OP>(a0, v0);
      a1 = fold<F, OP>(a1, v1);
      a2 = fold<F, OP>(a2, v2);
      a3 = fold<F, OP>(a3, v3);
    }
    for (; k < k1; ++k) a0 = fold<F, OP>(a0, __ldcs(base + k * pre));
    const double acc = combine<OP>(combine<OP>(a0, a1), combine<OP>(a2, a3));
    if (gridDim.y == 1) out[o] = (float)combine<OP>(init, acc);
    else partial[(int64_t)blockIdx.y * total + o] = acc;
  }
}

template <int OP>
__global__ void __launch_bounds__(256) fold_chunks(float* __restrict__ out, const double* __restrict__ partial,
                                                   int64_t total, int chunks, double init) {
  for (int64_t o = (int64_t)blockIdx.x * 256 + threadIdx.x; o < total; o += (int64_t)gridDim.x * 256) {
    double acc = neutral<OP>();
    for (int c = 0; c < chunks; ++c) acc = combine<OP>(acc, partial[(int64_t)c * total + o]);
    out[o] = (float)combine<OP>(init, acc);
  }
}

struct Args {
  float* out;
  const float* x;
  int64_t pre, len, post;
  double init;
  mk::Device* dev;
  cudaStream_t s;
};

template <int F, int OP>
int run(const Args& a) {
  const int64_t total = a.pre * a.post;
  const int64_t fill = (int64_t)a.dev->sms * 2048;  // threads that fill the GPU once
  if (a.pre == 1) {
    if (a.post >= (int64_t)a.dev->sms * 64 || a.len <= 1024) {
      int64_t blocks = mk::cdiv(a.post, 8);
      if (blocks > (int64_t)a.dev->sms * 32) blocks = (int64_t)a.dev->sms * 32;
      seg_warp<F, OP><<<(unsigned)blocks, 256, 0, a.s>>>(a.out, a.x, a.len, a.post, a.init);
    } else {
      int64_t blocks = a.post < (int64_t)a.dev->sms * 8 ? a.post : (int64_t)a.dev->sms * 8;
      seg_block<F, OP><<<(unsigned)blocks, 256, 0, a.s>>>(a.out, a.x, a.len, a.post, a.init);
    }
    return mk::check_launch("mk_mapreduce_dim_f32: launch");
  }
  int64_t chunks = 1;
  if (total < fill && a.len >= 128) {
    chunks = mk::cdiv(fill, total);
    if (chunks > a.len / 64) chunks = a.len / 64;
    if (chunks > 1024) chunks = 1024;
    if (chunks < 1) chunks = 1;
  }
  const int64_t chunk = mk::cdiv(a.len, chunks);
  chunks = mk::cdiv(a.len, chunk);
  double* partial = nullptr;
  if (chunks > 1) {
    void* ws = nullptr;
    int rc = mk::stream_workspace(a.dev, a.s, (size_t)chunks * (size_t)total * sizeof(double), &ws, mk::WS_DIMS);
    if (rc != MK_OK) return rc;
    partial = static_cast<double*>(ws);
  }
  int64_t bx = mk::cdiv(total, 256);
  if (bx > (int64_t)a.dev->sms * 16) bx = (int64_t)a.dev->sms * 16;
  strided<F, OP><<<dim3((unsigned)bx, (unsigned)chunks), 256, 0, a.s>>>(a.out, partial, a.x, a.pre, a.len, a.post,
                                                                      chunk, a.init);
  if (chunks > 1) fold_chunks<OP><<<(unsigned)bx, 256, 0, a.s>>>(a.out, partial, total, (int)chunks, a.init);
  return mk::check_launch("mk_mapreduce_dim_f32: launch");
}

template <int F>
int run_op(int op, const Args& a) {
  switch (op) {
    case MK_OP_ADD: return run<F, MK_OP_ADD>(a);
    case MK_OP_MAX: return run<F, MK_OP_MAX>(a);
    case MK_OP_MIN: return run<F, MK_OP_MIN>(a);
    default: return run<F, MK_OP_MUL>(a);
  }
}

__global__ void fill_value(float* out, int64_t n, float v) {
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) out[i] = v;
}

}  // namespace

extern "C" int mk_mapreduce_dim_f32(float* out, const float* x, int64_t pre, int64_t len, int64_t post, int f,
                                    int op, double init, void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (pre < 0 || len < 0 || post < 0) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_dim_f32: negative size");
  if (f < MK_F_IDENTITY || f > MK_F_GT0) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_dim_f32: unknown f");
  if (op < MK_OP_ADD || op > MK_OP_MUL) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_dim_f32: unknown op");
  const int64_t total = pre * post;
  if (total == 0) return MK_OK;
  if (!out || (len > 0 && !x)) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_dim_f32: null pointer");
  cudaStream_t s = mk::as_stream(stream);
  if (len == 0) {
    int64_t blocks = mk::cdiv(total, 256);
    if (blocks > (int64_t)dev->sms * 8) blocks = (int64_t)dev->sms * 8;
    fill_value<<<(unsigned)blocks, 256, 0, s>>>(out, total, (float)init);
    return mk::check_launch("mk_mapreduce_dim_f32: launch");
  }
  Args a{out, x, pre, len, post, init, dev, s};
  switch (f) {
    case MK_F_IDENTITY: return run_op<MK_F_IDENTITY>(op, a);
    case MK_F_ABS2: return run_op<MK_F_ABS2>(op, a);
    case MK_F_ABS: return run_op<MK_F_ABS>(op, a);
    default: return run_op<MK_F_GT0>(op, a);
  }
}
