// scan.cu — prefix scan of a Float32 vector: AK.accumulate! / cumsum on an
// MLIRArray (test/test_downstream_ka.jl:39-42 inclusive, :75-78 exclusive).
// AcceleratedKernels runs a decoupled look-back scan; this is the same
// single-pass scheme written for sm_100a, 8 bytes of HBM traffic per element.
//
//   * tiles of 8192 elements (256 threads x 32) are claimed in launch order
//     from an atomic counter, so every predecessor of a tile is already
//     running: waiting on it cannot deadlock;
//   * a tile loads with coalesced 16-byte vectors through shared memory, scans
//     each thread's 32 values and the 256 thread totals in fp64, publishes its
//     aggregate, then warp 0 looks back over 32 predecessors at a time: the
//     nearest inclusive prefix plus the aggregates after it give the tile's
//     exclusive prefix; the tile publishes its own inclusive prefix and writes
//     its outputs.  Value and kind share one 64-bit word (see ScanState);
//   * carries between threads and tiles are fp64; inside a thread the 32
//     values are combined in fp32 (a pairwise tree for the total, a running
//     sum for the outputs), so each output is within a few ulp of the exact
//     prefix, relative to the running sum of magnitudes (max/min exact).
//     Sequential fp32 summation (Base.cumsum) errs by up to n ulp;
//   * waits on predecessors are bounded (mk::wait_limit_cycles); a timeout
//     raises ERRBIT_TIMEOUT and publishes a prefix anyway so no successor waits
//     forever.
#include <stdlib.h>

#include "mk_common.cuh"
#include "reduce_ops.cuh"

namespace {

using namespace mk::rops;

constexpr int kThreads = 256;

// Per-tile state: one 64-bit word that is published with a single store, so
// a reader needs one load and no fence.  EMPTY is an all-ones NaN pattern
// (the workspace is memset to 0xFF); otherwise the word is an fp64 value whose
// lowest mantissa bit is replaced by the kind: 0 = tile aggregate, 1 =
// inclusive prefix.  Losing that bit (2^-52 relative) is far below the final
// Float32 rounding.
struct ScanState {
  unsigned* counter;              // tile ticket
  unsigned long long* word;       // per tile
};
constexpr unsigned long long EMPTY = ~0ull;

__device__ __forceinline__ unsigned long long pack(double v, unsigned kind) {
  unsigned long long w = (__double_as_longlong(v) & ~1ull) | kind;
  return w == EMPTY ? (EMPTY - 2ull) | kind : w;  // keep NaN, never EMPTY
}
__device__ __forceinline__ double unpack(unsigned long long w) { return __longlong_as_double(w & ~1ull); }

__device__ __forceinline__ void publish(unsigned long long* p, unsigned long long w) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long peek(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

__device__ __forceinline__ int pad(int i) { return i + (i >> 5); }

template <int OP, int kPer>
__global__ void __launch_bounds__(kThreads)
scan_kernel(float* out, const float* x,  // may alias: a tile reads all of its input before writing
            int64_t n, double init, int exclusive,
            ScanState st, unsigned long long limit, unsigned* __restrict__ err) {
  constexpr int kTile = kThreads * kPer;
  // one pad word per 32 floats: a thread's consecutive values and a warp's
  // float4 columns both map to 32 distinct banks
  extern __shared__ float buf[];  // kTile + kTile / 32 floats
  __shared__ double warp_tot[kThreads / 32];
  __shared__ unsigned s_tile;
  __shared__ double s_prefix;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_tile = atomicAdd(st.counter, 1u);
  __syncthreads();
  const int64_t t = s_tile;
  const int64_t base = t * kTile;
  const int64_t cnt = min((int64_t)kTile, n - base);

  // coalesced load into shared memory
  if (cnt == kTile && ((reinterpret_cast<uintptr_t>(x + base) & 15u) == 0)) {
    const float4* src = reinterpret_cast<const float4*>(x + base);
#pragma unroll
    for (int i = 0; i < kPer / 4; ++i) {
      const int e = 4 * (i * kThreads + tid);
      const float4 q = __ldcs(src + i * kThreads + tid);
      buf[pad(e)] = q.x;
      buf[pad(e + 1)] = q.y;
      buf[pad(e + 2)] = q.z;
      buf[pad(e + 3)] = q.w;
    }
  } else {
    for (int i = tid; i < kTile; i += kThreads) buf[pad(i)] = i < cnt ? x[base + i] : 0.0f;
  }
  __syncthreads();

  // per-thread total of its kPer values: an fp32 pairwise tree (relative
  // error <= log2(kPer) ulp of the sum of magnitudes), widened to fp64 for
  // the carries.  The values are re-read from shared memory for the output
  // pass, which keeps registers (and so occupancy) free for more tiles.
  double run;
  {
    float v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int idx = tid * kPer + j;
      v[j] = idx < cnt ? buf[pad(idx)] : neutral32<OP>();
    }
#pragma unroll
    for (int w = 1; w < kPer; w <<= 1)
#pragma unroll
      for (int j = 0; j + w < kPer; j += 2 * w) v[j] = combine32<OP>(v[j], v[j + w]);
    run = (double)v[0];
  }
  // block exclusive scan of thread totals
  double inc = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double u = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc = combine<OP>(u, inc);
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  double wexcl = neutral<OP>(), block_total = neutral<OP>();
  for (int w = 0; w < kThreads / 32; ++w) {
    if (w < warp) wexcl = combine<OP>(wexcl, warp_tot[w]);
    block_total = combine<OP>(block_total, warp_tot[w]);
  }
  double texcl = __shfl_up_sync(0xffffffffu, inc, 1);
  if (lane == 0) texcl = neutral<OP>();
  texcl = combine<OP>(wexcl, texcl);

  // decoupled look-back (warp 0)
  if (warp == 0) {
    double prefix;
    if (t == 0) {
      prefix = init;
    } else {
      if (lane == 0) publish(st.word + t, pack(block_total, 0u));
      double acc = neutral<OP>();
      int64_t j = t - 1 - lane;  // lane i looks at tile t-1-i
      bool found = false, timed_out = false;
      const long long t0 = clock64();
      while (!found) {
        unsigned long long w = (j >= 0) ? peek(st.word + j) : pack(init, 1u);
        // wait (warp-uniformly) until every lane of the window sees a value
        while (!__all_sync(0xffffffffu, w != EMPTY)) {
          if (__any_sync(0xffffffffu, (unsigned long long)(clock64() - t0) > limit)) {
            timed_out = true;
            break;
          }
          if (w == EMPTY) w = peek(st.word + j);
        }
        if (timed_out) break;
        const unsigned incl = __ballot_sync(0xffffffffu, (w & 1ull) != 0ull);
        const int stop = incl ? __ffs(incl) - 1 : 32;  // nearest lane holding an inclusive prefix
        double part = (lane <= stop) ? unpack(w) : neutral<OP>();
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part = combine<OP>(part, __shfl_xor_sync(0xffffffffu, part, o));
        acc = combine<OP>(part, acc);
        if (stop < 32) found = true;
        j -= 32;
      }
      if (timed_out) {
        if (lane == 0) atomicOr(err, mk::ERRBIT_TIMEOUT);
        acc = init;
      }
      prefix = acc;
    }
    if (lane == 0) {
      publish(st.word + t, pack(combine<OP>(prefix, block_total), 1u));
      s_prefix = prefix;
    }
  }
  __syncthreads();
  // output: the fp64 thread prefix rounded once to fp32, then an fp32
  // running combination of the thread's own values (<= kPer terms)
  const float pre = (float)combine<OP>(s_prefix, texcl);
  float loc = neutral32<OP>();
#pragma unroll 8
  for (int j = 0; j < kPer; ++j) {
    const int idx = tid * kPer + j;
    const float before = combine32<OP>(pre, loc);
    if (idx < cnt) loc = combine32<OP>(loc, buf[pad(idx)]);
    buf[pad(idx)] = exclusive ? before : combine32<OP>(pre, loc);
  }
  __syncthreads();
  if (cnt == kTile && ((reinterpret_cast<uintptr_t>(out + base) & 15u) == 0)) {
    float4* dst = reinterpret_cast<float4*>(out + base);
#pragma unroll
    for (int i = 0; i < kPer / 4; ++i) {
      const int e = 4 * (i * kThreads + tid);
      __stcs(dst + i * kThreads + tid, make_float4(buf[pad(e)], buf[pad(e + 1)], buf[pad(e + 2)], buf[pad(e + 3)]));
    }
  } else {
    for (int i = tid; i < cnt; i += kThreads) out[base + i] = buf[pad(i)];
  }
}

// elements per thread (tuning knob MK_TUNE_SCAN_PER: 16, 32 or 64)
int scan_per() {
  static int v = [] {
    const char* e = getenv("MK_TUNE_SCAN_PER");
    int p = e ? atoi(e) : 32;
    return (p == 16 || p == 32 || p == 64) ? p : 32;
  }();
  return v;
}

template <int OP, int PER>
int launch_per(int64_t tiles, size_t smem, cudaStream_t s, float* out, const float* x, int64_t n, double init,
               int exclusive, ScanState st, unsigned long long limit, unsigned* err) {
  int rc = mk::allow_dynamic_smem(reinterpret_cast<const void*>(scan_kernel<OP, PER>), smem);
  if (rc != MK_OK) return rc;
  scan_kernel<OP, PER><<<(unsigned)tiles, kThreads, smem, s>>>(out, x, n, init, exclusive, st, limit, err);
  return MK_OK;
}

template <int OP>
int launch(int per, int64_t tiles, size_t smem, cudaStream_t s, float* out, const float* x, int64_t n, double init,
           int exclusive, ScanState st, unsigned long long limit, unsigned* err) {
  if (per == 16) return launch_per<OP, 16>(tiles, smem, s, out, x, n, init, exclusive, st, limit, err);
  if (per == 64) return launch_per<OP, 64>(tiles, smem, s, out, x, n, init, exclusive, st, limit, err);
  return launch_per<OP, 32>(tiles, smem, s, out, x, n, init, exclusive, st, limit, err);
}

}  // namespace

extern "C" int mk_accumulate_f32(float* out, const float* x, int64_t n, int op, double init, int exclusive,
                                 void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n < 0) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: n must be >= 0");
  if (op < MK_OP_ADD || op > MK_OP_MUL) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: unknown op");
  if (n == 0) return MK_OK;
  if (!out || !x) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: null pointer");
  const int64_t tiles = mk::cdiv(n, (int64_t)kThreads * scan_per());
  if (tiles > (int64_t)UINT32_MAX / 2) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: n too large");
  cudaStream_t s = mk::as_stream(stream);
  // workspace: [counter (256 B) | one state word per tile]
  void* ws = nullptr;
  int rc = mk::stream_workspace(dev, s, 256 + (size_t)tiles * 8, &ws, mk::WS_SCAN);
  if (rc != MK_OK) return rc;
  char* b = static_cast<char*>(ws);
  ScanState st{reinterpret_cast<unsigned*>(b), reinterpret_cast<unsigned long long*>(b + 256)};
  cudaError_t e = cudaMemsetAsync(b, 0, 256, s);  // the ticket starts at zero
  if (e == cudaSuccess) e = cudaMemsetAsync(b + 256, 0xFF, (size_t)tiles * 8, s);  // every tile EMPTY
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_accumulate_f32: clearing tile state");
  const unsigned long long limit = mk::wait_limit_cycles();
  const int per = scan_per();
  const size_t smem = (size_t)(kThreads * per + kThreads * per / 32) * sizeof(float);
  switch (op) {
    case MK_OP_ADD: rc = launch<MK_OP_ADD>(per, tiles, smem, s, out, x, n, init, exclusive, st, limit, dev->err_word); break;
    case MK_OP_MAX: rc = launch<MK_OP_MAX>(per, tiles, smem, s, out, x, n, init, exclusive, st, limit, dev->err_word); break;
    case MK_OP_MIN: rc = launch<MK_OP_MIN>(per, tiles, smem, s, out, x, n, init, exclusive, st, limit, dev->err_word); break;
    default: rc = launch<MK_OP_MUL>(per, tiles, smem, s, out, x, n, init, exclusive, st, limit, dev->err_word); break;
  }
  if (rc != MK_OK) return rc;
  return mk::check_launch("mk_accumulate_f32: launch");
}
