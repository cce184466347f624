// scan.cu — prefix scan of a Float32 vector: AK.accumulate! / cumsum on an
// MLIRArray (test/test_downstream_ka.jl:39-42 inclusive, :75-78 exclusive).
// AcceleratedKernels runs a decoupled look-back scan; this is the same
// single-pass scheme written for sm_100a, 8 bytes of HBM traffic per element.
//
//   * tiles of 4096 elements (256 threads x 16) are claimed in launch order
//     from an atomic counter, so every predecessor of a tile is already
//     running: waiting on it cannot deadlock;
//   * a tile loads with coalesced 16-byte vectors through shared memory, scans
//     each thread's 16 values and the 256 thread totals in fp64, publishes its
//     aggregate (flag 1), then warp 0 looks back over 32 predecessors at a
//     time: the nearest inclusive prefix (flag 2) plus the aggregates after it
//     give the tile's exclusive prefix; the tile publishes its own inclusive
//     prefix (flag 2) and writes its outputs;
//   * values are carried in fp64 and rounded to Float32 once, so each output
//     is the correctly rounded prefix of the exact fp64 running value (max/min
//     exact).  Sequential fp32 summation (Base.cumsum) can only be less
//     accurate;
//   * waits on predecessors are bounded (mk::wait_limit_cycles); a timeout
//     raises ERRBIT_TIMEOUT and publishes a prefix anyway so no successor waits
//     forever.
#include "mk_common.cuh"
#include "reduce_ops.cuh"

namespace {

using namespace mk::rops;

constexpr int kThreads = 256;
constexpr int kPer = 16;
constexpr int kTile = kThreads * kPer;

struct ScanState {
  unsigned* counter;  // tile ticket
  unsigned* flags;    // per tile: 0 empty, 1 aggregate, 2 inclusive prefix
  double* agg;
  double* inc;
};

__device__ __forceinline__ int pad(int i) { return i + (i >> 5); }

__device__ __forceinline__ unsigned ld_flag(const unsigned* p) {
  return *reinterpret_cast<const volatile unsigned*>(p);
}

template <int OP>
__global__ void __launch_bounds__(kThreads)
scan_kernel(float* out, const float* x,  // may alias: a tile reads all of its input before writing
            int64_t n, double init, int exclusive,
            ScanState st, unsigned long long limit, unsigned* __restrict__ err) {
  // one pad word per 32 floats: a thread's 16 consecutive values and a warp's
  // float4 columns both map to 32 distinct banks
  __shared__ float buf[kTile + kTile / 32];
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

  // per-thread inclusive scan of 16 values (fp64)
  double v[kPer];
  double run = neutral<OP>();
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int idx = tid * kPer + j;
    const double e = idx < cnt ? (double)buf[pad(idx)] : neutral<OP>();
    run = combine<OP>(run, e);
    v[j] = run;
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
      if (lane == 0) {
        st.agg[t] = block_total;
        __threadfence();
        atomicExch(st.flags + t, 1u);
      }
      double acc = neutral<OP>();
      int64_t j = t - 1 - lane;  // lane i looks at tile t-1-i
      bool found = false, timed_out = false;
      const long long t0 = clock64();
      while (!found) {
        unsigned f = (j >= 0) ? ld_flag(st.flags + j) : 2u;
        // wait (warp-uniformly) until every lane of the window sees a value
        while (!__all_sync(0xffffffffu, f != 0u)) {
          if (__any_sync(0xffffffffu, (unsigned long long)(clock64() - t0) > limit)) {
            timed_out = true;
            break;
          }
          if (j >= 0 && f == 0u) f = ld_flag(st.flags + j);
        }
        if (timed_out) break;
        __threadfence();
        double val;
        if (j < 0) val = init;  // before tile 0: the initial value
        else val = (f == 2u) ? __ldcg(st.inc + j) : __ldcg(st.agg + j);
        const unsigned incl = __ballot_sync(0xffffffffu, f == 2u);
        const int stop = incl ? __ffs(incl) - 1 : 32;  // nearest lane holding an inclusive prefix
        double part = (lane <= stop) ? val : neutral<OP>();
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
      st.inc[t] = combine<OP>(prefix, block_total);
      __threadfence();
      atomicExch(st.flags + t, 2u);
      s_prefix = prefix;
    }
  }
  __syncthreads();
  const double pre = combine<OP>(s_prefix, texcl);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int idx = tid * kPer + j;
    const double before = (j == 0) ? pre : combine<OP>(pre, v[j - 1]);
    buf[pad(idx)] = (float)(exclusive ? before : combine<OP>(pre, v[j]));
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

}  // namespace

extern "C" int mk_accumulate_f32(float* out, const float* x, int64_t n, int op, double init, int exclusive,
                                 void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n < 0) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: n must be >= 0");
  if (op < MK_OP_ADD || op > MK_OP_MUL) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: unknown op");
  if (n == 0) return MK_OK;
  if (!out || !x) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: null pointer");
  const int64_t tiles = mk::cdiv(n, kTile);
  if (tiles > (int64_t)UINT32_MAX / 2) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: n too large");
  cudaStream_t s = mk::as_stream(stream);
  // workspace: [counter | flags(tiles) | agg(tiles) | inc(tiles)], 256-byte aligned parts
  const size_t flags_bytes = ((size_t)tiles * 4 + 255) & ~(size_t)255;
  const size_t val_bytes = ((size_t)tiles * 8 + 255) & ~(size_t)255;
  void* ws = nullptr;
  int rc = mk::stream_workspace(dev, s, 256 + flags_bytes + 2 * val_bytes, &ws, mk::WS_SCAN);
  if (rc != MK_OK) return rc;
  char* b = static_cast<char*>(ws);
  ScanState st{reinterpret_cast<unsigned*>(b), reinterpret_cast<unsigned*>(b + 256),
               reinterpret_cast<double*>(b + 256 + flags_bytes), reinterpret_cast<double*>(b + 256 + flags_bytes + val_bytes)};
  cudaError_t e = cudaMemsetAsync(b, 0, 256 + flags_bytes, s);  // ticket and flags start at zero
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_accumulate_f32: clearing tile flags");
  const unsigned long long limit = mk::wait_limit_cycles();
  switch (op) {
    case MK_OP_ADD: scan_kernel<MK_OP_ADD><<<(unsigned)tiles, kThreads, 0, s>>>(out, x, n, init, exclusive, st, limit, dev->err_word); break;
    case MK_OP_MAX: scan_kernel<MK_OP_MAX><<<(unsigned)tiles, kThreads, 0, s>>>(out, x, n, init, exclusive, st, limit, dev->err_word); break;
    case MK_OP_MIN: scan_kernel<MK_OP_MIN><<<(unsigned)tiles, kThreads, 0, s>>>(out, x, n, init, exclusive, st, limit, dev->err_word); break;
    default: scan_kernel<MK_OP_MUL><<<(unsigned)tiles, kThreads, 0, s>>>(out, x, n, init, exclusive, st, limit, dev->err_word); break;
  }
  return mk::check_launch("mk_accumulate_f32: launch");
}
