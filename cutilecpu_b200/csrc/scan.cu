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

// Decoupled look-back for tile t, run by one whole warp: publishes the tile's
// aggregate, combines the predecessors' words 32 at a time back to the
// nearest inclusive prefix, publishes the tile's inclusive prefix and returns
// the exclusive prefix.  The wait is bounded: on timeout ERRBIT_TIMEOUT is
// raised and `init` is used, so no successor waits forever.
template <int OP>
__device__ double look_back(ScanState st, int64_t t, double block_total, double init, unsigned long long limit,
                            unsigned* err, bool agg_published) {
  const int lane = threadIdx.x & 31;
  double prefix;
  if (t == 0) {
    prefix = init;
  } else {
    if (lane == 0 && !agg_published) publish(st.word + t, pack(block_total, 0u));
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
  if (lane == 0) publish(st.word + t, pack(combine<OP>(prefix, block_total), 1u));
  return prefix;
}

constexpr int kPer = 32;                 // elements per thread: one 128-byte row
constexpr int kTile = kThreads * kPer;   // 8192 elements per tile

// Shared-memory tile: row r (thread r's 32 values) is 8 16-byte chunks, and
// chunk c of row r is stored at slot c ^ (r & 7).  A thread then reads and
// writes its row as 8 conflict-free 16-byte accesses (a quarter-warp touches
// 8 rows at 8 distinct bank groups), and the coalesced global loads/stores
// (8 consecutive float4 = one row) are conflict-free too.
__device__ __forceinline__ int slot(int r, int c) { return r * 8 + (c ^ (r & 7)); }

template <int OP>
__global__ void __launch_bounds__(kThreads)
scan_kernel(float* out, const float* x,  // may alias: a tile reads all of its input before writing
            int64_t n, double init, int exclusive,
            ScanState st, unsigned long long limit, unsigned* __restrict__ err) {
  extern __shared__ float4 buf4[];  // kTile / 4 chunks
  __shared__ double warp_tot[kThreads / 32];
  __shared__ double warp_agg[kThreads / 32];  // early tile aggregate, per warp
  __shared__ unsigned s_tile;
  __shared__ double s_prefix;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // Tiles are claimed in block order in practice, so this block's own tile is
  // pulled into L2 (one bulk prefetch, no data to shared memory) while the
  // ticket's round trip is in flight; when the ticket differs the prefetched
  // tile is another block's and is read from L2 by it soon after.  This hides
  // the ticket's latency: 0.498 -> 0.419 ms at 2^28.  Prefetching a whole wave
  // of resident blocks further ahead measured no faster (0.420-0.486 ms).
  if (tid == 0) {
    const int64_t pb = (int64_t)blockIdx.x * kTile;
    if (pb + kTile <= n && ((reinterpret_cast<uintptr_t>(x + pb) & 15u) == 0))
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(x + pb), "r"((unsigned)(kTile * 4))
                   : "memory");
    s_tile = atomicAdd(st.counter, 1u);
  }
  __syncthreads();
  const int64_t t = s_tile;
  const int64_t base = t * kTile;
  const int64_t cnt = min((int64_t)kTile, n - base);
  const bool vec = cnt == kTile && ((reinterpret_cast<uintptr_t>(x + base) & 15u) == 0);

  // coalesced load into shared memory; past the end of x: the neutral element
  if (vec) {
    const float4* src = reinterpret_cast<const float4*>(x + base);
    float4 q[kPer / 4];
    // L2-cached loads of the lines the prefetch brought in (evict-first loads
    // measured 2 % slower: 0.4217 vs 0.4127 ms at 2^28)
#pragma unroll
    for (int i = 0; i < kPer / 4; ++i) q[i] = __ldcg(src + i * kThreads + tid);
#pragma unroll
    for (int i = 0; i < kPer / 4; ++i) {
      const int f = i * kThreads + tid;
      buf4[slot(f >> 3, f & 7)] = q[i];
    }
    // the tile's aggregate straight from the registers, so that successors
    // can use it before this tile has scanned anything (any fixed grouping:
    // it differs from the scan's own total only in rounding)
    float v[kPer / 4];
#pragma unroll
    for (int i = 0; i < kPer / 4; ++i)
      v[i] = combine32<OP>(combine32<OP>(q[i].x, q[i].y), combine32<OP>(q[i].z, q[i].w));
#pragma unroll
    for (int w = 1; w < kPer / 4; w <<= 1)
#pragma unroll
      for (int j = 0; j + w < kPer / 4; j += 2 * w) v[j] = combine32<OP>(v[j], v[j + w]);
    double a = (double)v[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = combine<OP>(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) warp_agg[warp] = a;
  } else {
    float* buf = reinterpret_cast<float*>(buf4);
    for (int e = tid; e < kTile; e += kThreads)
      buf[slot(e >> 5, (e >> 2) & 7) * 4 + (e & 3)] = e < cnt ? x[base + e] : neutral32<OP>();
  }
  __syncthreads();
  if (vec && warp == 0 && t > 0) {
    double a = lane < kThreads / 32 ? warp_agg[lane] : neutral<OP>();
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) a = combine<OP>(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) publish(st.word + t, pack(a, 0u));
  }

  float4* row = buf4 + tid * 8;
  const int sw = tid & 7;
  // per-thread total of its 32 values: an fp32 pairwise tree (relative error
  // <= 5 ulp of the sum of magnitudes), widened to fp64 for the carries.  The
  // values are re-read from shared memory for the output pass, which keeps
  // registers (and so occupancy) free for more tiles.
  double run;
  {
    float v[kPer];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 q = row[c ^ sw];
      v[4 * c] = q.x;
      v[4 * c + 1] = q.y;
      v[4 * c + 2] = q.z;
      v[4 * c + 3] = q.w;
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
    const double prefix = look_back<OP>(st, (int64_t)t, block_total, init, limit, err, vec);
    if (lane == 0) s_prefix = prefix;
  }
  __syncthreads();
  // output: the fp64 thread prefix rounded once to fp32, then an fp32
  // running combination of the thread's own values (<= 32 terms); values past
  // the end are the neutral element and are never stored
  const float pre = (float)combine<OP>(s_prefix, texcl);
  float loc = neutral32<OP>();
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const float4 q = row[c ^ sw];
    const float in[4] = {q.x, q.y, q.z, q.w};
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float before = combine32<OP>(pre, loc);
      loc = combine32<OP>(loc, in[e]);
      o[e] = exclusive ? before : combine32<OP>(pre, loc);
    }
    row[c ^ sw] = make_float4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  if (cnt == kTile && ((reinterpret_cast<uintptr_t>(out + base) & 15u) == 0)) {
    float4* dst = reinterpret_cast<float4*>(out + base);
#pragma unroll
    for (int i = 0; i < kPer / 4; ++i) {
      const int f = i * kThreads + tid;
      __stcs(dst + f, buf4[slot(f >> 3, f & 7)]);
    }
  } else {
    const float* buf = reinterpret_cast<const float*>(buf4);
    for (int e = tid; e < cnt; e += kThreads) out[base + e] = buf[slot(e >> 5, (e >> 2) & 7) * 4 + (e & 3)];
  }
}

template <int OP>
int launch(int64_t tiles, cudaStream_t s, float* out, const float* x, int64_t n, double init, int exclusive,
           ScanState st, unsigned long long limit, unsigned* err) {
  constexpr size_t smem = (size_t)kTile * sizeof(float);
  int rc = mk::allow_dynamic_smem(reinterpret_cast<const void*>(scan_kernel<OP>), smem);
  if (rc != MK_OK) return rc;
  scan_kernel<OP><<<(unsigned)tiles, kThreads, smem, s>>>(out, x, n, init, exclusive, st, limit, err);
  return MK_OK;
}

}  // namespace

extern "C" int mk_accumulate_f32(float* out, const float* x, int64_t n, int op, double init, int exclusive,
                                 void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n < 0) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: n must be >= 0");
  if (op < MK_OP_ADD || op > MK_OP_MUL) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: unknown op");
  if (n == 0) return MK_OK;
  if (!out || !x) return mk::fail(MK_ERR_INVALID, "mk_accumulate_f32: null pointer");
  const int64_t tiles = mk::cdiv(n, (int64_t)kTile);
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
  switch (op) {
    case MK_OP_ADD: rc = launch<MK_OP_ADD>(tiles, s, out, x, n, init, exclusive, st, limit, dev->err_word); break;
    case MK_OP_MAX: rc = launch<MK_OP_MAX>(tiles, s, out, x, n, init, exclusive, st, limit, dev->err_word); break;
    case MK_OP_MIN: rc = launch<MK_OP_MIN>(tiles, s, out, x, n, init, exclusive, st, limit, dev->err_word); break;
    default: rc = launch<MK_OP_MUL>(tiles, s, out, x, n, init, exclusive, st, limit, dev->err_word); break;
  }
  if (rc != MK_OK) return rc;
  return mk::check_launch("mk_accumulate_f32: launch");
}
