// mapreduce.cu — out = op(init, op_i f(x[i])) over an fp32 vector, in ONE
// launch: the fused replacement for the reference's reduce path
// (GPUArrays.mapreducedim! -> AK.mapreduce, ext/MLIRCUDAExt.jl:100-121), which
// materialises a broadcast `x.^2` first (:103) and then runs AcceleratedKernels'
// multi-launch block reductions with a host copy of the partials (:125-131).
//
// Design (HBM-bound: 4 bytes per element, read once):
//   * persistent grid of kBlocksPerSM x SMs blocks; every thread keeps kUnroll
//     16-byte loads in flight and accumulates in fp64 (sums/products), or exactly
//     in fp32 (max/min).  For f in {abs2, abs, x>0} the 8 mapped values of one
//     float4 pair are first added in fp32 (all terms >= 0: relative error of
//     that group <= 7 ulp), then added to the fp64 accumulator; identity sums
//     convert every term to fp64 because terms of mixed sign may cancel;
//   * warp shuffle + shared-memory combine -> one fp64 partial per block in the
//     per-stream scratch array;
//   * the last block to finish (atomic ticket) folds the partials in a fixed
//     order, applies `init`, writes out[0] and re-arms the ticket.  The result
//     depends only on n and the grid size, so it is deterministic per device.
// NaN handling of max/min follows Julia's `max`/`min` (a NaN operand wins) and
// +0.0 > -0.0, which is what `maximum`/`minimum` on Float32 give.
#include <math.h>
#include <stdlib.h>

#include <mutex>
#include <string>

#include "mk_common.cuh"
#include "peer.cuh"
#include "reduce_ops.cuh"

namespace {

using namespace mk::rops;

constexpr int kThreads = 256;
constexpr int kUnroll = 4;  // float4 loads in flight per thread

// Fold one float4 (already mapped) into the thread accumulator.
template <int F, int OP>
__device__ __forceinline__ void fold4(double& acc, float4 v) {
  const float m0 = mapf(F, v.x), m1 = mapf(F, v.y), m2 = mapf(F, v.z), m3 = mapf(F, v.w);
  if (OP == MK_OP_ADD) {
    if (F == MK_F_IDENTITY) {
      acc += (double)m0;
      acc += (double)m1;
      acc += (double)m2;
      acc += (double)m3;
    } else {
      acc += (double)((m0 + m1) + (m2 + m3));
    }
  } else if (OP == MK_OP_MUL) {
    acc = acc * (double)m0 * (double)m1 * (double)m2 * (double)m3;
  } else {
    acc = combine<OP>(acc, combine<OP>(combine<OP>((double)m0, (double)m1),
                                       combine<OP>((double)m2, (double)m3)));
  }
}

template <int F, int OP>
__device__ __forceinline__ void fold1(double& acc, float v) {
  acc = combine<OP>(acc, (double)mapf(F, v));
}

template <int OP>
__device__ __forceinline__ double block_reduce(double v, double* smem) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = combine<OP>(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  v = neutral<OP>();
  if (warp == 0) {
    if (lane < kThreads / 32) v = smem[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = combine<OP>(v, __shfl_xor_sync(0xffffffffu, v, o));
  }
  return v;  // valid in thread 0
}

// x: base pointer; the first `head` (0..3) elements precede the first 16-byte
// boundary and are folded by the first `head` threads, like the <4 tail.
// Registers fitted to 8 resident blocks per SM (32 a thread, no spills): the
// max/min and abs forms used 36-40 and ran 6 blocks per SM.  maximum over
// 2^28: 0.1703 -> 0.1676 ms; sum(x.^2): 0.1519 -> 0.1497 ms per graph step.
template <int F, int OP>
__global__ void __launch_bounds__(kThreads, 8)
mapreduce_kernel(const float* __restrict__ x, int64_t n, int head, double init,
                 double* __restrict__ partials, unsigned* __restrict__ ticket,
                 double* __restrict__ out, const mk::PeerArgs peer, unsigned* __restrict__ err) {
  __shared__ double smem[kThreads / 32];
  __shared__ bool is_last;
  __shared__ unsigned long long s_epoch;  // multi-GPU: the channel's last published epoch E
  if (peer.trace && blockIdx.x == 0 && threadIdx.x == 0)
    mk::peerdev::stamp(peer, mk::peerdev::read_epoch(peer) + 1, 0);
  const int64_t tid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  double acc = neutral<OP>();

  const float4* x4 = reinterpret_cast<const float4*>(x + head);
  const int64_t n4 = (n - head) / 4;
  float ext[4] = {neutral32<OP>(), neutral32<OP>(), neutral32<OP>(), neutral32<OP>()};
  int64_t i = tid;
  for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
    float4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = __ldcs(x4 + i + u * stride);
    if (OP == MK_OP_ADD && F != MK_F_IDENTITY) {
      // Pair-wise fp32 grouping: 8 non-negative mapped terms per fp64 add.
#pragma unroll
      for (int u = 0; u < kUnroll; u += 2) {
        float g0 = (mapf(F, v[u].x) + mapf(F, v[u].y)) + (mapf(F, v[u].z) + mapf(F, v[u].w));
        float g1 = (mapf(F, v[u + 1].x) + mapf(F, v[u + 1].y)) +
                   (mapf(F, v[u + 1].z) + mapf(F, v[u + 1].w));
        acc += (double)(g0 + g1);
      }
    } else if (OP == MK_OP_MAX || OP == MK_OP_MIN) {
      // max/min are exact: fold in fp32, one independent chain per vector lane
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        ext[0] = combine32<OP>(ext[0], mapf(F, v[u].x));
        ext[1] = combine32<OP>(ext[1], mapf(F, v[u].y));
        ext[2] = combine32<OP>(ext[2], mapf(F, v[u].z));
        ext[3] = combine32<OP>(ext[3], mapf(F, v[u].w));
      }
    } else {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) fold4<F, OP>(acc, v[u]);
    }
  }
  if (OP == MK_OP_MAX || OP == MK_OP_MIN)
    acc = combine<OP>(acc, (double)combine32<OP>(combine32<OP>(ext[0], ext[1]), combine32<OP>(ext[2], ext[3])));
  for (; i < n4; i += stride) fold4<F, OP>(acc, __ldcs(x4 + i));
  // Scalar head (before the first 16-byte boundary) and tail (< 4 elements).
  const int64_t tail_start = head + n4 * 4;
  if (tid < head) fold1<F, OP>(acc, x[tid]);
  if (tid < n - tail_start) fold1<F, OP>(acc, x[tail_start + tid]);

  double bsum = block_reduce<OP>(acc, smem);
  __shared__ bool is_first;
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = bsum;
    if (peer.world > 0) s_epoch = mk::peerdev::read_epoch(peer);  // before the ticket (see read_epoch)
    __threadfence();
    unsigned t = atomicAdd(ticket, 1u);
    is_last = (t == gridDim.x - 1);
    is_first = (t == 0);
  }
  __syncthreads();
  // Multi-GPU: the first block to finish its share finishes the previous
  // pipelined call's global result (epoch E) while the others are still
  // streaming, so the last block (which ends the kernel) only has to publish.
  const bool fold_early = peer.world > 0 && gridDim.x > 1;
  if (fold_early && is_first && threadIdx.x < 32) mk::peerdev::complete_pending(peer, s_epoch, err);
  if (!is_last) return;
  __threadfence();
  // Last block: fold the partials in a fixed order (strided per thread, then
  // the same shuffle tree), so the result does not depend on block timing.
  double v = neutral<OP>();
  for (int b = threadIdx.x; b < (int)gridDim.x; b += kThreads) v = combine<OP>(v, __ldcg(partials + b));
  __syncthreads();  // smem reuse
  v = block_reduce<OP>(v, smem);
  if (threadIdx.x < 32) {  // warp 0 (v is valid in lane 0)
    v = __shfl_sync(0xffffffffu, v, 0);
    if (threadIdx.x == 0) *ticket = 0u;  // re-arm for the next reduction on this stream
    if (peer.world == 0) {
      if (threadIdx.x == 0) out[0] = combine<OP>(init, v);
    } else {
      // multi-GPU: publish this rank's partial as epoch E+1, finish epoch E's
      // pending result unless the first block already did (its partials have
      // had a whole kernel to arrive), and in the blocking form wait for E+1
      const unsigned long long e1 = s_epoch + 1;
      if (threadIdx.x == 0) mk::peerdev::stamp(peer, e1, 1);
      mk::peerdev::publish(v, peer, e1);
      if (threadIdx.x == 0) mk::peerdev::stamp(peer, e1, 2);
      if (!fold_early) mk::peerdev::complete_pending(peer, s_epoch, err);
      if (threadIdx.x == 0) mk::peerdev::stamp(peer, e1, 3);
      if (peer.mode == mk::XMODE_BLOCKING) {
        const double g = mk::peerdev::fold(peer, e1, OP, err);
        if (threadIdx.x == 0) out[0] = combine<OP>(init, g);
      }
      if (threadIdx.x == 0) mk::peerdev::finish_epoch(peer, e1);
    }
  }
}

// Completes the pending pipelined result of mk_mapreduce_f32_allreduce_async.
__global__ void allreduce_complete_kernel(const mk::PeerArgs peer, unsigned* __restrict__ err) {
  if (threadIdx.x < 32) mk::peerdev::complete_pending(peer, mk::peerdev::read_epoch(peer), err);
}

// The grid is persistent: never more blocks than fit on the GPU at once (the
// resident count depends on each instantiation's registers), so no block
// waits for a second wave.
template <int F, int OP>
void launch(unsigned blocks, cudaStream_t s, const float* x, int64_t n, int head, double init,
            const mk::ReduceScratch& rs, double* out, const mk::PeerArgs& peer, unsigned* err) {
  static const int per_sm = [] {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, mapreduce_kernel<F, OP>, kThreads, 0) != cudaSuccess)
      b = 1;
    return b > 0 ? b : 1;
  }();
  const mk::Device* dev = mk::current_device();
  const unsigned resident = (unsigned)((dev ? dev->sms : 1) * per_sm);
  if (blocks > resident) blocks = resident;
  mapreduce_kernel<F, OP><<<blocks, kThreads, 0, s>>>(x, n, head, init, rs.partials, rs.ticket, out, peer, err);
}

template <int F>
int dispatch_op(int op, unsigned blocks, cudaStream_t s, const float* x, int64_t n, int head,
                double init, const mk::ReduceScratch& rs, double* out,
                const mk::PeerArgs& peer = mk::PeerArgs(), unsigned* err = nullptr) {
  switch (op) {
    case MK_OP_ADD: launch<F, MK_OP_ADD>(blocks, s, x, n, head, init, rs, out, peer, err); break;
    case MK_OP_MAX: launch<F, MK_OP_MAX>(blocks, s, x, n, head, init, rs, out, peer, err); break;
    case MK_OP_MIN: launch<F, MK_OP_MIN>(blocks, s, x, n, head, init, rs, out, peer, err); break;
    case MK_OP_MUL: launch<F, MK_OP_MUL>(blocks, s, x, n, head, init, rs, out, peer, err); break;
    default: return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: unknown op");
  }
  return MK_OK;
}

int blocks_per_sm() {
  static int v = [] {
    const char* e = getenv("MK_TUNE_REDUCE_BLOCKS_PER_SM");
    int b = e ? atoi(e) : 8;
    return (b >= 1 && b <= 16) ? b : 8;
  }();
  return v;
}

}  // namespace

namespace {

int mapreduce_impl(mk::Device* dev, double* out_dev, const float* x, int64_t n, int f, int op, double init,
                   void* stream, const mk::PeerArgs& peer) {
  if (n < 0) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: n must be >= 0");
  if (!out_dev || (n > 0 && !x)) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: null pointer");
  if (f < MK_F_IDENTITY || f > MK_F_GT0) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: unknown f");
  if (op < MK_OP_ADD || op > MK_OP_MUL) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: unknown op");
  cudaStream_t s = mk::as_stream(stream);
  mk::ReduceScratch rs;
  int rc = mk::reduce_scratch(dev, s, &rs);
  if (rc != MK_OK) return rc;
  int head = 0;
  if (n > 0) {
    head = (int)(((16u - (reinterpret_cast<uintptr_t>(x) & 15u)) & 15u) / 4u);
    if ((reinterpret_cast<uintptr_t>(x) & 3u) != 0)
      return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: x must be 4-byte aligned");
    if (head > n) head = (int)n;
  }
  int64_t want = mk::cdiv(n, (int64_t)kThreads * kUnroll * 4);
  int64_t cap = (int64_t)dev->sms * blocks_per_sm();
  if (cap > mk::kMaxReduceBlocks) cap = mk::kMaxReduceBlocks;
  unsigned blocks = (unsigned)(want < 1 ? 1 : (want > cap ? cap : want));
  switch (f) {
    case MK_F_IDENTITY: rc = dispatch_op<MK_F_IDENTITY>(op, blocks, s, x, n, head, init, rs, out_dev, peer, dev->err_word); break;
    case MK_F_ABS2: rc = dispatch_op<MK_F_ABS2>(op, blocks, s, x, n, head, init, rs, out_dev, peer, dev->err_word); break;
    case MK_F_ABS: rc = dispatch_op<MK_F_ABS>(op, blocks, s, x, n, head, init, rs, out_dev, peer, dev->err_word); break;
    default: rc = dispatch_op<MK_F_GT0>(op, blocks, s, x, n, head, init, rs, out_dev, peer, dev->err_word); break;
  }
  if (rc != MK_OK) return rc;
  return mk::check_launch("mk_mapreduce_f32: launch");
}

}  // namespace

extern "C" int mk_mapreduce_f32(double* out_dev, const float* x, int64_t n, int f, int op, double init,
                                void* stream) {
  MK_ENTRY_DEVICE(dev);
  return mapreduce_impl(dev, out_dev, x, n, f, op, init, stream, mk::PeerArgs());
}

namespace {

int allreduce_entry(bool blocking, double* out_dev, const float* x, int64_t n, int f, int op, double init,
                    void* stream) {
  MK_ENTRY_DEVICE(dev);
  // argument errors before an epoch is taken, so a rejected call leaves the
  // ranks' epoch counters in step
  if (n < 0) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: n must be >= 0");
  if (!out_dev || (n > 0 && !x)) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: null pointer");
  if (f < MK_F_IDENTITY || f > MK_F_GT0) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: unknown f");
  if (op < MK_OP_ADD || op > MK_OP_MUL) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: unknown op");
  if (n > 0 && (reinterpret_cast<uintptr_t>(x) & 3u) != 0)
    return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32: x must be 4-byte aligned");
  mk::PeerArgs peer;
  int rc = mk::peer_args(dev, mk::CH_REDUCE, blocking ? mk::XMODE_BLOCKING : mk::XMODE_PIPELINED, out_dev, op,
                         init, &peer);
  if (rc != MK_OK) return rc;
  return mapreduce_impl(dev, out_dev, x, n, f, op, init, stream, peer);
}

}  // namespace

extern "C" int mk_mapreduce_f32_allreduce(double* out_dev, const float* x, int64_t n, int f, int op, double init,
                                          void* stream) {
  return allreduce_entry(true, out_dev, x, n, f, op, init, stream);
}

extern "C" int mk_mapreduce_f32_allreduce_async(double* out_dev, const float* x, int64_t n, int f, int op,
                                                double init, void* stream) {
  return allreduce_entry(false, out_dev, x, n, f, op, init, stream);
}

extern "C" int mk_allreduce_complete(void* stream) {
  MK_ENTRY_DEVICE(dev);
  mk::PeerArgs peer;
  int rc = mk::peer_args(dev, mk::CH_REDUCE, mk::XMODE_COMPLETE, nullptr, 0, 0.0, &peer);
  if (rc != MK_OK) return rc;
  allreduce_complete_kernel<<<1, 32, 0, mk::as_stream(stream)>>>(peer, dev->err_word);
  return mk::check_launch("mk_allreduce_complete: launch");
}

extern "C" int mk_sum_sq_f32(double* out_dev, const float* x, int64_t n, void* stream) {
  return mk_mapreduce_f32(out_dev, x, n, MK_F_ABS2, MK_OP_ADD, 0.0, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot let a library call cudaMalloc:
// hosts whose device memory is owned by their own pool allocator (CUDA.jl's
// pool, torch's caching allocator) and must see every byte, or that run under
// a fixed memory budget set at start-up.  mk_mapreduce_f32 takes its
// per-stream scratch from cudaMalloc on first use; this entry point instead
// uses one file-scope device array that every GPU loading the library holds
// until exit: MK_NOALLOC_MAX_PARTIALS fp64 block partials (32 KiB) plus the
// u32 ticket, 256-byte aligned.  The reduction kernel is the same one, with
// the same grid, so the result is bit-identical to mk_mapreduce_f32.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocPartialBytes = sizeof(double) * MK_NOALLOC_MAX_PARTIALS;
constexpr size_t kNoAllocBytes = kNoAllocPartialBytes + 256;  // partials, then the ticket

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_addr[64] = {};  // device address of g_noalloc_scratch, per device

// Device address of the array on the current device.  Host code must not use
// the symbol itself: on the host it names a shadow variable, not device memory.
int noalloc_scratch(int device, unsigned char** out) {
  if (device < 0 || device >= 64) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32_noalloc: device out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return mk::fail_cuda(e, "mk_mapreduce_f32_noalloc: cudaGetSymbolAddress");
    g_noalloc_addr[device] = static_cast<unsigned char*>(p);
  }
  *out = g_noalloc_addr[device];
  return MK_OK;
}

}  // namespace

extern "C" int mk_mapreduce_f32_noalloc(double* out_dev, const float* x, int64_t n, int f, int op,
                                        double init, void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (n < 0) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32_noalloc: n must be >= 0");
  if (!out_dev || (n > 0 && !x)) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32_noalloc: null pointer");
  if (f < MK_F_IDENTITY || f > MK_F_GT0) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32_noalloc: unknown f");
  if (op < MK_OP_ADD || op > MK_OP_MUL) return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32_noalloc: unknown op");
  if (n > 0 && (reinterpret_cast<uintptr_t>(x) & 3u) != 0)
    return mk::fail(MK_ERR_INVALID, "mk_mapreduce_f32_noalloc: x must be 4-byte aligned");
  int64_t want = mk::cdiv(n, (int64_t)kThreads * kUnroll * 4);
  int64_t cap = (int64_t)dev->sms * blocks_per_sm();
  if (cap > mk::kMaxReduceBlocks) cap = mk::kMaxReduceBlocks;
  const int64_t blocks = want < 1 ? 1 : (want > cap ? cap : want);
  // One partial slot per block: the grid may not outgrow the static array.
  if (blocks > MK_NOALLOC_MAX_PARTIALS)
    return mk::fail(MK_ERR_INVALID,
                    "mk_mapreduce_f32_noalloc: the launch needs " + std::to_string(blocks) +
                        " block partials; the static scratch holds " + std::to_string(MK_NOALLOC_MAX_PARTIALS));
  unsigned char* base = nullptr;
  int rc = noalloc_scratch(dev->id, &base);
  if (rc != MK_OK) return rc;
  cudaStream_t s = mk::as_stream(stream);
  mk::ReduceScratch rs;
  rs.partials = reinterpret_cast<double*>(base);
  rs.ticket = reinterpret_cast<unsigned*>(base + kNoAllocPartialBytes);
  // The array keeps whatever the previous call left: the ticket must start at 0.
  cudaError_t e = cudaMemsetAsync(rs.ticket, 0, sizeof(unsigned), s);
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_mapreduce_f32_noalloc: clearing the ticket");
  int head = 0;
  if (n > 0) {
    head = (int)(((16u - (reinterpret_cast<uintptr_t>(x) & 15u)) & 15u) / 4u);
    if (head > n) head = (int)n;
  }
  const unsigned ub = (unsigned)blocks;
  switch (f) {
    case MK_F_IDENTITY: rc = dispatch_op<MK_F_IDENTITY>(op, ub, s, x, n, head, init, rs, out_dev); break;
    case MK_F_ABS2: rc = dispatch_op<MK_F_ABS2>(op, ub, s, x, n, head, init, rs, out_dev); break;
    case MK_F_ABS: rc = dispatch_op<MK_F_ABS>(op, ub, s, x, n, head, init, rs, out_dev); break;
    default: rc = dispatch_op<MK_F_GT0>(op, ub, s, x, n, head, init, rs, out_dev); break;
  }
  if (rc != MK_OK) return rc;
  return mk::check_launch("mk_mapreduce_f32_noalloc: launch");
}
