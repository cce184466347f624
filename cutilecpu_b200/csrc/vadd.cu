// vadd.cu — c[i] = a[i] + b[i] (fp32), the elementwise map of the reference's
// vadd kernel (test/test_gpu_simt.jl:13-16, examples/reflection_and_perf.jl:11-14).
//
// The reference lowers it to one scalar 4-byte load/store per thread with a
// masked tail (src/lower.jl:4110-4115, 4170-4174, valid_index :1895-1915).
// Here: 16-byte vector loads/stores, two float4 pairs in flight per thread,
// streaming (evict-first) cache hints, grid sized to fill every SM once and
// grid-striding beyond that.  Pure HBM traffic: 12 bytes per element.
#include "mbarrier.cuh"
#include "mk_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;  // float4 per operand in flight per thread
// Grid cap of the vector kernel: 5 blocks of 256 per SM (740 on a B200), not
// the 8 that fill every thread slot.  With PDL the next launch's blocks become
// resident while this one drains; at 2^20 elements in a CUDA graph a step
// took 3.41-3.44 us at 5 per SM against 3.58-3.62 at 8, 3.47 at 4 and 3.93
// at 2, and 2^24 / 2^26 streams stayed within 2 % of the 8-per-SM grid.
constexpr int kVecBlocksPerSM = 5;

// Device-clock stamps of a launch (probe builds only): [0] earliest block
// start, [1] latest block end, in ns of %globaltimer.
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// PDL: launched with programmatic stream serialization, the kernel lets the
// next kernel on the stream start launching at once (its blocks take free
// slots and wait in griddepcontrol.wait), and waits itself for the previous
// kernel's completion and memory flush before its first load.  Without the
// launch attribute both instructions are no-ops.
template <bool STAMP, bool PDL = false>
__global__ void __launch_bounds__(kThreads)
vadd_f32_vec4(float4* __restrict__ c, const float4* __restrict__ a,
              const float4* __restrict__ b, int64_t n4, unsigned long long* __restrict__ stamps) {
  if (PDL) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
  }
  if (STAMP && threadIdx.x == 0) atomicMin(stamps, globaltimer());
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
  if (STAMP) {
    __syncthreads();
    if (threadIdx.x == 0) atomicMax(stamps + 1, globaltimer());
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
  const int64_t max_vblocks = (int64_t)dev->sms * kVecBlocksPerSM;
  if (mk::aligned16(a) && mk::aligned16(b) && mk::aligned16(c)) {
    const int64_t n4 = n / 4;
    if (n4 > 0) {
      int64_t blocks = mk::cdiv(n4, kThreads);
      if (blocks > max_vblocks) blocks = max_vblocks;
      // A 2^20-element vadd is over in ~3 us on the device; launched with
      // programmatic dependent launch so back-to-back launches (a stream of
      // small maps, or a CUDA graph of them) overlap their launch latency.
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)blocks);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = 0;
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      cudaError_t e = cudaLaunchKernelEx(&cfg, vadd_f32_vec4<false, true>, reinterpret_cast<float4*>(c),
                                         reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b), n4,
                                         static_cast<unsigned long long*>(nullptr));
      if (e != cudaSuccess) return mk::fail_cuda(e, "mk_vadd_f32: launch");
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

// ---------------------------------------------------------------------------
// Measurement probes (no counterpart in the reference): the parts of a small
// vadd's time.  Each mode launches with the grid of the vector kernel above
// and records device-clock stamps (earliest block start, latest block end):
//   0  empty kernel: launch and block scheduling alone;
//   1  read-only: a and b streamed in, nothing but one word per block out;
//   2  the vector vadd itself (same code, with stamps);
//   3  bulk-copy vadd: one block per SM, each block moves its slice of a and b
//      global -> shared with cp.async.bulk (no multicast; this GPU's memory
//      only), adds in shared memory and writes its slice of c back with one
//      bulk store.
// ---------------------------------------------------------------------------
namespace {

__global__ void __launch_bounds__(kThreads) probe_empty(unsigned long long* __restrict__ stamps) {
  if (threadIdx.x == 0) {
    atomicMin(stamps, globaltimer());
    atomicMax(stamps + 1, globaltimer());
  }
}

__global__ void __launch_bounds__(kThreads)
probe_read2(unsigned* __restrict__ out, const float4* __restrict__ a, const float4* __restrict__ b, int64_t n4,
            unsigned long long* __restrict__ stamps) {
  if (threadIdx.x == 0) atomicMin(stamps, globaltimer());
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  unsigned acc = 0;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n4; i += stride) {
    const float4 va = __ldcs(a + i), vb = __ldcs(b + i);
    acc ^= __float_as_uint(va.x) ^ __float_as_uint(va.y) ^ __float_as_uint(va.z) ^ __float_as_uint(va.w) ^
           __float_as_uint(vb.x) ^ __float_as_uint(vb.y) ^ __float_as_uint(vb.z) ^ __float_as_uint(vb.w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ unsigned part[kThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned r = 0;
    for (int w = 0; w < kThreads / 32; ++w) r ^= part[w];
    out[blockIdx.x] = r;
    atomicMax(stamps + 1, globaltimer());
  }
}

constexpr int kBulkMaxTile = 8192;  // floats per operand per block (32 KiB)

// One tile of `tile` floats (a multiple of 4) per block; the last block's
// tile is shorter.  Shared memory: a-slice then b-slice; c overwrites a.
__global__ void __launch_bounds__(kThreads, 1)
vadd_f32_bulk(float* __restrict__ c, const float* __restrict__ a, const float* __restrict__ b, int64_t nv, int tile,
              unsigned long long* __restrict__ stamps) {
  using namespace mk::tma;
  extern __shared__ __align__(128) unsigned char bulk_smem[];
  __shared__ __align__(8) uint64_t full;
  float* sa = reinterpret_cast<float*>(bulk_smem);
  float* sb = sa + kBulkMaxTile;
  if (threadIdx.x == 0 && stamps) atomicMin(stamps, globaltimer());
  const int64_t start = (int64_t)blockIdx.x * tile;
  if (start >= nv) return;
  const int len = (int)min((int64_t)tile, nv - start);
  const uint32_t bytes = (uint32_t)len * 4u;
  const uint32_t bar = smem_u32(&full);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_expect_tx(bar, 2u * bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(sa)),
                 "l"(a + start), "r"(bytes), "r"(bar)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(sb)),
                 "l"(b + start), "r"(bytes), "r"(bar)
                 : "memory");
  }
  __syncthreads();  // barrier initialised before anyone waits on it
  volatile int no_abort = 0;
  // an issued copy lands in microseconds; the budget only bounds a fault
  const bool ok = wait_bounded(bar, 0, kDrainCycles, &no_abort);
  if (ok) {
    float4* sa4 = reinterpret_cast<float4*>(sa);
    const float4* sb4 = reinterpret_cast<const float4*>(sb);
    for (int j = threadIdx.x; j < len / 4; j += kThreads) {
      float4 x = sa4[j];
      const float4 y = sb4[j];
      x.x = __fadd_rn(x.x, y.x);
      x.y = __fadd_rn(x.y, y.y);
      x.z = __fadd_rn(x.z, y.z);
      x.w = __fadd_rn(x.w, y.w);
      sa4[j] = x;
    }
    fence_async_smem();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (ok) {
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(c + start), "r"(smem_u32(sa)),
                   "r"(bytes)
                   : "memory");
      bulk_commit();
      bulk_wait_all();
    }
    if (stamps) atomicMax(stamps + 1, globaltimer());
  }
}

}  // namespace

extern "C" int mk_probe_vadd_f32(int mode, float* c, const float* a, const float* b, int64_t n,
                                 unsigned long long* stamps, void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (mode < 0 || mode > 3) return mk::fail(MK_ERR_INVALID, "mk_probe_vadd_f32: mode must be 0..3");
  if (n < 4 || !c || !a || !b || (!stamps && mode < 2))
    return mk::fail(MK_ERR_INVALID, "mk_probe_vadd_f32: need n >= 4 and non-null pointers");
  if (!mk::aligned16(a) || !mk::aligned16(b) || !mk::aligned16(c))
    return mk::fail(MK_ERR_INVALID, "mk_probe_vadd_f32: a, b and c must be 16-byte aligned");
  cudaStream_t s = mk::as_stream(stream);
  const int64_t n4 = n / 4;
  const int64_t max_blocks = (int64_t)dev->sms * (2048 / kThreads);
  int64_t blocks = mk::cdiv(n4, kThreads);
  if (blocks > max_blocks) blocks = max_blocks;
  switch (mode) {
    case 0: probe_empty<<<(unsigned)blocks, kThreads, 0, s>>>(stamps); break;
    case 1: probe_read2<<<(unsigned)blocks, kThreads, 0, s>>>(reinterpret_cast<unsigned*>(c),
                                                             reinterpret_cast<const float4*>(a),
                                                             reinterpret_cast<const float4*>(b), n4, stamps);
      break;
    case 2:
      if (stamps)
        vadd_f32_vec4<true><<<(unsigned)blocks, kThreads, 0, s>>>(
            reinterpret_cast<float4*>(c), reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b), n4,
            stamps);
      else  // the vector vadd launched plainly (no programmatic dependent launch)
        vadd_f32_vec4<false><<<(unsigned)blocks, kThreads, 0, s>>>(
            reinterpret_cast<float4*>(c), reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b), n4,
            nullptr);
      break;
    default: {
      const int64_t nv = n4 * 4;
      int64_t tile = mk::cdiv(mk::cdiv(nv, (int64_t)dev->sms), 4) * 4;
      if (tile > kBulkMaxTile) return mk::fail(MK_ERR_INVALID, "mk_probe_vadd_f32: mode 3 needs n <= SMs x 8192");
      const size_t smem = 2 * kBulkMaxTile * sizeof(float);
      int rc = mk::allow_dynamic_smem(reinterpret_cast<const void*>(vadd_f32_bulk), smem);
      if (rc != MK_OK) return rc;
      vadd_f32_bulk<<<(unsigned)mk::cdiv(nv, tile), kThreads, smem, s>>>(c, a, b, nv, (int)tile, stamps);
    }
  }
  return mk::check_launch("mk_probe_vadd_f32: launch");
}
