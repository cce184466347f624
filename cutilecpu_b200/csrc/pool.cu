// pool.cu — device and pinned-host memory pools of libkernels.so.
//
// The reference allocates host buffers with posix_memalign-backed
// `aligned_array(T, dims; alignment)` (src/allocator.jl:32-61: alignment must
// be a positive power of two and a multiple of sizeof(void*)) and device
// buffers through CUDA.jl's pool (`KA.allocate`, ext/MLIRCUDAExt.jl:140).
// Here:
//   * device memory comes from a per-device CUDA stream-ordered memory pool
//     (cudaMallocFromPoolAsync) whose release threshold keeps freed memory
//     cached, so steady-state allocation costs no driver call;
//   * pinned host memory (the source/destination of fast H2D/D2H copies) is
//     cached per power-of-two size class; blocks are page-aligned, which
//     satisfies every alignment aligned_array accepts up to 4096.
#include <map>
#include <mutex>
#include <vector>

#include "mk_common.cuh"

namespace {

std::mutex g_mu;
cudaMemPool_t g_pools[64] = {};

struct PinnedStats {
  size_t live = 0, cached = 0;
};
std::map<size_t, std::vector<void*>> g_free_pinned;  // size class -> cached blocks
std::map<void*, size_t> g_pinned_class;              // live block -> size class
PinnedStats g_pstats;

size_t size_class(size_t bytes) {
  size_t c = 4096;
  while (c < bytes) c <<= 1;
  return c;
}

int device_pool(int dev, cudaMemPool_t* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t p;
    cudaError_t e = cudaMemPoolCreate(&p, &props);
    if (e != cudaSuccess) return mk::fail_cuda(e, "mk_pool: cudaMemPoolCreate");
    uint64_t keep = ~0ull;  // keep freed memory cached until mk_pool_trim
    e = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
    if (e != cudaSuccess) return mk::fail_cuda(e, "mk_pool: cudaMemPoolSetAttribute");
    g_pools[dev] = p;
  }
  *out = g_pools[dev];
  return MK_OK;
}

}  // namespace

extern "C" int mk_pool_alloc_device(void** ptr, size_t bytes, void* stream) {
  MK_ENTRY_DEVICE(dev);
  if (!ptr) return mk::fail(MK_ERR_INVALID, "mk_pool_alloc_device: null out pointer");
  *ptr = nullptr;
  if (bytes == 0) return MK_OK;
  cudaMemPool_t p;
  int rc = device_pool(dev->id, &p);
  if (rc != MK_OK) return rc;
  cudaError_t e = cudaMallocFromPoolAsync(ptr, bytes, p, mk::as_stream(stream));
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_pool_alloc_device: cudaMallocFromPoolAsync");
  return MK_OK;
}

extern "C" int mk_pool_free_device(void* ptr, void* stream) {
  mk::clear_error();
  if (!ptr) return MK_OK;
  cudaError_t e = cudaFreeAsync(ptr, mk::as_stream(stream));
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_pool_free_device: cudaFreeAsync");
  return MK_OK;
}

extern "C" int mk_host_alloc_aligned(void** ptr, size_t bytes, size_t alignment) {
  mk::clear_error();
  if (!ptr) return mk::fail(MK_ERR_INVALID, "mk_host_alloc_aligned: null out pointer");
  *ptr = nullptr;
  if (alignment == 0) return mk::fail(MK_ERR_INVALID, "alignment must be positive, got 0");
  if (alignment & (alignment - 1))
    return mk::fail(MK_ERR_INVALID, "alignment must be a power of two, got " + std::to_string(alignment));
  if (alignment % sizeof(void*))
    return mk::fail(MK_ERR_INVALID, "alignment (" + std::to_string(alignment) +
                                        ") must be a multiple of sizeof(void*) (=" + std::to_string(sizeof(void*)) + ")");
  if (alignment > 4096)
    return mk::fail(MK_ERR_INVALID, "alignment above the page size (4096) is not supported for pinned memory");
  if (bytes == 0) return MK_OK;
  const size_t c = size_class(bytes);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_free_pinned.find(c);
    if (it != g_free_pinned.end() && !it->second.empty()) {
      *ptr = it->second.back();
      it->second.pop_back();
      g_pinned_class[*ptr] = c;
      g_pstats.cached -= c;
      g_pstats.live += c;
      return MK_OK;
    }
  }
  void* p = nullptr;
  cudaError_t e = cudaHostAlloc(&p, c, cudaHostAllocPortable);
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_host_alloc_aligned: cudaHostAlloc");
  std::lock_guard<std::mutex> lk(g_mu);
  g_pinned_class[p] = c;
  g_pstats.live += c;
  *ptr = p;
  return MK_OK;
}

extern "C" int mk_host_free(void* ptr) {
  mk::clear_error();
  if (!ptr) return MK_OK;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_pinned_class.find(ptr);
  if (it == g_pinned_class.end()) return mk::fail(MK_ERR_INVALID, "mk_host_free: pointer not from mk_host_alloc_aligned");
  g_free_pinned[it->second].push_back(ptr);
  g_pstats.live -= it->second;
  g_pstats.cached += it->second;
  g_pinned_class.erase(it);
  return MK_OK;
}

extern "C" int mk_pool_stats(size_t* device_reserved, size_t* device_used, size_t* pinned_live,
                             size_t* pinned_cached) {
  MK_ENTRY_DEVICE(dev);
  cudaMemPool_t p;
  int rc = device_pool(dev->id, &p);
  if (rc != MK_OK) return rc;
  uint64_t reserved = 0, used = 0;
  cudaMemPoolGetAttribute(p, cudaMemPoolAttrReservedMemCurrent, &reserved);
  cudaMemPoolGetAttribute(p, cudaMemPoolAttrUsedMemCurrent, &used);
  if (device_reserved) *device_reserved = reserved;
  if (device_used) *device_used = used;
  std::lock_guard<std::mutex> lk(g_mu);
  if (pinned_live) *pinned_live = g_pstats.live;
  if (pinned_cached) *pinned_cached = g_pstats.cached;
  return MK_OK;
}

extern "C" int mk_pool_trim(void) {
  MK_ENTRY_DEVICE(dev);
  cudaMemPool_t p;
  int rc = device_pool(dev->id, &p);
  if (rc != MK_OK) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemPoolTrimTo(p, 0);
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_pool_trim");
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto& kv : g_free_pinned)
    for (void* q : kv.second) cudaFreeHost(q);
  g_free_pinned.clear();
  g_pstats.cached = 0;
  return MK_OK;
}
