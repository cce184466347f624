// api.cu — library-wide entry points of libkernels.so: version, last error,
// per-device initialisation, the device error word and reduction scratch.
//
// The reference resolves everything per launch in Julia (ext/MLIRCUDAExt.jl:
// 287-310 compiles and caches a CuFunction; :317-335 wires CUDA.jl's exception
// flag).  Here the kernels are precompiled for sm_100a, so "initialisation" is
// only: query the SM count, locate the error word, and hand out scratch.
#include <stdlib.h>

#include <atomic>
#include <map>
#include <tuple>
#include <mutex>
#include <utility>

#include <cudaTypedefs.h>

#include "mk_common.cuh"

// One error word per device: every module global exists once per device
// context.  Kernels receive its address as an argument.
static __device__ unsigned g_mk_error_word;

namespace mk {

static thread_local std::string t_last_error;
static std::mutex g_mu;
static constexpr int kMaxDevices = 64;
static Device g_devices[kMaxDevices];
// Set (release) once a device's state is complete; read (acquire) lock-free.
static std::atomic<int> g_ready[kMaxDevices];
static std::map<std::pair<int, cudaStream_t>, ReduceScratch> g_scratch;
struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};
static std::map<std::tuple<int, cudaStream_t, int>, Workspace> g_workspace;

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int fail_cuda(cudaError_t e, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return MK_ERR_CUDA;
}

void clear_error() { t_last_error.clear(); }

static int init_device_locked(int id) {
  Device& d = g_devices[id];
  if (d.id == id) return MK_OK;
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  if (prev != id && (e = cudaSetDevice(id)) != cudaSuccess) return fail_cuda(e, "cudaSetDevice");
  int sms = 0, smem = 0;
  int rc = MK_OK;
  void* word = nullptr;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, id)) != cudaSuccess)
    rc = fail_cuda(e, "cudaDeviceGetAttribute(MultiProcessorCount)");
  else if ((e = cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, id)) != cudaSuccess)
    rc = fail_cuda(e, "cudaDeviceGetAttribute(MaxSharedMemoryPerBlockOptin)");
  else if ((e = cudaGetSymbolAddress(&word, g_mk_error_word)) != cudaSuccess)
    rc = fail_cuda(e, "cudaGetSymbolAddress(error word)");
  if (rc == MK_OK) {
    d.sms = sms;
    d.max_smem_optin = smem;
    d.err_word = static_cast<unsigned*>(word);
    d.id = id;
    g_ready[id].store(1, std::memory_order_release);
  }
  if (prev != id) cudaSetDevice(prev);
  return rc;
}

Device* current_device() {
  int id = -1;
  cudaError_t e = cudaGetDevice(&id);
  if (e != cudaSuccess) {
    fail_cuda(e, "cudaGetDevice");
    return nullptr;
  }
  if (id < 0 || id >= kMaxDevices) {
    fail(MK_ERR_INVALID, "device ordinal out of range");
    return nullptr;
  }
  if (g_ready[id].load(std::memory_order_acquire)) return &g_devices[id];
  std::lock_guard<std::mutex> lk(g_mu);
  if (init_device_locked(id) != MK_OK) return nullptr;
  return &g_devices[id];
}

int reduce_scratch(Device* d, cudaStream_t s, ReduceScratch* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_pair(d->id, s);
  auto it = g_scratch.find(key);
  if (it != g_scratch.end()) {
    *out = it->second;
    return MK_OK;
  }
  // One allocation per (device, stream): partials then the ticket word.
  void* p = nullptr;
  size_t bytes = sizeof(double) * kMaxReduceBlocks + 256;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail_cuda(e, "cudaMalloc(reduce scratch)");
  // The ticket starts at zero; every reduction leaves it at zero again.  The
  // zeroing is ordered on `s` itself: a plain cudaMemset runs on the legacy
  // default stream, which does not order a non-blocking stream's next kernel.
  e = cudaMemsetAsync(p, 0, bytes, s);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail_cuda(e, "cudaMemsetAsync(reduce scratch)");
  }
  ReduceScratch rs;
  rs.partials = static_cast<double*>(p);
  rs.ticket = reinterpret_cast<unsigned*>(static_cast<char*>(p) + sizeof(double) * kMaxReduceBlocks);
  g_scratch[key] = rs;
  *out = rs;
  return MK_OK;
}

int stream_workspace(Device* d, cudaStream_t s, size_t bytes, void** out, int slot) {
  std::lock_guard<std::mutex> lk(g_mu);
  Workspace& w = g_workspace[std::make_tuple(d->id, s, slot)];
  if (w.bytes < bytes) {
    if (w.ptr) {
      // the old buffer may still be read by work queued on this stream
      cudaError_t e = cudaStreamSynchronize(s);
      if (e != cudaSuccess) return fail_cuda(e, "workspace: cudaStreamSynchronize");
      cudaFree(w.ptr);
      w.ptr = nullptr;
      w.bytes = 0;
    }
    cudaError_t e = cudaMalloc(&w.ptr, bytes);
    if (e != cudaSuccess) {
      w.ptr = nullptr;
      return fail_cuda(e, "workspace: cudaMalloc");
    }
    w.bytes = bytes;
  }
  *out = w.ptr;
  return MK_OK;
}

int allow_dynamic_smem(const void* kernel, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> done;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lk(mu);
  size_t& have = done[std::make_pair(dev, kernel)];
  if (have >= bytes) return MK_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return fail_cuda(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  have = bytes;
  return MK_OK;
}

unsigned long long wait_limit_cycles() {
  static unsigned long long v = [] {
    const char* e = getenv("MK_WAIT_LIMIT_CYCLES");
    unsigned long long x = e ? strtoull(e, nullptr, 10) : 0ull;
    return x ? x : (1ull << 32);
  }();
  return v;
}

int encode_rows_f32(CUtensorMap* map, const float* base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                    uint32_t box_rows, const char* who) {
  using Fn = PFN_cuTensorMapEncodeTiled_v12000;
  static Fn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<Fn>(p);
  }();
  if (!fn) return fail(MK_ERR_CUDA, std::string(who) + ": cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MK_ERR_CUDA, std::string(who) + ": cuTensorMapEncodeTiled failed");
  return MK_OK;
}

}  // namespace mk

extern "C" {

int mk_version(void) { return 100; }  // 0.1.0

const char* mk_last_error(void) { return mk::t_last_error.c_str(); }

int mk_init(int device) {
  mk::clear_error();
  if (device < 0 || device >= mk::kMaxDevices) return mk::fail(MK_ERR_INVALID, "mk_init: device ordinal out of range");
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_init: cudaGetDeviceCount");
  if (device >= count) return mk::fail(MK_ERR_INVALID, "mk_init: no such CUDA device");
  std::lock_guard<std::mutex> lk(mk::g_mu);
  return mk::init_device_locked(device);
}

int mk_error_poll(void* stream) {
  MK_ENTRY_DEVICE(dev);
  cudaStream_t s = mk::as_stream(stream);
  unsigned word = 0;
  cudaError_t e = cudaMemcpyAsync(&word, dev->err_word, sizeof(word), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_error_poll: reading the error word");
  if (word == 0) return MK_OK;
  const unsigned zero = 0;
  e = cudaMemcpyAsync(dev->err_word, &zero, sizeof(zero), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return mk::fail_cuda(e, "mk_error_poll: clearing the error word");
  std::string msg = "device fault:";
  if (word & mk::ERRBIT_GATHER_INDEX) msg += " gather index out of bounds;";
  if (word & mk::ERRBIT_HIST_KEY) msg += " histogram key out of range;";
  if (word & mk::ERRBIT_TIMEOUT) {
    msg += " bounded device wait timed out;";
    mk::fail(MK_ERR_TIMEOUT, msg);
    return MK_ERR_TIMEOUT;
  }
  return mk::fail(MK_ERR_DEVICE_FAULT, msg);
}

}  // extern "C"
