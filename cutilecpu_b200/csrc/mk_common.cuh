// mk_common.cuh — shared host/device plumbing of libkernels.so: status
// reporting, per-device state, launch-geometry helpers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string>

#include "../../include/mk_kernels.h"

namespace mk {

// Bits of the per-device error word (set by kernels with atomicOr).
enum : unsigned {
  ERRBIT_GATHER_INDEX = 1u << 0,  // gather index outside [1, na]
  ERRBIT_HIST_KEY = 1u << 1,      // histogram key outside [1, nbins]
  ERRBIT_TIMEOUT = 1u << 2,       // a bounded device wait gave up
};

// Per-device state, created once under a mutex (api.cu).
struct Device {
  int id = -1;
  int sms = 0;                 // multiprocessor count (148 on B200)
  int max_smem_optin = 0;      // bytes of shared memory a block may opt into
  unsigned* err_word = nullptr;  // device address of the error word
};

// Thread-local error message; returns `code` for tail-calling.
int fail(int code, const std::string& msg);
int fail_cuda(cudaError_t e, const char* what);
void clear_error();

// Current device's state (initialised lazily). nullptr + message on failure.
Device* current_device();

// Scratch for the deterministic two-level reductions, private to one
// (device, stream) pair: partials[kMaxReduceBlocks] doubles, then a u32 ticket
// that the last block of every reduction resets to zero.
constexpr int kMaxReduceBlocks = 4096;
struct ReduceScratch {
  double* partials = nullptr;
  unsigned* ticket = nullptr;
};
int reduce_scratch(Device* d, cudaStream_t s, ReduceScratch* out);

// Growable device workspace private to one (device, stream, slot), for kernels
// that stage re-laid-out operands (the 3xTF32 GEMM's hi/lo panels) or keep
// per-tile state (scan, dims reductions).  Grows with cudaMalloc (after a
// cudaFree of the smaller buffer, once the stream has drained); never shrinks.
enum : int { WS_GEMM = 0, WS_SCAN = 1, WS_DIMS = 2, WS_FIND = 3, WS_GEMM_SPLIT = 4 };
int stream_workspace(Device* d, cudaStream_t s, size_t bytes, void** out, int slot);

// Bounded device waits give up after this many SM clock cycles (env
// MK_WAIT_LIMIT_CYCLES overrides; default ~2 s at 1.9 GHz).
unsigned long long wait_limit_cycles();

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (device, kernel).
int allow_dynamic_smem(const void* kernel, size_t bytes);

// Tensor map of a row-major (rows x cols) fp32 array for 2-D TMA copies of
// box_rows x box_cols boxes with 128-byte swizzle (box_cols * 4 <= 128).
// base must be 16-byte aligned and cols a multiple of 4.
int encode_rows_f32(CUtensorMap* map, const float* base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                    uint32_t box_rows, const char* who);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch-result check: a bad launch configuration is reported immediately.
inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, what);
  return MK_OK;
}

}  // namespace mk

#define MK_ENTRY_DEVICE(dev)                      \
  mk::clear_error();                              \
  mk::Device* dev = mk::current_device();         \
  if (!dev) return MK_ERR_CUDA;
