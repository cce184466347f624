/*
 * mk_kernels.h — C ABI of libkernels.so, the B200 (sm_100a) kernel library
 * that replaces the JIT-compiled GPU path of MLIRKernels.jl (gbaraldi/cuTileCPU)
 * for five data-parallel kernels: vadd, mapreduce, gather, histogram and the
 * 16x16 @localmem tiled matmul.
 *
 * Conventions (all entry points):
 *   - Return an int status: MK_OK (0) or a negative MK_ERR_* code. On failure a
 *     human-readable message is available from mk_last_error() (thread-local),
 *     mirroring the descriptive Julia `error(...)` strings the reference raises
 *     in its launcher (ext/MLIRCUDAExt.jl:428-438, 483-497, 516-537).
 *   - Every pointer argument is a DEVICE pointer on the current CUDA device,
 *     owned by the caller; the library never frees caller memory
 *     (the reference launcher never allocates user data either:
 *     ext/MLIRCUDAExt.jl:540-548).
 *   - Every launch is asynchronous on the caller's stream (`stream` is a
 *     cudaStream_t passed as void*; NULL = legacy default stream), as CUDA.jl
 *     launches on its task-local stream (ext/MLIRCUDAExt.jl:546).
 *   - Index arrays (gather indices, histogram keys) are 1-BASED Int32, as in
 *     the Julia kernels.  Matrices are COLUMN-MAJOR (Julia layout).
 *   - Device-side faults that the reference turns into a KernelException at the
 *     next synchronize (src/lower.jl:1673-1703, ext/MLIRCUDAExt.jl:317-335) —
 *     here: an out-of-range gather index or histogram key — set a per-device
 *     error word; the offending element is skipped (gather writes 0).
 *     mk_error_poll() synchronises the stream and returns/clears that word.
 *   - Thread-safe: per-device state is created under a mutex; scratch used by
 *     the reductions is private to each (device, stream) pair.
 */
#ifndef MK_KERNELS_H
#define MK_KERNELS_H

#include <stdint.h>

#if defined(__GNUC__)
#define MK_API __attribute__((visibility("default")))
#else
#define MK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
#define MK_OK                 0
#define MK_ERR_INVALID       -1  /* bad argument (size, pointer, enum)              */
#define MK_ERR_CUDA          -2  /* a CUDA runtime/driver call failed                */
#define MK_ERR_NCCL          -3  /* reserved for collective failures                 */
#define MK_ERR_TIMEOUT       -4  /* a bounded device wait ran out                    */
#define MK_ERR_DEVICE_FAULT  -5  /* a kernel flagged bad input (index out of range)  */

/* ---- mapreduce selectors ------------------------------------------------ */
/* f: the element map applied before the reduction (Julia `f` in mapreduce). */
#define MK_F_IDENTITY 0   /* x            (sum, maximum, minimum, prod)       */
#define MK_F_ABS2     1   /* x*x          (sum(abs2, x), sum(x.^2))           */
#define MK_F_ABS      2   /* |x|                                              */
#define MK_F_GT0      3   /* x > 0 ? 1 : 0  (count(>(0), x))                  */
/* op: the associative reduction operator. */
#define MK_OP_ADD 0
#define MK_OP_MAX 1
#define MK_OP_MIN 2
#define MK_OP_MUL 3

/* Library version (major*10000 + minor*100 + patch). */
MK_API int mk_version(void);

/* Message for the last failing call on this host thread ("" if none). */
MK_API const char* mk_last_error(void);

/* Set up per-device state for `device` (SM count, error word).  Optional:
 * every entry point initialises the current device lazily.
 * Replaces the first-launch codegen/CuModule set-up of ext/MLIRCUDAExt.jl:287-310. */
MK_API int mk_init(int device);

/* Synchronise `stream`, then return MK_ERR_DEVICE_FAULT (and clear the word)
 * if any kernel on the current device flagged bad input since the last poll.
 * Replaces the KernelException check of ext/MLIRCUDAExt.jl:317-335. */
MK_API int mk_error_poll(void* stream);

/* c[i] = a[i] + b[i], i in [0, n).  fp32 IEEE round-to-nearest, bit-exact.
 * Replaces a KA launch of the vadd kernel (test/test_gpu_simt.jl:13-16,
 * examples/reflection_and_perf.jl:11-14) through ext/MLIRCUDAExt.jl:540-548. */
MK_API int mk_vadd_f32(float* c, const float* a, const float* b, int64_t n, void* stream);

/* Measurement probe with no counterpart in the reference: the parts of a
 * small vadd's time (mode 0 empty kernel, 1 read a and b only, 2 the vector
 * vadd, 3 a bulk-copy vadd through shared memory), each with the grid of
 * mk_vadd_f32.  stamps[0] / stamps[1] receive the earliest block start and
 * latest block end in ns of the device clock (the caller sets stamps[0] to
 * ~0 and stamps[1] to 0 first; stamps may be NULL for modes 2 and 3, and
 * mode 2 without stamps is the vector vadd launched without programmatic
 * dependent launch).  Mode 1 writes one u32 per block into c;
 * modes 2 and 3 write c = a + b.  a, b, c 16-byte aligned; mode 3 needs
 * n <= SMs x 8192. */
MK_API int mk_probe_vadd_f32(int mode, float* c, const float* a, const float* b, int64_t n,
                             unsigned long long* stamps, void* stream);

/* out[i] = alpha*x[i] + beta*y[i] (y may be NULL: out[i] = alpha*x[i]),
 * fp32 in Julia's order without FMA contraction, bit-exact.  Replaces
 * AK.map!(x -> a*x, dst, src) and broadcasts like 2f0 .* a, a .+ b
 * (test/test_downstream_ka.jl:18-20, test/test_gpuarrays.jl:31-32). */
MK_API int mk_axpby_f32(float* out, float alpha, const float* x, float beta, const float* y, int64_t n,
                        void* stream);

/* out_dev[0] = op(init, op_{i<n} f(x[i])) as fp64, written on the device.
 * Sums/products accumulate in fp64 (per-thread fp32 groups of <= 8 terms);
 * max/min are exact.  Deterministic for a given device model.  n == 0 gives init.
 * Replaces GPUArrays.mapreducedim! -> AK.mapreduce (ext/MLIRCUDAExt.jl:100-121)
 * and AK.reduce on an MLIRArray (test/test_downstream_ka.jl:27-31). */
MK_API int mk_mapreduce_f32(double* out_dev, const float* x, int64_t n,
                     int f, int op, double init, void* stream);

/* Allocation-free mk_mapreduce_f32, for callers that cannot let a library
 * call cudaMalloc (device memory owned by the host's own pool allocator, e.g.
 * CUDA.jl's or torch's, or a fixed budget set at start-up).  It has no
 * counterpart in the reference.  Its scratch is one static device array that
 * every GPU loading libkernels.so holds until exit: MK_NOALLOC_MAX_PARTIALS
 * fp64 block partials (32 KiB) and a ticket word.  It calls no cudaMalloc,
 * cudaFree or allocating library routine.  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress); make that first call
 * before any stream capture.  All calls on a device share the array, so calls
 * that overlap on the GPU (e.g. on two streams at once) race; serialise them.
 * Each call clears the ticket before its launch.  A launch that would need more
 * block partials than the array holds is rejected with MK_ERR_INVALID; n itself
 * is not limited because the grid strides over x.  Same result, bit for bit,
 * as mk_mapreduce_f32. */
#define MK_NOALLOC_MAX_PARTIALS 4096
MK_API int mk_mapreduce_f32_noalloc(double* out_dev, const float* x, int64_t n,
                                    int f, int op, double init, void* stream);

/* sum(x.^2) == mk_mapreduce_f32(out, x, n, MK_F_ABS2, MK_OP_ADD, 0.0, stream). */
MK_API int mk_sum_sq_f32(double* out_dev, const float* x, int64_t n, void* stream);

/* Reduction of one dimension of a column-major Float32 array viewed as
 * (pre, len, post), the reduced dimension in the middle:
 *   out[p + q*pre] = op(init, op_{k<len} f(x[p + k*pre + q*pre*len]))
 * for p < pre, q < post; out has pre*post Float32 elements (len == 0 gives
 * init).  fp64 accumulation, one rounding to Float32; deterministic.  May use
 * a per-stream workspace of up to 1024*pre*post doubles when pre*post is small.
 * Replaces the dims form of GPUArrays.mapreducedim! (ext/MLIRCUDAExt.jl:114-119;
 * sum/maximum/minimum(m; dims=d), test/test_gpuarrays.jl:98-107). */
MK_API int mk_mapreduce_dim_f32(float* out, const float* x, int64_t pre, int64_t len, int64_t post,
                                int f, int op, double init, void* stream);

/* Prefix scan: out[i] = op(init, x[0], ..., x[i]) (inclusive) or
 * op(init, x[0], ..., x[i-1]) (exclusive != 0; out[0] = init), op in
 * {MK_OP_ADD, MK_OP_MAX, MK_OP_MIN, MK_OP_MUL}.  Single-pass decoupled
 * look-back, fp64 carries, each output rounded once to Float32; bounded waits
 * (MK_ERR_TIMEOUT via mk_error_poll).  Uses a per-stream workspace of about
 * 5 bytes per 1024 elements.  out may alias x.  Replaces AK.accumulate! /
 * cumsum on an MLIRArray (test/test_downstream_ka.jl:39-42, 75-78). */
MK_API int mk_accumulate_f32(float* out, const float* x, int64_t n, int op, double init, int exclusive,
                             void* stream);

/* findmax (find_max != 0) or findmin of x[0, n), n >= 1: the extreme value
 * (as fp64) and its 1-based index, written on the device.  Julia's rules: NaN
 * counts as the maximum for findmax and as the minimum for findmin, +0.0 ranks
 * above -0.0, the first index wins ties.  Replaces findmax/findmin/argmax/
 * argmin on an MLIRArray (test/test_gpuarrays.jl:124-128). */
MK_API int mk_findext_f32(double* val_out, int64_t* idx_out, const float* x, int64_t n, int find_max,
                          void* stream);

/* c[i] = a[idx1[i] - 1], i in [0, n); idx1 is 1-based into a[0, na).
 * Out-of-range indices write 0 and set the device error word.  Bit-exact.
 * Replaces a KA launch of `c[i] = a[idx[i]]` (indexing semantics
 * src/lower.jl:4031-4140, 1-based -> 0-based at :4064-4077). */
MK_API int mk_gather_f32(float* c, const float* a, int64_t na, const int32_t* idx1,
                  int64_t n, void* stream);

/* Measurement probe with no counterpart in the reference: n independent
 * 4-byte reads of a[0, na) at positions hashed from the element number, with
 * the loads, grid and loads in flight of mk_gather_f32 but no index or output
 * stream.  Its duration is this GPU's ceiling for the gather's random reads.
 * sums receives one u32 (XOR of the bits read) per block: SMs x 8 values,
 * sums_len must be at least that.  seed varies the positions. */
MK_API int mk_probe_random_read_f32(unsigned* sums, int64_t sums_len, const float* a, int64_t na, int64_t n,
                                    unsigned seed, void* stream);

/* counts[keys1[i] - 1] += 1 for i in [0, n), u32 wrap-around, ACCUMULATING into
 * the caller's counts (as `@atomic bins[idx[i]] += 1` does).  Keys outside
 * [1, nbins] are skipped and set the device error word.  Bit-exact.
 * Replaces the histogram kernels of test/test_ka_cpu.jl:16-19 and
 * test/test_gpu_simt.jl:49-73 (atomic kind: src/lower.jl:3600-3623). */
MK_API int mk_hist_u32(uint32_t* counts, int32_t nbins, const int32_t* keys1, int64_t n,
                void* stream);

/* C[M,N] = A[M,K] * B[K,N], column-major with leading dimensions lda>=M,
 * ldb>=K, ldc>=M, fp32 in/out.  Computed on the tcgen05 tensor cores in 3xTF32
 * split precision (a_hi*b_hi + a_hi*b_lo + a_lo*b_hi, fp32 accumulation in
 * TMEM): within ~1e-6 relative (Frobenius) of an fp64 product for K=8192.
 * Only the first 16*floor(K/16) columns of A / rows of B take part, as in the
 * reference tiled kernel, which ignores the K % 16 remainder
 * (examples/tiled_matmul.jl:34).  Replaces mm_tiled! launches
 * (examples/tiled_matmul.jl:28-48).  Row-major callers compute C^T = B^T A^T by
 * swapping operands.  Uses a per-stream device workspace of (M+N)*2*K*4 bytes
 * for the split operands, plus up to 8*M*N*4 bytes of split-K partials when
 * the 128x256 tiles are fewer than the SMs (allocated on first use, grown as
 * needed). */
MK_API int mk_sgemm_3xtf32(float* C, const float* A, const float* B,
                           int64_t M, int64_t N, int64_t K,
                           int64_t lda, int64_t ldb, int64_t ldc, void* stream);

/* LinearAlgebra.mul!(C, A, B) on MLIRArrays: the same tcgen05 3xTF32 GEMM as
 * mk_sgemm_3xtf32 but over ALL K terms (the K % 16 remainder is zero-padded in
 * the split operands), i.e. the semantics of the naive kernel mm_naive!
 * (examples/tiled_matmul.jl:12-19, which the reference benchmarks against
 * CUBLAS mul! at :85).  Same layout, workspace and accuracy. */
MK_API int mk_sgemm_f32(float* C, const float* A, const float* B,
                        int64_t M, int64_t N, int64_t K,
                        int64_t lda, int64_t ldb, int64_t ldc, void* stream);

/* Histogram with the element types of the reference's other histogram forms:
 * bins of type bin_type (MK_BIN_U32: UInt32/Int32 bits, wrap-around;
 * MK_BIN_I64: Int64, two's complement; MK_BIN_F32: Float32, exact while a bin
 * stays below 2^24), 1-based keys of type key_type (MK_KEY_I32 / MK_KEY_I64).
 * Same accumulation and error rules as mk_hist_u32.  Covers the KA example of
 * test/test_gpu_simt.jl:49-73 (Int keys, Int bins) and the Float32 bins of
 * test/test_ka_cpu.jl:16-19, 67-79. */
#define MK_BIN_U32 0
#define MK_BIN_I64 1
#define MK_BIN_F32 2
#define MK_KEY_I32 0
#define MK_KEY_I64 1
MK_API int mk_hist(void* bins, int bin_type, int32_t nbins, const void* keys1, int key_type, int64_t n,
                   void* stream);

/* The reference's own algorithm on CUDA cores: one output per thread, 16x16
 * shared-memory tiles, K % 16 ignored (examples/tiled_matmul.jl:28-48).  Kept
 * as the SIMT comparison point for the tensor-core path; same argument rules. */
MK_API int mk_matmul_tiled16_f32(float* C, const float* A, const float* B,
                          int64_t M, int64_t N, int64_t K,
                          int64_t lda, int64_t ldb, int64_t ldc, void* stream);

/* ---- fused multi-GPU reduction (one process per GPU) ----------------------
 * The reference is single-GPU; this is the exchange step of the sharded
 * mapreduce.  Each rank creates a small peer mailbox on its device and gets
 * its CUDA IPC handle (mk_peer_handle_size() bytes); the host exchanges the
 * handles (e.g. an all-gather over the process group); every rank then maps
 * the others' mailboxes with mk_peer_connect(all world handles, rank order).
 * mk_mapreduce_f32_allreduce is mk_mapreduce_f32 whose last block also
 * writes its fp64 partial into every rank's mailbox over NVLink and folds
 * all ranks' partials in rank order (bounded wait; MK_ERR_TIMEOUT via
 * mk_error_poll if a rank never arrives): every rank gets the same result,
 * with no separate collective launch.  Each partial travels as one tagged
 * 8-byte word (its 4 lowest mantissa bits carry the epoch), which leaves
 * fp32-derived partials (max, min) exact and truncates an fp64 sum partial by
 * at most 2^-48 relative.  All ranks must call it the same number
 * of times, on their own GPU.  mk_peer_destroy synchronises the device and
 * releases the mailbox. */
MK_API int mk_peer_handle_size(void);
MK_API int mk_peer_create(int world, int rank, void* handle_out);
MK_API int mk_peer_connect(const void* handles);
MK_API int mk_peer_destroy(void);
MK_API int mk_mapreduce_f32_allreduce(double* out_dev, const float* x, int64_t n,
                                      int f, int op, double init, void* stream);

/* Pipelined form of mk_mapreduce_f32_allreduce for a stream of reductions
 * (no counterpart in the single-GPU reference).  The launch reduces this
 * rank's shard and publishes its partial to every rank, but does not wait
 * for the other ranks: the global result of a call is written to its out_dev
 * by the NEXT exchanging launch on this device (this function or the blocking
 * one), which folds it at its end, or by mk_allreduce_complete(stream).  So a
 * rank never stalls on a slower peer inside a step; only the completion waits.
 * The result is bit-identical to the blocking form's.  Until it is completed,
 * out_dev must stay allocated; all exchanging calls and the completion must
 * be issued on one stream per device, in the same order on every rank.
 * mk_allreduce_complete is a no-op when nothing is pending. */
MK_API int mk_mapreduce_f32_allreduce_async(double* out_dev, const float* x, int64_t n,
                                            int f, int op, double init, void* stream);
MK_API int mk_allreduce_complete(void* stream);

/* Fused multi-GPU histogram (no counterpart in the single-GPU reference):
 * mk_hist_u32 into this rank's `counts`, then, in the same launch, the
 * exchange that an NCCL all-reduce of the counts would do: global_out[b] =
 * sum over ranks of counts[b] (u32, wrapping), on every rank.  The last block
 * writes each count, tagged with the epoch, into every rank's mailbox over
 * NVLink.  The blocking form waits (bounded; MK_ERR_TIMEOUT via mk_error_poll
 * if a rank never arrives) and writes global_out before the launch ends.  The
 * _async form does not wait: its global_out is written by the next histogram
 * exchange on this device or by mk_hist_allreduce_complete(stream), with the
 * same rules as mk_mapreduce_f32_allreduce_async.  1 <= nbins <= 16384;
 * Int32 keys, UInt32 counts; counts and global_out are
 * distinct buffers. */
MK_API int mk_hist_u32_allreduce(uint32_t* global_out, uint32_t* counts, int32_t nbins,
                                 const int32_t* keys1, int64_t n, void* stream);
MK_API int mk_hist_u32_allreduce_async(uint32_t* global_out, uint32_t* counts, int32_t nbins,
                                       const int32_t* keys1, int64_t n, void* stream);
MK_API int mk_hist_allreduce_complete(void* stream);

/* Diagnostic with no counterpart in the reference: when entries > 0, every
 * exchanging launch on this device writes 4 device-clock stamps (ns of
 * %globaltimer) into log_dev[4*(epoch % entries) ...]: kernel start, start of
 * the last block's exchange, partial published, pending result folded.
 * entries = 0 turns it off.  Needs the mailbox (mk_peer_create). */
MK_API int mk_peer_trace(unsigned long long* log_dev, int entries);

/* ---- memory pools -------------------------------------------------------
 * Device memory from a per-device stream-ordered pool that keeps freed memory
 * cached (allocation and free are ordered on `stream`); replaces the CUDA.jl
 * pool behind KA.allocate(::MLIRCUDABackend, T, dims) (ext/MLIRCUDAExt.jl:140). */
#include <stddef.h>
MK_API int mk_pool_alloc_device(void** ptr, size_t bytes, void* stream);
MK_API int mk_pool_free_device(void* ptr, void* stream);

/* Pinned (page-locked) host memory, cached per power-of-two size class and
 * page-aligned, with the alignment rules of aligned_array
 * (src/allocator.jl:32-61): alignment must be positive, a power of two and a
 * multiple of sizeof(void*) (here also <= 4096); violations return
 * MK_ERR_INVALID with the reference's message.  The host side of fast
 * H2D/D2H copies. */
MK_API int mk_host_alloc_aligned(void** ptr, size_t bytes, size_t alignment);
MK_API int mk_host_free(void* ptr);

/* Pool occupancy (any out pointer may be NULL) and release of cached memory. */
MK_API int mk_pool_stats(size_t* device_reserved, size_t* device_used, size_t* pinned_live,
                         size_t* pinned_cached);
MK_API int mk_pool_trim(void);

#ifdef __cplusplus
}
#endif

#endif /* MK_KERNELS_H */
