/*
 * oracle.c — TEST INFRASTRUCTURE ONLY.  CPU restatement of the reference's
 * (gbaraldi/cuTileCPU, MLIRKernels.jl) algorithm for the five hot-path kernels.
 * Only the tests, __graft_entry__.smoke() and bench.py's CPU-baseline /
 * reference legs may load this library, and only as the checker or as the
 * timed CPU baseline; the product path (libkernels.so) never calls it.
 *
 * Two parts:
 *
 *  (1) Checkers (or_*): single-threaded, exact or fp64, following the
 *      reference's kernel semantics (1-based indices, column-major matrices,
 *      K % 16 ignored by the tiled matmul, u32 wrap-around histogram counts).
 *
 *  (2) The reference's CPU execution model restated (mlirb_*): KA @kernel on
 *      the CPU `MLIRBackend` runs `prod(ndrange)/W` blocks of W lanes on an
 *      OpenMP `parallel for` (src/lower.jl:626-786 emits scf.parallel over
 *      blocks with a vector<W> body; src/compile.jl:32-81 lowers scf->openmp;
 *      src/launch.jl:72-163 runs it), requires ndrange % W == 0
 *      (ext/KernelAbstractionsExt.jl:256-258), gathers indirect loads per lane
 *      (src/lower.jl:4134-4140) and scalarises per-lane atomics
 *      (src/lower.jl:3946-3965).  Compiled -O2 -march=native -fopenmp like the
 *      reference's `clang -O2 ... -lomp` (src/compile.jl:243-245).  The Julia
 *      reference itself cannot run here (no julia, unpinned deps), so this
 *      restatement is the CPU baseline ("kind": "port").
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_OK 0
#define OR_ERR_INVALID -1
#define OR_ERR_DEVICE_FAULT -5

/* selectors: identical values to include/mk_kernels.h */
enum { F_IDENTITY = 0, F_ABS2 = 1, F_ABS = 2, F_GT0 = 3 };
enum { OP_ADD = 0, OP_MAX = 1, OP_MIN = 2, OP_MUL = 3 };

int or_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void or_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------------------------------------------------- */
/* (1) checkers                                                               */
/* ------------------------------------------------------------------------- */

/* vadd: test/test_gpu_simt.jl:13-16 — c[i] = a[i] + b[i], fp32 RN. */
void or_vadd_f32(float* c, const float* a, const float* b, int64_t n) {
  for (int64_t i = 0; i < n; ++i) c[i] = a[i] + b[i];
}

static double map_f(int f, float v) {
  switch (f) {
    case F_ABS2: return (double)v * (double)v;
    case F_ABS: return fabs((double)v);
    case F_GT0: return v > 0.0f ? 1.0 : 0.0;
    default: return (double)v;
  }
}

/* Julia's max/min on floats: a NaN operand wins; +0.0 > -0.0. */
static double jl_max(double a, double b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
static double jl_min(double a, double b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}

/* mapreduce(f, op, x; init) in fp64, sequential: the semantics of Base
 * mapreduce that GPUArrays.mapreducedim! (ext/MLIRCUDAExt.jl:100-121) must
 * reproduce; x^2 is taken exactly in fp64 here (the oracle for rel 1e-5). */
double or_mapreduce_f64(const float* x, int64_t n, int f, int op, double init) {
  double acc = init;
  if (op == OP_ADD) {
    /* pairwise-free compensated sum: Neumaier, so the fp64 oracle itself is
     * accurate to ~1 ulp of fp64 even at n = 2^28 */
    double s = 0.0, comp = 0.0;
    for (int64_t i = 0; i < n; ++i) {
      double v = map_f(f, x[i]);
      double t = s + v;
      if (fabs(s) >= fabs(v)) comp += (s - t) + v;
      else comp += (v - t) + s;
      s = t;
    }
    return init + (s + comp);
  }
  for (int64_t i = 0; i < n; ++i) {
    double v = map_f(f, x[i]);
    if (op == OP_MUL) acc *= v;
    else if (op == OP_MAX) acc = jl_max(acc, v);
    else acc = jl_min(acc, v);
  }
  return acc;
}

/* dims reduction: out[p + q*pre] = op(init, op_k f(x[p + k*pre + q*pre*len]))
 * in fp64 (the dims form of mapreducedim!, ext/MLIRCUDAExt.jl:114-119). */
void or_mapreduce_dim_f64(double* out, const float* x, int64_t pre, int64_t len, int64_t post, int f, int op,
                          double init) {
  for (int64_t q = 0; q < post; ++q)
    for (int64_t p = 0; p < pre; ++p) {
      double acc = init;
      for (int64_t k = 0; k < len; ++k) {
        double v = map_f(f, x[p + k * pre + q * pre * len]);
        if (op == OP_ADD) acc += v;
        else if (op == OP_MUL) acc *= v;
        else if (op == OP_MAX) acc = jl_max(acc, v);
        else acc = jl_min(acc, v);
      }
      out[p + q * pre] = acc;
    }
}

/* prefix scan in fp64 (AK.accumulate!/cumsum semantics, inclusive or
 * exclusive with init first; test/test_downstream_ka.jl:39-42, 75-78). */
void or_accumulate_f64(double* out, const float* x, int64_t n, int op, double init, int exclusive) {
  double acc = init;
  for (int64_t i = 0; i < n; ++i) {
    if (exclusive) out[i] = acc;
    double v = (double)x[i];
    if (op == OP_ADD) acc += v;
    else if (op == OP_MUL) acc *= v;
    else if (op == OP_MAX) acc = jl_max(acc, v);
    else acc = jl_min(acc, v);
    if (!exclusive) out[i] = acc;
  }
}

/* findmax/findmin with Julia's rules (NaN counts as the extreme for both,
 * +0.0 > -0.0, first index wins); returns the 1-based index. */
int64_t or_findext_f32(double* val, const float* x, int64_t n, int find_max) {
  int64_t best = 0;
  for (int64_t i = 1; i < n; ++i) {
    const float a = x[i], b = x[best];
    int better;
    if (a != a || b != b) better = (a != a) && !(b != b);
    else if (a == b) better = (signbit(a) != signbit(b)) ? (find_max ? !signbit(a) : signbit(a)) : 0;
    else better = find_max ? a > b : a < b;
    if (better) best = i;
  }
  *val = (double)x[best];
  return best + 1;
}

/* CPU-baseline findmax/findmin: each OpenMP thread runs the or_findext_f32
 * rule over a contiguous chunk, and the chunk winners are combined in chunk
 * order with the same rule (an earlier chunk wins ties, so the first index
 * wins overall).  Returns the 1-based index. */
static int fe_better(float a, int64_t ia, float b, int64_t ib, int find_max) {
  if (a != a || b != b) return (a != a) && (!(b != b) || ia < ib);
  if (a == b) {
    if (signbit(a) != signbit(b)) return find_max ? !signbit(a) : signbit(a);
    return ia < ib;
  }
  return find_max ? a > b : a < b;
}

int64_t mlirb_findext_f32(double* val, const float* x, int64_t n, int find_max) {
  if (n <= 0) return 0;
  const int T = omp_get_max_threads();
  int64_t* best = (int64_t*)malloc(sizeof(int64_t) * (size_t)T);
#pragma omp parallel num_threads(T)
  {
    const int t = omp_get_thread_num(), nt = omp_get_num_threads();
    const int64_t lo = n * t / nt, hi = n * (t + 1) / nt;
    int64_t b = lo;
    for (int64_t i = lo + 1; i < hi; ++i)
      if (fe_better(x[i], i, x[b], b, find_max)) b = i;
    best[t] = hi > lo ? b : -1;
  }
  int64_t b = -1;
  for (int t = 0; t < T; ++t)
    if (best[t] >= 0 && (b < 0 || fe_better(x[best[t]], best[t], x[b], b, find_max))) b = best[t];
  free(best);
  *val = (double)x[b];
  return b + 1;
}

/* gather: c[i] = a[idx[i]], 1-based (src/lower.jl:4064-4077).  An index out of
 * [1, na] writes 0 and reports OR_ERR_DEVICE_FAULT (the reference raises a
 * BoundsError/KernelException without @inbounds). */
int or_gather_f32(float* c, const float* a, int64_t na, const int32_t* idx1, int64_t n) {
  int rc = OR_OK;
  for (int64_t i = 0; i < n; ++i) {
    int64_t k = (int64_t)idx1[i] - 1;
    if (k < 0 || k >= na) {
      c[i] = 0.0f;
      rc = OR_ERR_DEVICE_FAULT;
    } else {
      c[i] = a[k];
    }
  }
  return rc;
}

/* histogram: counts[key] += 1 with u32 wrap-around (atomic `addi`,
 * src/lower.jl:3600-3604), accumulating; bad keys skipped + reported. */
int or_hist_u32(uint32_t* counts, int32_t nbins, const int32_t* keys1, int64_t n) {
  int rc = OR_OK;
  for (int64_t i = 0; i < n; ++i) {
    int64_t k = (int64_t)keys1[i] - 1;
    if (k < 0 || k >= nbins) rc = OR_ERR_DEVICE_FAULT;
    else counts[k] += 1u;
  }
  return rc;
}

/* fp64 matmul with the tiled kernel's K rule (examples/tiled_matmul.jl:34:
 * only 16*floor(K/16) terms), column-major, C64 leading dimension M.
 * OpenMP over columns so 1-2k^3 checks finish in seconds. */
void or_matmul_f64(double* C, const float* A, const float* B, int64_t M, int64_t N, int64_t K,
                   int64_t lda, int64_t ldb) {
  const int64_t Kt = (K / 16) * 16;
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < N; ++j) {
    double* cj = C + j * M;
    for (int64_t i = 0; i < M; ++i) cj[i] = 0.0;
    for (int64_t k = 0; k < Kt; ++k) {
      const double b = (double)B[k + j * ldb];
      const float* ak = A + k * lda;
      for (int64_t i = 0; i < M; ++i) cj[i] += (double)ak[i] * b;
    }
  }
}

/* C[i,j] for a list of (i,j) pairs in fp64 (full-size spot checks). */
void or_matmul_entries_f64(double* out, const int64_t* ii, const int64_t* jj, int64_t cnt,
                           const float* A, const float* B, int64_t K, int64_t lda, int64_t ldb) {
  const int64_t Kt = (K / 16) * 16;
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < cnt; ++e) {
    double s = 0.0;
    for (int64_t k = 0; k < Kt; ++k) s += (double)A[ii[e] + k * lda] * (double)B[k + jj[e] * ldb];
    out[e] = s;
  }
}

/* y = A * (B * v) in fp64 (a size-independent property check of C = A*B:
 * C*v must equal A*(B*v)); v has N entries, y has M. */
void or_matvec_chain_f64(double* y, const float* A, const float* B, const double* v, int64_t M, int64_t N,
                         int64_t K, int64_t lda, int64_t ldb) {
  const int64_t Kt = (K / 16) * 16;
  double* t = (double*)calloc((size_t)(Kt > 0 ? Kt : 1), sizeof(double));
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < Kt; ++k) {
    double s = 0.0;
    for (int64_t j = 0; j < N; ++j) s += (double)B[k + j * ldb] * v[j];
    t[k] = s;
  }
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < M; ++i) {
    double s = 0.0;
    for (int64_t k = 0; k < Kt; ++k) s += (double)A[i + k * lda] * t[k];
    y[i] = s;
  }
  free(t);
}

/* y = C * v in fp64 for an fp32 column-major C (ldc). */
void or_matvec_f64(double* y, const float* C, const double* v, int64_t M, int64_t N, int64_t ldc) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < M; ++i) {
    double s = 0.0;
    for (int64_t j = 0; j < N; ++j) s += (double)C[i + j * ldc] * v[j];
    y[i] = s;
  }
}

/* The tiled kernel's exact fp32 arithmetic (examples/tiled_matmul.jl:28-48):
 * per 16-wide k-tile, out = fma chain over kk = 0..15 starting from 0, then
 * acc += out.  With FMA contraction (what NVPTX emits for `out += a*b`) this is
 * the bit pattern every correct 16x16 SIMT implementation produces. */
void or_mm_tiled16_f32(float* C, const float* A, const float* B, int64_t M, int64_t N, int64_t K,
                       int64_t lda, int64_t ldb, int64_t ldc) {
  const int64_t nkt = K / 16;
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < N; ++j) {
    for (int64_t i = 0; i < M; ++i) {
      float acc = 0.0f;
      for (int64_t kt = 0; kt < nkt; ++kt) {
        float out = 0.0f;
        for (int kk = 0; kk < 16; ++kk) {
          int64_t k = kt * 16 + kk;
          out = fmaf(A[i + k * lda], B[k + j * ldb], out);
        }
        acc = acc + out;
      }
      C[i + j * ldc] = acc;
    }
  }
}

/* ------------------------------------------------------------------------- */
/* (2) the reference's CPU MLIRBackend execution model, restated              */
/* ------------------------------------------------------------------------- */

/* KA launch check of ext/KernelAbstractionsExt.jl:256-258: ndrange must be a
 * multiple of the workgroup size W on the CPU backend. */
static int check_grid(int64_t n, int W) { return (W > 0 && n % W == 0) ? OR_OK : OR_ERR_INVALID; }

/* vadd on MLIRBackend: blocks of W lanes, contiguous lanes vectorised
 * (vector.transfer_read/write, src/lower.jl:4120-4131, 4184-4191). */
int mlirb_vadd_f32(float* c, const float* a, const float* b, int64_t n, int W) {
  if (check_grid(n, W)) return OR_ERR_INVALID;
  const int64_t blocks = n / W;
#pragma omp parallel for schedule(static)
  for (int64_t blk = 0; blk < blocks; ++blk) {
    const int64_t o = blk * W;
#pragma omp simd
    for (int l = 0; l < W; ++l) c[o + l] = a[o + l] + b[o + l];
  }
  return OR_OK;
}

/* sum(x.^2) on the reference: GPUArrays.mapreducedim! materialises the
 * broadcast x.^2 into a new array (ext/MLIRCUDAExt.jl:103), then
 * AcceleratedKernels' reduce runs block reductions in the element type (fp32):
 * each block of W lanes folds 2W elements through a shared-memory tree, the
 * per-block partials are reduced again the same way until one block is left.
 * `tmp` must hold n floats (the materialised x.^2) and n/(2W)+1 partials. */
static float block_tree_f32(const float* v, int64_t cnt, int W) {
  /* 2W slots; slots past cnt hold the neutral 0 */
  float s[2048];
  const int m = 2 * W;
  for (int l = 0; l < m; ++l) s[l] = (l < cnt) ? v[l] : 0.0f;
  for (int w = W; w >= 1; w >>= 1)
    for (int l = 0; l < w; ++l) s[l] = s[l] + s[l + w];
  return s[0];
}

double mlirb_sum_sq_f32(const float* x, int64_t n, int W, float* tmp) {
  if (W < 1 || W > 1024 || (W & (W - 1))) return NAN;
  if (n == 0) return 0.0;
  float* sq = tmp;
  /* broadcast kernel: y = x .^ 2 */
  const int64_t nb = (n + W - 1) / W;
#pragma omp parallel for schedule(static)
  for (int64_t blk = 0; blk < nb; ++blk) {
    const int64_t o = blk * W;
    const int64_t e = (o + W < n) ? o + W : n;
#pragma omp simd
    for (int64_t i = o; i < e; ++i) sq[i] = x[i] * x[i];
  }
  /* reduction rounds, ping-ponging inside tmp */
  float* src = sq;
  int64_t len = n;
  float* part = tmp + n;
  while (len > 1) {
    const int64_t blocks = (len + 2 * W - 1) / (2 * W);
#pragma omp parallel for schedule(static)
    for (int64_t blk = 0; blk < blocks; ++blk) {
      const int64_t o = blk * 2 * W;
      const int64_t cnt = (len - o < 2 * W) ? len - o : 2 * W;
      part[blk] = block_tree_f32(src + o, cnt, W);
    }
    /* next round reads the partials; write the round after into src space */
    float* t = src;
    src = part;
    part = t;
    len = blocks;
  }
  return (double)src[0];
}

/* gather on MLIRBackend: per-lane vector.gather (src/lower.jl:4134-4140). */
int mlirb_gather_f32(float* c, const float* a, int64_t na, const int32_t* idx1, int64_t n, int W) {
  if (check_grid(n, W)) return OR_ERR_INVALID;
  const int64_t blocks = n / W;
  int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
  for (int64_t blk = 0; blk < blocks; ++blk) {
    const int64_t o = blk * W;
    for (int l = 0; l < W; ++l) {
      const int64_t k = (int64_t)idx1[o + l] - 1;
      const int ok = (k >= 0) & (k < na);
      bad |= !ok;
      c[o + l] = ok ? a[k] : 0.0f;
    }
  }
  return bad ? OR_ERR_DEVICE_FAULT : OR_OK;
}

/* histogram on MLIRBackend: the per-lane index makes the atomic scalarised
 * into W atomic RMWs per block (src/lower.jl:3946-3965). */
int mlirb_hist_u32(uint32_t* counts, int32_t nbins, const int32_t* keys1, int64_t n, int W) {
  if (check_grid(n, W)) return OR_ERR_INVALID;
  const int64_t blocks = n / W;
  int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
  for (int64_t blk = 0; blk < blocks; ++blk) {
    const int64_t o = blk * W;
    for (int l = 0; l < W; ++l) {
      const int64_t k = (int64_t)keys1[o + l] - 1;
      if (k < 0 || k >= nbins) {
        bad = 1;
        continue;
      }
#pragma omp atomic update
      counts[k] += 1u;
    }
  }
  return bad ? OR_ERR_DEVICE_FAULT : OR_OK;
}

/* mm_tiled! on MLIRBackend: one block per 16x16 output tile (W = 256 lanes),
 * @localmem tiles as per-block buffers, @synchronize a no-op
 * (src/lower.jl:3786-3791, 1881-1890).  Same arithmetic as or_mm_tiled16_f32.
 * Rows [i0, i0+mrows) x columns [j0, j0+ncols) only (bounded samples). */
int mlirb_mm_tiled16_f32(float* C, const float* A, const float* B, int64_t M, int64_t N, int64_t K,
                         int64_t lda, int64_t ldb, int64_t ldc, int64_t j0, int64_t ncols) {
  if (M % 16 || N % 16 || j0 % 16 || ncols % 16) return OR_ERR_INVALID;
  const int64_t nkt = K / 16;
  const int64_t tm = M / 16, tn = ncols / 16;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t bj = 0; bj < tn; ++bj) {
    for (int64_t bi = 0; bi < tm; ++bi) {
      float tA[16][16], tB[16][16], acc[16][16], out[16][16];
      memset(acc, 0, sizeof(acc));
      const int64_t I0 = bi * 16, J0 = j0 + bj * 16;
      for (int64_t kt = 0; kt < nkt; ++kt) {
        const int64_t kb = kt * 16;
        for (int jj = 0; jj < 16; ++jj)
          for (int ii = 0; ii < 16; ++ii) {
            tA[jj][ii] = A[(I0 + ii) + (kb + jj) * lda];
            tB[jj][ii] = B[(kb + ii) + (J0 + jj) * ldb];
          }
        memset(out, 0, sizeof(out));
        for (int kk = 0; kk < 16; ++kk)
          for (int jj = 0; jj < 16; ++jj) {
            const float bv = tB[jj][kk];
#pragma omp simd
            for (int ii = 0; ii < 16; ++ii) out[jj][ii] = fmaf(tA[kk][ii], bv, out[jj][ii]);
          }
        for (int jj = 0; jj < 16; ++jj)
          for (int ii = 0; ii < 16; ++ii) acc[jj][ii] += out[jj][ii];
      }
      for (int jj = 0; jj < 16; ++jj)
        for (int ii = 0; ii < 16; ++ii) C[(I0 + ii) + (J0 + jj) * ldc] = acc[jj][ii];
    }
  }
  return OR_OK;
}

/* accumulate!(+) on MLIRBackend: AcceleratedKernels' block scan restated as
 * blocks of 2W elements scanned per block in fp32 (OpenMP), block totals
 * scanned sequentially, then a second parallel pass adding the block prefix. */
int mlirb_cumsum_f32(float* out, const float* x, int64_t n, int W, float* block_tot) {
  if (W < 1) return OR_ERR_INVALID;
  const int64_t B = 2 * (int64_t)W;
  const int64_t nb = (n + B - 1) / B;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) {
    float acc = 0.0f;
    const int64_t e = (b + 1) * B < n ? (b + 1) * B : n;
    for (int64_t i = b * B; i < e; ++i) out[i] = (acc += x[i]);
    block_tot[b] = acc;
  }
  float run = 0.0f;
  for (int64_t b = 0; b < nb; ++b) {
    const float t = block_tot[b];
    block_tot[b] = run;
    run += t;
  }
#pragma omp parallel for schedule(static)
  for (int64_t b = 1; b < nb; ++b) {
    const float p = block_tot[b];
    const int64_t e = (b + 1) * B < n ? (b + 1) * B : n;
#pragma omp simd
    for (int64_t i = b * B; i < e; ++i) out[i] += p;
  }
  return OR_OK;
}

/* sum(m; dims=1) on MLIRBackend for a column-major rows x cols Float32
 * matrix: OpenMP over columns, fp32 accumulation per column. */
void mlirb_sum_dims1_f32(float* out, const float* x, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < cols; ++j) {
    float acc = 0.0f;
    const float* c = x + j * rows;
#pragma omp simd reduction(+ : acc)
    for (int64_t i = 0; i < rows; ++i) acc += c[i];
    out[j] = acc;
  }
}
