/*
 * lanczos_b200.h — C ABI of the B200 Lanczos engine (liblanczos_b200.so).
 *
 * Plain pointers and sizes only.  Two groups of entry points:
 *
 *  1. Reference-compatible: `compute_eigsh` and `compute_eigsh_sigma` keep the
 *     exact signatures and argument meaning of the reference's C ABI
 *     (python/gpu_eigsh/_cuda_eigsh.cu:29-33 and :82-87; declared for its
 *     binding in python/gpu_eigsh/_bindings.cpp:19-30).  Host pointers in,
 *     host pointers out, synchronous.  Differences: errors come back as
 *     negative return codes instead of terminating the process, and the
 *     convergence test uses ARPACK's eps^(2/3) floor.
 *
 *  2. lg_*: plan-based eigsh with scipy/ARPACK semantics (which, tol, ncv,
 *     maxiter as restarts, v0), host or device buffers, status codes and an
 *     info record; and the stochastic-Lanczos-quadrature kernels behind
 *     `slq_logdet` (device pointers, caller's CUDA stream).
 */
#ifndef LANCZOS_B200_H
#define LANCZOS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
enum {
  LG_OK = 0,
  LG_NOCONV = 1,          /* iteration limit reached; info.nconv < k, outputs hold the best pairs */
  LG_ERR_INVALID = -1,    /* bad argument or malformed CSR */
  LG_ERR_CUDA = -2,       /* CUDA runtime error (text via lg_last_error) */
  LG_ERR_NOMEM = -3,      /* device allocation failed */
  LG_ERR_TIMEOUT = -4,    /* a bounded device-side wait gave up */
  LG_ERR_NUMERIC = -5,    /* tridiagonal QR did not converge, or non-finite values */
  LG_ERR_CG_NOCONV = -6   /* shift-invert inner CG did not reach cg_tol */
};

enum { LG_WHICH_LM = 0, LG_WHICH_SM = 1, LG_WHICH_LA = 2, LG_WHICH_SA = 3, LG_WHICH_BE = 4 };

typedef struct lg_eigsh_opts {
  int k;               /* eigenpairs wanted (1 <= k < n) */
  int ncv;             /* Lanczos basis size; 0 = min(n, max(2k+1, 20)) (scipy default) */
  int maxiter;         /* implicit restarts (ARPACK iterations); 0 = 10*n */
  long long max_steps; /* Lanczos step budget (reference meaning of max_iters); 0 = none */
  double tol;          /* relative accuracy of Ritz values; 0 = machine precision */
  int which;           /* LG_WHICH_*; with use_sigma it applies to (A - sigma I)^-1 */
  int use_sigma;       /* 1: shift-invert about sigma */
  double sigma;
  int cg_max_iters;    /* shift-invert: CG iterations per solve; 0 = 10*n */
  double cg_tol;       /* shift-invert: CG relative residual */
  int mixed;           /* 1: fp32 matrix values, fp64 accumulation and fp64 basis */
  uint64_t seed;       /* seed of the starting vector when v0 is NULL */
  int return_vectors;  /* 1: fill evecs */
  int evecs_rowmajor;  /* 1: evecs is n x k row-major; 0: column-major with ld = n */
  int profile;         /* 1: time every kernel with CUDA events (info.kernel_*) */
} lg_eigsh_opts;

/* Kernel classes of info.kernel_* */
enum {
  LG_K_SPMV = 0,     /* normalise + SpMV of a Lanczos step */
  LG_K_PROJECT = 1,  /* Gram-Schmidt pass 1: h = V^T w */
  LG_K_CORRPROJ = 2, /* pass 2: r = w - V h, s = V^T r */
  LG_K_CORRECT = 3,  /* pass 3: r -= V s */
  LG_K_RESTART = 4,  /* one-CTA tridiagonal QR + shifts */
  LG_K_BASIS = 5,    /* V*Q restart update / Ritz vectors */
  LG_K_CG = 6,       /* shift-invert CG iteration kernels */
  LG_K_OTHER = 7,
  LG_K_CLASSES = 8
};

typedef struct lg_eigsh_info {
  int nconv;           /* Ritz pairs that passed the convergence test */
  int restarts;        /* implicit restarts performed */
  long long steps;     /* Lanczos steps (operator applications) */
  int pass3;           /* DGKS third Gram-Schmidt passes */
  int breakdowns;      /* invariant subspaces met (random restart vectors) */
  long long cg_iters;  /* shift-invert: total inner CG iterations */
  int cg_failures;     /* shift-invert: solves that stopped at cg_max_iters */
  double ms;           /* device time of the solve */
  long long launches;  /* kernels launched by the solve */
  double kernel_ms[8];          /* profile: summed device time per kernel class */
  long long kernel_calls[8];    /* profile: launches per class */
  double kernel_bytes[8];       /* profile: algorithmic DRAM bytes per class */
} lg_eigsh_info;

typedef struct lg_eigsh_plan lg_eigsh_plan;

/* Fill *o with the defaults (k = 6, which = LM, tol = 0, seed = 42, vectors on). */
int lg_eigsh_opts_default(lg_eigsh_opts* o);

/* Own a device copy of the CSR matrix (int32 indices, fp64 values, n x n,
 * symmetric) plus the solver workspace for up to `max_ncv` basis vectors.
 * device_ptrs = 1: the three arrays are device pointers (copied on device).
 * mixed = 1 also keeps an fp32 copy of the values (made on the device). */
int lg_eigsh_plan_create(lg_eigsh_plan** plan, int n, long long nnz, const int* row_ptr,
                         const int* col_idx, const double* vals, int device_ptrs, int max_ncv,
                         int mixed);

/* Solve.  evals: host, k doubles, ascending.  evecs: n x k per opts layout.
 * io_on_device = 1: v0 and evecs are device pointers.  v0 may be NULL. */
int lg_eigsh_plan_run(lg_eigsh_plan* plan, const lg_eigsh_opts* opts, const double* v0, double* evals,
                      double* evecs, int io_on_device, lg_eigsh_info* info);

int lg_eigsh_plan_destroy(lg_eigsh_plan* plan);

/* One-shot convenience: create + run + destroy with host pointers. */
int lg_eigsh(int n, long long nnz, const int* row_ptr, const int* col_idx, const double* vals,
             const lg_eigsh_opts* opts, const double* v0, double* evals, double* evecs,
             lg_eigsh_info* info);

/* m Lanczos steps (CGS2) from the host vector v0 without restarts: alpha
 * (m doubles) and beta (m+1 doubles; beta[0] = 0, beta[m] = final residual
 * norm) of the tridiagonal, copied to the host.  A test and debugging hook
 * (the reference's compute_funm_debug, python/gpu_eigsh/_cuda_funm.cu:132-178,
 * serves the same purpose for its matrix-function path). */
int lg_eigsh_plan_factorize(lg_eigsh_plan* plan, const double* v0, int m, double* alpha, double* beta);

/* y = A x with the plan's matrix (device pointers, n doubles each). */
int lg_eigsh_plan_matvec(lg_eigsh_plan* plan, const double* x, double* y);

/* Two classical Gram-Schmidt passes of w against the first ncols columns of a
 * row-major basis V (n x ldv doubles on the device, 16-byte aligned, even ldv
 * >= ncols):  h1 = V^T w, r1 = w - V h1, s = V^T r1, r = r1 - V s.
 * Outputs on the device: r (n doubles, must not alias w), coef = h1 + s
 * (ncols doubles), norms = {||w||, ||r1||, ||r||}.  Asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream).  1 <= ncols <= 128.
 * Counterpart of cgs_orthogonalize + dgks_reorth
 * (src/lanczos_ops.cuh:113-192), always with the second pass. */
int lg_cgs2_orthogonalize(const double* V, int ldv, int n, int ncols, const double* w, double* r, double* coef,
                          double* norms, void* stream);

/* Same contract and results as lg_cgs2_orthogonalize, for callers that must
 * not allocate device memory (e.g. code running inside a device allocator or
 * memory-pool hook, or a service whose device memory budget is fixed at
 * start-up): no cudaMalloc/cudaFree or other allocating call is made.  The
 * workspace is a fixed 0.5 MiB device array inside the library that every GPU
 * loading it keeps until exit; 1 <= ncols <= 128.  The first call on a device
 * resolves the array's address (make it before capturing any stream).  All
 * calls share the array: calls that overlap on the GPU race, so order them on
 * one stream.  This entry point has no counterpart in the reference. */
int lg_cgs2_orthogonalize_noalloc(const double* V, int ldv, int n, int ncols, const double* w, double* r,
                                  double* coef, double* norms, void* stream);

const char* lg_status_string(int status);
/* Copies the last error message of the calling thread; returns its length. */
int lg_last_error(char* buf, int len);

/* ---- reference-compatible entry points ---------------------------------- */

/* k smallest-algebraic eigenpairs of the symmetric CSR matrix.
 * ncv = 0: min(max(3k, 40), n).  max_iters: Lanczos step budget.
 * out_eigenvectors: column-major n x k.  Returns the number of pairs
 * written (min(k, ncv)) or a negative LG_ERR_* code.
 * Replaces compute_eigsh, python/gpu_eigsh/_cuda_eigsh.cu:29-74. */
int compute_eigsh(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals, int k,
                  int ncv, int max_iters, double tol, double* out_eigenvalues, double* out_eigenvectors);

/* k eigenpairs nearest sigma by shift-invert Lanczos with an inner CG solve
 * of (A - sigma I) y = x.  Eigenvalues ascending.
 * Replaces compute_eigsh_sigma, python/gpu_eigsh/_cuda_eigsh.cu:82-163. */
int compute_eigsh_sigma(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals, int k,
                        int ncv, int max_iters, double tol, double sigma, int cg_max_iters, double cg_tol,
                        double* out_eigenvalues, double* out_eigenvectors);

#ifdef __cplusplus
}
#endif

#endif /* LANCZOS_B200_H */
