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
  LG_K_PROJECT = 1,  /* Gram-Schmidt pass 1: h = V^T w (lag steps: s = V^T u, t = V^T z in one stream) */
  LG_K_CORRPROJ = 2, /* pass 2: r = w - V h, s = V^T r (lag steps: the correction finishing v_j and r1) */
  LG_K_CORRECT = 3,  /* pass 3: r -= V s (also the delayed pass of an extension's last residual) */
  LG_K_RESTART = 4,  /* one-CTA tridiagonal QR + shifts */
  LG_K_BASIS = 5,    /* V*Q restart update / Ritz vectors */
  LG_K_CG = 6,       /* shift-invert CG iteration kernels */
  LG_K_OTHER = 7,
  LG_K_COMM = 8,     /* partitioned plans: the reductions over the ranks and the residual exchanges (waits included) */
  LG_K_CLASSES = 9
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
  double kernel_ms[LG_K_CLASSES];        /* profile: summed device time per kernel class */
  long long kernel_calls[LG_K_CLASSES];  /* profile: launches per class */
  double kernel_bytes[LG_K_CLASSES];     /* profile: algorithmic DRAM bytes per class */
} lg_eigsh_info;

typedef struct lg_eigsh_plan lg_eigsh_plan;

/* Fill *o with the defaults (k = 6, which = LM, tol = 0, seed = 42, vectors on). */
int lg_eigsh_opts_default(lg_eigsh_opts* o);

/* Own a device copy of the CSR matrix (int32 indices, fp64 values, n x n,
 * symmetric) plus the solver workspace for up to `max_ncv` basis vectors.
 * device_ptrs = 1: the three arrays are device pointers (copied on device, on
 * the plan's own non-blocking stream: the caller makes sure the work that
 * writes them has finished; the same holds for device v0 / evecs buffers
 * passed to lg_eigsh_plan_run).
 * mixed = 1 also keeps an fp32 copy of the values (made on the device). */
int lg_eigsh_plan_create(lg_eigsh_plan** plan, int n, long long nnz, const int* row_ptr,
                         const int* col_idx, const double* vals, int device_ptrs, int max_ncv,
                         int mixed);

/* lg_eigsh_plan_create with flags.  LG_PLAN_REORDER_BFS renumbers the rows
 * inside the plan in Cuthill-McKee order (BFS levels from a
 * pseudo-peripheral vertex, each level in the order of the vertices that found
 * it; the matrix pattern must be symmetric), so that the gathers of the sparse
 * product stay in L1 / L2 for graphs whose input numbering has no locality
 * (the kNN graph of randomly ordered points).  The caller sees its own
 * numbering everywhere: v0, the eigenvectors and lg_eigsh_plan_matvec are
 * mapped through the permutation; the eigenvalues are those of the same
 * matrix.  Creation computes the order on the host (a few hundred ms at
 * n = 1e6), so the flag pays off for plans that solve more than once. */
#define LG_PLAN_REORDER_BFS 1
/* LG_PLAN_CGS2_INLINE keeps both classical Gram-Schmidt passes inside every
 * Lanczos step (three streams of the basis per step).  By default the second
 * pass of step j-1 is delayed into step j (two streams per step: the
 * projection of the new vector and the delayed projection share one read of
 * V, and so do the two corrections); the basis, alpha and beta agree with the
 * in-step passes to rounding, and the DGKS and breakdown tests are the same.
 * Shift-invert solves always use the in-step passes. */
#define LG_PLAN_CGS2_INLINE 2
/* LG_PLAN_REORDER_DEGREE renumbers the rows by descending row length (ties by
 * the caller's index) instead, for power-law graphs (R-MAT, web and social
 * graphs) where Cuthill-McKee finds no bandwidth: the hub vertices, which
 * most column indices name, get the first numbers, so the entries of the
 * vector that the sparse product gathers most often share cache sectors and
 * stay in L2, and the rows of one length class are consecutive.  Mapped for
 * the caller exactly like LG_PLAN_REORDER_BFS; the two flags exclude each
 * other.  Creation sorts on the host in O(n + max row length). */
#define LG_PLAN_REORDER_DEGREE 4
int lg_eigsh_plan_create_ex(lg_eigsh_plan** plan, int n, long long nnz, const int* row_ptr,
                            const int* col_idx, const double* vals, int device_ptrs, int max_ncv,
                            int mixed, int flags);

/* ---- matrix-free operators ---------------------------------------------
 *
 * A plan whose operator is the caller's function y = A x instead of a CSR
 * matrix (A symmetric, n x n).  Replaces FunctionOperator
 * (src/matvec_operator.cuh:149-163), whose callback type lg_matvec_fn keeps:
 * x and y are n doubles, `user` is passed through untouched.  Three kinds:
 *   LG_OP_DEVICE  fn gets device pointers.  The plan's stream is drained
 *                 before each call and the whole device after it, so fn may
 *                 use any stream (the reference's contract).
 *   LG_OP_HOST    fn gets host pointers (pinned copies made by the plan):
 *                 operators that live on the host, e.g. a Python
 *                 scipy.sparse.linalg.LinearOperator.
 *   LG_OP_STREAM  sfn gets device pointers and the plan's cudaStream_t; it
 *                 enqueues y = A x on that stream and returns without
 *                 waiting, so the solve keeps its one host wait per restart.
 * fn / sfn run on the thread that calls lg_eigsh_plan_run (or _matvec,
 * _factorize, _funm), once per Lanczos step.  The Lanczos steps keep both
 * Gram-Schmidt passes inside every step (the delayed second pass of CSR plans
 * folds 1/||r|| into the sparse product).  Shift-invert needs a CSR plan. */
typedef void (*lg_matvec_fn)(const double* x, double* y, int n, void* user);
typedef void (*lg_matvec_stream_fn)(const double* x, double* y, int n, void* user, void* stream);
#define LG_OP_DEVICE 0
#define LG_OP_HOST 1
#define LG_OP_STREAM 2
/* kind LG_OP_DEVICE / LG_OP_HOST: fn set, sfn NULL; LG_OP_STREAM: sfn set,
 * fn NULL.  n >= 2; workspace for up to max_ncv basis vectors. */
int lg_eigsh_plan_create_op(lg_eigsh_plan** plan, int n, int kind, lg_matvec_fn fn, lg_matvec_stream_fn sfn,
                            void* user, int max_ncv);

/* Solve.  evals: host, k doubles, ascending.  evecs: n x k per opts layout.
 * io_on_device = 1: v0 and evecs are device pointers.  v0 may be NULL. */
int lg_eigsh_plan_run(lg_eigsh_plan* plan, const lg_eigsh_opts* opts, const double* v0, double* evals,
                      double* evecs, int io_on_device, lg_eigsh_info* info);

int lg_eigsh_plan_destroy(lg_eigsh_plan* plan);

/* One-shot convenience: create + run + destroy with host pointers. */
int lg_eigsh(int n, long long nnz, const int* row_ptr, const int* col_idx, const double* vals,
             const lg_eigsh_opts* opts, const double* v0, double* evals, double* evecs,
             lg_eigsh_info* info);

/* ---- row-partitioned eigsh over several GPUs (one process per GPU) --------
 *
 * Rank r owns the rows [r*nb, min((r+1)*nb, n)) of the n x n matrix, with
 * nb = lg_partition_block(n, nranks); its CSR holds those rows with global
 * column indices.  Before every sparse product the residual rows that other
 * ranks read reach them (NCCL): by a halo exchange (grouped point-to-point
 * sends of exactly the rows the other ranks' columns name) when the halos
 * are small, else by an in-place all-gather of the whole residual; one row
 * of partial sums is all-reduced per Gram-Schmidt pass; the restart logic
 * runs replicated on every rank.  With a
 * partitioned plan, lg_eigsh_plan_run takes this rank's slice of v0 and
 * returns this rank's rows of the eigenvectors (n_local x k); the
 * eigenvalues are returned on every rank.  Shift-invert, factorize and
 * matvec are single-GPU only.  The communicator is NCCL's, created from a
 * unique id that rank 0 draws and the caller distributes (e.g. with
 * torch.distributed); NCCL is loaded on first use. */
typedef struct lg_comm lg_comm;
#define LG_COMM_ID_BYTES 128
int lg_comm_unique_id(void* out, int len);
int lg_comm_create(lg_comm** comm, const void* id, int len, int nranks, int rank);
int lg_comm_destroy(lg_comm* comm);
int lg_partition_block(int n, int nranks);
int lg_eigsh_plan_create_dist(lg_eigsh_plan** plan, lg_comm* comm, int n_global, int n_local, long long nnz,
                              const int* row_ptr, const int* col_idx, const double* vals, int device_ptrs,
                              int max_ncv, int mixed);

/* Residual exchange of a partitioned plan.  lg_eigsh_plan_create_dist builds
 * the halo lists (a collective call) and picks LG_EXCHANGE_HALO when every
 * rank receives at most half of the rows an all-gather would bring, else
 * LG_EXCHANGE_ALLGATHER.  set_exchange overrides the choice (LG_EXCHANGE_AUTO
 * restores it); every rank must pass the same mode before its next run.
 * exchange_info reports the mode in use and this rank's halo sizes in rows
 * (received from / sent to the other ranks).  Single-GPU plans: LG_ERR_INVALID. */
#define LG_EXCHANGE_AUTO 0
#define LG_EXCHANGE_ALLGATHER 1
#define LG_EXCHANGE_HALO 2
int lg_eigsh_plan_set_exchange(lg_eigsh_plan* plan, int mode);
int lg_eigsh_plan_exchange_info(const lg_eigsh_plan* plan, int* mode, long long* recv_rows, long long* send_rows);

/* Transport of a partitioned plan's reductions and residual exchange.
 * LG_TRANSPORT_PEER: each reduction and each exchange is one kernel that
 * stores straight into the other ranks' memory over NVLink (buffers mapped
 * with CUDA IPC at plan creation) and waits, bounded, on flags the other
 * ranks raise; every rank adds the ranks' partial rows in rank order, so all
 * ranks hold bitwise the same sums.  LG_TRANSPORT_NCCL: NCCL all-reduce and
 * grouped send/receive (or all-gather).  lg_eigsh_plan_create_dist picks the
 * peer transport when every rank has its own GPU and every mapping opens
 * (environment LG_PEER_TRANSPORT=0 keeps NCCL), identically on every rank;
 * set_transport overrides it (every rank must pass the same mode before its
 * next run; LG_TRANSPORT_PEER fails where the mappings are missing).  A wait
 * that gives up (about ten seconds) ends the run with LG_ERR_TIMEOUT.
 * No counterpart in the reference (single device). */
#define LG_TRANSPORT_AUTO 0
#define LG_TRANSPORT_NCCL 1
#define LG_TRANSPORT_PEER 2
int lg_eigsh_plan_set_transport(lg_eigsh_plan* plan, int mode);
int lg_eigsh_plan_transport(const lg_eigsh_plan* plan, int* mode);

/* Host-side halo planning of a partitioned plan (the steps
 * lg_eigsh_plan_create_dist runs between its collectives), callable without a
 * GPU so that the plan can be checked on CPU ranks.  No counterpart in the
 * reference (single device).
 * lg_halo_recv_list: the global rows of other ranks that this rank's columns
 *   (host array col, nnz entries, global indices) name, grouped by owner
 *   (ascending owner, then row) into recv_pos (capacity entries); recv_cnt
 *   (nranks) the count per owner, *total the list length (also when the
 *   capacity is too small, which returns LG_ERR_INVALID).
 * lg_halo_send_plan: from the all-reduced count matrix counts (nranks x
 *   nranks doubles, row r = rows rank r receives from each rank) this rank's
 *   rows sent to each peer (send_cnt, nranks) and the exchange mode
 *   (LG_EXCHANGE_HALO or LG_EXCHANGE_ALLGATHER) every rank derives alike.
 * The rows a rank sends to peer p are p's receive positions owned by this
 * rank, in p's order; the receiver writes them at the same global positions. */
int lg_halo_recv_list(int n_global, int nranks, int rank, long long nnz, const int* col, int* recv_pos,
                      long long capacity, long long* recv_cnt, long long* total);
int lg_halo_send_plan(int n_global, int nranks, int rank, const double* counts, long long* send_cnt, int* mode);

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
 * resolves the array's address and caches it.  With CUDA's lazy module
 * loading that first call is also when the library's device code is loaded
 * on the device, which takes driver memory: make the first call on each
 * device outside the no-allocation context (at start-up, for example), and
 * before capturing any stream.  The cached address does not survive a
 * cudaDeviceReset of that device; do not call this entry point after one.
 * All calls share the array: calls that overlap on the GPU race, so order
 * them on one stream.  This entry point has no counterpart in the reference. */
int lg_cgs2_orthogonalize_noalloc(const double* V, int ldv, int n, int ncols, const double* w, double* r,
                                  double* coef, double* norms, void* stream);

/* ---- stochastic Lanczos quadrature (SLQ) and the Kraemer adjoint ---------
 *
 * All pointers are device pointers; every call is asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream) and allocates nothing.
 *
 * Blocks of probe vectors are n x ld row-major arrays of the operator's
 * element type (LG_F32 / LG_F64), ld even, 8-byte (fp32) or 16-byte (fp64)
 * aligned; columns [0, B) are the probes, 1 <= B <= 128.  When B is odd,
 * column B is padding: it is read as zero and written as zero.  Reductions
 * accumulate in fp64 and are bitwise repeatable.  Per-probe scalars (alpha,
 * beta, g_alpha, g_beta: B x m row-major; znorm: B) are fp64.
 *
 * `ws` is a 256-byte aligned device workspace of at least
 * lg_slq_workspace_bytes(op, B, ld) bytes (op = NULL: the size for the
 * lg_slq_small_side / lg_slq_block_* calls alone).  Calls sharing a workspace
 * must be ordered on one stream.
 */
enum { LG_F32 = 0, LG_F64 = 1 };
enum { LG_FUNC_LOG = 0, LG_FUNC_EXP = 1, LG_FUNC_SQRT = 2, LG_FUNC_INV = 3 };

/* P = A^power with A = shift I + L; L symmetric, given as its diagonal and its
 * off-diagonal entries in CSR (every off-diagonal pair stored both ways).
 * ddiag / doffval: dL/dq for one scalar parameter q of L (NULL: no q).
 * The IMGP precision operator (python/gpu_eigsh/imgp.py:234-289) is
 * shift = 2 nu / lengthscale^2, L = L_sym(graphbandwidth), power = nu. */
typedef struct lg_slq_op {
  int n;
  long long nnz;          /* off-diagonal entries, < 2^31 */
  const int* rowptr;      /* n + 1 */
  const int* col;         /* nnz */
  const void* offval;     /* nnz */
  const void* diag;       /* n */
  const void* doffval;    /* nnz or NULL */
  const void* ddiag;      /* n or NULL */
  double shift;
  int power;              /* 1 .. 8 */
  int dtype;              /* LG_F32 or LG_F64 */
} lg_slq_op;

size_t lg_slq_workspace_bytes(const lg_slq_op* op, int B, int ld);

/* Batched three-term Lanczos without re-orthogonalisation of B probe columns
 * of Z through P, m steps: V holds m+1 blocks (v_0 .. v_m, block stride n*ld),
 * Y holds m*(power-1) blocks A^p v_j (j-major; NULL when power = 1), kept for
 * lg_slq_backward; alpha/beta (B x m) the tridiagonals (beta[:, m-1] is the
 * final residual norm), znorm the column norms of Z.
 * Replaces lanczos_torch_noreortho_batched (python/gpu_eigsh/funm_torch.py:120-173)
 * on the operator of python/gpu_eigsh/imgp.py:234-289. */
int lg_slq_forward(const lg_slq_op* op, int B, int m, int ld, const void* Z, void* V, void* Y, double* alpha,
                   double* beta, double* znorm, void* ws, size_t ws_bytes, void* stream);

/* Kraemer reverse sweep of the batched recurrence for a scalar loss with
 * gradient *g_out * (g_alpha, g_beta) with respect to (alpha, beta):
 * g_params[0] = d loss / dq (through ddiag/doffval; 0 without them),
 * g_params[1] = d loss / d shift.  g_out may be NULL (= 1).
 * Replaces the sweep of _SLQLogdetBatched.backward
 * (python/gpu_eigsh/funm_torch.py:681-727) with the parameter VJP formed
 * inside the sparse products instead of by autograd through the matvec. */
int lg_slq_backward(const lg_slq_op* op, int B, int m, int ld, const void* V, const void* Y, const double* alpha,
                    const double* beta, const double* g_alpha, const double* g_beta, const double* g_out,
                    double* g_params, void* ws, size_t ws_bytes, void* stream);

/* Y = P X (B columns).  Replaces the precision matvec of
 * make_imgp_precision_matvec (python/gpu_eigsh/imgp.py:279-287). */
int lg_slq_apply(const lg_slq_op* op, int B, int ld, const void* X, void* Y, void* ws, size_t ws_bytes,
                 void* stream);

/* VJP of Y = P X for the cotangent G: gX = P G, g_params[0] = sum <G, (dP/dq) X>,
 * g_params[1] = sum <G, (dP/dshift) X>. */
int lg_slq_apply_vjp(const lg_slq_op* op, int B, int ld, const void* X, const void* G, void* gX,
                     double* g_params, void* ws, size_t ws_bytes, void* stream);

/* Small side of every probe b (T_b = tridiag(alpha[b, :], beta[b, :m-1]),
 * f = LG_FUNC_*):
 *   mode 0: out[b] = znorm[b]^2 e1^T f(T_b) e1, g_alpha/g_beta = g_scale * its gradient;
 *   mode 1: out[b*m .. b*m+m) = f(T_b) e1;
 *   mode 2: g_alpha/g_beta = g_scale * gradient of <gu[b, :], f(T_b) e1>.
 * *status becomes nonzero when a T_b holds non-finite values (outputs NaN).
 * Replaces the eigh-based small side of python/gpu_eigsh/funm_torch.py:62-76,
 * 595-607 and its autograd (:634-660). */
int lg_slq_small_side(int B, int m, int func, int mode, const double* alpha, const double* beta,
                      const double* znorm, const double* gu, double g_scale, double* out, double* g_alpha,
                      double* g_beta, int* status, void* ws, size_t ws_bytes, void* stream);

/* Recurrence and reverse-sweep steps around a product P x formed by the
 * caller (any operator the caller can apply):
 *   block_start:  V0 = Z / ||Z|| per column, znorm = ||Z||;
 *   block_step:   given W = P v_j: alpha_j = <v_j, W>, R = W - alpha_j v_j -
 *                 beta_{j-1} v_{j-1}, beta_j = ||R||, Vnext = R / beta_j;
 *   block_lambda: lambda of step j (xi = NULL starts the sweep at j = m-1);
 *   block_xi:     given Plam = P lambda: xi of step j-1, i.e.
 *                 -dcoef[b] G[:, b] - Plam + alpha_j lambda + beta_j lplus -
 *                 beta_j nu_j xplus (dcoef, G optional; lplus NULL at j = m-1;
 *                 xjm1 NULL at j = 0);
 *   block_start_grad: gZ = (<xi, V0> V0 - xi) / znorm + g_znorm * Z / znorm.
 * The workspace carries column sums from block_xi to the next block_lambda.
 * Same arithmetic as lanczos_torch_noreortho(_batched) and the Kraemer sweeps
 * of python/gpu_eigsh/funm_torch.py:83-173, 317-365, 681-727, 503-560. */
int lg_slq_block_start(int n, int B, int ld, int dtype, const void* Z, void* V0, double* znorm, void* ws,
                       size_t ws_bytes, void* stream);
int lg_slq_block_step(int n, int B, int ld, int dtype, int j, int m, const void* W, const void* Vj,
                      const void* Vjm1, void* R, void* Vnext, double* alpha, double* beta, void* ws,
                      size_t ws_bytes, void* stream);
int lg_slq_block_lambda(int n, int B, int ld, int dtype, int j, int m, const void* xi, const void* xplus,
                        const void* xj, const double* beta, const double* g_alpha, const double* g_beta,
                        const double* g_out, void* lam, void* ws, size_t ws_bytes, void* stream);
int lg_slq_block_xi(int n, int B, int ld, int dtype, int j, int m, const void* Plam, const void* lam,
                    const void* lplus, const void* xplus, const void* xj, const void* xjm1, const double* alpha,
                    const double* beta, const double* dcoef, const void* G, void* xi, void* ws, size_t ws_bytes,
                    void* stream);
int lg_slq_block_start_grad(int n, int B, int ld, int dtype, const void* xi, const void* V0, const void* Z,
                            const double* znorm, const double* g_znorm, void* gZ, void* ws, size_t ws_bytes,
                            void* stream);

/* The IMGP graph Laplacian L_sym(graphbandwidth) (symmetric normalisation,
 * optional self loops) in the order of a CSR that stores every edge in both
 * directions: d2 holds the squared edge distance of every CSR entry; outputs
 * offval (nnz), diag (n) and, when doffval/ddiag are not NULL, dL/d
 * graphbandwidth.  work: 4n doubles of device scratch.
 * Replaces _build_laplacian_cache (python/gpu_eigsh/imgp.py:142-189). */
int lg_imgp_laplacian(int n, long long nnz, const int* rowptr, const int* col, int dtype, const void* d2,
                      double graphbandwidth, int self_loops, void* offval, void* diag, void* doffval, void* ddiag,
                      double* work, void* stream);

/* Breadth-first levels of the graph of a CSR (every edge stored both ways)
 * from vertex `start`: level[v] = hop distance, -1 where unreachable.  work:
 * 2n + 2 ints of device scratch.  Synchronises `stream` every 16 levels;
 * *nlevels receives the number of expansion rounds run.  Used to order the
 * rows of the SLQ operator for locality (no counterpart in the reference,
 * which keeps the caller's order). */
int lg_graph_bfs_levels(int n, const int* rowptr, const int* col, int start, int* level, int* work, int* nlevels,
                        void* stream);

/* Matrix Market files (host).  lg_mtx_read parses a `coordinate` file
 * (real, integer or pattern; general, symmetric or skew-symmetric, mirrored
 * entries added) on all host cores into a CSR held by the returned handle:
 * 0-based, columns sorted inside each row, duplicate entries summed;
 * lg_mtx_copy copies it out (row_ptr: nrows + 1, col and vals: nnz),
 * lg_mtx_free releases it.  lg_mtx_write writes a CSR as `coordinate real
 * general` (symmetric = 1: `symmetric`, lower triangle only), every value in
 * the shortest form that reads back to the same double.  Replaces
 * load_matrix_market / export_matrix_market (src/main.cu:129-244). */
typedef struct lg_mtx lg_mtx;
int lg_mtx_read(const char* path, lg_mtx** out, int* nrows, int* ncols, long long* nnz);
int lg_mtx_copy(const lg_mtx* m, int* row_ptr, int* col, double* vals);
int lg_mtx_free(lg_mtx* m);
int lg_mtx_write(const char* path, int nrows, int ncols, const int* row_ptr, const int* col, const double* vals,
                 int symmetric);

/* Cuthill-McKee order of the graph of a HOST CSR (every edge stored both
 * ways): perm[new] = old, n ints.  Each connected component starts from a
 * pseudo-peripheral vertex; inside a BFS level the vertices follow the order
 * of their discoverers, unvisited neighbours by increasing degree.  Orders the
 * rows of the SLQ operator and of large differentiable-eigsh matrices so that
 * consecutive rows gather neighbouring rows (no counterpart in the reference). */
int lg_graph_cm_order(int n, const int* rowptr, const int* col, int* perm);

/* Exact k nearest neighbours of n DEVICE points (row-major n x dim fp64),
 * self excluded: out_idx (n x k int64) and out_d2 (n x k squared distances,
 * sums of squared coordinate differences in coordinate order, no fused
 * multiply-add), each row ascending by (distance, index) — the order of the
 * reference driver's partial_sort over (dist2, j) pairs (src/main.cu:42-63),
 * which replaces it, and of cKDTree.query in
 * benchmark/generate_large_laplacian.py:36-44 up to exact ties.
 * method: LG_KNN_AUTO (cells for dim <= 3, else brute), LG_KNN_CELLS (uniform
 * cell grid, dim <= 3), LG_KNN_BRUTE (tiled all-pairs, dim <= 32).
 * 1 <= k <= min(64, n - 1).  Synchronises `stream` once (coordinate bounds). */
#define LG_KNN_AUTO 0
#define LG_KNN_CELLS 1
#define LG_KNN_BRUTE 2
int lg_knn(int n, int dim, int k, const double* pts, long long* out_idx, double* out_d2, int method, void* stream);

/* The kNN graph Laplacian L = D - A on the device, in two calls.
 * A_ij = exp(-d2_ij / denom) for j in i's list or i in j's list (union
 * symmetrisation: src/main.cu:65-74, the A.maximum(A.T) of
 * benchmark/generate_large_laplacian.py:58); D_ii = sum_j A_ij summed in
 * column order.  Rows hold their entries in ascending column order with the
 * diagonal included (src/main.cu:76-107).  denom = 4 bw^2 gives both
 * reference builders' weights.
 * lg_knn_laplacian_rows: row_ptr (device, n + 1) and *nnz (host); checks that
 *   every list holds distinct indices in [0, n) other than its row.
 * lg_knn_laplacian_fill: col (nnz int32) and vals (nnz fp64) for that row_ptr. */
int lg_knn_laplacian_rows(int n, int k, const long long* idx, int* rowptr, long long* nnz, void* stream);
int lg_knn_laplacian_fill(int n, int k, const long long* idx, const double* d2, double denom, const int* rowptr,
                          int* col, double* vals, void* stream);

/* y = A x for a dense row-major n x n A (vectors with element strides ldx, ldy),
 * and gA += lam x^T (fp64 gA, vectors with element stride ld): the dense-matrix
 * operations of funm_apply_kraemer (python/gpu_eigsh/funm_torch.py:284, 347). */
int lg_dense_matvec(int n, int dtype, const void* A, const void* x, int ldx, void* y, int ldy, void* stream);
int lg_outer_accumulate(int n, int dtype, const void* lam, const void* x, int ld, double* gA, void* stream);

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

/* Backward of eigsh (implicit differentiation, Xie et al. 2020), device
 * pointers on `stream`.  For every eigenpair i (eigenvalue evals[i],
 * eigenvector column i of X, n x k row-major) the solution xi_i of
 *   (A - evals[i] I) xi_i = (I - X X^T) g_evecs[:, i],   xi_i orthogonal to X,
 * is found by conjugate gradients (relative residual cg_tol, at most
 * cg_max_iters iterations; the k systems advance together as one block, each
 * with its own shift and convergence test), and for every stored entry
 * p = (r, c) of the CSR
 *   grad_vals[p] = sum_i (g_evals[i] X[r, i] - xi_i[r]) X[c, i].
 * g_evals (k) and g_evecs (n x k row-major) may be NULL (zero).  cg_iters
 * (host, k ints, may be NULL) receives the iterations per pair, negative when
 * a pair stopped at the limit or at a breakdown, as the reference's CG
 * reports.  1 <= k <= min(n, 128); the CSR is checked on the device first.
 * Replaces compute_adjoint_eigsh, python/gpu_eigsh/_cuda_eigsh.cu:183-326. */
int lg_eigsh_adjoint(int n, long long nnz, const int* row_ptr, const int* col_idx, const double* vals, int k,
                     const double* evals, const double* X, const double* g_evals, const double* g_evecs,
                     double* grad_vals, int cg_max_iters, double cg_tol, int* cg_iters, void* stream);

/* Matrix functions by m-step Lanczos quadrature (no restart; the steps stop
 * at an invariant subspace), f = LG_FUNC_LOG / _EXP / _SQRT / _INV:
 *   mode 1: y = f(A) v ~ ||v|| V S f(Theta) S^T e1   (n doubles)
 *   mode 0: *value = v^T f(A) v ~ ||v||^2 sum_i S[0, i]^2 f(Theta_i).
 * v, y: host (io_on_device = 0) or device pointers, in the caller's numbering.
 * *m_actual receives the depth reached (1 <= m <= min(n, max_ncv)), or the
 * reference's negative status: -2 f undefined at a Ritz value (log: theta <= 0,
 * sqrt: theta < 0, inv: theta = 0), -3 zero v (y = 0), -4 tridiagonal
 * eigensolver failure; the call itself then still returns LG_OK.  Single-GPU
 * plans only.  Replaces compute_funm_apply / compute_funm_qform
 * (python/gpu_eigsh/_cuda_funm.cu:40-251, src/matrix_function.cuh:82-274). */
int lg_eigsh_plan_funm(lg_eigsh_plan* plan, const double* v, int io_on_device, int m, int func, int mode, double* y,
                       double* value, int* m_actual);

/* Reference-compatible matrix functions with the reference's signatures and
 * return values (depth reached, or -1 unknown func_name, -2, -3, -4 as above);
 * failures the reference cannot report return -100 + LG_ERR_*.  m is capped at
 * min(n, 127).  compute_funm_debug returns the basis (n x m_actual,
 * column-major), alpha (m_actual) and beta (m_actual + 1; beta[0] = 0,
 * beta[m_actual] = the final residual norm) as the reference's test hook
 * (python/gpu_eigsh/_cuda_funm.cu:132-178). */
int compute_funm_apply(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals,
                       const double* v_host, int m, const char* func_name, double* out_y);
int compute_funm_qform(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals,
                       const double* v_host, int m, const char* func_name, double* out_value);
int compute_funm_debug(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals,
                       const double* v_host, int m, double* out_V, double* out_alpha, double* out_beta);

/* Reference-compatible form of lg_eigsh_adjoint: host arrays, returns 0 (or a
 * negative LG_ERR_* status; the reference aborts the process instead).
 * Same signature as compute_adjoint_eigsh (python/gpu_eigsh/_cuda_eigsh.cu:183-194). */
int compute_adjoint_eigsh(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals, int k,
                          const double* eigenvalues, const double* eigenvectors, const double* grad_evals,
                          const double* grad_evecs, double* grad_vals, int cg_max_iters, double cg_tol);

#ifdef __cplusplus
}
#endif

#endif /* LANCZOS_B200_H */
