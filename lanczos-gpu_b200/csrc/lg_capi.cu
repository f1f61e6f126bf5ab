// lg_capi.cu — extern "C" entry points of liblanczos_b200.so (declared in
// include/lanczos_b200.h).
#include "lg_common.cuh"
#include "lg_solver.h"

#include <algorithm>
#include <cstring>
#include <new>
#include <string>

struct lg_eigsh_plan {
  lg::Solver solver;
};

extern "C" {

int lg_eigsh_opts_default(lg_eigsh_opts* o) {
  if (!o) return LG_ERR_INVALID;
  std::memset(o, 0, sizeof(*o));
  o->k = 6;
  o->ncv = 0;
  o->maxiter = 0;
  o->max_steps = 0;
  o->tol = 0.0;
  o->which = LG_WHICH_LM;
  o->use_sigma = 0;
  o->sigma = 0.0;
  o->cg_max_iters = 0;
  o->cg_tol = 1e-12;
  o->mixed = 0;
  o->seed = 42;
  o->return_vectors = 1;
  o->evecs_rowmajor = 0;
  return LG_OK;
}

int lg_eigsh_plan_create(lg_eigsh_plan** plan, int n, long long nnz, const int* row_ptr, const int* col_idx,
                         const double* vals, int device_ptrs, int max_ncv, int mixed) {
  return lg_eigsh_plan_create_ex(plan, n, nnz, row_ptr, col_idx, vals, device_ptrs, max_ncv, mixed, 0);
}

int lg_eigsh_plan_create_ex(lg_eigsh_plan** plan, int n, long long nnz, const int* row_ptr, const int* col_idx,
                            const double* vals, int device_ptrs, int max_ncv, int mixed, int flags) {
  if (!plan) return LG_ERR_INVALID;
  *plan = nullptr;
  if (flags & ~(LG_PLAN_REORDER_BFS | LG_PLAN_CGS2_INLINE | LG_PLAN_REORDER_DEGREE)) {
    lg::g_last_error = "unknown plan flags";
    return LG_ERR_INVALID;
  }
  if ((flags & LG_PLAN_REORDER_BFS) && (flags & LG_PLAN_REORDER_DEGREE)) {
    lg::g_last_error = "LG_PLAN_REORDER_BFS and LG_PLAN_REORDER_DEGREE exclude each other";
    return LG_ERR_INVALID;
  }
  lg_eigsh_plan* p = new (std::nothrow) lg_eigsh_plan();
  if (!p) return LG_ERR_NOMEM;
  const int rc = p->solver.create(n, nnz, row_ptr, col_idx, vals, device_ptrs, max_ncv, mixed, flags);
  if (rc != LG_OK) {
    delete p;
    return rc;
  }
  *plan = p;
  return LG_OK;
}

int lg_eigsh_plan_create_op(lg_eigsh_plan** plan, int n, int kind, lg_matvec_fn fn, lg_matvec_stream_fn sfn,
                            void* user, int max_ncv) {
  if (!plan) return LG_ERR_INVALID;
  *plan = nullptr;
  lg_eigsh_plan* p = new (std::nothrow) lg_eigsh_plan();
  if (!p) return LG_ERR_NOMEM;
  const int rc = p->solver.create_op(n, kind, fn, sfn, user, max_ncv);
  if (rc != LG_OK) {
    delete p;
    return rc;
  }
  *plan = p;
  return LG_OK;
}

int lg_partition_block(int n, int nranks) {
  if (n < 1 || nranks < 1) return 0;
  const long long per = ((long long)n + nranks - 1) / nranks;
  return (int)((per + lg::kRowAlign - 1) / lg::kRowAlign * lg::kRowAlign);
}

int lg_eigsh_plan_create_dist(lg_eigsh_plan** plan, lg_comm* comm, int n_global, int n_local, long long nnz,
                              const int* row_ptr, const int* col_idx, const double* vals, int device_ptrs,
                              int max_ncv, int mixed) {
  if (!plan) return LG_ERR_INVALID;
  *plan = nullptr;
  lg_eigsh_plan* p = new (std::nothrow) lg_eigsh_plan();
  if (!p) return LG_ERR_NOMEM;
  const int rc = p->solver.create_dist(comm, n_global, n_local, nnz, row_ptr, col_idx, vals, device_ptrs, max_ncv,
                                       mixed);
  if (rc != LG_OK) {
    delete p;
    return rc;
  }
  *plan = p;
  return LG_OK;
}

int lg_eigsh_plan_set_exchange(lg_eigsh_plan* plan, int mode) {
  if (!plan) return LG_ERR_INVALID;
  return plan->solver.set_exchange(mode);
}

int lg_eigsh_plan_exchange_info(const lg_eigsh_plan* plan, int* mode, long long* recv_rows, long long* send_rows) {
  if (!plan) return LG_ERR_INVALID;
  return plan->solver.exchange_info(mode, recv_rows, send_rows);
}

int lg_eigsh_plan_set_transport(lg_eigsh_plan* plan, int mode) {
  if (!plan) return LG_ERR_INVALID;
  return plan->solver.set_transport(mode);
}

int lg_eigsh_plan_transport(const lg_eigsh_plan* plan, int* mode) {
  if (!plan || !mode) return LG_ERR_INVALID;
  *mode = plan->solver.transport_mode();
  return LG_OK;
}

int lg_eigsh_plan_funm(lg_eigsh_plan* plan, const double* v, int io_on_device, int m, int func, int mode, double* y,
                       double* value, int* m_actual) {
  if (!plan) return LG_ERR_INVALID;
  return plan->solver.funm(v, io_on_device, m, func, mode, y, value, m_actual);
}

int lg_eigsh_plan_run(lg_eigsh_plan* plan, const lg_eigsh_opts* opts, const double* v0, double* evals,
                      double* evecs, int io_on_device, lg_eigsh_info* info) {
  if (!plan || !opts || !evals) {
    lg::g_last_error = "null plan, opts or evals";
    return LG_ERR_INVALID;
  }
  return plan->solver.run(*opts, v0, evals, evecs, io_on_device, info);
}

int lg_eigsh_plan_destroy(lg_eigsh_plan* plan) {
  delete plan;
  return LG_OK;
}

int lg_eigsh_plan_matvec(lg_eigsh_plan* plan, const double* x, double* y) {
  if (!plan || !x || !y) return LG_ERR_INVALID;
  return plan->solver.matvec(x, y);
}

int lg_eigsh_plan_factorize(lg_eigsh_plan* plan, const double* v0, int m, double* alpha, double* beta) {
  if (!plan || !v0 || !alpha || !beta) return LG_ERR_INVALID;
  return plan->solver.factorize(v0, m, alpha, beta);
}

int lg_eigsh(int n, long long nnz, const int* row_ptr, const int* col_idx, const double* vals,
             const lg_eigsh_opts* opts, const double* v0, double* evals, double* evecs, lg_eigsh_info* info) {
  if (!opts) return LG_ERR_INVALID;
  int ncv = opts->ncv > 0 ? opts->ncv : std::min(n, std::max(2 * opts->k + 1, 20));
  lg_eigsh_plan* p = nullptr;
  int rc = lg_eigsh_plan_create(&p, n, nnz, row_ptr, col_idx, vals, 0, ncv, opts->mixed);
  if (rc != LG_OK) return rc;
  rc = lg_eigsh_plan_run(p, opts, v0, evals, evecs, 0, info);
  lg_eigsh_plan_destroy(p);
  return rc;
}

const char* lg_status_string(int status) {
  switch (status) {
    case LG_OK: return "ok";
    case LG_NOCONV: return "iteration limit reached before all Ritz pairs converged";
    case LG_ERR_INVALID: return "invalid argument";
    case LG_ERR_CUDA: return "CUDA error";
    case LG_ERR_NOMEM: return "device memory allocation failed";
    case LG_ERR_TIMEOUT: return "bounded device wait timed out";
    case LG_ERR_NUMERIC: return "numerical failure";
    case LG_ERR_CG_NOCONV: return "inner CG did not converge";
    default: return "unknown status";
  }
}

int lg_last_error(char* buf, int len) {
  const std::string& s = lg::g_last_error;
  if (buf && len > 0) {
    const int c = std::min<int>(len - 1, (int)s.size());
    std::memcpy(buf, s.data(), c);
    buf[c] = '\0';
  }
  return (int)s.size();
}

// ---- reference-compatible ABI ---------------------------------------------

// Reference behaviour kept: k smallest-algebraic pairs, ncv = 0 means
// min(max(3k, 40), n), max_iters is a Lanczos-step budget, the return value
// is min(k, ncv), eigenvectors are column-major.
int compute_eigsh(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals, int k, int ncv,
                  int max_iters, double tol, double* out_eigenvalues, double* out_eigenvectors) {
  if (n < 2 || k < 1 || k >= n || !out_eigenvalues) return LG_ERR_INVALID;
  lg_eigsh_opts o;
  lg_eigsh_opts_default(&o);
  o.k = k;
  o.ncv = ncv > 0 ? std::min(ncv, n) : std::min(std::max(3 * k, 40), n);
  if (o.ncv <= k) o.ncv = std::min(n, k + 1);
  o.which = LG_WHICH_SA;
  o.tol = tol;
  o.max_steps = max_iters > 0 ? max_iters : 0;
  o.maxiter = 2147483647;
  o.return_vectors = out_eigenvectors != nullptr;
  o.evecs_rowmajor = 0;
  lg_eigsh_info info;
  const int rc = lg_eigsh(n, nnz, row_ptr, col_idx, vals, &o, nullptr, out_eigenvalues, out_eigenvectors, &info);
  if (rc < 0) return rc;
  return std::min(k, o.ncv);
}

int compute_eigsh_sigma(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals, int k,
                        int ncv, int max_iters, double tol, double sigma, int cg_max_iters, double cg_tol,
                        double* out_eigenvalues, double* out_eigenvectors) {
  if (n < 2 || k < 1 || k >= n || !out_eigenvalues) return LG_ERR_INVALID;
  lg_eigsh_opts o;
  lg_eigsh_opts_default(&o);
  o.k = k;
  o.ncv = ncv > 0 ? std::min(ncv, n) : std::min(std::max(3 * k, 40), n);
  if (o.ncv <= k) o.ncv = std::min(n, k + 1);
  o.which = LG_WHICH_LM;   // largest |mu| of (A - sigma I)^-1 = nearest sigma
  o.tol = tol;
  o.max_steps = max_iters > 0 ? max_iters : 0;
  o.maxiter = 2147483647;
  o.use_sigma = 1;
  o.sigma = sigma;
  o.cg_max_iters = cg_max_iters;
  o.cg_tol = cg_tol;
  o.return_vectors = out_eigenvectors != nullptr;
  lg_eigsh_info info;
  const int rc = lg_eigsh(n, nnz, row_ptr, col_idx, vals, &o, nullptr, out_eigenvalues, out_eigenvectors, &info);
  if (rc < 0 && rc != LG_ERR_CG_NOCONV) return rc;
  return std::min(k, o.ncv);
}

}  // extern "C"

// ---- reference-compatible matrix functions (python/gpu_eigsh/_cuda_funm.cu) --
// Return values keep the reference's meaning: the depth reached (> 0), or -1
// unknown function, -2 f undefined at a Ritz value, -3 zero vector, -4
// tridiagonal eigensolver failure.  Failures the reference cannot report (it
// exits the process) come back as kFunmLibErr + LG_ERR_* (text in lg_last_error).
static const int kFunmLibErr = -100;

static int funm_code(const char* name) {
  if (!name) return -1;
  if (std::strcmp(name, "log") == 0) return LG_FUNC_LOG;
  if (std::strcmp(name, "exp") == 0) return LG_FUNC_EXP;
  if (std::strcmp(name, "sqrt") == 0) return LG_FUNC_SQRT;
  if (std::strcmp(name, "inv") == 0) return LG_FUNC_INV;
  return -1;
}

static int funm_host(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals, const double* v,
                     int m, const char* func_name, int mode, double* y, double* value) {
  const int func = funm_code(func_name);
  if (func < 0) return -1;   // the reference's "unknown func"
  if (n < 1 || m < 1 || !v) {
    lg::g_last_error = "compute_funm: invalid arguments";
    return kFunmLibErr + LG_ERR_INVALID;
  }
  lg_eigsh_plan* p = nullptr;
  int rc = lg_eigsh_plan_create(&p, n, nnz, row_ptr, col_idx, vals, 0, std::min(m, n), 0);
  if (rc != LG_OK) return kFunmLibErr + rc;
  int ma = 0;
  rc = p->solver.funm(v, 0, std::min(m, n), func, mode, y, value, &ma);
  lg_eigsh_plan_destroy(p);
  return rc != LG_OK ? kFunmLibErr + rc : ma;
}

extern "C" {

int compute_funm_apply(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals,
                       const double* v_host, int m, const char* func_name, double* out_y) {
  if (!out_y) return kFunmLibErr + LG_ERR_INVALID;
  return funm_host(n, nnz, row_ptr, col_idx, vals, v_host, m, func_name, 1, out_y, nullptr);
}

int compute_funm_qform(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals,
                       const double* v_host, int m, const char* func_name, double* out_value) {
  if (!out_value) return kFunmLibErr + LG_ERR_INVALID;
  return funm_host(n, nnz, row_ptr, col_idx, vals, v_host, m, func_name, 0, nullptr, out_value);
}

int compute_funm_debug(int n, int nnz, const int* row_ptr, const int* col_idx, const double* vals,
                       const double* v_host, int m, double* out_V, double* out_alpha, double* out_beta) {
  if (n < 1 || m < 1 || !v_host || !out_V || !out_alpha || !out_beta) return kFunmLibErr + LG_ERR_INVALID;
  lg_eigsh_plan* p = nullptr;
  int rc = lg_eigsh_plan_create(&p, n, nnz, row_ptr, col_idx, vals, 0, std::min(m, n), 0);
  if (rc != LG_OK) return kFunmLibErr + rc;
  int ma = 0;
  rc = p->solver.funm_debug(v_host, std::min(m, n), out_V, out_alpha, out_beta, &ma);
  lg_eigsh_plan_destroy(p);
  return rc != LG_OK ? kFunmLibErr + rc : ma;
}

}  // extern "C"

