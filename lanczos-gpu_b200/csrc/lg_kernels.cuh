// lg_kernels.cuh — launch interfaces of the eigsh kernels (host side).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace lg {

// Layout of a basis: element (r, c) is at V + (c >> 3) * ps + r * rs + (c & 7).
//  * the solver's panel layout: columns in panels of 8, each panel an
//    n_pad x 8 row-major block (rs = 8, ps = 8 n_pad).  Reading c live
//    columns streams ceil(c / 8) contiguous panels, and a new column lands 8
//    bytes every 64 (a row's entry of one panel), not every row stride;
//  * a row-major n x ld array (the caller's basis of lg_cgs2_orthogonalize):
//    rs = ld, ps = 8.
// A 16-byte chunk of two columns (c even) never straddles a panel.
struct VLayout {
  long long rs = 0, ps = 0;
};
__host__ __device__ __forceinline__ long long vidx(const VLayout& L, long long r, int c) {
  return (long long)(c >> 3) * L.ps + r * L.rs + (c & 7);
}

// Launch geometry of the Gram-Schmidt pass kernels (lg_gs.cu).  V has the
// layout L; `ncols` live columns.
struct GsPlan {
  int lpr = 32;      // lanes per basis row
  int ch = 1;        // 2*lpr-column chunks per row
  int grid = 0;      // CTAs (each owns a contiguous row range)
};

GsPlan gs_plan(int n, int ncols, int grid);

cudaError_t gs_project(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n,
                       const double* vec, double* part_out, int* state);
cudaError_t gs_correct_project(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n,
                               const double* W, double* R, const double* part_in, int nrows_in,
                               double* part_out, double* scal, int* state);
cudaError_t gs_correct(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n, double* R,
                       const double* part_in, int nrows_in, double* part_out, double* scal, double* alpha,
                       int j, int alpha_mode, int* state);

// Lag step j (second Gram-Schmidt pass of step j-1 delayed into step j; V has
// j finished columns, R = u the once-orthogonalised residual of step j-1,
// W = z = A u / ||u||):
//   gs_lag_project: partS rows = [V^T u | ||u||^2 in column j], scalar u^T z;
//                   partT rows = [V^T z], scalar ||z||^2
//   gs_lag_correct: DGKS / breakdown checks, alpha_{j-1} += s_{j-1},
//                   beta[j], v_j = (u - V s) / beta_j into V[:, j],
//                   R = (rho / beta_j) (z - V t - (v_j^T z) v_j), alpha[j]
//                   (first pass); part_out: ||R||^2.
cudaError_t gs_lag_project(const GsPlan& p, cudaStream_t st, const double* V, VLayout L, int ncols, int n,
                           const double* U, const double* Z, double* partS, double* partT, int* state);
// Partial-sum rows gs_lag_project writes per table (the CTAs of a cluster
// combine theirs into one row when the grid allows it).
int gs_lag_rows(const GsPlan& p);
cudaError_t gs_lag_correct(const GsPlan& p, cudaStream_t st, double* V, VLayout L, int ncols, int n, double* R,
                           const double* Z, const double* partS, const double* partT, int nrows_in,
                           double* part_out, double* scal, double* alpha, double* beta, int* state);

// SpMV step (lg_spmv.cu).  beta_mode says what the norm of R means.
enum BetaMode {
  BETA_INIT = 0,      // starting vector: normalise only
  BETA_STEP = 1,      // residual of step j-1: store beta[j], run the DGKS / breakdown checks
  BETA_RESTART = 2,   // residual after an implicit restart: store beta[j], breakdown check only
  BETA_ZERO = 3,      // fresh vector after an invariant subspace: beta[j] = 0
  BETA_LAG = 4,       // lag step: w = A r / ||r|| only (V[:, j] and beta[j] come from gs_lag_correct)
};

struct CsrDev {
  int n = 0;
  long long nnz = 0;
  const int* rowptr = nullptr;
  const int* col = nullptr;
  const double* val64 = nullptr;   // fp64 values (or null)
  const float* val32 = nullptr;    // fp32 values (mixed mode) (or null)
  int lanes = 8;                   // lanes per row of the vector kernel
  // Rows with more than kLongRow nonzeros (power-law graphs): the row kernels
  // of spmv_step / spmv_plain stop after kLongRow; the remainder is split into
  // chunks of kLongRow summed by one warp each and added in a fixed order.
  int nlong = 0, nchunks = 0;
  const int* long_rows = nullptr;    // nlong row indices
  const int* long_first = nullptr;   // nlong + 1: chunk range of each long row
  const int* chunk_begin = nullptr;  // nchunks
  const int* chunk_end = nullptr;    // nchunks
  double* chunk_sum = nullptr;       // nchunks
  // Skewed row lengths (power-law graphs): rows bucketed by the lane count
  // that suits them (2, 4, 8, 16, 32 lanes); one launch per non-empty bucket
  // over its row list.  nclasses == 0: all rows with `lanes`.
  int nclasses = 0;
  int class_lanes[5] = {0, 0, 0, 0, 0};
  int class_count[5] = {0, 0, 0, 0, 0};
  const int* class_rows[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
};

// Vj points at column j of the basis, its rows ldv doubles apart (the layout's rs).
cudaError_t spmv_step(const CsrDev& A, cudaStream_t st, int grid, const double* R, double* W, double* Vj,
                      int ldv, const double* part_in, int nrows_in, int j, int beta_mode, double* alpha,
                      double* beta, double* scal, int* state, const double* R_own = nullptr);

// Normalise R into V[:, j] (same checks as spmv_step) without applying A;
// optionally also into the contiguous vector `out`.
cudaError_t normalize_step(cudaStream_t st, int grid, int n, const double* R, double* Vj, int ldv, double* out,
                           const double* part_in,
                           int nrows_in, int j, int beta_mode, double* alpha, double* beta, double* scal,
                           int* state);

// y = A x (+ shift * x) for plain vectors, used by CG and checks.
cudaError_t spmv_plain(const CsrDev& A, cudaStream_t st, int grid, const double* x, double* y,
                       double shift);

// Misc vector kernels (lg_spmv.cu).
cudaError_t fill_random(cudaStream_t st, double* x, int n, int ld, uint64_t seed, long long index0 = 0);
cudaError_t norm_partials(cudaStream_t st, int grid, const double* x, int ld, double* part_out);

// Restart (lg_restart.cu).
struct RestartArgs {
  int m = 0;            // ncv
  int nev0 = 0;         // requested eigenpairs
  int which = 0;        // Which enum
  double tol = 0.0;
  int iter = 0;         // restart counter (1-based, ARPACK convention)
  int maxiter = 0;
  int force_done = 0;   // stop after this Ritz computation (e.g. step budget exhausted)
  int skip_checks = 0;  // residual known to be exactly zero (invariant subspace at the last step)
  const double* part_in = nullptr;
  int nrows_in = 0;
  double* alpha = nullptr;
  double* beta = nullptr;
  double* scal = nullptr;
  double* ritz_out = nullptr;   // m: selected Ritz values (ascending) when done
  double* bounds_out = nullptr; // m
  int* conv_out = nullptr;      // m: converged flag of each selected value
  double* zsel = nullptr;       // m x m col-major: eigenvectors of T for the selection
  double* Q = nullptr;          // m x m col-major: accumulated shift rotations
  double* scratch = nullptr;    // restart_scratch_doubles(): LU factors of the inverse iterations
  int* state = nullptr;
};
enum Which { WHICH_LM = 0, WHICH_SM = 1, WHICH_LA = 2, WHICH_SA = 3, WHICH_BE = 4 };
size_t restart_scratch_doubles();
cudaError_t restart_step(const RestartArgs& a, cudaStream_t st);

// Basis update (lg_basis.cu): out = V[:, 0:m] * Q[:, 0:kq], V with layout vl.
//  restart mode: V[:, 0:kq-1] <- out[:, 0:kq-1] in place;
//                R <- rcoef * R + tau * out[:, kq-1];  norm partials of R.
//  ritz mode   : Y[:, 0:kq] = out (column-major ldy, or row-major when rowmajor).
struct BasisArgs {
  double* V = nullptr;
  VLayout vl;
  int n = 0;
  int m = 0;            // columns of V used
  int kq = 0;           // columns of Q used
  const double* Q = nullptr;   // m x kq col-major, leading dim ldq
  int ldq = 0;
  int restart = 0;
  double* R = nullptr;
  const double* scal = nullptr;  // SC_RCOEF, SC_TAU
  double* part_out = nullptr;
  double* Y = nullptr;
  long long ldy = 0;
  int rowmajor = 0;
  const int* ymap = nullptr;   // ritz mode: row r of out goes to row ymap[r] of Y (null: r)
  int* state = nullptr;
};
struct BasisPlan {
  int TR = 32, grid = 0;
  size_t smem = 0;
};
BasisPlan basis_plan(int n, int m, int kq, int grid);
cudaError_t basis_update(const BasisPlan& p, const BasisArgs& a, cudaStream_t st);

}  // namespace lg
