// lg_irlm.cu — host driver of the implicitly restarted Lanczos method.
//
// Reference: src/irlm_lanczos.cu:153-394 (irlm_lanczos), :110-148
// (lanczos_extend) and the C ABI wrappers python/gpu_eigsh/_cuda_eigsh.cu.
//
// Differences in structure (same mathematics):
//  * all vectors, alpha/beta, the restart logic and the convergence test stay
//    on the device; the host enqueues a whole Lanczos extension
//    (3 kernels per lag step, 4 with in-step CGS2) without waiting and synchronises once per
//    restart to read a 16-word state record;
//  * rare events (a third DGKS pass, an invariant subspace) are detected on
//    the device, which then turns the rest of the queued work into no-ops;
//    the host handles the event at the next sync and resumes at the next step;
//  * workspace lives in a plan that can be reused across solves; nothing is
//    allocated inside the iteration.
#include "lg_common.cuh"
#include "lg_csr.cuh"
#include "lg_halo.h"
#include "lg_pool.h"
#include "lg_kernels.cuh"
#include "lg_solver.h"
#include "lg_staging.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace lg {

thread_local std::string g_last_error;

void set_error(const char* fmt, const char* a, int line) {
  char buf[512];
  snprintf(buf, sizeof(buf), fmt, a, line);
  g_last_error = buf;
}

#define LG_TRY(expr)                                                     \
  do {                                                                   \
    cudaError_t _e = (expr);                                             \
    if (_e != cudaSuccess) {                                             \
      set_error("CUDA error %s at lg_irlm.cu:%d", cudaGetErrorString(_e), __LINE__); \
      return (_e == cudaErrorMemoryAllocation) ? LG_ERR_NOMEM : LG_ERR_CUDA; \
    }                                                                    \
  } while (0)

static int pick_lanes(double mean) {
  if (mean < 3.0) return 2;
  if (mean < 8.0) return 4;   // 7-point stencils: 4 lanes keep the CG products 21 % faster than 8
  if (mean < 16.0) return 8;
  if (mean < 32.0) return 16;
  return 32;
}

__global__ void cast_f64_f32_kernel(const double* __restrict__ a, float* __restrict__ b, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    b[i] = (float)a[i];
}

// Sets *bad when a column index lies outside [0, ncols) (device-pointer CSR
// input is checked before any kernel gathers through it).
__global__ void check_cols_kernel(const int* __restrict__ col, long long nnz, int ncols, int* bad) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nnz; i += (long long)gridDim.x * blockDim.x) {
    const int c = col[i];
    if (c < 0 || c >= ncols) *bad = 1;
  }
}

__global__ void scale_kernel(double* x, int n, double s) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) x[i] *= s;
}

Solver::~Solver() { release(); }

void Solver::release() {
  release_peer();
  if (Rfull) {
    cudaFree(Rfull);
    Rfull = nullptr;
    R = nullptr;
  }
  if (red) dfree(red);
  red = nullptr;
  for (void* p : {(void*)d_send_idx, (void*)d_recv_pos, (void*)d_send_buf, (void*)d_recv_buf, (void*)d_perm,
                  (void*)funm_ws})
    if (p) dfree(p);
  d_perm = nullptr;
  funm_ws = nullptr;
  d_send_idx = d_recv_pos = nullptr;
  d_send_buf = d_recv_buf = nullptr;
  send_off.clear();
  send_cnt.clear();
  recv_off.clear();
  recv_cnt.clear();
  halo_send = halo_recv = 0;
  void* ptrs[] = {d_rowptr, d_col, d_val64, d_val32, d_long, d_chunk_sum, d_classes, V, W, R, partA, partB, partC, alpha, beta, scal,
                  ritz, bounds, zsel, Q, rs_scratch, conv, state, Ytmp, cg_ws, cg_part, cg_scal, cg_counter, cg_flags};
  for (void* p : ptrs)
    if (p) dfree(p);
  d_rowptr = d_col = nullptr;
  d_val64 = nullptr;
  d_val32 = nullptr;
  d_long = nullptr;
  d_chunk_sum = nullptr;
  d_classes = nullptr;
  A = CsrDev();
  V = W = R = partA = partB = partC = alpha = beta = scal = ritz = bounds = zsel = Q = rs_scratch = Ytmp = cg_ws = nullptr;
  cg_part = cg_scal = nullptr;
  cg_counter = nullptr;
  conv = state = cg_flags = nullptr;
  if (op_x) dfree(op_x);
  op_x = nullptr;
  if (h_op_x) cudaFreeHost(h_op_x);
  if (h_op_y) cudaFreeHost(h_op_y);
  h_op_x = h_op_y = nullptr;
  if (h_state) cudaFreeHost(h_state);
  if (h_cg_flags) cudaFreeHost(h_cg_flags);
  h_state = h_cg_flags = nullptr;
  for (cudaEvent_t e : ev_pool) cudaEventDestroy(e);
  ev_pool.clear();
  if (ev0) cudaEventDestroy(ev0);
  if (ev1) cudaEventDestroy(ev1);
  ev0 = ev1 = nullptr;
  if (stream) cudaStreamDestroy(stream);
  stream = nullptr;
}

// Plan buffers come from the library's device pool (lg_pool.h) on the plan's
// stream, so creating and destroying plans in a loop maps no memory after the
// first plan; buffers other ranks map with CUDA IPC stay plain allocations.
cudaError_t Solver::dalloc(void** p, size_t bytes) {
  cudaError_t e = pool_alloc(p, bytes, stream);
  if (e == cudaSuccess) pooled.insert(*p);
  return e;
}

void Solver::dfree(void* p) {
  if (!p) return;
  auto it = pooled.find(p);
  if (it != pooled.end()) {
    pool_free(p, stream);
    pooled.erase(it);
  } else {
    cudaFree(p);
  }
}

int Solver::init_device() {
  LG_TRY(cudaGetDevice(&device));
  LG_TRY(cudaDeviceGetAttribute(&num_sm, cudaDevAttrMultiProcessorCount, device));
  int smem_optin = 0;
  LG_TRY(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  smem_budget = (size_t)smem_optin;
  LG_TRY(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  LG_TRY(cudaEventCreate(&ev0));
  LG_TRY(cudaEventCreate(&ev1));

  grid_gs = num_sm;
  grid_spmv = num_sm * 8;
  grid_basis = num_sm * 4;
  return LG_OK;
}

// The Krylov basis, the operator output and residual, the partial-sum rows,
// the tridiagonal and the restart state (n, ld, ldv and the stream are set).
int Solver::alloc_workspace() {
  LG_TRY(dalloc((void**)&V, sizeof(double) * vsize()));
  LG_TRY(dalloc((void**)&W, sizeof(double) * (size_t)ld));
  if (comm) {
    LG_TRY(cudaMalloc(&Rfull, sizeof(double) * (size_t)ld * nranks));
    LG_TRY(cudaMemsetAsync(Rfull, 0, sizeof(double) * (size_t)ld * nranks, stream));
    R = Rfull + (size_t)rank * ld;
    LG_TRY(dalloc((void**)&red, sizeof(double) * 3 * kPartStride));
    LG_TRY(cudaMemsetAsync(red, 0, sizeof(double) * 3 * kPartStride, stream));
  } else {
    LG_TRY(dalloc((void**)&R, sizeof(double) * (size_t)ld));
    LG_TRY(cudaMemsetAsync(R, 0, sizeof(double) * (size_t)ld, stream));
  }
  LG_TRY(cudaMemsetAsync(V, 0, sizeof(double) * vsize(), stream));
  LG_TRY(cudaMemsetAsync(W, 0, sizeof(double) * (size_t)ld, stream));
  const int prow = std::max(grid_gs, std::max(grid_basis, num_sm)) ;
  for (double** p : {&partA, &partB, &partC}) {
    LG_TRY(dalloc((void**)p, sizeof(double) * (size_t)prow * kPartStride));
    LG_TRY(cudaMemsetAsync(*p, 0, sizeof(double) * (size_t)prow * kPartStride, stream));
  }
  LG_TRY(dalloc((void**)&alpha, sizeof(double) * (kMaxCols + 2)));
  LG_TRY(dalloc((void**)&beta, sizeof(double) * (kMaxCols + 2)));
  LG_TRY(dalloc((void**)&scal, sizeof(double) * SC_WORDS));
  LG_TRY(dalloc((void**)&ritz, sizeof(double) * kMaxCols));
  LG_TRY(dalloc((void**)&bounds, sizeof(double) * kMaxCols));
  LG_TRY(dalloc((void**)&zsel, sizeof(double) * kMaxCols * kMaxCols));
  LG_TRY(dalloc((void**)&Q, sizeof(double) * kMaxCols * kMaxCols));
  LG_TRY(dalloc((void**)&rs_scratch, sizeof(double) * restart_scratch_doubles()));
  LG_TRY(dalloc((void**)&conv, sizeof(int) * kMaxCols));
  LG_TRY(dalloc((void**)&state, sizeof(int) * ST_WORDS));
  LG_TRY(cudaMallocHost(&h_state, sizeof(int) * ST_WORDS));
  return LG_OK;
}

int Solver::create_op(int n_, int kind, lg_matvec_fn fn, lg_matvec_stream_fn sfn, void* user, int max_ncv_) {
  if (n_ < 2) {
    g_last_error = "matrix-free plan: n must be at least 2";
    return LG_ERR_INVALID;
  }
  if (kind != LG_OP_DEVICE && kind != LG_OP_HOST && kind != LG_OP_STREAM) {
    g_last_error = "matrix-free plan: kind must be LG_OP_DEVICE, LG_OP_HOST or LG_OP_STREAM";
    return LG_ERR_INVALID;
  }
  if ((kind == LG_OP_STREAM) != (sfn != nullptr) || (kind != LG_OP_STREAM) != (fn != nullptr)) {
    g_last_error = "matrix-free plan: LG_OP_STREAM takes sfn only, LG_OP_DEVICE / LG_OP_HOST take fn only";
    return LG_ERR_INVALID;
  }
  comm = nullptr;
  n_global = n_;
  row0 = 0;
  nranks = 1;
  rank = 0;
  n = n_;
  nnz = 0;
  mixed = 0;
  op_kind = kind;
  op_fn = fn;
  op_sfn = sfn;
  op_user = user;
  max_ncv = std::max(2, std::min(max_ncv_ > 0 ? max_ncv_ : kMaxCols - 1, kMaxCols - 1));
  ld = round_up(n, kRowAlign);
  ldv = round_up(max_ncv + 1, 8);
  vl.rs = 8;
  vl.ps = 8ll * round_up(n, 8);
  int rc = init_device();
  if (rc != LG_OK) return rc;
  rc = alloc_workspace();
  if (rc != LG_OK) return rc;
  LG_TRY(dalloc((void**)&op_x, sizeof(double) * (size_t)ld));
  LG_TRY(cudaMemsetAsync(op_x, 0, sizeof(double) * (size_t)ld, stream));
  if (kind == LG_OP_HOST) {
    LG_TRY(cudaMallocHost(&h_op_x, sizeof(double) * (size_t)n));
    LG_TRY(cudaMallocHost(&h_op_y, sizeof(double) * (size_t)n));
  }
  lag_steps = false;   // the lag steps fold 1/||u|| into the sparse product; a callback gets v_j itself
  LG_TRY(cudaStreamSynchronize(stream));
  return LG_OK;
}

// y = OP(x) by the caller's callback (x, y: device vectors of n doubles).
//  LG_OP_STREAM: the callback enqueues its work on the plan's stream.
//  LG_OP_DEVICE: the callback may use any stream; the plan's stream is
//    drained before the call and the whole device after it.
//  LG_OP_HOST:   x goes to pinned host memory, the callback runs on host
//    vectors, y comes back.
int Solver::call_user_op(const double* x, double* y) {
  const size_t bytes = sizeof(double) * (size_t)n;
  if (op_kind == LG_OP_STREAM) {
    op_sfn(x, y, n, op_user, (void*)stream);
    LG_TRY(cudaGetLastError());
    return LG_OK;
  }
  if (op_kind == LG_OP_HOST) {
    LG_TRY(cudaMemcpyAsync(h_op_x, x, bytes, cudaMemcpyDeviceToHost, stream));
    LG_TRY(cudaStreamSynchronize(stream));
    op_fn(h_op_x, h_op_y, n, op_user);
    LG_TRY(cudaMemcpyAsync(y, h_op_y, bytes, cudaMemcpyHostToDevice, stream));
    // h_op_y is rewritten by the next call: wait for this copy
    LG_TRY(cudaStreamSynchronize(stream));
    return LG_OK;
  }
  LG_TRY(cudaStreamSynchronize(stream));
  op_fn(x, y, n, op_user);
  LG_TRY(cudaGetLastError());
  LG_TRY(cudaDeviceSynchronize());
  return LG_OK;
}

// Matrix-free step j: v_j = R / beta_j into V[:, j] and op_x (the same DGKS /
// breakdown checks as the sparse step), then W = OP(v_j).
int Solver::apply_user_op(int j, int beta_mode) {
  double* Vj = V + vidx(vl, 0, j);
  LG_TRY(timed(LG_K_OTHER, 24.0 * n, 1, [&] {
    return normalize_step(stream, num_sm * 8, n, R, Vj, (int)vl.rs, op_x, inC, nrowsC, j, beta_mode, alpha, beta, scal,
                          state);
  }));
  return call_user_op(op_x, W);
}

int Solver::create(int n_, long long nnz_, const int* rowptr, const int* col, const double* vals, int device_ptrs,
                   int max_ncv_, int mixed_, int flags) {
  comm = nullptr;
  n_global = n_;
  row0 = 0;
  nranks = 1;
  rank = 0;
  return create_impl(n_, n_, nnz_, rowptr, col, vals, device_ptrs, max_ncv_, mixed_, flags);
}

int Solver::create_dist(lg_comm* c, int n_glob, int n_local, long long nnz_, const int* rowptr, const int* col,
                        const double* vals, int device_ptrs, int max_ncv_, int mixed_) {
  if (!c) {
    g_last_error = "null communicator";
    return LG_ERR_INVALID;
  }
  comm = c;
  nranks = comm_size(c);
  rank = comm_rank(c);
  n_global = n_glob;
  const int nb = lg_partition_block(n_glob, nranks);
  row0 = rank * nb;
  const int expect = std::min(nb, n_glob - row0);
  if (nb <= 0 || expect < 1 || n_local != expect) {
    char buf[200];
    snprintf(buf, sizeof(buf), "rank %d must own rows [%d, %d) (block %d of n=%d over %d ranks; every rank needs rows)",
             rank, row0, row0 + std::max(expect, 0), nb, n_glob, nranks);
    g_last_error = buf;
    return LG_ERR_INVALID;
  }
  return create_impl(n_local, n_glob, nnz_, rowptr, col, vals, device_ptrs, max_ncv_, mixed_, 0);
}

int Solver::create_impl(int n_, int n_cols, long long nnz_, const int* rowptr, const int* col, const double* vals,
                        int device_ptrs, int max_ncv_, int mixed_, int flags) {
  if (n_ < 1 || nnz_ < 0 || !rowptr || (nnz_ > 0 && (!col || !vals))) {
    g_last_error = "invalid CSR arguments";
    return LG_ERR_INVALID;
  }
  if (nnz_ > 2147483647ll) {
    g_last_error = "nnz exceeds int32 indexing";
    return LG_ERR_INVALID;
  }
  if (!device_ptrs) {
    // Host-side structural checks (the reference performs none).
    if (rowptr[0] != 0 || (long long)rowptr[n_] != nnz_) {
      g_last_error = "row_ptr must start at 0 and end at nnz";
      return LG_ERR_INVALID;
    }
    for (int i = 0; i < n_; ++i)
      if (rowptr[i + 1] < rowptr[i]) {
        g_last_error = "row_ptr is not monotone";
        return LG_ERR_INVALID;
      }
    // column range on all host cores (tens of millions of entries)
    const int nth = (int)std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    std::vector<char> bad((size_t)nth, 0);
    std::vector<std::thread> pool;
    for (int w = 0; w < nth; ++w)
      pool.emplace_back([&, w] {
        const long long b = nnz_ * w / nth, e = nnz_ * (w + 1) / nth;
        for (long long k = b; k < e; ++k)
          if (col[k] < 0 || col[k] >= n_cols) {
            bad[w] = 1;
            return;
          }
      });
    for (std::thread& th : pool) th.join();
    for (char b : bad)
      if (b) {
        g_last_error = "column index out of range";
        return LG_ERR_INVALID;
      }
  }
  n = n_;
  nnz = nnz_;
  mixed = mixed_;
  max_ncv = std::max(2, std::min(max_ncv_ > 0 ? max_ncv_ : kMaxCols - 1, kMaxCols - 1));
  ld = comm ? lg_partition_block(n_global, nranks) : round_up(n, kRowAlign);
  ldv = round_up(max_ncv + 1, 8);
  vl.rs = 8;
  vl.ps = 8ll * round_up(n, 8);

  {
    int rc = init_device();
    if (rc != LG_OK) return rc;
  }

  LG_TRY(dalloc((void**)&d_rowptr, sizeof(int) * (size_t)(n + 1)));
  LG_TRY(dalloc((void**)&d_col, sizeof(int) * (size_t)std::max<long long>(nnz, 1)));
  LG_TRY(dalloc((void**)&d_val64, sizeof(double) * (size_t)std::max<long long>(nnz, 1)));
  if (device_ptrs) {
    LG_TRY(cudaMemcpyAsync(d_rowptr, rowptr, sizeof(int) * (size_t)(n + 1), cudaMemcpyDeviceToDevice, stream));
    if (nnz > 0) {
      LG_TRY(cudaMemcpyAsync(d_col, col, sizeof(int) * (size_t)nnz, cudaMemcpyDeviceToDevice, stream));
      LG_TRY(cudaMemcpyAsync(d_val64, vals, sizeof(double) * (size_t)nnz, cudaMemcpyDeviceToDevice, stream));
    }
  } else {   // pageable host arrays: through the pinned staging pool
    LG_TRY(staged_h2d(d_rowptr, rowptr, sizeof(int) * (size_t)(n + 1), stream));
    if (nnz > 0) {
      LG_TRY(staged_h2d(d_col, col, sizeof(int) * (size_t)nnz, stream));
      LG_TRY(staged_h2d(d_val64, vals, sizeof(double) * (size_t)nnz, stream));
    }
  }

  {
    int rc = alloc_workspace();
    if (rc != LG_OK) return rc;
  }

  A.n = n;
  A.nnz = nnz;
  A.rowptr = d_rowptr;
  A.col = d_col;
  A.val64 = d_val64;
  A.val32 = nullptr;   // set once the fp32 copy exists (after any reordering)
  A.lanes = pick_lanes(nnz / (double)n);

  std::vector<int> hrp((size_t)n + 1);
  if (device_ptrs) {
    // the same structural checks as for host input: row_ptr on the host,
    // column indices by a kernel
    LG_TRY(cudaMemcpyAsync(hrp.data(), rowptr, sizeof(int) * hrp.size(), cudaMemcpyDeviceToHost, stream));
    LG_TRY(cudaMemsetAsync(state, 0, sizeof(int) * ST_WORDS, stream));
    if (nnz > 0) {
      check_cols_kernel<<<num_sm * 4, 256, 0, stream>>>(d_col, nnz, n_cols, state);
      LG_TRY(cudaGetLastError());
    }
    LG_TRY(cudaMemcpyAsync(h_state, state, sizeof(int), cudaMemcpyDeviceToHost, stream));
    LG_TRY(cudaStreamSynchronize(stream));
    if (hrp[0] != 0 || (long long)hrp[n] != nnz) {
      g_last_error = "row_ptr must start at 0 and end at nnz";
      return LG_ERR_INVALID;
    }
    for (int i = 0; i < n; ++i)
      if (hrp[i + 1] < hrp[i]) {
        g_last_error = "row_ptr is not monotone";
        return LG_ERR_INVALID;
      }
    if (h_state[0] != 0) {
      g_last_error = "column index out of range";
      return LG_ERR_INVALID;
    }
  } else {
    std::copy(rowptr, rowptr + n + 1, hrp.begin());
  }
  lag_steps = !(flags & LG_PLAN_CGS2_INLINE);
  if ((flags & (LG_PLAN_REORDER_BFS | LG_PLAN_REORDER_DEGREE)) && !comm) {
    int rc = reorder_rows(hrp, (flags & LG_PLAN_REORDER_DEGREE) != 0);
    if (rc != LG_OK) return rc;
  }
  if (mixed) {
    LG_TRY(dalloc((void**)&d_val32, sizeof(float) * (size_t)std::max<long long>(nnz, 1)));
    cast_f64_f32_kernel<<<num_sm * 4, 256, 0, stream>>>(d_val64, d_val32, nnz);
    LG_TRY(cudaGetLastError());
    A.val32 = d_val32;
  }
  {
    int rc = build_long_rows(hrp.data());
    if (rc != LG_OK) return rc;
  }
  if (comm) {
    int rc = setup_halo();
    if (rc != LG_OK) return rc;
    rc = setup_peer();
    if (rc != LG_OK) return rc;
  }

  LG_TRY(cudaStreamSynchronize(stream));
  return LG_OK;
}

// Row i of the renumbered CSR is row perm[i] of the caller's, its column
// indices mapped through pos = perm^-1 (one warp per row, entries in the
// caller's order).
__global__ void permute_csr_kernel(int n, const int* __restrict__ perm, const int* __restrict__ pos,
                                   const int* __restrict__ rp_old, const int* __restrict__ col_old,
                                   const double* __restrict__ val_old, const int* __restrict__ rp_new,
                                   int* __restrict__ col_new, double* __restrict__ val_new) {
  const int lane = threadIdx.x & 31;
  for (long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; w < n;
       w += ((long long)gridDim.x * blockDim.x) >> 5) {
    const int i = (int)w;
    const int src = rp_old[perm[i]], len = rp_old[perm[i] + 1] - src, dst = rp_new[i];
    for (int k = lane; k < len; k += 32) {
      col_new[dst + k] = pos[col_old[src + k]];
      val_new[dst + k] = val_old[src + k];
    }
  }
}

// out[i] = in[perm[i]]  (caller's order -> plan order)
__global__ void gather_perm_kernel(double* __restrict__ out, const double* __restrict__ in,
                                   const int* __restrict__ perm, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = in[perm[i]];
}

// out[perm[i]] = in[i]  (plan order -> caller's order)
__global__ void scatter_perm_kernel(double* __restrict__ out, const double* __restrict__ in,
                                    const int* __restrict__ perm, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[perm[i]] = in[i];
}

// perm[new] = old: the rows by descending length, ties by index (a counting
// sort, O(n + longest row)).
static void degree_order(int n, const int* hrp, int* perm) {
  int maxlen = 0;
  for (int i = 0; i < n; ++i) maxlen = std::max(maxlen, hrp[i + 1] - hrp[i]);
  std::vector<long long> start((size_t)maxlen + 2, 0);
  for (int i = 0; i < n; ++i) ++start[(size_t)(maxlen - (hrp[i + 1] - hrp[i])) + 1];
  for (size_t d = 1; d < start.size(); ++d) start[d] += start[d - 1];
  for (int i = 0; i < n; ++i) perm[start[(size_t)(maxlen - (hrp[i + 1] - hrp[i]))]++] = i;
}

// Renumbers the rows for locality of the sparse product's gathers.  Without
// by_degree: Cuthill-McKee order (BFS levels from a pseudo-peripheral vertex,
// each level in the order of the vertices that found it; lg_graph_cm_order
// on the host), so that neighbouring rows get nearby numbers and the gathers
// hit L1 / L2.  With by_degree: descending row length, so that the hubs of a
// power-law graph (the entries most gathers read) are packed together at the
// front.  The plan keeps perm (plan row -> caller row): v0 is gathered
// through it and the Ritz vectors are written through it, so the caller sees
// its own numbering.  hrp (host row pointer) becomes the new one.
int Solver::reorder_rows(std::vector<int>& hrp, bool by_degree) {
  std::vector<int> perm((size_t)n), pos((size_t)n), nrp((size_t)n + 1);
  if (by_degree) {
    degree_order(n, hrp.data(), perm.data());
  } else {
    // Cuthill-McKee order on the host from the column indices already on
    // the device
    std::vector<int> hcol((size_t)std::max<long long>(nnz, 1));
    if (nnz > 0) {
      LG_TRY(cudaMemcpyAsync(hcol.data(), d_col, sizeof(int) * (size_t)nnz, cudaMemcpyDeviceToHost, stream));
      LG_TRY(cudaStreamSynchronize(stream));
    }
    int rc = lg_graph_cm_order(n, hrp.data(), hcol.data(), perm.data());
    if (rc != LG_OK) return rc;
  }
  for (int i = 0; i < n; ++i) pos[(size_t)perm[i]] = i;
  nrp[0] = 0;
  for (int i = 0; i < n; ++i) nrp[(size_t)i + 1] = nrp[i] + (hrp[(size_t)perm[i] + 1] - hrp[perm[i]]);

  int *d_pos = nullptr, *rp2 = nullptr, *col2 = nullptr;
  double* val2 = nullptr;
  cudaError_t e = cudaSuccess;
  LG_TRY(dalloc((void**)&d_perm, sizeof(int) * (size_t)n));
  LG_TRY(dalloc((void**)&d_pos, sizeof(int) * (size_t)n));
  e = dalloc((void**)&rp2, sizeof(int) * ((size_t)n + 1));
  if (e == cudaSuccess) e = dalloc((void**)&col2, sizeof(int) * (size_t)std::max<long long>(nnz, 1));
  if (e == cudaSuccess) e = dalloc((void**)&val2, sizeof(double) * (size_t)std::max<long long>(nnz, 1));
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_perm, perm.data(), sizeof(int) * (size_t)n, cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_pos, pos.data(), sizeof(int) * (size_t)n, cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(rp2, nrp.data(), sizeof(int) * ((size_t)n + 1), cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess && nnz > 0) {
    permute_csr_kernel<<<num_sm * 8, 256, 0, stream>>>(n, d_perm, d_pos, d_rowptr, d_col, d_val64, rp2, col2, val2);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);   // the host vectors go out of scope
  dfree(d_pos);
  if (e != cudaSuccess) {
    dfree(rp2);
    dfree(col2);
    dfree(val2);
    LG_TRY(e);
  }
  dfree(d_rowptr);
  dfree(d_col);
  dfree(d_val64);
  d_rowptr = rp2;
  d_col = col2;
  d_val64 = val2;
  A.rowptr = d_rowptr;
  A.col = d_col;
  A.val64 = d_val64;
  hrp.swap(nrp);
  return LG_OK;
}

// Marks every column outside this rank's rows [lo, hi) in a bitmap over the
// global index range.
__global__ void mark_remote_kernel(const int* __restrict__ col, long long nnz, int lo, int hi, int ncols,
                                   unsigned* bits) {
  for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < nnz;
       k += (long long)gridDim.x * blockDim.x) {
    const int c = col[k];
    if ((c >= lo && c < hi) || c < 0 || c >= ncols) continue;
    const unsigned m = 1u << (c & 31);
    if (!(__ldcg(bits + (c >> 5)) & m)) atomicOr(bits + (c >> 5), m);
  }
}

__global__ void halo_pack_kernel(const double* __restrict__ full, const int* __restrict__ idx, long long cnt,
                                 double* __restrict__ out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < cnt; i += (long long)gridDim.x * blockDim.x)
    out[i] = full[idx[i]];
}

__global__ void halo_unpack_kernel(const double* __restrict__ in, const int* __restrict__ pos, long long cnt,
                                   double* __restrict__ full) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < cnt; i += (long long)gridDim.x * blockDim.x)
    full[pos[i]] = in[i];
}

// Halo lists of a partitioned plan (collective: every rank calls it once, at
// creation; the host steps are lg_halo.cu's halo_recv_lists / halo_send_plan).  The columns of this rank's rows that other ranks own, grouped by
// owner in ascending order, are the rows it receives; one all-reduce of the
// ranks x ranks count matrix tells every rank what it sends to whom, and one
// grouped exchange hands each owner the positions it must pack.  Halo mode is
// chosen (identically on every rank, from the all-reduced counts) when every
// rank receives at most half of the rows an all-gather would bring.
int Solver::setup_halo() {
  const long long total = (long long)ld * nranks;
  const size_t words = (size_t)((total + 31) / 32);
  unsigned* d_bits = nullptr;
  LG_TRY(cudaMalloc(&d_bits, sizeof(unsigned) * words));
  cudaError_t e = cudaMemsetAsync(d_bits, 0, sizeof(unsigned) * words, stream);
  if (e == cudaSuccess && nnz > 0) {
    mark_remote_kernel<<<num_sm * 4, 256, 0, stream>>>(d_col, nnz, row0, row0 + n, n_global, d_bits);
    e = cudaGetLastError();
  }
  std::vector<unsigned> bits(words);
  if (e == cudaSuccess) e = cudaMemcpyAsync(bits.data(), d_bits, sizeof(unsigned) * words, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  cudaFree(d_bits);
  LG_TRY(e);

  std::vector<int> pos;
  halo_recv_lists(bits.data(), ld, nranks, rank, n_global, pos, recv_off, recv_cnt);
  halo_recv = (long long)pos.size();

  // count matrix: row r = the rows rank r receives from each rank
  const size_t nn = (size_t)nranks * nranks;
  std::vector<double> cnt(nn, 0.0);
  for (int o = 0; o < nranks; ++o) cnt[(size_t)rank * nranks + o] = (double)recv_cnt[o];
  double* d_cnt = nullptr;
  LG_TRY(cudaMalloc(&d_cnt, sizeof(double) * nn));
  e = cudaMemcpyAsync(d_cnt, cnt.data(), sizeof(double) * nn, cudaMemcpyHostToDevice, stream);
  int rc = LG_OK;
  if (e == cudaSuccess) rc = comm_allreduce_sum(comm, d_cnt, nn, stream);
  if (e == cudaSuccess && rc == LG_OK)
    e = cudaMemcpyAsync(cnt.data(), d_cnt, sizeof(double) * nn, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess && rc == LG_OK) e = cudaStreamSynchronize(stream);
  cudaFree(d_cnt);
  if (rc != LG_OK) return rc;
  LG_TRY(e);
  exchange_auto = halo_send_plan(cnt.data(), nranks, rank, ld, send_off, send_cnt, &halo_send);
  exchange = exchange_auto;

  LG_TRY(cudaMalloc(&d_recv_pos, sizeof(int) * (size_t)std::max<long long>(halo_recv, 1)));
  LG_TRY(cudaMalloc(&d_send_idx, sizeof(int) * (size_t)std::max<long long>(halo_send, 1)));
  LG_TRY(cudaMalloc(&d_recv_buf, sizeof(double) * (size_t)std::max<long long>(halo_recv, 1)));
  LG_TRY(cudaMalloc(&d_send_buf, sizeof(double) * (size_t)std::max<long long>(halo_send, 1)));
  if (halo_recv > 0)
    LG_TRY(cudaMemcpyAsync(d_recv_pos, pos.data(), sizeof(int) * (size_t)halo_recv, cudaMemcpyHostToDevice, stream));
  // my receive positions go to their owners, which keep them as send lists
  rc = comm_sendrecv(comm, 4, d_recv_pos, recv_off.data(), recv_cnt.data(), d_send_idx, send_off.data(),
                     send_cnt.data(), stream);
  if (rc != LG_OK) return rc;
  // Each send segment ascends (the readers scanned their bitmaps in order):
  // its last entry is the highest row of this block that the peer reads.
  // An all-gather then sends each peer only the rows up to that one (a graph
  // numbered by descending degree keeps its never-named rows at the end).
  ag_need.assign((size_t)nranks, 0);
  for (int q = 0; q < nranks; ++q)
    if (q != rank && send_cnt[q] > 0)
      LG_TRY(cudaMemcpyAsync(&ag_need[q], d_send_idx + send_off[q] + send_cnt[q] - 1, sizeof(int),
                             cudaMemcpyDeviceToHost, stream));
  LG_TRY(cudaStreamSynchronize(stream));   // pos goes out of scope, ag_need has arrived
  for (int q = 0; q < nranks; ++q) ag_need[q] = (q != rank && send_cnt[q] > 0) ? ag_need[q] - row0 + 1 : 0;
  return LG_OK;
}

int Solver::set_exchange(int mode) {
  if (!comm) {
    g_last_error = "set_exchange: not a partitioned plan";
    return LG_ERR_INVALID;
  }
  if (mode == LG_EXCHANGE_AUTO) exchange = exchange_auto;
  else if (mode == LG_EXCHANGE_ALLGATHER || mode == LG_EXCHANGE_HALO) exchange = mode;
  else {
    g_last_error = "set_exchange: mode must be LG_EXCHANGE_AUTO, _ALLGATHER or _HALO";
    return LG_ERR_INVALID;
  }
  return LG_OK;
}

int Solver::exchange_info(int* mode, long long* recv_rows, long long* send_rows) const {
  if (!comm) {
    g_last_error = "exchange_info: not a partitioned plan";
    return LG_ERR_INVALID;
  }
  if (mode) *mode = exchange;
  if (recv_rows) *recv_rows = halo_recv;
  if (send_rows) *send_rows = halo_send;
  return LG_OK;
}

// Tables of the rows longer than kLongRow (see CsrDev): row index, range of
// chunks, chunk bounds; nothing is allocated for graphs without such rows.
int Solver::build_long_rows(const int* hrp) {
  std::vector<int> rows, first{0}, cb, ce;
  for (int i = 0; i < n; ++i) {
    const int b = hrp[i], e = hrp[i + 1];
    if (e - b <= kLongRow) continue;
    rows.push_back(i);
    for (int k = b + kLongRow; k < e; k += kLongRow) {
      cb.push_back(k);
      ce.push_back(std::min(e, k + kLongRow));
    }
    first.push_back((int)cb.size());
  }
  // Row-length classes: when no single lane count suits 90 % of the rows
  // (power-law graphs), each class gets its own launch over its row list.
  {
    static const int kLanes[5] = {2, 4, 8, 16, 32};
    // class of a row: the index of pick_lanes(len) in kLanes (len < 3, < 8,
    // < 16, < 32, else), one byte per row
    std::vector<unsigned char> cls((size_t)n);
    int hist[5] = {0, 0, 0, 0, 0};
    for (int i = 0; i < n; ++i) {
      const int len = hrp[i + 1] - hrp[i];
      const int c = len < 3 ? 0 : len < 8 ? 1 : len < 16 ? 2 : len < 32 ? 3 : 4;
      cls[(size_t)i] = (unsigned char)c;
      ++hist[c];
    }
    const int top = *std::max_element(hist, hist + 5);
    if ((double)top < 0.9 * n) {
      std::vector<int> lists;
      lists.reserve(n);
      int off[5];
      A.nclasses = 0;
      for (int c = 0; c < 5; ++c) {
        off[c] = (int)lists.size();
        for (int i = 0; i < n; ++i)
          if (cls[i] == c) lists.push_back(i);
        if (hist[c] > 0) {
          A.class_lanes[A.nclasses] = kLanes[c];
          A.class_count[A.nclasses] = hist[c];
          A.class_rows[A.nclasses] = reinterpret_cast<const int*>((size_t)off[c]);   // offset, fixed below
          ++A.nclasses;
        }
      }
      LG_TRY(dalloc((void**)&d_classes, sizeof(int) * (size_t)n));
      LG_TRY(cudaMemcpyAsync(d_classes, lists.data(), sizeof(int) * (size_t)n, cudaMemcpyHostToDevice, stream));
      LG_TRY(cudaStreamSynchronize(stream));
      for (int c = 0; c < A.nclasses; ++c)
        A.class_rows[c] = d_classes + reinterpret_cast<size_t>(A.class_rows[c]);
    }
  }
  A.nlong = (int)rows.size();
  A.nchunks = (int)cb.size();
  if (A.nlong == 0) return LG_OK;
  const size_t total = rows.size() + first.size() + cb.size() + ce.size();
  LG_TRY(dalloc((void**)&d_long, sizeof(int) * total));
  LG_TRY(dalloc((void**)&d_chunk_sum, sizeof(double) * cb.size()));
  int* p = d_long;
  for (const std::vector<int>* v : {&rows, &first, &cb, &ce}) {
    LG_TRY(cudaMemcpyAsync(p, v->data(), sizeof(int) * v->size(), cudaMemcpyHostToDevice, stream));
    p += v->size();
  }
  LG_TRY(cudaStreamSynchronize(stream));   // the host vectors go out of scope
  A.long_rows = d_long;
  A.long_first = d_long + rows.size();
  A.chunk_begin = A.long_first + first.size();
  A.chunk_end = A.chunk_begin + cb.size();
  A.chunk_sum = d_chunk_sum;
  return LG_OK;
}

// Fixed-order sum of `nrows` partial rows into one row (one thread per entry).
__global__ void sum_rows_kernel(const double* __restrict__ part, int nrows, double* __restrict__ out) {
  for (int i = threadIdx.x; i < kPartStride; i += blockDim.x) {
    double s = 0.0;
    for (int r = 0; r < nrows; ++r) s += part[(size_t)r * kPartStride + i];
    out[i] = s;
  }
}

int Solver::reduce_partials_all(double* part, int nrows, int slot, const double** in, int* nin) {
  if (!comm) {
    *in = part;
    *nin = nrows;
    return LG_OK;
  }
  double* row = red + (size_t)slot * kPartStride;
  if (transport == LG_TRANSPORT_PEER) {
    int rc = peer_reduce(part, nullptr, nrows, 1, slot);
    if (rc != LG_OK) return rc;
    *in = row;
    *nin = 1;
    return LG_OK;
  }
  sum_rows_kernel<<<1, 160, 0, stream>>>(part, nrows, row);
  LG_TRY(cudaGetLastError());
  launches += 2;
  int rc = comm_allreduce_sum(comm, row, kPartStride, stream);
  if (rc != LG_OK) return rc;
  *in = row;
  *nin = 1;
  return LG_OK;
}

int Solver::reduce_partials_all2(double* pa, double* pb, int nrows, int slot, const double** ina,
                                 const double** inb, int* nin) {
  if (comm && transport == LG_TRANSPORT_PEER) {
    int rc = peer_reduce(pa, pb, nrows, 2, slot);
    if (rc != LG_OK) return rc;
    *ina = red + (size_t)slot * kPartStride;
    *inb = red + (size_t)(slot + 1) * kPartStride;
    *nin = 1;
    return LG_OK;
  }
  int na = 0, nb = 0;
  int rc = reduce_partials_all(pa, nrows, slot, ina, &na);
  if (rc != LG_OK) return rc;
  rc = reduce_partials_all(pb, nrows, slot + 1, inb, &nb);
  *nin = na;
  return rc;
}

// Before a sparse product: the other ranks' residual rows that this rank's
// columns name into Rfull, by the halo exchange (pack the rows others read,
// grouped sends and receives, unpack at their global positions) or by an
// in-place all-gather of every block.
int Solver::gather_residual() {
  if (!comm) return LG_OK;
  if (transport == LG_TRANSPORT_PEER) return peer_exchange();
  if (exchange == LG_EXCHANGE_HALO) {
    if (halo_send > 0) {
      const int g = (int)std::min<long long>((long long)num_sm * 4, (halo_send + 255) / 256);
      halo_pack_kernel<<<g, 256, 0, stream>>>(Rfull, d_send_idx, halo_send, d_send_buf);
      LG_TRY(cudaGetLastError());
      ++launches;
    }
    int rc = comm_sendrecv(comm, 8, d_send_buf, send_off.data(), send_cnt.data(), d_recv_buf, recv_off.data(),
                           recv_cnt.data(), stream);
    if (rc != LG_OK) return rc;
    ++launches;
    if (halo_recv > 0) {
      const int g = (int)std::min<long long>((long long)num_sm * 4, (halo_recv + 255) / 256);
      halo_unpack_kernel<<<g, 256, 0, stream>>>(d_recv_buf, d_recv_pos, halo_recv, Rfull);
      LG_TRY(cudaGetLastError());
      ++launches;
    }
    return LG_OK;
  }
  ++launches;
  return comm_allgather_inplace(comm, Rfull, (size_t)ld, stream);
}

int Solver::sync_state() {
  LG_TRY(cudaMemcpyAsync(h_state, state, sizeof(int) * ST_WORDS, cudaMemcpyDeviceToHost, stream));
  LG_TRY(cudaStreamSynchronize(stream));
  return LG_OK;
}

int Solver::clear_status() {
  LG_TRY(cudaMemsetAsync(state, 0, sizeof(int) * 2, stream));
  return LG_OK;
}

// w = OP(v_j) preceded by the normalisation of R into V[:, j].
int Solver::apply_step(int j, int beta_mode) {
  if (op_kind >= 0) return apply_user_op(j, beta_mode);
  double* Vj = V + vidx(vl, 0, j);   // column j of the basis
  if (!opts.use_sigma) {
    // CSR stream + x gather (counted once) + v_j and w written
    const double vb = mixed ? 4.0 : 8.0;
    const double bytes = (4.0 + vb) * (double)nnz + 4.0 * (n + 1) + 8.0 * n + 16.0 * n;
    int rc = gather_residual();
    if (rc != LG_OK) return rc;
    const double* Rg = comm ? Rfull : R;
    LG_TRY(timed(LG_K_SPMV, bytes, (A.nclasses > 0 ? A.nclasses : 1) + (A.nlong ? 2 : 0), [&] {
      return spmv_step(A, stream, grid_spmv, Rg, W, Vj, (int)vl.rs, inC, nrowsC, j, beta_mode, alpha, beta, scal, state,
                       R);
    }));
    return LG_OK;
  }
  return apply_shift_invert(j, beta_mode);
}

int Solver::extend(int j0, int j1, int first_mode, bool lag) {
  bool last_lag = false;
  deferred_norm_rows = 0;
  for (int j = j0; j < j1; ++j) {
    // a lag step needs a previous column and a residual whose coupling is
    // its norm (not after a fresh start, an explicit third pass or a random
    // restart, whose first step keeps the in-step passes and their checks)
    if (lag && j > 0 && (j > j0 || first_mode == BETA_RESTART)) {
      // on the peer transport the norm of this step's residual is reduced
      // by the next lag step's exchange (every step but the last)
      const bool defer = comm && transport == LG_TRANSPORT_PEER && j + 1 < j1;
      int rc = lag_step(j, defer);
      if (rc != LG_OK) return rc;
      last_lag = true;
      continue;
    }
    last_lag = false;
    int rc = apply_step(j, j == j0 ? first_mode : BETA_STEP);
    if (rc != LG_OK) return rc;
    const int ncols = j + 1;
    const GsPlan p = gs_plan(n, ncols, grid_gs);
    const double vbytes = 8.0 * (double)n * ncols;
    const double *inA = nullptr, *inB = nullptr;
    int nA = 0, nB = 0;
    LG_TRY(timed(LG_K_PROJECT, vbytes + 8.0 * n, 1,
                 [&] { return gs_project(p, stream, V, vl, ncols, n, W, partA, state); }));
    rc = reduce_partials_all(partA, p.grid, 0, &inA, &nA);
    if (rc != LG_OK) return rc;
    LG_TRY(timed(LG_K_CORRPROJ, vbytes + 16.0 * n, 1, [&] {
      return gs_correct_project(p, stream, V, vl, ncols, n, W, R, inA, nA, partB, scal, state);
    }));
    rc = reduce_partials_all(partB, p.grid, 1, &inB, &nB);
    if (rc != LG_OK) return rc;
    LG_TRY(timed(LG_K_CORRECT, vbytes + 16.0 * n, 1, [&] {
      return gs_correct(p, stream, V, vl, ncols, n, R, inB, nB, partC, scal, alpha, j, 1, state);
    }));
    rc = reduce_partials_all(partC, p.grid, 2, &inC, &nrowsC);
    if (rc != LG_OK) return rc;
  }
  if (last_lag) return finish_lag(j1 - 1);
  return LG_OK;
}

// Lag step j: z = A u / ||u|| from the once-orthogonalised residual u of step
// j-1, then one stream of V for s = V^T u and t = V^T z, and one that
// finishes v_j = (u - V s) / beta_j and forms the next once-orthogonalised
// residual (lg_gs.cu, gs_lag_project / gs_lag_correct).
int Solver::lag_step(int j, bool defer_norm) {
  const double vb = mixed ? 4.0 : 8.0;
  const double sbytes = (4.0 + vb) * (double)nnz + 4.0 * (n + 1) + 8.0 * n + 8.0 * n;
  int rc = LG_OK;
  if (deferred_norm_rows > 0) {
    // the previous step's ||R||^2 partial rows, reduced by the exchange
    rc = peer_exchange(partC, deferred_norm_rows, 2);
    inC = red + (size_t)2 * kPartStride;
    nrowsC = 1;
    deferred_norm_rows = 0;
  } else {
    rc = gather_residual();
  }
  if (rc != LG_OK) return rc;
  const double* Rg = comm ? Rfull : R;
  LG_TRY(timed(LG_K_SPMV, sbytes, (A.nclasses > 0 ? A.nclasses : 1) + (A.nlong ? 2 : 0), [&] {
    return spmv_step(A, stream, grid_spmv, Rg, W, nullptr, (int)vl.rs, inC, nrowsC, j, BETA_LAG, alpha, beta, scal, state,
                     R);
  }));
  const GsPlan p = gs_plan(n, j, grid_gs);
  const double vbytes = 8.0 * (double)n * j;
  LG_TRY(timed(LG_K_PROJECT, vbytes + 16.0 * n, 1,
               [&] { return gs_lag_project(p, stream, V, vl, j, n, R, W, partA, partB, state); }));
  const double *inS = nullptr, *inT = nullptr;
  int nS = 0;
  rc = reduce_partials_all2(partA, partB, gs_lag_rows(p), 0, &inS, &inT, &nS);
  if (rc != LG_OK) return rc;
  LG_TRY(timed(LG_K_CORRPROJ, vbytes + 32.0 * n, 1, [&] {
    return gs_lag_correct(p, stream, V, vl, j, n, R, W, inS, inT, nS, partC, scal, alpha, beta, state);
  }));
  if (defer_norm) {
    deferred_norm_rows = p.grid;
    inC = partC;
    nrowsC = p.grid;
    return LG_OK;
  }
  return reduce_partials_all(partC, p.grid, 2, &inC, &nrowsC);
}

// The delayed second pass of the last residual of an extension (step s):
// R -= V[:, 0..s] (V^T R), alpha_s += its coefficient, ||R||^2 partials for
// the restart (whose DGKS / breakdown tests then read them).
int Solver::finish_lag(int s) {
  const int ncols = s + 1;
  const GsPlan p = gs_plan(n, ncols, grid_gs);
  const double vbytes = 8.0 * (double)n * ncols;
  const double* inA = nullptr;
  int nA = 0;
  LG_TRY(timed(LG_K_PROJECT, vbytes + 8.0 * n, 1,
               [&] { return gs_project(p, stream, V, vl, ncols, n, R, partA, state); }));
  int rc = reduce_partials_all(partA, p.grid, 0, &inA, &nA);
  if (rc != LG_OK) return rc;
  LG_TRY(timed(LG_K_CORRECT, vbytes + 16.0 * n, 1, [&] {
    return gs_correct(p, stream, V, vl, ncols, n, R, inA, nA, partC, scal, alpha, s, 2, state);
  }));
  return reduce_partials_all(partC, p.grid, 2, &inC, &nrowsC);
}

cudaEvent_t Solver::next_event() {
  if (ev_used == ev_pool.size()) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    ev_pool.push_back(e);
  }
  return ev_pool[ev_used++];
}

void Solver::collect_profile(lg_eigsh_info* info) {
  for (const KTime& kt : ktimes) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, kt.a, kt.b) == cudaSuccess && kt.cls >= 0 && kt.cls < LG_K_CLASSES) {
      info->kernel_ms[kt.cls] += ms;
      info->kernel_calls[kt.cls] += 1;
      info->kernel_bytes[kt.cls] += kt.bytes;
    }
  }
  ktimes.clear();
  ev_used = 0;
}

// Third DGKS pass on the residual of step s (reference: the second
// refinement pass of dgks_reorth, src/lanczos_ops.cuh:158-191).
int Solver::pass3(int s) {
  const int ncols = s + 1;
  const GsPlan p = gs_plan(n, ncols, grid_gs);
  launches += 2;
  const double* inA = nullptr;
  int nA = 0;
  LG_TRY(gs_project(p, stream, V, vl, ncols, n, R, partA, state));
  int rc = reduce_partials_all(partA, p.grid, 0, &inA, &nA);
  if (rc != LG_OK) return rc;
  LG_TRY(gs_correct(p, stream, V, vl, ncols, n, R, inA, nA, partC, scal, alpha, s, 2, state));
  return reduce_partials_all(partC, p.grid, 2, &inC, &nrowsC);
}

// Invariant subspace after step s: a random vector made orthogonal to
// V[:, 0..s] by two Gram-Schmidt passes (reference: inject_random_restart,
// src/lanczos_ops.cuh:229-253; ARPACK dgetv0).  The coupling beta_{s+1} is
// set to zero (as ARPACK does), so T decouples.
int Solver::random_restart(int s) {
  const int ncols = s + 1;
  ++breakdowns;
  LG_TRY(fill_random(stream, R, n, ld, mix64(opts.seed + 0x5bd1e995ull * (uint64_t)(breakdowns + 1) + (uint64_t)s),
                     row0));
  const GsPlan p = gs_plan(n, ncols, grid_gs);
  launches += 5;
  for (int pass = 0; pass < 2; ++pass) {
    const double* inA = nullptr;
    int nA = 0;
    LG_TRY(gs_project(p, stream, V, vl, ncols, n, R, partA, state));
    int rc = reduce_partials_all(partA, p.grid, 0, &inA, &nA);
    if (rc != LG_OK) return rc;
    LG_TRY(gs_correct(p, stream, V, vl, ncols, n, R, inA, nA, partC, scal, alpha, s, 0, state));
    rc = reduce_partials_all(partC, p.grid, 2, &inC, &nrowsC);
    if (rc != LG_OK) return rc;
  }
  return LG_OK;
}

int Solver::run(const lg_eigsh_opts& o, const double* v0, double* evals, double* evecs, int io_on_device,
                lg_eigsh_info* info) {
  opts = o;
  const int k = o.k;
  if (k < 1 || k >= n) {
    g_last_error = "k must satisfy 1 <= k < n";
    return LG_ERR_INVALID;
  }
  int m = o.ncv > 0 ? o.ncv : std::min(n, std::max(2 * k + 1, 20));
  if (m > n) m = n;
  if (m <= k || m > max_ncv) {
    char buf[160];
    snprintf(buf, sizeof(buf), "ncv must satisfy k < ncv <= min(n, %d); got ncv=%d k=%d", max_ncv, m, k);
    g_last_error = buf;
    return LG_ERR_INVALID;
  }
  if (o.which < 0 || o.which > 4) {
    g_last_error = "unknown which";
    return LG_ERR_INVALID;
  }
  const int maxiter = o.maxiter > 0 ? o.maxiter : (n > 214748364 ? 2147483647 : 10 * n);
  breakdowns = 0;
  int pass3_count = 0;
  cg_iters = 0;
  cg_failures = 0;
  skip_checks_next = 0;
  launches = 0;
  ktimes.clear();
  ev_used = 0;

  if (comm && o.use_sigma) {
    g_last_error = "shift-invert is not available with a row-partitioned plan";
    return LG_ERR_INVALID;
  }
  if (op_kind >= 0 && o.use_sigma) {
    g_last_error = "shift-invert needs a CSR plan (its inner CG multiplies by the matrix)";
    return LG_ERR_INVALID;
  }
  if (o.use_sigma) {
    int rc = prepare_shift_invert();
    if (rc != LG_OK) return rc;
  }

  LG_TRY(cudaEventRecord(ev0, stream));
  LG_TRY(cudaMemsetAsync(state, 0, sizeof(int) * ST_WORDS, stream));
  LG_TRY(cudaMemsetAsync(scal, 0, sizeof(double) * SC_WORDS, stream));
  LG_TRY(cudaMemsetAsync(alpha, 0, sizeof(double) * (kMaxCols + 2), stream));
  LG_TRY(cudaMemsetAsync(beta, 0, sizeof(double) * (kMaxCols + 2), stream));
  LG_TRY(cudaMemsetAsync(V, 0, sizeof(double) * vsize(), stream));

  // Starting vector into R.
  if (v0) {
    LG_TRY(cudaMemsetAsync(R, 0, sizeof(double) * (size_t)ld, stream));
    const cudaMemcpyKind kind = io_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    if (d_perm) {   // caller's numbering -> the plan's
      LG_TRY(cudaMemcpyAsync(W, v0, sizeof(double) * (size_t)n, kind, stream));
      gather_perm_kernel<<<num_sm * 4, 256, 0, stream>>>(R, W, d_perm, n);
      LG_TRY(cudaGetLastError());
      ++launches;
    } else {
      LG_TRY(cudaMemcpyAsync(R, v0, sizeof(double) * (size_t)n, kind, stream));
    }
  } else {
    LG_TRY(fill_random(stream, R, n, ld, o.seed, row0));
    ++launches;
  }
  LG_TRY(norm_partials(stream, grid_gs, R, ld, partC));
  ++launches;
  {
    int rc0 = reduce_partials_all(partC, grid_gs, 2, &inC, &nrowsC);
    if (rc0 != LG_OK) return rc0;
  }

  long long steps = 0;
  const bool lag = lag_steps && !o.use_sigma;
  int rc = extend(0, m, BETA_INIT, lag);
  if (rc != LG_OK) return rc;
  steps += m;

  int iter = 1;
  int last_pass3_step = -1;
  for (;;) {
    RestartArgs ra;
    ra.m = m;
    ra.nev0 = k;
    ra.which = o.which;
    ra.tol = o.tol;
    ra.iter = iter;
    ra.maxiter = maxiter;
    ra.force_done = (o.max_steps > 0 && steps >= o.max_steps) ? 1 : 0;
    ra.skip_checks = skip_checks_next;
    skip_checks_next = 0;
    ra.part_in = inC;
    ra.nrows_in = nrowsC;
    ra.alpha = alpha;
    ra.beta = beta;
    ra.scal = scal;
    ra.ritz_out = ritz;
    ra.bounds_out = bounds;
    ra.conv_out = conv;
    ra.zsel = zsel;
    ra.Q = Q;
    ra.scratch = rs_scratch;
    ra.state = state;
    LG_TRY(timed(LG_K_RESTART, 0.0, 1, [&] { return restart_step(ra, stream); }));
    rc = sync_state();
    if (rc != LG_OK) return rc;

    const int status = h_state[ST_STATUS];
    if (status == STATUS_TIMEOUT) {
      g_last_error = "bounded device wait timed out";
      return LG_ERR_TIMEOUT;
    }
    if (status == STATUS_TRIDIAG_FAIL) {
      g_last_error = "tridiagonal QR iteration did not converge (non-finite values?)";
      return LG_ERR_NUMERIC;
    }
    if (status == STATUS_PASS3 || status == STATUS_BREAKDOWN || status == STATUS_PASS3_LAG) {
      const int s = h_state[ST_STEP];
      if (s < 0 || s >= m) {
        g_last_error = "internal: bad step index in device state";
        return LG_ERR_NUMERIC;
      }
      rc = clear_status();
      if (rc != LG_OK) return rc;
      int next_mode = BETA_STEP;
      if (status == STATUS_PASS3_LAG) {
        // the delayed second pass of step s, applied, then the third pass
        rc = pass3(s);
        if (rc == LG_OK) rc = pass3(s);
        ++pass3_count;
        last_pass3_step = s;
      } else if (status == STATUS_PASS3 && s != last_pass3_step) {
        rc = pass3(s);
        ++pass3_count;
        last_pass3_step = s;
      } else {
        // breakdown, or a third pass that did not restore the norm
        rc = random_restart(s);
        next_mode = BETA_ZERO;
        last_pass3_step = -1;
      }
      if (rc != LG_OK) return rc;
      if (s + 1 < m) {
        rc = extend(s + 1, m, next_mode, lag);
        if (rc != LG_OK) return rc;
        steps += m - (s + 1);
      } else if (next_mode == BETA_ZERO) {
        // invariant subspace at the last step: the residual is exactly zero
        LG_TRY(cudaMemsetAsync(R, 0, sizeof(double) * (size_t)ld, stream));
        LG_TRY(norm_partials(stream, grid_gs, R, ld, partC));
        ++launches;
        rc = reduce_partials_all(partC, grid_gs, 2, &inC, &nrowsC);
        if (rc != LG_OK) return rc;
        skip_checks_next = 1;
      }
      continue;  // re-run the Ritz computation for this restart
    }
    last_pass3_step = -1;

    if (h_state[ST_DONE]) break;
    const int nev_use = h_state[ST_NEV_USE];
    if (nev_use < 1 || nev_use >= m) {
      g_last_error = "internal: bad nev in device state";
      return LG_ERR_NUMERIC;
    }
    BasisArgs ba;
    ba.V = V;
    ba.vl = vl;
    ba.n = n;
    ba.m = m;
    ba.kq = nev_use + 1;
    ba.Q = Q;
    ba.ldq = m;
    ba.restart = 1;
    ba.R = R;
    ba.scal = scal;
    ba.part_out = partC;
    ba.state = state;
    const BasisPlan bp = basis_plan(n, m, ba.kq, grid_basis);
    LG_TRY(timed(LG_K_BASIS, 8.0 * n * (m + nev_use) + 16.0 * n, 1, [&] { return basis_update(bp, ba, stream); }));
    rc = reduce_partials_all(partC, bp.grid, 2, &inC, &nrowsC);
    if (rc != LG_OK) return rc;
    rc = extend(nev_use, m, BETA_RESTART, lag);
    if (rc != LG_OK) return rc;
    steps += m - nev_use;
    ++iter;
  }

  const int ksel = h_state[ST_KSEL];
  const int nconv = h_state[ST_NCONV];
  std::vector<double> hr(ksel);
  std::vector<int> hconv(ksel);
  LG_TRY(cudaMemcpyAsync(hr.data(), ritz, sizeof(double) * ksel, cudaMemcpyDeviceToHost, stream));
  LG_TRY(cudaMemcpyAsync(hconv.data(), conv, sizeof(int) * ksel, cudaMemcpyDeviceToHost, stream));
  LG_TRY(cudaStreamSynchronize(stream));

  // Final eigenvalues, ascending.  Shift-invert: lambda = sigma + 1/mu
  // (reference _cuda_eigsh.cu:121-152), which reorders the pairs.
  std::vector<double> lam(ksel);
  std::vector<int> order(ksel);
  for (int i = 0; i < ksel; ++i) {
    order[i] = i;
    lam[i] = hr[i];
    if (o.use_sigma) lam[i] = (fabs(hr[i]) > kSafeMin) ? o.sigma + 1.0 / hr[i] : o.sigma;
  }
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return lam[a] < lam[b]; });
  bool identity = true;
  for (int i = 0; i < ksel; ++i) identity = identity && order[i] == i;
  if (!identity && o.return_vectors && evecs) {
    std::vector<double> zs((size_t)m * ksel), zp((size_t)m * ksel);
    LG_TRY(cudaMemcpyAsync(zs.data(), zsel, sizeof(double) * zs.size(), cudaMemcpyDeviceToHost, stream));
    LG_TRY(cudaStreamSynchronize(stream));
    for (int c = 0; c < ksel; ++c)
      std::copy(zs.begin() + (size_t)order[c] * m, zs.begin() + (size_t)(order[c] + 1) * m, zp.begin() + (size_t)c * m);
    LG_TRY(cudaMemcpyAsync(zsel, zp.data(), sizeof(double) * zp.size(), cudaMemcpyHostToDevice, stream));
  }

  if (o.return_vectors && evecs) {
    double* Y = evecs;
    if (!io_on_device) {
      if (!Ytmp || ytmp_elems < (size_t)n * ksel) {
        if (Ytmp) dfree(Ytmp);
        Ytmp = nullptr;
        LG_TRY(dalloc((void**)&Ytmp, sizeof(double) * (size_t)n * ksel));
        ytmp_elems = (size_t)n * ksel;
      }
      Y = Ytmp;
    }
    BasisArgs ba;
    ba.V = V;
    ba.vl = vl;
    ba.n = n;
    ba.m = m;
    ba.kq = ksel;
    ba.Q = zsel;
    ba.ldq = m;
    ba.restart = 0;
    ba.Y = Y;
    ba.ldy = n;
    ba.rowmajor = o.evecs_rowmajor;
    ba.ymap = d_perm;   // rows back in the caller's numbering
    ba.state = state;
    const BasisPlan bp = basis_plan(n, m, ksel, grid_basis);
    LG_TRY(timed(LG_K_BASIS, 8.0 * n * (m + ksel), 1, [&] { return basis_update(bp, ba, stream); }));
    if (!io_on_device) LG_TRY(staged_d2h(evecs, Ytmp, sizeof(double) * (size_t)n * ksel, stream));
  }
  LG_TRY(cudaEventRecord(ev1, stream));
  LG_TRY(cudaStreamSynchronize(stream));
  rc = sync_state();
  if (rc != LG_OK) return rc;
  if (h_state[ST_STATUS] == STATUS_TIMEOUT) {
    g_last_error = "bounded device wait timed out";
    return LG_ERR_TIMEOUT;
  }
  for (int i = 0; i < ksel; ++i) evals[i] = lam[order[i]];

  float ms = 0.f;
  cudaEventElapsedTime(&ms, ev0, ev1);
  if (info) {
    info->nconv = nconv;
    info->restarts = iter - 1;
    info->steps = steps;
    info->pass3 = pass3_count;
    info->breakdowns = breakdowns;
    info->cg_iters = cg_iters;
    info->cg_failures = cg_failures;
    info->ms = ms;
    info->launches = launches;
    for (int c = 0; c < LG_K_CLASSES; ++c) {
      info->kernel_ms[c] = 0.0;
      info->kernel_calls[c] = 0;
      info->kernel_bytes[c] = 0.0;
    }
    collect_profile(info);
  }
  ktimes.clear();
  ev_used = 0;
  for (int i = 0; i < ksel; ++i)
    if (!std::isfinite(hr[i])) {
      g_last_error = "non-finite Ritz value";
      return LG_ERR_NUMERIC;
    }
  if (o.use_sigma && cg_failures > 0) {
    char buf[200];
    snprintf(buf, sizeof(buf), "%d inner CG solves stopped before cg_tol (cg_max_iters=%d)", cg_failures,
             o.cg_max_iters);
    g_last_error = buf;
    return LG_ERR_CG_NOCONV;
  }
  return nconv >= k ? LG_OK : LG_NOCONV;
}

// m Lanczos steps from v0 (host vector) without restarts; returns the
// tridiagonal (alpha[0..m), beta[0..m], beta[m] = final residual norm).
int Solver::factorize(const double* v0, int m, double* alpha_out, double* beta_out) {
  if (comm) {
    g_last_error = "factorize is not available with a row-partitioned plan";
    return LG_ERR_INVALID;
  }
  if (m < 1 || m > max_ncv || m > n || !v0) {
    g_last_error = "factorize: need 1 <= m <= min(n, max_ncv) and a starting vector";
    return LG_ERR_INVALID;
  }
  lg_eigsh_opts o;
  std::memset(&o, 0, sizeof(o));
  opts = o;
  LG_TRY(cudaMemsetAsync(state, 0, sizeof(int) * ST_WORDS, stream));
  LG_TRY(cudaMemsetAsync(scal, 0, sizeof(double) * SC_WORDS, stream));
  LG_TRY(cudaMemsetAsync(alpha, 0, sizeof(double) * (kMaxCols + 2), stream));
  LG_TRY(cudaMemsetAsync(beta, 0, sizeof(double) * (kMaxCols + 2), stream));
  LG_TRY(cudaMemsetAsync(V, 0, sizeof(double) * vsize(), stream));
  LG_TRY(cudaMemsetAsync(R, 0, sizeof(double) * (size_t)ld, stream));
  if (d_perm) {
    LG_TRY(cudaMemcpyAsync(W, v0, sizeof(double) * (size_t)n, cudaMemcpyHostToDevice, stream));
    gather_perm_kernel<<<num_sm * 4, 256, 0, stream>>>(R, W, d_perm, n);
    LG_TRY(cudaGetLastError());
  } else {
    LG_TRY(cudaMemcpyAsync(R, v0, sizeof(double) * (size_t)n, cudaMemcpyHostToDevice, stream));
  }
  LG_TRY(norm_partials(stream, grid_gs, R, ld, partC));
  nrowsC = grid_gs;
  inC = partC;
  int rc = extend(0, m, BETA_INIT);
  if (rc != LG_OK) return rc;
  std::vector<double> part((size_t)nrowsC * kPartStride);
  LG_TRY(cudaMemcpyAsync(alpha_out, alpha, sizeof(double) * m, cudaMemcpyDeviceToHost, stream));
  LG_TRY(cudaMemcpyAsync(beta_out, beta, sizeof(double) * m, cudaMemcpyDeviceToHost, stream));
  LG_TRY(cudaMemcpyAsync(part.data(), partC, sizeof(double) * part.size(), cudaMemcpyDeviceToHost, stream));
  rc = sync_state();
  if (rc != LG_OK) return rc;
  if (h_state[ST_STATUS] != STATUS_RUNNING) {
    g_last_error = "factorize: invariant subspace or DGKS third pass met (not handled in this entry point)";
    return LG_ERR_NUMERIC;
  }
  double s = 0.0;
  for (int r = 0; r < nrowsC; ++r) s += part[(size_t)r * kPartStride + kPartScalar];
  beta_out[m] = std::sqrt(s);
  return LG_OK;
}

int Solver::matvec(const double* x, double* y) {
  if (comm) {
    g_last_error = "matvec is not available with a row-partitioned plan";
    return LG_ERR_INVALID;
  }
  if (op_kind >= 0) {
    int rc = call_user_op(x, y);
    if (rc != LG_OK) return rc;
    LG_TRY(cudaStreamSynchronize(stream));
    return LG_OK;
  }
  if (d_perm) {   // y = A x in the caller's numbering: gather x, product, scatter y
    gather_perm_kernel<<<num_sm * 4, 256, 0, stream>>>(R, x, d_perm, n);
    LG_TRY(cudaGetLastError());
    LG_TRY(spmv_plain(A, stream, grid_spmv, R, W, 0.0));
    scatter_perm_kernel<<<num_sm * 4, 256, 0, stream>>>(y, W, d_perm, n);
    LG_TRY(cudaGetLastError());
  } else {
    LG_TRY(spmv_plain(A, stream, grid_spmv, x, y, 0.0));
  }
  LG_TRY(cudaStreamSynchronize(stream));
  return LG_OK;
}

}  // namespace lg
