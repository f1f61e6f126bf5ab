// lg_solver.h — host-side solver object behind the lg_eigsh_plan handle.
#pragma once

#include <cuda_runtime.h>
#include <string>
#include <unordered_set>
#include <vector>

#include "../../include/lanczos_b200.h"
#include "lg_comm.h"
#include "lg_kernels.cuh"

namespace lg {

extern thread_local std::string g_last_error;

// Peer-memory transport of partitioned plans (lg_peer.cu): every rank's
// exchange buffer (mailbox, then flag words) and residual buffer, as this
// rank addresses them (its own, or mapped with CUDA IPC).
constexpr int kMaxPeerRanks = 16;
struct PeerPtrs {
  double* mail[kMaxPeerRanks];
  unsigned long long* flags[kMaxPeerRanks];
  double* R[kMaxPeerRanks];
  // all-gather mode: rank q reads only the first ag_len[q] rows of this
  // rank's block (the last one its columns name, plus one; 0 for none)
  int ag_len[kMaxPeerRanks];
};

class Solver {
 public:
  ~Solver();
  int create(int n, long long nnz, const int* rowptr, const int* col, const double* vals, int device_ptrs,
             int max_ncv, int mixed, int flags);
  // Matrix-free plan: the operator is the caller's callback (LG_OP_DEVICE /
  // LG_OP_HOST: fn; LG_OP_STREAM: sfn), no CSR.  Shift-invert is not
  // available (its inner CG multiplies by the CSR).
  int create_op(int n, int kind, lg_matvec_fn fn, lg_matvec_stream_fn sfn, void* user, int max_ncv);
  // Row-partitioned solver: this rank's n_local rows of an n_global x n_global matrix.
  int create_dist(lg_comm* comm, int n_global, int n_local, long long nnz, const int* rowptr, const int* col,
                  const double* vals, int device_ptrs, int max_ncv, int mixed);
  int run(const lg_eigsh_opts& o, const double* v0, double* evals, double* evecs, int io_on_device,
          lg_eigsh_info* info);
  int matvec(const double* x, double* y);
  int factorize(const double* v0, int m, double* alpha_out, double* beta_out);
  // Partitioned runs: how the residual reaches the other ranks before each
  // sparse product (LG_EXCHANGE_*); the same mode on every rank.
  // m-step Lanczos quadrature of f(A) v (mode 1) or v^T f(A) v (mode 0), no
  // restart (lg_funm.cu); *m_actual: depth reached, or the reference's
  // negative status (-2 f undefined at a Ritz value, -3 zero v, -4 T failed)
  int funm(const double* v, int io_on_device, int m, int func, int mode, double* y, double* value, int* m_actual);
  int funm_debug(const double* v, int m, double* V_out, double* alpha_out, double* beta_out, int* m_actual);
  int set_exchange(int mode);
  // Partitioned runs: LG_TRANSPORT_* of the reductions and the exchange.
  int set_transport(int mode);
  int transport_mode() const { return transport; }
  int exchange_info(int* mode, long long* recv_rows, long long* send_rows) const;

 private:
  void release();
  cudaError_t dalloc(void** p, size_t bytes);
  void dfree(void* p);
  std::unordered_set<void*> pooled;   // buffers from the device pool
  int init_device();
  int alloc_workspace();
  int create_impl(int n_rows, int n_cols, long long nnz, const int* rowptr, const int* col, const double* vals,
                  int device_ptrs, int max_ncv, int mixed, int flags);
  int reorder_rows(std::vector<int>& host_rowptr, bool by_degree);
  // Partitioned runs: sum `nrows` partial-sum rows into row `slot` of `red`
  // and all-reduce it over the ranks; *in / *nin become that single row.
  // Single GPU: *in = part, *nin = nrows.
  int reduce_partials_all(double* part, int nrows, int slot, const double** in, int* nin);
  int gather_residual();
  int setup_halo();
  // peer transport (lg_peer.cu)
  int setup_peer();
  void release_peer();
  int peer_reduce(const double* partA, const double* partB, int nrows, int ntables, int slot);
  // The residual exchange; with `part`, also the all-reduce of its nrows
  // partial rows into row `slot` of `red` (one wait for both).
  int peer_exchange(const double* part = nullptr, int nrows = 0, int slot = 0);
  // reduce_partials_all of two tables of one producer (rows `slot` and
  // slot + 1 of red): one peer all-reduce, or two NCCL ones.
  int reduce_partials_all2(double* pa, double* pb, int nrows, int slot, const double** ina, const double** inb,
                           int* nin);
  int build_long_rows(const int* host_rowptr);
  int funm_factor(const double* v, int io_on_device, int m, int* m_actual, double* vnorm);
  int sync_state();
  int clear_status();
  int apply_step(int j, int beta_mode);
  // Matrix-free plans: normalise R into V[:, j] and op_x, then y = OP(op_x)
  // by the caller's callback.
  int apply_user_op(int j, int beta_mode);
  int call_user_op(const double* x, double* y);
  // Lanczos steps j0 .. j1-1.  lag: steps after the first take the second
  // Gram-Schmidt pass delayed into the next step (lag_step), and the last
  // residual gets that pass at the end (finish_lag).
  int extend(int j0, int j1, int first_mode, bool lag = false);
  // defer_norm: leave the ||R||^2 partial rows of the correction unreduced
  // (nrowsC = their count, inC = partC); the next lag step reduces them
  // together with its residual exchange (peer transport).
  int lag_step(int j, bool defer_norm = false);
  int deferred_norm_rows = 0;   // partial rows of partC awaiting the next lag step's exchange
  int finish_lag(int s);
  bool lag_steps = true;   // false: LG_PLAN_CGS2_INLINE (both passes inside every step)
  int pass3(int s);
  int random_restart(int s);
  // shift-invert (lg_cg.cu)
  int prepare_shift_invert();
  int apply_shift_invert(int j, int beta_mode);
  int cg_solve(const double* b, double* x);

  int n = 0, ld = 0, ldv = 0, max_ncv = 0, mixed = 0;   // ld: vector length padding; ldv: basis columns (a multiple of 8)
  VLayout vl;   // the basis in panels of 8 columns (lg_kernels.cuh): rs = 8, ps = 8 * round_up(n, 8)
  size_t vsize() const { return (size_t)vl.ps * (size_t)(ldv / 8); }   // doubles of the basis
  // matrix-free plans: LG_OP_* (-1: the plan owns a CSR), the callback and
  // its argument; op_x: the contiguous operand; host operators: pinned
  // copies of x and y
  int op_kind = -1;
  lg_matvec_fn op_fn = nullptr;
  lg_matvec_stream_fn op_sfn = nullptr;
  void* op_user = nullptr;
  double* op_x = nullptr;
  double* h_op_x = nullptr;
  double* h_op_y = nullptr;
  // row partition (comm set): this rank owns global rows [row0, row0 + n); the
  // residuals of all ranks live in Rfull (nranks blocks of ld = nb doubles)
  // and R is this rank's block, so global column indices address Rfull.
  lg_comm* comm = nullptr;
  int n_global = 0, row0 = 0, nranks = 1, rank = 0;
  double* Rfull = nullptr;
  double* red = nullptr;          // 3 x kPartStride: all-reduced partial rows
  const double* inC = nullptr;    // partial sums read by the next step / restart
  // Halo exchange: the residual rows of other ranks that this rank's sparse
  // product reads (recv, by global position in Rfull) and the rows of this
  // rank that others read (send, by global position); per-peer offsets and
  // counts in rows, host side.
  int exchange = LG_EXCHANGE_ALLGATHER, exchange_auto = LG_EXCHANGE_ALLGATHER;
  std::vector<long long> send_off, send_cnt, recv_off, recv_cnt;
  long long halo_send = 0, halo_recv = 0;
  int transport = LG_TRANSPORT_NCCL;
  bool peer_ok = false;
  unsigned long long peer_seq = 0;   // calls of the peer transport (the same sequence on every rank)
  long long peer_wait_cycles = 0;    // bound of every wait of the peer kernels
  void* peer_xch = nullptr;          // this rank's mailbox + flags (mapped by the peers)
  unsigned* peer_counter = nullptr;  // last-CTA counter of the exchange kernel
  long long* d_peer_send_off = nullptr;
  void* peer_open_mail[kMaxPeerRanks] = {};
  void* peer_open_R[kMaxPeerRanks] = {};
  PeerPtrs peer_ptrs{};
  int* d_send_idx = nullptr;
  std::vector<int> ag_need;   // per peer: leading rows of this block it reads (setup_halo)
  int* d_recv_pos = nullptr;
  double* d_send_buf = nullptr;
  double* d_recv_buf = nullptr;
  long long nnz = 0;
  int device = 0, num_sm = 0, grid_gs = 0, grid_spmv = 0, grid_basis = 0;
  size_t smem_budget = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;

  CsrDev A;
  int* d_rowptr = nullptr;
  int* d_col = nullptr;
  double* d_val64 = nullptr;
  float* d_val32 = nullptr;
  int* d_long = nullptr;          // long-row tables (rows, chunk ranges, chunk bounds)
  int* d_classes = nullptr;       // row lists of the row-length classes
  int* d_perm = nullptr;          // reordered plans: plan row -> caller row
  double* funm_ws = nullptr;      // funm small side: Z, inverse-iteration scratch, q, scalars
  double* d_chunk_sum = nullptr;  // one partial per long-row chunk

  double* V = nullptr;      // basis, ldv columns in panels of 8 (vl), ldv >= max_ncv + 1
  double* W = nullptr;      // operator output
  double* R = nullptr;      // residual (unnormalised next basis vector)
  double* partA = nullptr;  // partial sums: pass 1
  double* partB = nullptr;  // pass 2
  double* partC = nullptr;  // pass 3 / norms of R
  int nrowsC = 0;
  double* alpha = nullptr;
  double* beta = nullptr;
  double* scal = nullptr;
  double* ritz = nullptr;
  double* bounds = nullptr;
  double* zsel = nullptr;
  double* Q = nullptr;
  double* rs_scratch = nullptr;
  int* conv = nullptr;
  int* state = nullptr;
  int* h_state = nullptr;
  double* Ytmp = nullptr;
  size_t ytmp_elems = 0;

  // shift-invert CG workspace: x r pa pb Ap (ld each) + scalars
  double* cg_ws = nullptr;
  double* cg_part = nullptr;
  double* cg_scal = nullptr;
  unsigned* cg_counter = nullptr;
  int* cg_flags = nullptr;
  int* h_cg_flags = nullptr;
  int cg_grid = 0;
  int cg_chunk = 64;

  // launch accounting and optional per-kernel-class event timing
  struct KTime {
    int cls;
    cudaEvent_t a, b;
    double bytes;
  };
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  std::vector<KTime> ktimes;
  long long launches = 0;
  cudaEvent_t next_event();
  // Records an event pair around `launch` when profiling; counts `nlaunch`.
  template <class F>
  cudaError_t timed(int cls, double bytes, int nlaunch, F&& launch) {
    launches += nlaunch;
    if (!opts.profile) return launch();
    KTime kt{cls, next_event(), next_event(), bytes};
    cudaEventRecord(kt.a, stream);
    cudaError_t e = launch();
    cudaEventRecord(kt.b, stream);
    ktimes.push_back(kt);
    return e;
  }
  void collect_profile(lg_eigsh_info* info);

  lg_eigsh_opts opts{};
  int breakdowns = 0;
  long long cg_iters = 0;
  int cg_failures = 0;
  int skip_checks_next = 0;
};

}  // namespace lg
