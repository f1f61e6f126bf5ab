// lg_peer.cu — peer-memory transport of row-partitioned eigsh plans.
//
// A partitioned Lanczos step needs three reductions of one partial-sum row
// (136 doubles) over the ranks and, before its sparse product, the residual
// rows that other ranks own.  Through NCCL that is a row-sum kernel plus an
// all-reduce per reduction and a pack kernel, a grouped send/receive and an
// unpack kernel per exchange, each with its launch and protocol latency.
// Here each of them is ONE kernel that writes straight into the other ranks'
// memory over NVLink (buffers mapped with CUDA IPC at plan creation):
//
//   peer_allreduce_kernel (1 CTA): sums this rank's partial rows of one or
//     two tables in a fixed order, stores the sums into slot [rank] of every
//     rank's mailbox, fences, raises its flag on every rank (a release store of
//     the call's sequence number), waits for every rank's flag in its own
//     memory, and adds the ranks' rows in rank order — the same additions in
//     the same order on every rank, so every rank gets bitwise the same row.
//   peer_exchange_kernel (a grid): stores the residual rows each peer reads
//     (halo lists) or this rank's whole block (all-gather mode) at their
//     global positions in every peer's residual buffer; the last CTA to
//     finish fences, raises the flags and waits for every peer's.
//
// Buffers per rank (one allocation, mapped by every peer): the mailbox
// [2 parities][2 tables][ranks][136 doubles] and the flags [2 parities][ranks].
// Consecutive calls alternate the parity.  A rank can be at most one call
// ahead of another (it cannot finish call c before every rank has entered
// it), so a parity is never rewritten while a rank may still read it.
//
// Every wait is bounded (ten seconds at the highest SM clock; the
// environment variable LG_PEER_WAIT_MS, read at plan creation, sets it).  A rank that gives
// up records STATUS_TIMEOUT in the plan's state word, which turns the rest of
// its queued work into no-ops; the host reports LG_ERR_TIMEOUT at its next
// synchronisation, and the other ranks' waits give up the same way.  The
// transport is only used when every rank sits on its own GPU and every peer
// mapping opened; otherwise the plan keeps NCCL, decided alike on every rank.
// Only plain stores and loads touch peer memory (no bulk or tensor copies).
#include "lg_common.cuh"
#include "lg_comm.h"
#include "lg_solver.h"

#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace lg {

namespace {

constexpr double kPeerWaitMs = 10000.0;   // default bound of every wait (LG_PEER_WAIT_MS overrides)
constexpr int kReduceThreads = 1024;
constexpr int kExchangeThreads = 256;

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ size_t mail_index(int par, int table, int src, int nranks) {
  return ((size_t)(par * 2 + table) * nranks + src) * kPartStride;
}

// Threads [0, nranks) wait until flag[src] >= seq; returns false (every
// thread) when a wait gave up.
__device__ bool wait_flags(const unsigned long long* flags, int nranks, unsigned long long seq, long long wait_cycles,
                           int* sh_fail) {
  const int t = threadIdx.x;
  if (t == 0) *sh_fail = 0;
  __syncthreads();
  if (t < nranks) {
    const long long t0 = clock64();
    while (ld_acquire_sys(flags + t) < seq) {
      if (clock64() - t0 > wait_cycles) {
        atomicExch(sh_fail, 1);
        break;
      }
      __nanosleep(40);
    }
  }
  __syncthreads();
  return *sh_fail == 0;
}

__global__ void __launch_bounds__(kReduceThreads)
peer_allreduce_kernel(const double* __restrict__ partA, const double* __restrict__ partB, int nrows, int ntables,
                      double* out, PeerPtrs P, int nranks, int rank, unsigned long long seq, long long wait_cycles,
                      int* state) {
  griddep_wait();   // the partial rows come from the kernel just before
  // the next kernel (the correction) may start prefetching its basis rows
  // while this one waits for the other ranks; it waits for this kernel's sums
  griddep_launch_dependents();
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  constexpr int NW = kReduceThreads / 32;          // 32 warps
  constexpr int CPL = (kPartStride + 31) / 32;     // columns per lane (5)
  __shared__ double wsum[NW][kPartStride];
  __shared__ double sums[2][kPartStride];
  __shared__ int sh_fail;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int par = (int)(seq & 1ull);
  // 1. this rank's rows: warp w sums rows w, w + 32, ... (every load of a
  //    lane independent, so they are in flight together), lanes across the
  //    columns; then the warps' sums in warp order.  A fixed order.
  for (int tb = 0; tb < ntables; ++tb) {
    const double* part = tb == 0 ? partA : partB;
    double acc[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) acc[c] = 0.0;
    for (int r = warp; r < nrows; r += NW) {
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int col = lane + 32 * c;
        if (col < kPartStride) acc[c] += __ldcg(part + (size_t)r * kPartStride + col);
      }
    }
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      const int col = lane + 32 * c;
      if (col < kPartStride) wsum[warp][col] = acc[c];
    }
    __syncthreads();
    if (t < kPartStride) {
      double s = 0.0;
      for (int w = 0; w < NW; ++w) s += wsum[w][t];
      sums[tb][t] = s;
    }
    __syncthreads();
  }
  // 2. into slot [rank] of every rank's mailbox, then the flags
  if (t < ntables * kPartStride) {
    const int tb = t / kPartStride, col = t - tb * kPartStride;
    const double v = sums[tb][col];
    for (int q = 0; q < nranks; ++q) P.mail[q][mail_index(par, tb, rank, nranks) + col] = v;
    __threadfence_system();
  }
  __syncthreads();
  if (t == 0) {
    __threadfence_system();
    for (int q = 0; q < nranks; ++q) st_release_sys(P.flags[q] + (size_t)par * nranks + rank, seq);
  }
  // 3. every rank's row has arrived: add them in rank order
  if (!wait_flags(P.flags[rank] + (size_t)par * nranks, nranks, seq, wait_cycles, &sh_fail)) {
    if (t == 0) {
      state[ST_ERRINFO] = 1;
      state[ST_STATUS] = STATUS_TIMEOUT;
    }
    return;
  }
  if (t < ntables * kPartStride) {
    const int tb = t / kPartStride, col = t - tb * kPartStride;
    const double* mail = P.mail[rank];
    double s = 0.0;
    for (int q = 0; q < nranks; ++q) s += __ldcg(mail + mail_index(par, tb, q, nranks) + col);
    out[(size_t)tb * kPartStride + col] = s;
  }
}

// Halo mode (send_off != nullptr): entry i of the send list (global position
// send_idx[i], peer p with send_off[p] <= i < send_off[p + 1]) goes to the
// same position of peer p's residual buffer.  All-gather mode: this rank's
// rows [row0, row0 + P.ag_len[p]) go to peer p (the rows it reads).
//
// With `part` (nrows partial-sum rows of the kernel just before), the same
// call also all-reduces them into `out`: CTA 0 first sums this rank's rows in
// a fixed order (warp w takes rows w, w + 8, ..., then the warps in order)
// and stores the sum into slot [rank] of every rank's mailbox (table 0); the
// flags that announce the exchanged rows then announce that row too, and the
// CTA that waits for them adds the ranks' rows in rank order.  One wait per
// Lanczos step instead of two (the residual's norm and its rows).
__global__ void __launch_bounds__(kExchangeThreads)
peer_exchange_kernel(const double* __restrict__ Rfull, const int* __restrict__ send_idx,
                     const long long* __restrict__ send_off, long long total, int row0, int n_local, PeerPtrs P,
                     int nranks, int rank, unsigned long long seq, long long wait_cycles, unsigned* counter,
                     const double* __restrict__ part, int nrows, double* out, int* state) {
  griddep_wait();   // the residual rows come from the kernel just before
  if (state[ST_STATUS] != STATUS_RUNNING) return;
  __shared__ int sh_last, sh_fail;
  const int t = threadIdx.x;
  const int par = (int)(seq & 1ull);
  if (part && blockIdx.x == 0) {
    constexpr int NW = kExchangeThreads / 32;
    constexpr int CPL = (kPartStride + 31) / 32;
    __shared__ double wsum[NW][kPartStride];
    const int lane = t & 31, warp = t >> 5;
    double acc[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) acc[c] = 0.0;
    for (int r = warp; r < nrows; r += NW) {
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int col = lane + 32 * c;
        if (col < kPartStride) acc[c] += __ldcg(part + (size_t)r * kPartStride + col);
      }
    }
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      const int col = lane + 32 * c;
      if (col < kPartStride) wsum[warp][col] = acc[c];
    }
    __syncthreads();
    if (t < kPartStride) {
      double v = 0.0;
      for (int w = 0; w < NW; ++w) v += wsum[w][t];
      for (int q = 0; q < nranks; ++q) P.mail[q][mail_index(par, 0, rank, nranks) + t] = v;
    }
  }
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long i0 = (long long)blockIdx.x * blockDim.x + t;
  if (send_off) {
    for (long long i = i0; i < total; i += stride) {
      int p = 0;
      while (p + 1 < nranks && i >= __ldg(send_off + p + 1)) ++p;
      const int idx = __ldg(send_idx + i);
      P.R[p][idx] = __ldg(Rfull + idx);
    }
  } else {
    // 16-byte stores: row0 is a multiple of 256, so pairs stay aligned
    const double2* src = reinterpret_cast<const double2*>(Rfull + row0);
    for (int q = 0; q < nranks; ++q) {
      if (q == rank) continue;
      const int len = min(P.ag_len[q], n_local);
      const long long npairs = len / 2;
      double2* dst = reinterpret_cast<double2*>(P.R[q] + row0);
      for (long long i = i0; i < npairs; i += stride) dst[i] = __ldg(src + i);
      if ((len & 1) && i0 == 0) P.R[q][row0 + len - 1] = Rfull[row0 + len - 1];
    }
  }
  __threadfence_system();
  __syncthreads();
  if (t == 0) sh_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!sh_last) return;
  if (t == 0) {
    *counter = 0u;   // for the next call (stream-ordered)
    __threadfence_system();
    for (int q = 0; q < nranks; ++q)
      if (q != rank) st_release_sys(P.flags[q] + (size_t)par * nranks + rank, seq);
    // own slot, so that the wait below covers every rank uniformly
    st_release_sys(P.flags[rank] + (size_t)par * nranks + rank, seq);
  }
  if (!wait_flags(P.flags[rank] + (size_t)par * nranks, nranks, seq, wait_cycles, &sh_fail)) {
    if (t == 0) {
      state[ST_ERRINFO] = 2;
      state[ST_STATUS] = STATUS_TIMEOUT;
    }
    return;
  }
  if (part && t < kPartStride) {
    const double* mail = P.mail[rank];
    double v = 0.0;
    for (int q = 0; q < nranks; ++q) v += __ldcg(mail + mail_index(par, 0, q, nranks) + t);
    out[t] = v;
  }
}

}  // namespace

#define LG_PTRY(expr)                                                                          \
  do {                                                                                         \
    cudaError_t _e = (expr);                                                                   \
    if (_e != cudaSuccess) {                                                                   \
      g_last_error = std::string("CUDA error in the peer transport: ") + cudaGetErrorString(_e); \
      return LG_ERR_CUDA;                                                                      \
    }                                                                                          \
  } while (0)

void Solver::release_peer() {
  for (int q = 0; q < kMaxPeerRanks; ++q) {
    if (q == rank) continue;
    if (peer_open_mail[q]) cudaIpcCloseMemHandle(peer_open_mail[q]);
    if (peer_open_R[q]) cudaIpcCloseMemHandle(peer_open_R[q]);
    peer_open_mail[q] = peer_open_R[q] = nullptr;
  }
  if (peer_xch) cudaFree(peer_xch);
  if (peer_counter) cudaFree(peer_counter);
  if (d_peer_send_off) cudaFree(d_peer_send_off);
  peer_xch = nullptr;
  peer_counter = nullptr;
  d_peer_send_off = nullptr;
  peer_ok = false;
  std::memset(&peer_ptrs, 0, sizeof(peer_ptrs));
}

// Collective (every rank of a partitioned plan, once, after setup_halo).
// Maps every rank's exchange buffer and residual buffer; keeps NCCL when any
// rank cannot (environment LG_PEER_TRANSPORT=0, two ranks on one GPU, more
// ranks than kMaxPeerRanks, a mapping that does not open).
int Solver::setup_peer() {
  peer_ok = false;
  const char* env = std::getenv("LG_PEER_TRANSPORT");
  int ok = (env && env[0] == '0') ? 0 : 1;
  if (nranks > kMaxPeerRanks || nranks < 2) ok = 0;
  const size_t mail_doubles = (size_t)2 * 2 * nranks * kPartStride;
  const size_t xch_bytes = sizeof(double) * mail_doubles + sizeof(unsigned long long) * 2 * (size_t)nranks;
  LG_PTRY(cudaMalloc(&peer_xch, xch_bytes));
  LG_PTRY(cudaMemsetAsync(peer_xch, 0, xch_bytes, stream));
  LG_PTRY(cudaMalloc(&peer_counter, sizeof(unsigned)));
  LG_PTRY(cudaMemsetAsync(peer_counter, 0, sizeof(unsigned), stream));
  {
    std::vector<long long> off((size_t)nranks + 1, 0);
    for (int p = 0; p < nranks; ++p) off[p + 1] = off[p] + send_cnt[p];
    LG_PTRY(cudaMalloc(&d_peer_send_off, sizeof(long long) * off.size()));
    LG_PTRY(cudaMemcpyAsync(d_peer_send_off, off.data(), sizeof(long long) * off.size(), cudaMemcpyHostToDevice,
                            stream));
    LG_PTRY(cudaStreamSynchronize(stream));
  }

  // record per rank: the two IPC handles, the GPU's UUID, the ok flag
  struct Rec {
    cudaIpcMemHandle_t mail, R;
    char uuid[16];
    int ok;
    int pad[3];
  };
  Rec mine;
  std::memset(&mine, 0, sizeof(mine));
  cudaDeviceProp prop;
  LG_PTRY(cudaGetDeviceProperties(&prop, device));
  std::memcpy(mine.uuid, &prop.uuid, 16);
  {
    // the bound of every wait, in SM clock cycles at the highest clock
    const char* w = std::getenv("LG_PEER_WAIT_MS");
    const double ms = (w && std::atof(w) > 0.0) ? std::atof(w) : kPeerWaitMs;
    int khz = 0;
    if (cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, device) != cudaSuccess || khz <= 0) khz = 2000000;
    peer_wait_cycles = (long long)(ms * (double)khz);
  }
  if (ok) {
    if (cudaIpcGetMemHandle(&mine.mail, peer_xch) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine.R, Rfull) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
    }
  }
  mine.ok = ok;
  void* d_recs = nullptr;
  LG_PTRY(cudaMalloc(&d_recs, sizeof(Rec) * (size_t)nranks));
  std::vector<Rec> recs((size_t)nranks);
  cudaError_t e = cudaMemcpyAsync(static_cast<char*>(d_recs) + sizeof(Rec) * rank, &mine, sizeof(Rec),
                                  cudaMemcpyHostToDevice, stream);
  int rc = e == cudaSuccess ? comm_allgather_bytes(comm, d_recs, sizeof(Rec), stream) : LG_ERR_CUDA;
  if (rc == LG_OK) e = cudaMemcpyAsync(recs.data(), d_recs, sizeof(Rec) * recs.size(), cudaMemcpyDeviceToHost, stream);
  if (rc == LG_OK && e == cudaSuccess) e = cudaStreamSynchronize(stream);
  cudaFree(d_recs);
  if (rc != LG_OK) return rc;
  LG_PTRY(e);
  for (int q = 0; q < nranks && ok; ++q) {
    if (!recs[q].ok) ok = 0;
    for (int p = 0; p < q && ok; ++p)
      if (std::memcmp(recs[p].uuid, recs[q].uuid, 16) == 0) ok = 0;   // two ranks on one GPU
  }
  std::memset(&peer_ptrs, 0, sizeof(peer_ptrs));
  if (ok) {
    for (int q = 0; q < nranks && ok; ++q) {
      if (q == rank) {
        peer_ptrs.mail[q] = static_cast<double*>(peer_xch);
        peer_ptrs.R[q] = Rfull;
      } else {
        void* pm = nullptr;
        void* pr = nullptr;
        if (cudaIpcOpenMemHandle(&pm, recs[q].mail, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess ||
            cudaIpcOpenMemHandle(&pr, recs[q].R, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
          cudaGetLastError();
          if (pm) cudaIpcCloseMemHandle(pm);
          ok = 0;
          break;
        }
        peer_open_mail[q] = pm;
        peer_open_R[q] = pr;
        peer_ptrs.mail[q] = static_cast<double*>(pm);
        peer_ptrs.R[q] = static_cast<double*>(pr);
      }
      peer_ptrs.flags[q] = reinterpret_cast<unsigned long long*>(peer_ptrs.mail[q] + mail_doubles);
    }
  }
  // every rank learns whether every mapping opened (and every buffer is
  // zeroed before any rank writes into it: the all-reduce is the barrier)
  double* d_bad = nullptr;
  LG_PTRY(cudaMalloc(&d_bad, sizeof(double)));
  const double bad = ok ? 0.0 : 1.0;
  e = cudaMemcpyAsync(d_bad, &bad, sizeof(double), cudaMemcpyHostToDevice, stream);
  rc = e == cudaSuccess ? comm_allreduce_sum(comm, d_bad, 1, stream) : LG_ERR_CUDA;
  double all_bad = 1.0;
  if (rc == LG_OK) e = cudaMemcpyAsync(&all_bad, d_bad, sizeof(double), cudaMemcpyDeviceToHost, stream);
  if (rc == LG_OK && e == cudaSuccess) e = cudaStreamSynchronize(stream);
  cudaFree(d_bad);
  if (rc != LG_OK) return rc;
  LG_PTRY(e);
  if (all_bad != 0.0) {
    release_peer();
    transport = LG_TRANSPORT_NCCL;
    return LG_OK;
  }
  for (int q = 0; q < nranks; ++q) peer_ptrs.ag_len[q] = q < (int)ag_need.size() ? ag_need[q] : n;
  peer_ok = true;
  peer_seq = 0;
  transport = LG_TRANSPORT_PEER;
  return LG_OK;
}

int Solver::set_transport(int mode) {
  if (!comm) {
    g_last_error = "set_transport: not a partitioned plan";
    return LG_ERR_INVALID;
  }
  if (mode == LG_TRANSPORT_AUTO) {
    transport = peer_ok ? LG_TRANSPORT_PEER : LG_TRANSPORT_NCCL;
  } else if (mode == LG_TRANSPORT_NCCL) {
    transport = mode;
  } else if (mode == LG_TRANSPORT_PEER) {
    if (!peer_ok) {
      g_last_error = "set_transport: the peer mappings of this plan are not available (NCCL only)";
      return LG_ERR_INVALID;
    }
    transport = mode;
  } else {
    g_last_error = "set_transport: mode must be LG_TRANSPORT_AUTO, _NCCL or _PEER";
    return LG_ERR_INVALID;
  }
  return LG_OK;
}

// One peer all-reduce of `ntables` partial tables (nrows rows each) into rows
// slot, slot + 1 of `red`.
int Solver::peer_reduce(const double* partA, const double* partB, int nrows, int ntables, int slot) {
  double* out = red + (size_t)slot * kPartStride;
  ++peer_seq;
  LG_PTRY(timed(LG_K_COMM, 0.0, 1, [&] {
    return launch_pdl(peer_allreduce_kernel, dim3(1), dim3(kReduceThreads), 0, stream, partA, partB, nrows, ntables,
                      out, peer_ptrs, nranks, rank, peer_seq, peer_wait_cycles, state);
  }));
  return LG_OK;
}

int Solver::peer_exchange(const double* part, int nrows, int slot) {
  ++peer_seq;
  const bool halo = exchange == LG_EXCHANGE_HALO;
  long long ag_pairs = 0;
  for (int q = 0; q < nranks; ++q) ag_pairs += (peer_ptrs.ag_len[q] + 1) / 2;
  const long long work = halo ? halo_send : ag_pairs;
  const int grid = (int)std::max<long long>(1, std::min<long long>((long long)num_sm * 4,
                                                                    (work + kExchangeThreads - 1) / kExchangeThreads));
  LG_PTRY(timed(LG_K_COMM, 0.0, 1, [&] {
    return launch_pdl(peer_exchange_kernel, dim3(grid), dim3(kExchangeThreads), 0, stream, (const double*)Rfull,
                      (const int*)d_send_idx, (const long long*)(halo ? d_peer_send_off : nullptr), halo_send, row0,
                      n, peer_ptrs, nranks, rank, peer_seq, peer_wait_cycles, peer_counter, part, part ? nrows : 0,
                      part ? red + (size_t)slot * kPartStride : nullptr, state);
  }));
  return LG_OK;
}

}  // namespace lg
