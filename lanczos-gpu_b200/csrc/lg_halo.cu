// lg_halo.cu — host-side planning of the halo exchange of a row-partitioned
// eigsh plan.
//
// Rank r owns the global rows [r*nb, min((r+1)*nb, n)); its CSR names global
// columns.  Before every sparse product each rank needs the residual entries
// of the columns it names that other ranks own (its halo).  The plan is made
// once, at plan creation (Solver::setup_halo, lg_irlm.cu), in three steps:
//   1. the columns outside the rank's own block are marked in a bitmap over
//      the global index range (a device kernel there; a host loop in
//      lg_halo_recv_list below), and halo_recv_lists turns the bitmap into the
//      receive list: global positions grouped by owner (ascending owner,
//      ascending row);
//   2. one all-reduce of the ranks x ranks count matrix (row r = how many rows
//      rank r receives from each rank) tells every rank how many rows it
//      sends to each peer, and halo_send_plan derives its send offsets and
//      the exchange mode, the same on every rank because every rank decides
//      from the same all-reduced matrix;
//   3. every rank hands each owner its receive positions, which the owner
//      keeps as its send list (the pack positions); the receiver unpacks at
//      the same global positions.
// Steps 1 and 2 are plain host functions so that they can be checked without
// GPUs: lg_halo_recv_list and lg_halo_send_plan expose them through the C ABI.
// There is no counterpart in the reference (single device).
#include "lg_common.cuh"
#include "lg_halo.h"
#include "lg_solver.h"

#include <algorithm>
#include <vector>

namespace lg {

void halo_recv_lists(const unsigned* bits, long long ld, int nranks, int rank, int n_global, std::vector<int>& pos,
                     std::vector<long long>& recv_off, std::vector<long long>& recv_cnt) {
  pos.clear();
  recv_off.assign(nranks, 0);
  recv_cnt.assign(nranks, 0);
  for (int o = 0; o < nranks; ++o) {
    recv_off[o] = (long long)pos.size();
    if (o == rank) continue;
    const long long lo = (long long)o * ld, hi = std::min<long long>((long long)(o + 1) * ld, n_global);
    for (long long c = lo; c < hi; ++c) {
      const unsigned w = bits[(size_t)(c >> 5)];
      if (w == 0u) {   // skip the rest of an empty word (block starts are multiples of 32)
        c |= 31;
        continue;
      }
      if ((w >> (c & 31)) & 1u) pos.push_back((int)c);
    }
    recv_cnt[o] = (long long)pos.size() - recv_off[o];
  }
}

int halo_send_plan(const double* cnt, int nranks, int rank, long long ld, std::vector<long long>& send_off,
                   std::vector<long long>& send_cnt, long long* total_send) {
  send_off.assign(nranks, 0);
  send_cnt.assign(nranks, 0);
  long long off = 0;
  bool small = true;
  for (int p = 0; p < nranks; ++p) {
    send_off[p] = off;
    send_cnt[p] = p == rank ? 0 : (long long)cnt[(size_t)p * nranks + rank];
    off += send_cnt[p];
    double recv_p = 0.0;
    for (int o = 0; o < nranks; ++o) recv_p += cnt[(size_t)p * nranks + o];
    // halo when every rank receives at most half of what an all-gather brings
    if (2.0 * recv_p > (double)(nranks - 1) * (double)ld) small = false;
  }
  *total_send = off;
  return small ? LG_EXCHANGE_HALO : LG_EXCHANGE_ALLGATHER;
}

}  // namespace lg

extern "C" {

int lg_halo_recv_list(int n_global, int nranks, int rank, long long nnz, const int* col, int* recv_pos,
                      long long capacity, long long* recv_cnt, long long* total) {
  using namespace lg;
  if (n_global < 1 || nranks < 1 || rank < 0 || rank >= nranks || nnz < 0 || (nnz > 0 && !col) || !recv_cnt ||
      !total || capacity < 0) {
    g_last_error = "lg_halo_recv_list: invalid arguments";
    return LG_ERR_INVALID;
  }
  const long long ld = lg_partition_block(n_global, nranks);
  const long long lo = (long long)rank * ld, hi = std::min<long long>(lo + ld, n_global);
  std::vector<unsigned> bits((size_t)((ld * nranks + 31) / 32), 0u);
  // the marking rule of the device kernel: a column outside this rank's rows
  // and inside [0, n_global)
  for (long long k = 0; k < nnz; ++k) {
    const int c = col[k];
    if ((c >= lo && c < hi) || c < 0 || c >= n_global) continue;
    bits[(size_t)(c >> 5)] |= 1u << (c & 31);
  }
  std::vector<int> pos;
  std::vector<long long> off, cnt;
  halo_recv_lists(bits.data(), ld, nranks, rank, n_global, pos, off, cnt);
  *total = (long long)pos.size();
  for (int o = 0; o < nranks; ++o) recv_cnt[o] = cnt[o];
  if ((long long)pos.size() > capacity || (!recv_pos && !pos.empty())) {
    g_last_error = "lg_halo_recv_list: recv_pos holds fewer entries than the halo (see *total)";
    return LG_ERR_INVALID;
  }
  std::copy(pos.begin(), pos.end(), recv_pos);
  return LG_OK;
}

int lg_halo_send_plan(int n_global, int nranks, int rank, const double* counts, long long* send_cnt, int* mode) {
  using namespace lg;
  if (n_global < 1 || nranks < 1 || rank < 0 || rank >= nranks || !counts || !send_cnt || !mode) {
    g_last_error = "lg_halo_send_plan: invalid arguments";
    return LG_ERR_INVALID;
  }
  std::vector<long long> off, cnt;
  long long total = 0;
  *mode = halo_send_plan(counts, nranks, rank, lg_partition_block(n_global, nranks), off, cnt, &total);
  for (int p = 0; p < nranks; ++p) send_cnt[p] = cnt[p];
  return LG_OK;
}

}  // extern "C"
