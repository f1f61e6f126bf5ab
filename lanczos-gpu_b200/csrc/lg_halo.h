// lg_halo.h — host-side halo planning of row-partitioned plans (lg_halo.cu).
#pragma once

#include <vector>

namespace lg {

// Receive list from the bitmap of marked global columns (bit c set: this rank
// reads row c of another rank): global positions grouped by owner rank
// (ascending owner, ascending row); per-owner offsets and counts in rows.
// ld: rows per rank block (a multiple of 32).
void halo_recv_lists(const unsigned* bits, long long ld, int nranks, int rank, int n_global, std::vector<int>& pos,
                     std::vector<long long>& recv_off, std::vector<long long>& recv_cnt);

// From the all-reduced ranks x ranks count matrix (row r = rows rank r
// receives from each rank): this rank's send offsets and counts per peer and
// their total; returns the exchange mode (LG_EXCHANGE_HALO when every rank
// receives at most half of what an all-gather brings, else
// LG_EXCHANGE_ALLGATHER), identical on every rank.
int halo_send_plan(const double* cnt, int nranks, int rank, long long ld, std::vector<long long>& send_off,
                   std::vector<long long>& send_cnt, long long* total_send);

}  // namespace lg
