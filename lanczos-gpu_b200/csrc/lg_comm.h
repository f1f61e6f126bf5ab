// lg_comm.h — collectives used by the row-partitioned eigensolver (lg_comm.cu).
#pragma once

#include <cuda_runtime.h>

#include "../../include/lanczos_b200.h"

namespace lg {

int comm_rank(const lg_comm* c);
int comm_size(const lg_comm* c);
// Sum of `count` doubles over all ranks, in place, on stream `st`.
int comm_allreduce_sum(const lg_comm* c, double* buf, size_t count, cudaStream_t st);
// full holds nranks blocks of count_per_rank doubles; this rank's block is
// already in place; afterwards every rank holds all blocks.
int comm_allgather_inplace(const lg_comm* c, double* full, size_t count_per_rank, cudaStream_t st);
// full holds nranks blocks of bytes_per_rank bytes (this rank's in place);
// afterwards every rank holds all blocks.
int comm_allgather_bytes(const lg_comm* c, void* full, size_t bytes_per_rank, cudaStream_t st);
// One grouped exchange: to every other rank p, send_cnt[p] elements from
// sendbuf + send_off[p]; from p, recv_cnt[p] elements into recvbuf +
// recv_off[p] (offsets and counts in elements, host arrays of nranks entries;
// elements are 4-byte integers or doubles).  The counts of a pair must agree
// on both sides.
int comm_sendrecv(const lg_comm* c, int elem_bytes, const void* sendbuf, const long long* send_off,
                  const long long* send_cnt, void* recvbuf, const long long* recv_off, const long long* recv_cnt,
                  cudaStream_t st);

}  // namespace lg
