// lg_comm.cu — NCCL communicator for the row-partitioned eigensolver.
//
// One process per GPU.  The library does not link NCCL: the first
// communicator opens libnccl.so.2 with dlopen (if the process already loaded
// it — torch.distributed does — the loaded copy is reused) and resolves the
// handful of entry points it needs.  Collectives run on the solver's stream:
//   all-reduce (sum) of one partial-sum row per Gram-Schmidt pass, and
//   before each sparse product either the in-place all-gather of the residual
//   or the halo exchange (grouped point-to-point sends and receives of the
//   residual rows that other ranks' sparse products read).
// Every rank issues the same collectives in the same order; the solver's
// control decisions derive only from all-reduced values, so they agree.
#include "lg_comm.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

namespace lg {

extern thread_local std::string g_last_error;

namespace {

struct NcclApi {
  void* lib = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

bool load_nccl() {
  std::lock_guard<std::mutex> lk(g_nccl_mu);
  if (g_nccl.lib) return true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    g_last_error = std::string("cannot load libnccl.so.2: ") + dlerror();
    return false;
  }
  NcclApi a;
  a.lib = h;
  a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
  a.CommInitRank = reinterpret_cast<decltype(a.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
  a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
  a.AllReduce = reinterpret_cast<decltype(a.AllReduce)>(dlsym(h, "ncclAllReduce"));
  a.AllGather = reinterpret_cast<decltype(a.AllGather)>(dlsym(h, "ncclAllGather"));
  a.Send = reinterpret_cast<decltype(a.Send)>(dlsym(h, "ncclSend"));
  a.Recv = reinterpret_cast<decltype(a.Recv)>(dlsym(h, "ncclRecv"));
  a.GroupStart = reinterpret_cast<decltype(a.GroupStart)>(dlsym(h, "ncclGroupStart"));
  a.GroupEnd = reinterpret_cast<decltype(a.GroupEnd)>(dlsym(h, "ncclGroupEnd"));
  a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
  if (!a.GetUniqueId || !a.CommInitRank || !a.CommDestroy || !a.AllReduce || !a.AllGather || !a.Send || !a.Recv ||
      !a.GroupStart || !a.GroupEnd || !a.GetErrorString) {
    g_last_error = "libnccl.so.2 lacks a required entry point";
    dlclose(h);
    return false;
  }
  g_nccl = a;
  return true;
}

int nccl_fail(const char* what, ncclResult_t r) {
  g_last_error = std::string(what) + ": " + (g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "NCCL error");
  return LG_ERR_CUDA;
}

}  // namespace

struct CommImpl {
  ncclComm_t comm = nullptr;
  int rank = 0, nranks = 1;
};

int comm_rank(const lg_comm* c) { return reinterpret_cast<const CommImpl*>(c)->rank; }
int comm_size(const lg_comm* c) { return reinterpret_cast<const CommImpl*>(c)->nranks; }

int comm_allreduce_sum(const lg_comm* c, double* buf, size_t count, cudaStream_t st) {
  const CommImpl* ci = reinterpret_cast<const CommImpl*>(c);
  ncclResult_t r = g_nccl.AllReduce(buf, buf, count, ncclDouble, ncclSum, ci->comm, st);
  return r == ncclSuccess ? LG_OK : nccl_fail("ncclAllReduce", r);
}

int comm_allgather_inplace(const lg_comm* c, double* full, size_t count_per_rank, cudaStream_t st) {
  const CommImpl* ci = reinterpret_cast<const CommImpl*>(c);
  ncclResult_t r = g_nccl.AllGather(full + (size_t)ci->rank * count_per_rank, full, count_per_rank, ncclDouble,
                                    ci->comm, st);
  return r == ncclSuccess ? LG_OK : nccl_fail("ncclAllGather", r);
}

int comm_allgather_bytes(const lg_comm* c, void* full, size_t bytes_per_rank, cudaStream_t st) {
  const CommImpl* ci = reinterpret_cast<const CommImpl*>(c);
  char* base = static_cast<char*>(full);
  ncclResult_t r = g_nccl.AllGather(base + (size_t)ci->rank * bytes_per_rank, base, bytes_per_rank, ncclChar,
                                    ci->comm, st);
  return r == ncclSuccess ? LG_OK : nccl_fail("ncclAllGather", r);
}

int comm_sendrecv(const lg_comm* c, int elem_bytes, const void* sendbuf, const long long* send_off,
                  const long long* send_cnt, void* recvbuf, const long long* recv_off, const long long* recv_cnt,
                  cudaStream_t st) {
  const CommImpl* ci = reinterpret_cast<const CommImpl*>(c);
  const ncclDataType_t t = elem_bytes == 8 ? ncclDouble : ncclInt32;
  ncclResult_t r = g_nccl.GroupStart();
  if (r != ncclSuccess) return nccl_fail("ncclGroupStart", r);
  ncclResult_t first = ncclSuccess;
  for (int p = 0; p < ci->nranks; ++p) {
    if (p == ci->rank) continue;
    if (send_cnt[p] > 0) {
      r = g_nccl.Send(static_cast<const char*>(sendbuf) + (size_t)send_off[p] * elem_bytes, (size_t)send_cnt[p], t, p,
                      ci->comm, st);
      if (r != ncclSuccess && first == ncclSuccess) first = r;
    }
    if (recv_cnt[p] > 0) {
      r = g_nccl.Recv(static_cast<char*>(recvbuf) + (size_t)recv_off[p] * elem_bytes, (size_t)recv_cnt[p], t, p,
                      ci->comm, st);
      if (r != ncclSuccess && first == ncclSuccess) first = r;
    }
  }
  r = g_nccl.GroupEnd();   // always closes the group, also after a failed call inside it
  if (first != ncclSuccess) return nccl_fail("ncclSend/ncclRecv", first);
  return r == ncclSuccess ? LG_OK : nccl_fail("ncclGroupEnd", r);
}

}  // namespace lg

using namespace lg;

extern "C" int lg_comm_unique_id(void* out, int len) {
  if (!out || len < (int)sizeof(ncclUniqueId)) {
    g_last_error = "lg_comm_unique_id: need a buffer of LG_COMM_ID_BYTES bytes";
    return LG_ERR_INVALID;
  }
  if (!load_nccl()) return LG_ERR_CUDA;
  ncclUniqueId id;
  ncclResult_t r = g_nccl.GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
  std::memcpy(out, &id, sizeof(id));
  return LG_OK;
}

extern "C" int lg_comm_create(lg_comm** out, const void* id, int len, int nranks, int rank) {
  if (!out || !id || len < (int)sizeof(ncclUniqueId) || nranks < 1 || rank < 0 || rank >= nranks) {
    g_last_error = "lg_comm_create: invalid arguments";
    return LG_ERR_INVALID;
  }
  if (!load_nccl()) return LG_ERR_CUDA;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  CommImpl* c = new CommImpl;
  c->rank = rank;
  c->nranks = nranks;
  ncclResult_t r = g_nccl.CommInitRank(&c->comm, nranks, uid, rank);
  if (r != ncclSuccess) {
    delete c;
    return nccl_fail("ncclCommInitRank", r);
  }
  *out = reinterpret_cast<lg_comm*>(c);
  return LG_OK;
}

extern "C" int lg_comm_destroy(lg_comm* c) {
  if (!c) return LG_OK;
  CommImpl* ci = reinterpret_cast<CommImpl*>(c);
  if (ci->comm) g_nccl.CommDestroy(ci->comm);
  delete ci;
  return LG_OK;
}
