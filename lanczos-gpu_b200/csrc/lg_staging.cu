// lg_staging.cu — host <-> device copies of pageable host memory through a
// process-wide pinned staging pool.
//
// A one-shot solve from host arrays moves the CSR matrix up (12 bytes per
// nonzero) and the eigenvectors down (8 n k bytes).  From pageable memory the
// driver stages those copies itself at a fraction of the link rate.  Here two
// pinned slots of kSlotBytes, allocated on first use and kept for the process,
// carry the data in chunks: the host side of a chunk is copied by several host
// threads while the previous chunk's DMA is in flight, so the copy runs at
// close to the slower of the link and the host memcpy rate.  The pool is shared
// by all plans and threads (one copy at a time, under a mutex).
#include "lg_staging.h"

#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace lg {

namespace {

constexpr size_t kSlotBytes = size_t(32) << 20;
constexpr size_t kMinStaged = size_t(4) << 20;   // smaller copies go straight through the driver

std::mutex g_stage_mu;
void* g_slot[2] = {nullptr, nullptr};
cudaEvent_t g_ev[2] = {nullptr, nullptr};
int g_stage_dev = -1;

// Host workers kept for the process (started on first use, never joined: the
// pool outlives every caller), so a copy of a few chunks does not pay for
// creating and joining a dozen threads per chunk.
class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool* p = new CopyPool();   // intentionally never destroyed
    return *p;
  }
  int size() const { return (int)workers_.size() + 1; }
  // Runs fn(0 .. parts-1) on the workers and the calling thread; returns when
  // all parts are done.  One job at a time (callers hold g_stage_mu).
  void run(int parts, const std::function<void(int)>& fn) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      job_ = &fn;
      parts_ = parts;
      next_ = 1;   // part 0 is the caller's
      done_ = 0;
      ++gen_;
    }
    cv_.notify_all();
    fn(0);
    std::unique_lock<std::mutex> lk(mu_);
    ++done_;
    for (;;) {   // help with parts no worker has taken yet
      if (next_ >= parts_) break;
      const int part = next_++;
      lk.unlock();
      fn(part);
      lk.lock();
      ++done_;
    }
    cv_done_.wait(lk, [&] { return done_ == parts_; });
    job_ = nullptr;
  }

 private:
  CopyPool() {
    const int nth = (int)std::max(1u, std::min(16u, std::thread::hardware_concurrency())) - 1;
    for (int w = 0; w < nth; ++w) workers_.emplace_back([this] { loop(); });
    for (std::thread& t : workers_) t.detach();
  }
  void loop() {
    unsigned long long seen = 0;
    std::unique_lock<std::mutex> lk(mu_);
    for (;;) {
      cv_.wait(lk, [&] { return gen_ != seen && job_ != nullptr && next_ < parts_; });
      seen = gen_;
      while (job_ && next_ < parts_) {
        const int part = next_++;
        const std::function<void(int)>* f = job_;
        lk.unlock();
        (*f)(part);
        lk.lock();
        if (++done_ == parts_) cv_done_.notify_all();
      }
    }
  }
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, cv_done_;
  const std::function<void(int)>* job_ = nullptr;
  int parts_ = 0, next_ = 0, done_ = 0;
  unsigned long long gen_ = 0;
};

void parallel_copy(void* dst, const void* src, size_t bytes) {
  const size_t per = size_t(2) << 20;
  CopyPool& pool = CopyPool::get();
  const int nth = (int)std::max<size_t>(1, std::min<size_t>((size_t)pool.size(), (bytes + per - 1) / per));
  if (nth <= 1) {
    std::memcpy(dst, src, bytes);
    return;
  }
  pool.run(nth, [=](int w) {
    const size_t b = bytes * w / nth, e = bytes * (w + 1) / nth;
    std::memcpy(static_cast<char*>(dst) + b, static_cast<const char*>(src) + b, e - b);
  });
}

// Slots of the current device (re-created when the caller's device changes).
cudaError_t ensure_slots() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (g_slot[0] && g_stage_dev == dev) return cudaSuccess;
  for (int i = 0; i < 2; ++i) {
    if (g_slot[i]) cudaFreeHost(g_slot[i]);
    if (g_ev[i]) cudaEventDestroy(g_ev[i]);
    g_slot[i] = nullptr;
    g_ev[i] = nullptr;
  }
  for (int i = 0; i < 2; ++i) {
    e = cudaHostAlloc(&g_slot[i], kSlotBytes, cudaHostAllocDefault);
    if (e != cudaSuccess) return e;
    e = cudaEventCreateWithFlags(&g_ev[i], cudaEventDisableTiming);
    if (e != cudaSuccess) return e;
  }
  g_stage_dev = dev;
  return cudaSuccess;
}

}  // namespace

cudaError_t staged_h2d(void* dst, const void* src, size_t bytes, cudaStream_t st) {
  if (bytes < kMinStaged) return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st);
  std::lock_guard<std::mutex> lock(g_stage_mu);
  cudaError_t e = ensure_slots();
  if (e != cudaSuccess) return e;
  size_t off = 0;
  for (int c = 0; off < bytes; ++c) {
    const int s = c & 1;
    const size_t n = std::min(kSlotBytes, bytes - off);
    if (c >= 2) {   // the DMA that last read this slot has finished
      e = cudaEventSynchronize(g_ev[s]);
      if (e != cudaSuccess) return e;
    }
    parallel_copy(g_slot[s], static_cast<const char*>(src) + off, n);
    e = cudaMemcpyAsync(static_cast<char*>(dst) + off, g_slot[s], n, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return e;
    e = cudaEventRecord(g_ev[s], st);
    if (e != cudaSuccess) return e;
    off += n;
  }
  // the slots may be refilled by the next copy only after these DMAs
  return cudaStreamSynchronize(st);
}

cudaError_t staged_d2h(void* dst, const void* src, size_t bytes, cudaStream_t st) {
  if (bytes < kMinStaged) {
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(st);
  }
  std::lock_guard<std::mutex> lock(g_stage_mu);
  cudaError_t e = ensure_slots();
  if (e != cudaSuccess) return e;
  // chunk c lands in slot c & 1; chunk c + 1's DMA overlaps chunk c's host copy
  const size_t nchunks = (bytes + kSlotBytes - 1) / kSlotBytes;
  auto issue = [&](size_t c) -> cudaError_t {
    const size_t o = c * kSlotBytes, n = std::min(kSlotBytes, bytes - o);
    cudaError_t r = cudaMemcpyAsync(g_slot[c & 1], static_cast<const char*>(src) + o, n, cudaMemcpyDeviceToHost, st);
    if (r != cudaSuccess) return r;
    return cudaEventRecord(g_ev[c & 1], st);
  };
  e = issue(0);
  if (e != cudaSuccess) return e;
  for (size_t c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks) {
      e = issue(c + 1);
      if (e != cudaSuccess) return e;
    }
    e = cudaEventSynchronize(g_ev[c & 1]);
    if (e != cudaSuccess) return e;
    const size_t o = c * kSlotBytes, n = std::min(kSlotBytes, bytes - o);
    parallel_copy(static_cast<char*>(dst) + o, g_slot[c & 1], n);
  }
  return cudaSuccess;
}

}  // namespace lg
