// Host -> device upload of row-major float32 rows that live in ordinary
// (pageable) host memory -- the way numpy hands them to the library.
//
// A plain cudaMemcpy from pageable memory is staged by the driver through its
// own small pinned buffers, one host thread at a time (well below the PCIe
// rate). Here the rows go through a ring of large page-locked buffers instead:
// worker threads copy chunk i + 1 into a free buffer while the DMA engine
// moves chunk i to the device, and an event per buffer keeps a buffer from
// being refilled before its DMA has finished. Page-locked and device sources
// are copied directly.
#include <cuda_runtime.h>

#include <algorithm>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <thread>
#include <vector>

#include "driver.h"

namespace skm {

namespace {

constexpr size_t kStageChunk = 16u << 20;  // bytes per staging buffer
constexpr int kStageBuffers = 4;
constexpr size_t kStageMin = 4u << 20;     // smaller uploads go straight through the driver

// Persistent worker threads for splitting a large memcpy. One job at a time
// (callers serialise on the pool's mutex); the calling thread copies a piece
// too.
class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool pool;
    return pool;
  }

  void copy(void* dst, const void* src, size_t bytes) {
    std::lock_guard<std::mutex> job_lock(job_mutex_);
    const int parts = static_cast<int>(workers_.size()) + 1;
    if (parts == 1 || bytes < (1u << 20)) {
      memcpy(dst, src, bytes);
      return;
    }
    {
      std::lock_guard<std::mutex> lk(m_);
      dst_ = static_cast<char*>(dst);
      src_ = static_cast<const char*>(src);
      bytes_ = bytes;
      parts_ = parts;
      pending_ = parts - 1;
      ++generation_;
    }
    cv_work_.notify_all();
    piece(0);
    std::unique_lock<std::mutex> lk(m_);
    cv_done_.wait(lk, [&] { return pending_ == 0; });
  }

 private:
  CopyPool() {
    int n = 0;
    if (const char* e = getenv("SKMETAL_COPY_THREADS")) n = atoi(e);
    if (n <= 0) n = std::min(8, std::max(1, static_cast<int>(std::thread::hardware_concurrency()) / 2));
    for (int i = 1; i < n; ++i) workers_.emplace_back([this, i] { run(i); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(m_);
      stop_ = true;
    }
    cv_work_.notify_all();
    for (auto& t : workers_) t.join();
  }

  // bytes [i * B / P, (i + 1) * B / P) rounded to 64-byte boundaries
  void piece(int i) {
    const size_t lo = (bytes_ * i / parts_) & ~size_t(63), hi = i + 1 == parts_ ? bytes_ : (bytes_ * (i + 1) / parts_) & ~size_t(63);
    if (hi > lo) memcpy(dst_ + lo, src_ + lo, hi - lo);
  }

  void run(int i) {
    unsigned long long seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(m_);
        cv_work_.wait(lk, [&] { return stop_ || generation_ != seen; });
        if (stop_) return;
        seen = generation_;
      }
      piece(i);
      {
        std::lock_guard<std::mutex> lk(m_);
        if (--pending_ == 0) cv_done_.notify_one();
      }
    }
  }

  std::mutex job_mutex_, m_;
  std::condition_variable cv_work_, cv_done_;
  std::vector<std::thread> workers_;
  char* dst_ = nullptr;
  const char* src_ = nullptr;
  size_t bytes_ = 0;
  int parts_ = 1, pending_ = 0;
  unsigned long long generation_ = 0;
  bool stop_ = false;
};

// The calling thread's staging ring on one device.
struct StageRing {
  void* buf[kStageBuffers] = {};
  cudaEvent_t done[kStageBuffers] = {};
  bool used[kStageBuffers] = {};
  int next = 0;
};

thread_local std::map<int, StageRing> t_rings;

int stage_ring(StageRing** out) {
  int dev = 0;
  SKM_CUDA(cudaGetDevice(&dev));
  StageRing& r = t_rings[dev];
  if (!r.buf[0]) {
    for (int i = 0; i < kStageBuffers; ++i) {
      SKM_CUDA(cudaMallocHost(&r.buf[i], kStageChunk));
      SKM_CUDA(cudaEventCreateWithFlags(&r.done[i], cudaEventDisableTiming));
    }
  }
  *out = &r;
  return OK;
}

bool is_pageable(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return a.type == cudaMemoryTypeUnregistered;
}

}  // namespace

int upload_rows(float* dst, int ld, const float* src, long long n, int d, cudaStream_t s) {
  if (n == 0) return OK;
  const size_t row_bytes = sizeof(float) * (size_t)d;
  const size_t total = row_bytes * (size_t)n;
  if (total < kStageMin || row_bytes > kStageChunk || !is_pageable(src)) {
    if (ld == d) {
      SKM_CUDA(cudaMemcpyAsync(dst, src, total, cudaMemcpyDefault, s));
    } else {
      SKM_CUDA(cudaMemcpy2DAsync(dst, sizeof(float) * ld, src, row_bytes, row_bytes, n, cudaMemcpyDefault, s));
    }
  } else {
    StageRing* r = nullptr;
    SKM_TRY(stage_ring(&r));
    const long long rows_per = (long long)(kStageChunk / row_bytes);
    for (long long r0 = 0; r0 < n; r0 += rows_per) {
      const long long rows = std::min(rows_per, n - r0);
      const int b = r->next;
      r->next = (b + 1) % kStageBuffers;
      if (r->used[b]) SKM_CUDA(cudaEventSynchronize(r->done[b]));  // its previous DMA has finished
      CopyPool::get().copy(r->buf[b], src + r0 * d, row_bytes * (size_t)rows);
      if (ld == d) {
        SKM_CUDA(cudaMemcpyAsync(dst + r0 * ld, r->buf[b], row_bytes * (size_t)rows, cudaMemcpyHostToDevice, s));
      } else {
        SKM_CUDA(cudaMemcpy2DAsync(dst + r0 * ld, sizeof(float) * ld, r->buf[b], row_bytes, row_bytes, rows,
                                   cudaMemcpyHostToDevice, s));
      }
      SKM_CUDA(cudaEventRecord(r->done[b], s));
      r->used[b] = true;
    }
  }
  if (ld != d)
    SKM_CUDA(cudaMemset2DAsync(dst + d, sizeof(float) * ld, 0, sizeof(float) * (ld - d), n, s));
  return OK;
}

}  // namespace skm
