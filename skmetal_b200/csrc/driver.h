// Host-side helpers shared by the translation units of the library.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <vector>

#include "skm.cuh"

#define SKM_CUDA(call)                                                                                  \
  do {                                                                                                  \
    cudaError_t e_ = (call);                                                                            \
    if (e_ != cudaSuccess) {                                                                            \
      const int c_ = e_ == cudaErrorMemoryAllocation ? ::skm::ERR_OOM : ::skm::ERR_CUDA;                \
      ::skm::set_error(c_, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
      return c_;                                                                                        \
    }                                                                                                   \
  } while (0)

#define SKM_TRY(expr)          \
  do {                         \
    const int rc_ = (expr);    \
    if (rc_ != 0) return rc_;  \
  } while (0)

namespace skm {

extern std::atomic<unsigned long long> g_launches;

int check_injected(const char* where);
int current_device(int* dev);
int thread_stream(cudaStream_t* s, double** pinned);
int sm_count();
int check_launch(const char* what);
int upload_rows(float* dst, int ld, const float* src, long long n, int d, cudaStream_t s);

// Stream-ordered device allocations freed (stream-ordered) when the owner
// goes out of scope.
struct DevBuffers {
  cudaStream_t stream;
  std::vector<void*> ptrs;
  explicit DevBuffers(cudaStream_t s) : stream(s) {}
  ~DevBuffers();
  DevBuffers(const DevBuffers&) = delete;
  DevBuffers& operator=(const DevBuffers&) = delete;
  int alloc(void** p, size_t bytes);
  template <class T>
  int alloc_n(T** p, size_t count) {
    return alloc(reinterpret_cast<void**>(p), sizeof(T) * count);
  }
};

}  // namespace skm
