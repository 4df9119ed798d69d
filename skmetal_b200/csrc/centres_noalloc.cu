// Centroid update that allocates no device memory.
//
// skmetal_kmeans_update_centers_noalloc computes, for rows and labels that
// already live in device memory, every cluster's mean with the same exact
// fixed-point sums as the fit's M-step (max |x| -> scale 2^F, integer sums,
// mean = sum * (2^-F / count)), so its centres are bit-identical to the ones
// skmetal_kmeans_lloyd_iter returns for the same labels when no cluster is
// empty. It exists for callers that cannot allocate device memory at the time
// they call: a process whose free device memory is already claimed by another
// allocator's pool (a cudaMalloc would fail there), or a loop that cannot
// afford the device-wide waits a cudaMalloc / cudaFree may cause. Those
// callers pass their own device buffers and stream, and nothing here calls
// cudaMalloc, cudaFree or a library routine that allocates.
//
// Its scratch (max |x| bits, a bad-label counter, per-cluster row counts and
// fixed-point column sums) lives in one static device array of
// SKMETAL_NOALLOC_SCRATCH_BYTES, which every device that loads this library
// holds until the process exits. Every call looks up that array's device
// address with cudaGetSymbolAddress (the first call on a device can load this
// library's device code there) and waits for its work on the caller's stream
// before it returns. There is one array per device, shared by every caller,
// so calls on the same device that overlap in time race on it.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "device_util.cuh"
#include "driver.h"
#include "../../include/skmetal_cuda.h"

constexpr size_t kNoallocScratchWords = SKMETAL_NOALLOC_SCRATCH_BYTES / sizeof(long long);

// word 0: [max |x| float bits | count of labels outside [0, k)] as two u32;
// words 1 .. k: row count per cluster; then k x d fixed-point column sums
static __device__ __align__(256) long long g_noalloc_scratch[kNoallocScratchWords];

namespace skm {
namespace {

constexpr size_t kScratchWords = kNoallocScratchWords;
constexpr int kMaxDevices = 64;

// Same formula as the fit's fixed-point scale: 2^F with F = 62 - E - L, where
// max |x| < 2^E and n <= 2^L, so no sum of up to n values can reach 2^62.
__device__ double noalloc_fixed_scale(unsigned int maxabs_bits, double n) {
  const float mx = __uint_as_float(maxabs_bits);
  int E = -60;
  if (mx > 0.0f) frexp((double)mx, &E);
  int L = 0;
  frexp(fmax(n, 1.0), &L);
  int F = 62 - E - L;
  F = max(-1000, min(1000, F));
  return ldexp(1.0, F);
}

// max |x| over the n x d row-major rows (NaN keeps its bits, above +inf)
__global__ void noalloc_maxabs_kernel(const float* __restrict__ X, long long total, unsigned int* __restrict__ hdr) {
  unsigned int m = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x)
    m = max(m, __float_as_uint(X[i]) & 0x7fffffffu);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(&hdr[0], m);
}

// Fixed-point sums: one warp per row, lanes over the columns. Integer
// additions are exact, so the result does not depend on their order. Rows
// whose label lies outside [0, k) are counted and skipped.
__global__ void noalloc_sums_kernel(const float* __restrict__ X, long long n, int d,
                                    const int32_t* __restrict__ labels, int k, unsigned int* __restrict__ hdr,
                                    long long* __restrict__ counts, long long* __restrict__ S) {
  const unsigned int mx = hdr[0];
  if (mx >= 0x7f800000u) return;  // non-finite X: reported by the host
  const double scale = noalloc_fixed_scale(mx, (double)n);
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += warps) {
    const int c = labels[r];
    if (c < 0 || c >= k) {
      if (lane == 0) atomicAdd(&hdr[1], 1u);
      continue;
    }
    const float* xr = X + r * d;
    long long* sr = S + (long long)c * d;
    for (int j = lane; j < d; j += 32) {
      const long long v = to_fixed(xr[j], scale);
      if (v != 0) red_add_s64(sr + j, v);
    }
    if (lane == 0) red_add_s64(counts + c, 1);
  }
}

// centres[c][j] = S[c][j] * (2^-F / count[c]) for every non-empty cluster (the
// fit's averaging expression, centre_from_sum); rows of empty clusters are
// left as they are.
// Nothing is written when the sums reported an error.
__global__ void noalloc_centres_kernel(const long long* __restrict__ S, const long long* __restrict__ counts,
                                       long long n, int d, int k, const unsigned int* __restrict__ hdr,
                                       float* __restrict__ centres, float* __restrict__ weight) {
  if (hdr[0] >= 0x7f800000u || hdr[1] != 0) return;
  const double inv_scale = 1.0 / noalloc_fixed_scale(hdr[0], (double)n);
  const long long total = (long long)k * d;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += stride) {
    const long long cnt = counts[i / d];
    if (cnt > 0) centres[i] = centre_from_sum(S[i], centre_factor(inv_scale, cnt));
  }
  if (weight)
    for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < k; c += stride)
      weight[c] = (float)counts[c];
}

// Device address of the static scratch on the current device `dev`. Looked
// up on every call (with that device current): the lookup allocates nothing,
// costs little once the library's device code is loaded, and stays right
// after a cudaDeviceReset, which gives the scratch a new address in the new
// context. The first lookup on a device can load the library's device code
// there.
int scratch_for_device(int dev, long long** out) {
  long long* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    cudaGetLastError();
    set_error(ERR_CUDA, "kmeans_update_centers_noalloc: cudaGetSymbolAddress of the static scratch failed on device %d: %s",
              dev, cudaGetErrorString(e));
    return ERR_CUDA;
  }
  *out = ptr;
  return OK;
}

int require_device_memory(const void* p, int dev, const char* what) {
  cudaPointerAttributes a{};
  const cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error(ERR_INVALID, "kmeans_update_centers_noalloc: %s is not a valid pointer: %s", what, cudaGetErrorString(e));
    return ERR_INVALID;
  }
  const bool on_device = a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
  if (!on_device || a.device != dev) {
    set_error(ERR_INVALID, "kmeans_update_centers_noalloc: %s must point to device memory of the current device %d", what,
              dev);
    return ERR_INVALID;
  }
  return OK;
}

}  // namespace
}  // namespace skm

using namespace skm;

extern "C" int skmetal_kmeans_update_centers_noalloc(const float* X, const int32_t* labels, size_t n, size_t d,
                                                     size_t k, float* centers, float* weight, void* stream) {
  SKM_TRY(check_injected("kmeans_update_centers_noalloc"));
  if (X == nullptr || labels == nullptr || centers == nullptr) {
    set_error(ERR_INVALID, "kmeans_update_centers_noalloc: X, labels and centers must not be NULL");
    return ERR_INVALID;
  }
  if (n == 0 || d == 0 || k == 0 || n >= (size_t(1) << 31)) {
    set_error(ERR_INVALID, "kmeans_update_centers_noalloc: invalid shape n=%zu d=%zu k=%zu", n, d, k);
    return ERR_INVALID;
  }
  // scratch words: 1 header + k counts + k*d sums (k, d < 2^31 keeps k*d in range)
  if (k >= kScratchWords || d >= kScratchWords || 1 + k + k * d > kScratchWords) {
    set_error(ERR_INVALID,
              "kmeans_update_centers_noalloc: k=%zu, d=%zu needs %zu bytes of scratch; the static scratch holds %zu "
              "bytes (k * (d + 1) must be at most %zu)",
              k, d, (k < kScratchWords && d < kScratchWords) ? sizeof(long long) * (1 + k + k * d) : (size_t)-1,
              (size_t)SKMETAL_NOALLOC_SCRATCH_BYTES, kScratchWords - 1);
    return ERR_INVALID;
  }
  int dev = 0;
  SKM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) {
    set_error(ERR_UNSUPPORTED, "kmeans_update_centers_noalloc: device %d is beyond the %d supported", dev, kMaxDevices);
    return ERR_UNSUPPORTED;
  }
  SKM_TRY(require_device_memory(X, dev, "X"));
  SKM_TRY(require_device_memory(labels, dev, "labels"));
  SKM_TRY(require_device_memory(centers, dev, "centers"));
  if (weight) SKM_TRY(require_device_memory(weight, dev, "weight"));

  long long* scratch = nullptr;
  SKM_TRY(scratch_for_device(dev, &scratch));
  unsigned int* hdr = reinterpret_cast<unsigned int*>(scratch);
  long long* counts = scratch + 1;
  long long* S = counts + k;
  const size_t words = 1 + k + k * d;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // the max, the bad-label count, the counts and the sums all accumulate from zero
  SKM_CUDA(cudaMemsetAsync(scratch, 0, sizeof(long long) * words, s));
  const long long nsm = sm_count();
  const long long total = (long long)n * (long long)d;
  const int mx_blocks = (int)std::max(1LL, std::min(nsm * 4, (total + 255) / 256));
  noalloc_maxabs_kernel<<<mx_blocks, 256, 0, s>>>(X, total, hdr);
  SKM_TRY(check_launch("noalloc_maxabs_kernel"));
  const int sum_blocks = (int)std::max(1LL, std::min(nsm * 8, ((long long)n + 7) / 8));
  noalloc_sums_kernel<<<sum_blocks, 256, 0, s>>>(X, (long long)n, (int)d, labels, (int)k, hdr, counts, S);
  SKM_TRY(check_launch("noalloc_sums_kernel"));
  const int c_blocks = (int)std::max(1LL, std::min(nsm * 2, ((long long)(k * d) + 255) / 256));
  noalloc_centres_kernel<<<c_blocks, 256, 0, s>>>(S, counts, (long long)n, (int)d, (int)k, hdr, centers, weight);
  SKM_TRY(check_launch("noalloc_centres_kernel"));

  unsigned int h[2] = {0, 0};
  SKM_CUDA(cudaMemcpyAsync(h, hdr, sizeof(h), cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  if (h[0] >= 0x7f800000u) {
    set_error(ERR_INVALID, "kmeans_update_centers_noalloc: X holds a non-finite value");
    return ERR_INVALID;
  }
  if (h[1] != 0) {
    set_error(ERR_INVALID, "kmeans_update_centers_noalloc: %u labels lie outside [0, %zu)", h[1], k);
    return ERR_INVALID;
  }
  return OK;
}
