// Squared Euclidean distance matrix of the rows of X (n x d float32):
//   D[i][j] = max(||x_i||^2 + ||x_j||^2 - 2 x_i . x_j, 0)
// in float32, the expanded formula of the reference's pairwise path
// (skmetal_bridge/Sources/SkMetalBridge/KMeansBridge.swift:8-85: row norms,
// X X^T, then Kernels/PairwiseDistKernels.metal:10-22 per element).
//
// The output (4 n^2 bytes) is written once. D is symmetric, so the kernel
// computes the tiles on and above the diagonal only and writes each
// off-diagonal tile twice, as itself and transposed: half the dot products
// of the full matrix. A CTA of 256 threads owns a 128 x 128 tile; its rows
// and columns of X go through shared memory in slices of 16 columns, stored
// column-major (k, row) so that a thread reads four consecutive rows as one
// 16-byte word; thread (tx, ty) accumulates the 8 x 8 products of rows
// {4 ty + r, 64 + 4 ty + r} and columns {4 tx + c, 64 + 4 tx + c} in
// registers (float32 fma, the k order ascending). Stores are 16-byte when n
// is a multiple of 4, else scalar.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "driver.h"
#include "kernels.cuh"
#include "../../include/skmetal_cuda.h"

namespace skm {

namespace {

constexpr int PT = 128;  // tile edge
constexpr int PK = 16;   // columns of X per shared-memory slice
constexpr int PTHREADS = 256;

// ||x_i||^2 in float32, one warp per row, lanes over columns then a xor butterfly
__global__ void pair_norms_kernel(const float* __restrict__ X, int ld, long long n, int d, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long w0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long r = w0; r < n; r += nw) {
    float s = 0.f;
    for (int j = lane; j < d; j += 32) {
      const float v = X[r * ld + j];
      s = fmaf(v, v, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[r] = s;
  }
}

// tile (bi, bj), bj >= bi, of the upper triangle from its linear index t
__device__ __forceinline__ void tri_tile(long long t, long long nb, long long* bi, long long* bj) {
  // row bi starts at S(bi) = bi nb - bi (bi - 1) / 2; invert, then correct by one step
  const double fb = (double)nb + 0.5;
  long long i = (long long)floor(fb - sqrt(fb * fb - 2.0 * (double)t));
  if (i < 0) i = 0;
  if (i > nb - 1) i = nb - 1;
  auto start = [nb](long long r) { return r * nb - r * (r - 1) / 2; };
  while (i > 0 && start(i) > t) --i;
  while (i + 1 < nb && start(i + 1) <= t) ++i;
  *bi = i;
  *bj = i + (t - start(i));
}

__device__ __forceinline__ void store4(float* D, long long n, long long row, long long col, const float v[4],
                                       bool vec) {
  if (row >= n) return;
  float* p = D + row * n + col;
  if (vec && col + 3 < n) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (col + c < n) p[c] = v[c];
  }
}

__global__ void __launch_bounds__(PTHREADS) pairwise_kernel(const float* __restrict__ X, int ld, long long n, int d,
                                                           const float* __restrict__ nrm, float* __restrict__ D,
                                                           long long n_tiles) {
  __shared__ __align__(16) float As[PK][PT];
  __shared__ __align__(16) float Bs[PK][PT];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const long long nb = (n + PT - 1) / PT;
  const bool vec = (n & 3) == 0;
  for (long long t = blockIdx.x; t < n_tiles; t += gridDim.x) {
    long long bi, bj;
    tri_tile(t, nb, &bi, &bj);
    const long long I0 = bi * PT, J0 = bj * PT;
    float acc[8][8];
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int b = 0; b < 8; ++b) acc[a][b] = 0.f;
    for (int k0 = 0; k0 < d; k0 += PK) {
      __syncthreads();  // the previous slice is consumed
      // each thread stages 8 elements of each operand: row = idx / PK, k = idx % PK
#pragma unroll
      for (int e = 0; e < (PT * PK) / PTHREADS; ++e) {
        const int idx = threadIdx.x + e * PTHREADS;
        const int r = idx / PK, kk = idx % PK;
        const int kg = k0 + kk;
        const long long ra = I0 + r, rb = J0 + r;
        As[kk][r] = (ra < n && kg < d) ? X[ra * ld + kg] : 0.f;
        Bs[kk][r] = (rb < n && kg < d) ? X[rb * ld + kg] : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < PK; ++kk) {
        const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][4 * ty]);
        const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][64 + 4 * ty]);
        const float4 b0 = *reinterpret_cast<const float4*>(&Bs[kk][4 * tx]);
        const float4 b1 = *reinterpret_cast<const float4*>(&Bs[kk][64 + 4 * tx]);
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
          for (int b = 0; b < 8; ++b) acc[a][b] = fmaf(av[a], bv[b], acc[a][b]);
      }
    }
    // epilogue: distances, the tile and (off the diagonal) its transpose
    float ni[8], nj[8];
#pragma unroll
    for (int a = 0; a < 8; ++a) {
      const long long i = I0 + (a < 4 ? 4 * ty + a : 64 + 4 * ty + a - 4);
      const long long j = J0 + (a < 4 ? 4 * tx + a : 64 + 4 * tx + a - 4);
      ni[a] = i < n ? nrm[i] : 0.f;
      nj[a] = j < n ? nrm[j] : 0.f;
    }
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int b = 0; b < 8; ++b) acc[a][b] = fmaxf(ni[a] + nj[b] - 2.0f * acc[a][b], 0.f);
#pragma unroll
    for (int a = 0; a < 8; ++a) {
      const long long i = I0 + (a < 4 ? 4 * ty + a : 64 + 4 * ty + a - 4);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float v[4] = {acc[a][4 * h], acc[a][4 * h + 1], acc[a][4 * h + 2], acc[a][4 * h + 3]};
        store4(D, n, i, J0 + 64 * h + 4 * tx, v, vec);
      }
    }
    if (bi != bj) {
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        const long long j = J0 + (b < 4 ? 4 * tx + b : 64 + 4 * tx + b - 4);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float v[4] = {acc[4 * h][b], acc[4 * h + 1][b], acc[4 * h + 2][b], acc[4 * h + 3][b]};
          store4(D, n, j, I0 + 64 * h + 4 * ty, v, vec);
        }
      }
    }
  }
}

}  // namespace

// Device-resident form: X (n rows at stride ld floats) and D (n x n) on the
// device; norms = n floats of scratch. Launches on `s`.
int pairwise_device(const float* X, int ld, long long n, int d, float* norms, float* D, cudaStream_t s) {
  const int nsm = sm_count();
  pair_norms_kernel<<<std::max(1, std::min<int>((int)((n + 7) / 8), nsm * 8)), 256, 0, s>>>(X, ld, n, d, norms);
  SKM_TRY(check_launch("pair_norms_kernel"));
  const long long nb = (n + PT - 1) / PT;
  const long long tiles = nb * (nb + 1) / 2;
  const int grid = (int)std::max(1LL, std::min<long long>(tiles, (long long)nsm * 4));
  pairwise_kernel<<<grid, PTHREADS, 0, s>>>(X, ld, n, d, norms, D, tiles);
  SKM_TRY(check_launch("pairwise_kernel"));
  return OK;
}

}  // namespace skm

using namespace skm;

extern "C" int skmetal_pairwise_distance(const float* X, float* D, size_t n, size_t d) {
  SKM_TRY(check_injected("pairwise_distance"));
  if (n == 0 || d == 0 || X == nullptr || D == nullptr) {
    set_error(ERR_INVALID, "pairwise_distance: invalid arguments n=%zu d=%zu", n, d);
    return ERR_INVALID;
  }
  if (n >= (size_t)1 << 31 || d > ((size_t)1 << 20)) {
    set_error(ERR_INVALID, "pairwise_distance: shape too large n=%zu d=%zu", n, d);
    return ERR_INVALID;
  }
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  DevBuffers buf(s);
  const int ld = (int)((d + 3) & ~(size_t)3);
  float *Xd = nullptr, *nrm = nullptr, *Dd = nullptr;
  SKM_TRY(buf.alloc_n(&Xd, n * (size_t)ld));
  SKM_TRY(buf.alloc_n(&nrm, n));
  SKM_TRY(buf.alloc_n(&Dd, n * n));
  SKM_TRY(upload_rows(Xd, ld, X, (long long)n, (int)d, s));
  SKM_TRY(pairwise_device(Xd, ld, (long long)n, (int)d, nrm, Dd, s));
  SKM_CUDA(cudaMemcpyAsync(D, Dd, sizeof(float) * n * n, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  return OK;
}
