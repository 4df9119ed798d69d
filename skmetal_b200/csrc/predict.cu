// Assignment for small d and k: the memory-bound predict workload (X of
// 400M x 8, k = 16), KMeans.predict of the reference
// (skmetal/estimators/cluster.py:118-126 -> skmetal_kmeans_assign,
// KMeansBridge.swift:138-181; kernel kmeans_assign, KMeansKernels.metal:6-43).
//
// The work per row is tiny (d * k multiply-adds), so the kernel must not
// spend more instructions per row than HBM takes to deliver it:
//   * the centres travel in the kernel's parameter block (the constant bank),
//     so every multiply-add takes its centre operand from there: no loads;
//   * distances are compared through the expansion
//         score_c = ||c - m||^2 - 2 (x - m).(c - m)      (= ||x - c||^2 - ||x - m||^2)
//     with m the centres' mean, one FMA per element and centre; the offset m
//     keeps the terms small, so float32 rounding stays near that of the
//     distances themselves;
//   * each row's best and second-best scores are kept; when their gap does
//     not exceed twice a bound on the scores' rounding error (which the
//     expansion's terms give per row), the row is recomputed with direct
//     differences, sum_j (x_j - c_j)^2 in column order, over every centre
//     in index order with strict '<' -- the reference's own arithmetic -- so
//     the label is that of the direct computation whenever rounding could
//     matter, and the true argmin otherwise;
//   * one thread per row (few registers: the centres are operands, not
//     registers), so many rows' loads are in flight per SM; X is read once
//     with an evict-first hint.
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>

#include "driver.h"
#include "kernels.cuh"

namespace skm {

namespace {

template <int D, int KM>
struct ConstCentres {
  float cm2[D][KM];  // -2 (c - m), centre-minor: centres c and c + 1 of a column are one 8-byte pair
  float nrm[KM];     // ||c - m||^2, +inf for padding centres (c >= k)
  float m[D];        // offset: the centres' column means
  float a_max;       // max over centres of ||c - m||^2
  float b_max;       // max over centres and columns of |c - m|
  float eps;         // error-bound factor (d + 4) 2^-24, with margin
  int k;
};

template <int D, int KM>
__global__ void __launch_bounds__(256) assign_const_kernel(const float* __restrict__ X, long long n,
                                                           const ConstCentres<D, KM> P,
                                                           const float* __restrict__ C, int ldc,
                                                           int32_t* __restrict__ labels) {
  static_assert(D % 4 == 0, "rows are read as float4");
  static_assert(KM % 2 == 0, "centres are scored in pairs");
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += stride) {
    float x[D];
    const float4* xr = reinterpret_cast<const float4*>(X + r * D);
#pragma unroll
    for (int q = 0; q < D / 4; ++q) {
      const float4 v = __ldcs(xr + q);
      x[4 * q] = v.x;
      x[4 * q + 1] = v.y;
      x[4 * q + 2] = v.z;
      x[4 * q + 3] = v.w;
    }
    float xm[D];
    float l1 = 0.0f;
#pragma unroll
    for (int j = 0; j < D; ++j) {
      xm[j] = x[j] - P.m[j];
      l1 += fabsf(xm[j]);
    }
    // x - m broadcast to both halves of a pair, once per row
    unsigned long long xx[D];
#pragma unroll
    for (int j = 0; j < D; ++j) asm("mov.b64 %0, {%1, %1};" : "=l"(xx[j]) : "f"(xm[j]));
    float s1 = INFINITY, s2 = INFINITY;
    int i1 = 0;
#pragma unroll
    for (int c = 0; c < KM; c += 2) {
      // the scores of centres c and c + 1 together: one fma.rn.f32x2 per
      // column (each half rounds exactly as fmaf, in the same order)
      unsigned long long sp;
      asm("mov.b64 %0, {%1, %2};" : "=l"(sp) : "f"(P.nrm[c]), "f"(P.nrm[c + 1]));
#pragma unroll
      for (int j = 0; j < D; ++j) {
        unsigned long long cp;
        asm("mov.b64 %0, {%1, %2};" : "=l"(cp) : "f"(P.cm2[j][c]), "f"(P.cm2[j][c + 1]));
        asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(sp) : "l"(xx[j]), "l"(cp));
      }
      float sc[2];
      asm("mov.b64 {%0, %1}, %2;" : "=f"(sc[0]), "=f"(sc[1]) : "l"(sp));
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float s = sc[u];
        const bool lt = s < s1;
        s2 = lt ? s1 : fminf(s2, s);
        i1 = lt ? c + u : i1;
        s1 = lt ? s : s1;
      }
    }
    // |rounding error| of every score <= eps (a_max + 2 b_max ||x - m||_1)
    const float e = P.eps * (P.a_max + 2.0f * P.b_max * l1);
    if (!(s2 - s1 > 2.0f * e)) {
      // rounding could decide the order (or a value is not finite): direct
      // differences, index order, strict '<'
      float best = FLT_MAX;
      int bl = 0;
      for (int c = 0; c < P.k; ++c) {
        const float* cr = C + (long long)c * ldc;
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < D; ++j) {
          const float t = x[j] - __ldg(cr + j);
          acc = fmaf(t, t, acc);
        }
        if (acc < best) {
          best = acc;
          bl = c;
        }
      }
      i1 = bl;
    }
    __stcs(labels + r, i1);
  }
}

template <int D, int KM>
int launch_const(const float* X, long long n, const float* C_host, const float* C_dev, int ldc, int k,
                 int32_t* labels, cudaStream_t s) {
  ConstCentres<D, KM> P{};
  double m[D] = {};
  for (int c = 0; c < k; ++c)
    for (int j = 0; j < D; ++j) m[j] += C_host[(size_t)c * D + j];
  for (int j = 0; j < D; ++j) P.m[j] = (float)(m[j] / k);
  double a_max = 0.0, b_max = 0.0;
  for (int c = 0; c < KM; ++c) {
    if (c >= k) {
      P.nrm[c] = INFINITY;
      for (int j = 0; j < D; ++j) P.cm2[j][c] = 0.0f;
      continue;
    }
    // the kernel's offset is the float P.m; c - m is exact in float64
    double nrm = 0.0;
    for (int j = 0; j < D; ++j) {
      const double t = (double)C_host[(size_t)c * D + j] - (double)P.m[j];
      P.cm2[j][c] = (float)(-2.0 * t);
      nrm += t * t;
      b_max = std::max(b_max, std::fabs(t));
    }
    P.nrm[c] = (float)nrm;
    a_max = std::max(a_max, nrm);
  }
  // x - m (rounded), then D FMAs on top of the rounded ||c - m||^2, each of
  // relative error 2^-24 on terms bounded by a_max + 2 b_max |x - m|_1;
  // rounding of -2 (c - m) and of ||c - m||^2 adds two more; x 1.5 margin
  P.a_max = (float)a_max;
  P.b_max = (float)(b_max * (1.0 + 1e-6));
  P.eps = (float)(1.5 * (D + 4) * std::ldexp(1.0, -24));
  P.k = k;
  const int threads = 256;
  const int blocks = (int)std::max(1LL, std::min((n + threads - 1) / threads, (long long)sm_count() * 8));
  assign_const_kernel<D, KM><<<blocks, threads, 0, s>>>(X, n, P, C_dev, ldc, labels);
  return check_launch("assign_const_kernel");
}

}  // namespace

// Labels of n rows of X (n x d, ld == d, device) against k centres given on
// the host (C_host, k x d row-major) and on the device (C_dev, k x ldc). Sets
// *used = false (and launches nothing) when (d, k) has no specialisation.
int launch_assign_const(const float* X, int ld, long long n, int d, const float* C_host, const float* C_dev, int ldc,
                        int k, int32_t* labels, cudaStream_t s, bool* used) {
  *used = false;
  if (ld != d || !C_host || k < 1) return OK;
  for (long long i = 0; i < (long long)k * d; ++i)
    if (!std::isfinite(C_host[i])) return OK;  // non-finite centres: the generic kernels report them
  int rc = OK;
  if (d == 8 && k <= 16) rc = launch_const<8, 16>(X, n, C_host, C_dev, ldc, k, labels, s);
  else if (d == 8 && k <= 32) rc = launch_const<8, 32>(X, n, C_host, C_dev, ldc, k, labels, s);
  else if (d == 4 && k <= 16) rc = launch_const<4, 16>(X, n, C_host, C_dev, ldc, k, labels, s);
  else if (d == 4 && k <= 32) rc = launch_const<4, 32>(X, n, C_host, C_dev, ldc, k, labels, s);
  else if (d == 16 && k <= 16) rc = launch_const<16, 16>(X, n, C_host, C_dev, ldc, k, labels, s);
  else return OK;
  *used = rc == OK;
  return rc;
}

}  // namespace skm
