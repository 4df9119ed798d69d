// k-means++ seeding on the device: scikit-learn's greedy k-means++
// (sklearn/cluster/_kmeans.py, _kmeans_plusplus; reached from the
// reference's KMeans on this platform through skmetal/estimators/
// _registry.py:50-51), with the caller's random stream.
//
// The host draws what scikit-learn draws from its RandomState, in the same
// order: the first centre (random_state.choice over w / sum(w)) and, for every
// further centre, n_local_trials uniforms. Everything that touches the rows
// runs here, once per centre:
//   * pp_trial_kernel: for every row and every candidate t, the squared
//     distance formed as scikit-learn's float32 path forms it (float64:
//     (-2 x.c_t + |c_t|^2) + |x|^2, rounded to float32, then max(., 0)), the
//     new closest distance min(closest, d_t), written out per candidate, and
//     per-chunk float64 sums of w * new (fixed order within a chunk of 2048
//     rows);
//   * pp_pick_kernel (one block): each candidate's potential as the ordered
//     sum of its chunk sums, the first candidate of smallest potential (as
//     np.argmin), the chosen row as the next centre, then the next centre's
//     candidates: targets u_t * pot, the first chunk whose inclusive prefix
//     reaches a target, and inside that chunk the first row whose running
//     sum reaches it (np.searchsorted, left side; clipped to n - 1).
// Rows are centred on the fly (x - mean in float32, the fit's centring), so
// the centres are those scikit-learn draws from its centred copy of X; the
// returned rows are the raw rows. The cumulative sum and the potentials are
// float64 here; scikit-learn accumulates both in float32 (np.cumsum of a
// float32 array, a float32 matrix-vector product), so on large inputs its
// candidate rows can differ by a few positions.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "driver.h"
#include "kernels.cuh"

namespace skm {

namespace {

constexpr int PP_CHUNK = 2048;   // rows per partial sum
constexpr int PP_THREADS = 256;  // trial kernel
constexpr int PP_PICK_THREADS = 1024;

// block-wide float64 sum in a fixed order (warp xor trees, then warp 0 over the warps)
__device__ double block_sum_fixed(double v, double* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  double r = 0.0;
  if (warp == 0) {
    r = lane < nw ? sh[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  }
  __syncthreads();
  if (threadIdx.x == 0) sh[0] = r;
  __syncthreads();
  r = sh[0];
  __syncthreads();
  return r;
}

struct TrialArgs {
  const float* X;  // n x ld raw rows
  int ld, d, T;
  long long n;
  const float* mean;  // nullable
  const float* w;     // nullable: unit weights
  const int* cand;    // T candidate rows
  const float* closest_base;  // nullable (first centre): closest = closest_base + (*best) * n
  const int* best;
  float* out;     // T x n new closest distances
  double* part;   // T x n_chunks
  int n_chunks;
};

__global__ void __launch_bounds__(PP_THREADS) pp_trial_kernel(TrialArgs a) {
  extern __shared__ __align__(16) double pp_sm[];
  double* cs = pp_sm;                      // T x d centred candidate rows (float64)
  double* cc = cs + (size_t)a.T * a.d;     // T norms
  double* red = cc + a.T;                  // 32 reduction slots
  for (int i = threadIdx.x; i < a.T * a.d; i += blockDim.x) {
    const int t = i / a.d, j = i - t * a.d;
    float v = a.X[(long long)a.cand[t] * a.ld + j];
    if (a.mean) v = v - a.mean[j];
    cs[i] = (double)v;
  }
  __syncthreads();
  if (threadIdx.x < a.T) {
    double s = 0.0;
    for (int j = 0; j < a.d; ++j) s = fma(cs[threadIdx.x * a.d + j], cs[threadIdx.x * a.d + j], s);
    cc[threadIdx.x] = s;
  }
  __syncthreads();
  const float* closest = a.closest_base ? a.closest_base + (long long)(*a.best) * a.n : nullptr;
  constexpr int MAXT = 16;
  for (int ch = blockIdx.x; ch < a.n_chunks; ch += gridDim.x) {
    double psum[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) psum[t] = 0.0;
    for (int m = 0; m < PP_CHUNK / PP_THREADS; ++m) {
      const long long r = (long long)ch * PP_CHUNK + m * PP_THREADS + threadIdx.x;
      if (r >= a.n) break;
      const float* xr = a.X + r * a.ld;
      double dot[MAXT];
#pragma unroll
      for (int t = 0; t < MAXT; ++t) dot[t] = 0.0;
      double yy = 0.0;
      for (int j = 0; j < a.d; ++j) {
        float v = xr[j];
        if (a.mean) v = v - a.mean[j];
        const double x = (double)v;
        yy = fma(x, x, yy);
#pragma unroll
        for (int t = 0; t < MAXT; ++t)
          if (t < a.T) dot[t] = fma(x, cs[t * a.d + j], dot[t]);
      }
      const float cl = closest ? closest[r] : INFINITY;
      const double wr = a.w ? (double)a.w[r] : 1.0;
#pragma unroll
      for (int t = 0; t < MAXT; ++t) {
        if (t < a.T) {
          double dd = -2.0 * dot[t];
          dd += cc[t];
          dd += yy;
          float df = (float)dd;
          df = df > 0.f ? df : 0.f;         // np.maximum(d, 0)
          const float nw = cl < df ? cl : df;  // np.minimum(closest, d)
          a.out[(long long)t * a.n + r] = nw;
          psum[t] += wr * (double)nw;
        }
      }
    }
    for (int t = 0; t < a.T; ++t) {
      const double s = block_sum_fixed(psum[t], red);
      if (threadIdx.x == 0) a.part[(long long)t * a.n_chunks + ch] = s;
    }
  }
}

struct PickArgs {
  const float* X;
  int ld, d, T, T_next;
  long long n;
  const float* w;
  const float* news;   // T x n new closest distances of this centre's candidates
  const double* part;  // T x n_chunks
  int n_chunks;
  int* cand;           // in: this centre's candidates; out: the next centre's
  int* best;           // out: index of the chosen candidate
  double* prefix;      // n_chunks scratch
  const double* u;     // T_next uniforms of the next centre (nullable: last centre)
  float* centers;      // k x d raw rows
  long long* indices;  // k
  int c;               // this centre
};

__global__ void __launch_bounds__(PP_PICK_THREADS) pp_pick_kernel(PickArgs a) {
  __shared__ double red[32];
  __shared__ double pots[16];
  __shared__ double wtot[32];
  __shared__ int best_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // potentials: thread i sums chunks i, i + B, ... in order, then a fixed tree
  for (int t = 0; t < a.T; ++t) {
    double s = 0.0;
    for (int b = tid; b < a.n_chunks; b += blockDim.x) s += a.part[(long long)t * a.n_chunks + b];
    s = block_sum_fixed(s, red);
    if (tid == 0) pots[t] = s;
  }
  __syncthreads();
  if (tid == 0) {
    int bt = 0;
    for (int t = 1; t < a.T; ++t)
      if (pots[t] < pots[bt]) bt = t;  // np.argmin: the first smallest
    best_s = bt;
    *a.best = bt;
  }
  __syncthreads();
  const int bt = best_s;
  const long long row = a.cand[bt];
  for (int j = tid; j < a.d; j += blockDim.x) a.centers[(long long)a.c * a.d + j] = a.X[row * a.ld + j];
  if (tid == 0) a.indices[a.c] = row;
  if (!a.u) return;
  // inclusive prefix of the chosen candidate's chunk sums: contiguous ranges per thread
  const double* pb = a.part + (long long)bt * a.n_chunks;
  const int per = (a.n_chunks + blockDim.x - 1) / blockDim.x;
  const int b0 = tid * per, b1 = min(a.n_chunks, b0 + per);
  double loc = 0.0;
  for (int b = b0; b < b1; ++b) loc += pb[b];
  // exclusive scan of the thread totals: warps, then warp totals (fixed order)
  double incl = loc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wtot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    double v = lane < (int)(blockDim.x >> 5) ? wtot[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double x = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += x;
    }
    wtot[lane] = v;  // inclusive over warps
  }
  __syncthreads();
  double run = (warp > 0 ? wtot[warp - 1] : 0.0) + (incl - loc);
  for (int b = b0; b < b1; ++b) {
    run += pb[b];
    a.prefix[b] = run;
  }
  __syncthreads();
  const double pot = pots[bt];
  const float* nb = a.news + (long long)bt * a.n;
  // one warp per target
  for (int t = warp; t < a.T_next; t += blockDim.x >> 5) {
    const double target = a.u[t] * pot;
    // first chunk whose inclusive prefix reaches the target
    int lo = 0, hi = a.n_chunks;  // answer in [lo, hi]; hi = n_chunks: none
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (a.prefix[mid] >= target) hi = mid;
      else lo = mid + 1;
    }
    long long pick;
    if (lo >= a.n_chunks) {
      pick = a.n - 1;  // beyond the total (np.clip to n - 1)
    } else {
      const long long r0 = (long long)lo * PP_CHUNK;
      const long long r1 = min(a.n, r0 + PP_CHUNK);
      const double base = lo > 0 ? a.prefix[lo - 1] : 0.0;
      // lane l walks rows r0 + 64 l .. r0 + 64 l + 63 from its running prefix
      const long long l0 = r0 + 64LL * lane, l1 = min(r1, l0 + 64);
      double ls = 0.0;
      for (long long r = l0; r < l1; ++r) ls += (a.w ? (double)a.w[r] : 1.0) * (double)nb[r];
      double inc = ls;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
      }
      double s = base + (inc - ls);
      long long hit = -1;
      for (long long r = l0; r < l1; ++r) {
        s += (a.w ? (double)a.w[r] : 1.0) * (double)nb[r];
        if (s >= target) {
          hit = r;
          break;
        }
      }
      const unsigned int m = __ballot_sync(0xffffffffu, hit >= 0);
      if (m) {
        pick = __shfl_sync(0xffffffffu, hit, __ffs(m) - 1);
      } else {
        pick = r1 - 1;  // the chunk's prefix reached the target: its last row
      }
    }
    if (lane == 0) a.cand[t] = (int)pick;
  }
}

}  // namespace

size_t kmeanspp_scratch_bytes(long long n, int T) {
  const long long n_chunks = (n + PP_CHUNK - 1) / PP_CHUNK;
  return 2 * (size_t)T * n * sizeof(float) + (size_t)T * n_chunks * sizeof(double) +
         (size_t)n_chunks * sizeof(double) + 64 * sizeof(int);
}

// Seeds k centres from X (n rows of d at stride ld, raw; mean nullable) on
// stream s. u: (k - 1) x T uniforms on the device; w nullable; scratch of
// kmeanspp_scratch_bytes(n, T) bytes; centers (k x d) and indices (k) on the
// device.
int kmeanspp_device(const float* X, int ld, long long n, int d, int k, const float* mean, const float* w,
                    long long first, const double* u, int T, void* scratch, float* centers, long long* indices,
                    cudaStream_t s) {
  if (T < 1 || T > 16 || (long long)T * d > 8192 || n < 1 || first < 0 || first >= n) {
    set_error(ERR_INVALID, "kmeans_plusplus: unsupported n_local_trials=%d, d=%d, or first row", T, d);
    return ERR_INVALID;
  }
  const int n_chunks = (int)((n + PP_CHUNK - 1) / PP_CHUNK);
  float* news = reinterpret_cast<float*>(scratch);            // 2 sets of T x n
  double* part = reinterpret_cast<double*>(news + 2 * (size_t)T * n);
  double* prefix = part + (size_t)T * n_chunks;
  int* cand = reinterpret_cast<int*>(prefix + n_chunks);      // 16 entries
  int* best = cand + 32;
  const int first_i = (int)first;
  SKM_CUDA(cudaMemcpyAsync(cand, &first_i, sizeof(int), cudaMemcpyHostToDevice, s));
  SKM_CUDA(cudaMemsetAsync(best, 0, sizeof(int), s));
  const size_t trial_smem = sizeof(double) * ((size_t)T * d + T + 32);
  if (trial_smem > 48 * 1024)
    SKM_CUDA(cudaFuncSetAttribute(pp_trial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)trial_smem));
  const int grid = std::max(1, std::min(n_chunks, sm_count() * 8));
  for (int c = 0; c < k; ++c) {
    const int Tc = c == 0 ? 1 : T;
    float* out = news + (size_t)(c & 1) * T * n;
    TrialArgs ta{X, ld, d, Tc, n, mean, w, cand,
                 c == 0 ? nullptr : news + (size_t)((c - 1) & 1) * T * n, best, out, part, n_chunks};
    pp_trial_kernel<<<grid, PP_THREADS, trial_smem, s>>>(ta);
    SKM_TRY(check_launch("pp_trial_kernel"));
    PickArgs pa{X, ld, d, Tc, T, n, w, out, part, n_chunks, cand, best, prefix,
                c + 1 < k ? u + (size_t)c * T : nullptr, centers, indices, c};
    pp_pick_kernel<<<1, PP_PICK_THREADS, 0, s>>>(pa);
    SKM_TRY(check_launch("pp_pick_kernel"));
  }
  return OK;
}

}  // namespace skm
