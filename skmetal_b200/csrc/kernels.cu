// SIMT kernels of the KMeans Lloyd path: data preparation (mean, centring,
// scales), the direct-difference assignment used for predict and for small
// shapes, the bulk fixed-point centroid sums, the M-step (relocation, average,
// shift, convergence) and the inertia / distance outputs.
//
// Semantics follow scikit-learn 1.9.0's Lloyd, which is what the reference's
// accelerate(KMeans) runs off Apple hardware:
//   argmin with strict '<', first index wins  (_k_means_lloyd.pyx:205-213)
//   relocation of empty clusters              (_k_means_common.pyx:167-211)
//   averaging, empty -> heaviest cluster      (_k_means_common.pyx:274-295)
//   centre shift                              (_k_means_common.pyx:298-311)
//   strict convergence / tol / max_iter       (_kmeans.py:705-758)
#include "kernels.cuh"
#include "device_util.cuh"
#include "mstep_dev.cuh"

#include <cfloat>
#include <cmath>

namespace skm {


// ---------------------------------------------------------------------------
// data preparation
// ---------------------------------------------------------------------------

// The padding columns [d, ld) of X are zero and the mean is zero there, so
// the elementwise passes below run over the whole row-major buffer as float4
// (ld is a multiple of 4) without masking. A thread that needs the column of
// its float4 keeps c4 = i mod (ld/4) updated by addition instead of division.

// max |x| (float bits; |x| >= 0 so unsigned order = float order)
__global__ void maxabs_kernel(const float* __restrict__ X, int ld, long long n, int d,
                              unsigned int* __restrict__ out_bits) {
  (void)d;
  const float4* X4 = reinterpret_cast<const float4*>(X);
  const long long total = n * (long long)(ld >> 2);
  unsigned int m = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 v = __ldcs(X4 + i);
    m = max(m, __float_as_uint(v.x) & 0x7fffffffu);
    m = max(m, __float_as_uint(v.y) & 0x7fffffffu);
    m = max(m, __float_as_uint(v.z) & 0x7fffffffu);
    m = max(m, __float_as_uint(v.w) & 0x7fffffffu);
  }
  m = min(m, 0x7f800000u);  // NaN counts as +inf (rejected by the host)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out_bits, m);
}

// Column sums of X in fixed point (exact): colsum[j] = sum_r round(x_rj * scale).
// blockDim = q * g with q = ld / 4: thread t owns column group t % q and the
// rows r = (block, t / q) strided, so its four int64 partials stay in
// registers; partials meet in shared memory (integer atomics, exact).
__global__ void colsum_fixed_kernel(const float* __restrict__ X, int ld, long long n, int d,
                                    const double* __restrict__ scale_ptr, long long* __restrict__ colsum) {
  extern __shared__ long long cs_acc[];
  (void)d;
  const double scale = *scale_ptr;
  const int q = ld >> 2;
  const int g = blockDim.x / q;
  const int c4 = threadIdx.x % q, rg = threadIdx.x / q;
  const float4* X4 = reinterpret_cast<const float4*>(X);
  long long a0 = 0, a1 = 0, a2 = 0, a3 = 0;
  if (g == 0) {
    // more column groups than threads: one thread per column group, straight
    // to global memory
    for (int cc = threadIdx.x; cc < q; cc += blockDim.x) {
      long long b0 = 0, b1 = 0, b2 = 0, b3 = 0;
      for (long long r = blockIdx.x; r < n; r += gridDim.x) {
        const float4 v = __ldcs(X4 + r * q + cc);
        b0 += to_fixed(v.x, scale);
        b1 += to_fixed(v.y, scale);
        b2 += to_fixed(v.z, scale);
        b3 += to_fixed(v.w, scale);
      }
      red_add_s64(&colsum[4 * cc + 0], b0);
      red_add_s64(&colsum[4 * cc + 1], b1);
      red_add_s64(&colsum[4 * cc + 2], b2);
      red_add_s64(&colsum[4 * cc + 3], b3);
    }
    return;
  }
  if (rg < g) {
    for (long long r = (long long)blockIdx.x * g + rg; r < n; r += (long long)gridDim.x * g) {
      const float4 v = __ldcs(X4 + r * q + c4);
      a0 += to_fixed(v.x, scale);
      a1 += to_fixed(v.y, scale);
      a2 += to_fixed(v.z, scale);
      a3 += to_fixed(v.w, scale);
    }
  }
  for (int i = threadIdx.x; i < ld; i += blockDim.x) cs_acc[i] = 0;
  block_sync();
  if (rg < g) {
    atomicAdd(reinterpret_cast<unsigned long long*>(&cs_acc[4 * c4 + 0]), (unsigned long long)a0);
    atomicAdd(reinterpret_cast<unsigned long long*>(&cs_acc[4 * c4 + 1]), (unsigned long long)a1);
    atomicAdd(reinterpret_cast<unsigned long long*>(&cs_acc[4 * c4 + 2]), (unsigned long long)a2);
    atomicAdd(reinterpret_cast<unsigned long long*>(&cs_acc[4 * c4 + 3]), (unsigned long long)a3);
  }
  block_sync();
  for (int i = threadIdx.x; i < ld; i += blockDim.x)
    if (cs_acc[i] != 0) red_add_s64(&colsum[i], cs_acc[i]);
}

// mean[j] = colsum[j] * inv_scale / n (float32; zero in the padding)
__global__ void mean_from_colsum_kernel(const long long* __restrict__ colsum, int d, const double* __restrict__ scale_ptr,
                                        double n_total, float* __restrict__ mean) {
  const double inv_scale = 1.0 / *scale_ptr;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < d; j += gridDim.x * blockDim.x)
    mean[j] = (float)((double)colsum[j] * inv_scale / n_total);
}

// X -= mean (float32, in place), max |x - mean|, and per-block float64
// partials of sum (x - mean)^2 (for the scaled tolerance) when `partial`.
__global__ void center_kernel(float* __restrict__ X, int ld, long long n, int d, const float* __restrict__ mean,
                              unsigned int* __restrict__ maxabs_bits, double* __restrict__ partial) {
  __shared__ double scratch[32];
  (void)d;
  float4* X4 = reinterpret_cast<float4*>(X);
  const int q = ld >> 2;
  const long long total = n * (long long)q;
  const long long start = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int sq = (int)(stride % q);
  int c4 = (int)(start % q);
  const float4* M4 = reinterpret_cast<const float4*>(mean);
  unsigned int m = 0;
  double ss = 0.0;
  for (long long i = start; i < total; i += stride) {
    float4 v = X4[i];
    const float4 mu = M4[c4];
    v.x -= mu.x;
    v.y -= mu.y;
    v.z -= mu.z;
    v.w -= mu.w;
    X4[i] = v;
    m = max(m, max(max(__float_as_uint(v.x) & 0x7fffffffu, __float_as_uint(v.y) & 0x7fffffffu),
                   max(__float_as_uint(v.z) & 0x7fffffffu, __float_as_uint(v.w) & 0x7fffffffu)));
    ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    c4 += sq;
    if (c4 >= q) c4 -= q;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && maxabs_bits) atomicMax(maxabs_bits, m);
  if (partial) {
    ss = block_sum_f64(ss, scratch);
    if (threadIdx.x == 0) partial[blockIdx.x] = ss;
  }
}

// Blocked working copy of X (layout: see xblk_index): out = raw - mean (or
// raw when mean is null), zero in padding rows; also max |out| and per-block
// float64 partials of sum out^2 (when `partial`). Threads walk the blocked
// output in order (consecutive threads write consecutive 16-byte rows of a
// quad), so the writes are coalesced and each raw row is read as 16-byte
// pieces that neighbouring warps share through L1/L2.
__global__ void center_block_kernel(const float* __restrict__ raw, int ld, long long n, int d,
                                    const float* __restrict__ mean, float* __restrict__ out,
                                    unsigned int* __restrict__ maxabs_bits, double* __restrict__ partial) {
  __shared__ double scratch[32];
  (void)d;
  const int q4 = ld >> 2;  // quads per row
  const long long n_pad = (n + 127) / 128 * 128;
  const long long total = n_pad * q4;  // float4 elements
  const float4* R4 = reinterpret_cast<const float4*>(raw);
  float4* O4 = reinterpret_cast<float4*>(out);
  const float4* M4 = reinterpret_cast<const float4*>(mean);
  unsigned int m = 0;
  double ss = 0.0;
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < total;
       g += (long long)gridDim.x * blockDim.x) {
    // g = (tile * q4 + q) * 128 + rr
    const long long tq = g >> 7;
    const int rr = (int)(g & 127);
    const long long t = tq / q4;
    const int q = (int)(tq - t * q4);
    const long long r = t * 128 + rr;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < n) {
      v = __ldg(R4 + r * q4 + q);
      if (mean) {
        const float4 mu = M4[q];
        v.x -= mu.x;
        v.y -= mu.y;
        v.z -= mu.z;
        v.w -= mu.w;
      }
    }
    O4[g] = v;
    m = max(m, max(max(__float_as_uint(v.x) & 0x7fffffffu, __float_as_uint(v.y) & 0x7fffffffu),
                   max(__float_as_uint(v.z) & 0x7fffffffu, __float_as_uint(v.w) & 0x7fffffffu)));
    ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  m = min(m, 0x7f800000u);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && maxabs_bits) atomicMax(maxabs_bits, m);
  if (partial) {
    ss = block_sum_f64(ss, scratch);
    if (threadIdx.x == 0) partial[blockIdx.x] = ss;
  }
}

// Per-block float64 partials of sum x^2 (uncentred fits with a relative tolerance).
__global__ void sumsq_partial_kernel(const float* __restrict__ X, int ld, long long n, int d,
                                     double* __restrict__ partial) {
  __shared__ double scratch[32];
  (void)d;
  const float4* X4 = reinterpret_cast<const float4*>(X);
  const long long total = n * (long long)(ld >> 2);
  double ss = 0.0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 v = X4[i];
    ss += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  ss = block_sum_f64(ss, scratch);
  if (threadIdx.x == 0) partial[blockIdx.x] = ss;
}

// Fixed-point scale 2^F for sums of up to n_total values bounded by the max |x|
// recorded in maxabs_bits: F = 62 - E - L with max < 2^E and n_total <= 2^L,
// so no partial or total sum can reach 2^62.
__device__ double fixed_scale(unsigned int maxabs_bits, double n_total) {
  const float mx = __uint_as_float(maxabs_bits);
  int E = -60;
  if (mx > 0.0f) frexp((double)mx, &E);
  int L = 0;
  frexp(fmax(n_total, 1.0), &L);  // n_total < 2^L
  int F = 62 - E - L;
  F = max(-1000, min(1000, F));
  return ldexp(1.0, F);
}

__global__ void scale_kernel(const unsigned int* __restrict__ maxabs_bits, double n_total, double* __restrict__ out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *out = fixed_scale(*maxabs_bits, n_total);
}

// Initialise the fit state. tol_mode 0: `tol` is already absolute; 1: `tol` is
// relative and is scaled by the mean column variance sumsq / (n_total * d).
__global__ void init_state_kernel(FitState* st, int max_iter, double tol, int tol_mode, const double* sumsq,
                                  double n_total, int d, const unsigned int* maxabs_bits, int bulk_always,
                                  const float* w, const unsigned int* wmax_bits, int bulk_divisor) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  st->iter = 0;
  st->done = max_iter <= 0;
  st->strict = 0;
  st->max_iter = max_iter;
  st->n_empty = 0;
  st->relocated = 0;
  st->error = 0;
  st->full_update = 1;
  st->changed = 0;
  st->sel_count = 0;
  st->barrier_count = 0;
  st->ticket = 0;
  st->barrier_gen = 0;
  st->shift_tot = 0.0;
  st->inertia = 0.0;
  double t = tol;
  if (tol_mode == 1) t = (tol == 0.0 || sumsq == nullptr) ? 0.0 : (*sumsq / (n_total * (double)d)) * tol;
  st->tol = t;
  st->maxabs_bits = *maxabs_bits;
  st->bulk = 1;  // the first iteration starts from labels -1: every row changes
  st->bulk_always = bulk_always;
  st->bulk_threshold = (long long)fmax(1.0, n_total / (double)bulk_divisor);
  st->xexp = split_exp(*maxabs_bits);
  st->cexp = st->xexp;
  // weighted fits: the sums hold w * x (wmax_bits[0] = max |w x|) and the
  // cluster weights w (wmax_bits[1] = max w), each with its own scale
  st->w = w;
  st->scale = fixed_scale(w ? wmax_bits[0] : *maxabs_bits, n_total);
  st->wscale = w ? fixed_scale(wmax_bits[1], n_total) : 1.0;
  st->inv_scale = st->wscale / st->scale;
}

// max |w_r x_rj| (float32 products, as the sums take them) and max w_r over
// the rows of the blocked copy, as float bits (non-negative values order as
// their bits); atomicMax into out[0], out[1]
__global__ void weight_max_kernel(const float* __restrict__ X, int ld, long long n, const float* __restrict__ w,
                                  unsigned int* __restrict__ out) {
  unsigned int mx = 0u, mw = 0u;
  for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < n; r += (long long)gridDim.x * blockDim.x) {
    const float wr = w[r];
    mw = max(mw, __float_as_uint(fabsf(wr)));
    for (int j = 0; j < ld; ++j) mx = max(mx, __float_as_uint(fabsf(X[xblk_index(r, j, ld)] * wr)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mw = max(mw, __shfl_xor_sync(0xffffffffu, mw, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMax(out, mx);
    atomicMax(out + 1, mw);
  }
}

// centres: C[c][j] = init[c][j] - mean[j] for j < d, 0 in the padding
__global__ void center_init_kernel(const float* __restrict__ init, int d, int k, const float* __restrict__ mean,
                                   float* __restrict__ C, int ld) {
  const int total = k * ld;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int c = i / ld, j = i % ld;
    C[i] = j < d ? (mean ? init[c * d + j] - mean[j] : init[c * d + j]) : 0.0f;
  }
}

// ---------------------------------------------------------------------------
// assignment (direct differences, float32): labels, min distance, change count
// ---------------------------------------------------------------------------

// Generic kernel: one thread per row, centres staged through shared memory.
__global__ void assign_simt_kernel(const float* __restrict__ X, int ld, long long n, int d,
                                   const float* __restrict__ C, int k,
                                   int32_t* __restrict__ labels, float* __restrict__ mind,
                                   const FitState* __restrict__ st, unsigned long long* __restrict__ changed,
                                   long long* __restrict__ D, int skip_if_strict, int blocked) {
  extern __shared__ float csh[];
  if (st) {
    if (skip_if_strict ? (st->strict != 0) : (st->done != 0)) return;
  }
  const int chunk = max(1, min(k, (int)(kAssignSmemFloats / ld)));
  const long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const bool active = r < n;
  // blocked X: quad q of the row at xr + 512 q; row-major: at xr + 4 q
  const float* xr = blocked ? X + xblk_index(active ? r : 0, 0, ld) : X + (active ? r : 0) * ld;
  const int qstride = blocked ? 512 : 4;
  float best = FLT_MAX;
  int bl = 0;
  for (int c0 = 0; c0 < k; c0 += chunk) {
    const int cn = min(chunk, k - c0);
    block_sync();
    for (int i = threadIdx.x; i < cn * ld; i += blockDim.x) csh[i] = C[(long long)c0 * ld + i];
    block_sync();
    if (active) {
      for (int c = 0; c < cn; ++c) {
        const float* cr = csh + c * ld;
        float acc = 0.0f;
        int j = 0;
        for (; j + 4 <= d; j += 4) {
          const float4 xv = *reinterpret_cast<const float4*>(xr + (j >> 2) * qstride);
          const float d0 = xv.x - cr[j], d1 = xv.y - cr[j + 1], d2 = xv.z - cr[j + 2], d3 = xv.w - cr[j + 3];
          acc = fmaf(d0, d0, acc);
          acc = fmaf(d1, d1, acc);
          acc = fmaf(d2, d2, acc);
          acc = fmaf(d3, d3, acc);
        }
        for (; j < d; ++j) {
          const float t = xr[(j >> 2) * qstride + (j & 3)] - cr[j];
          acc = fmaf(t, t, acc);
        }
        if (acc < best) {
          best = acc;
          bl = c0 + c;
        }
      }
    }
  }
  bool ch = false;
  int old = -1;
  if (active) {
    if (changed) {
      old = labels[r];
      ch = old != bl;
    }
    labels[r] = bl;
    if (mind) mind[r] = best;
  }
  if (changed) {
    const unsigned int b = __ballot_sync(0xffffffffu, ch);
    if ((threadIdx.x & 31) == 0 && b) atomicAdd(changed, (unsigned long long)__popc(b));
    if (D && !st->bulk) warp_apply_changed(X, ld, d, k, r, old, bl, ch, D, st);
  }
}

// Small-d specialisation: the row lives in registers, all centres in shared memory.
template <int D>
__global__ void assign_small_kernel(const float* __restrict__ X, int ld, long long n,
                                    const float* __restrict__ C, int k,
                                    int32_t* __restrict__ labels, float* __restrict__ mind) {
  extern __shared__ float csh[];
  for (int i = threadIdx.x; i < k * D; i += blockDim.x) csh[i] = C[(i / D) * ld + (i % D)];
  block_sync();
  for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < n;
       r += (long long)gridDim.x * blockDim.x) {
    float x[D];
#pragma unroll
    for (int j = 0; j < D; j += 4) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(X + r * ld + j));
      x[j] = v.x; x[j + 1] = v.y; x[j + 2] = v.z; x[j + 3] = v.w;
    }
    float best = FLT_MAX;
    int bl = 0;
    for (int c = 0; c < k; ++c) {
      float acc = 0.0f;
#pragma unroll
      for (int j = 0; j < D; ++j) {
        const float t = x[j] - csh[c * D + j];
        acc = fmaf(t, t, acc);
      }
      if (acc < best) { best = acc; bl = c; }
    }
    __stcs(labels + r, bl);
    if (mind) mind[r] = best;
  }
}

bool launch_assign_small(int d, int blocks, int threads, size_t smem, cudaStream_t s, const float* X, int ld,
                         long long n, const float* C, int k, int32_t* labels, float* mind) {
  switch (d) {
    case 4: assign_small_kernel<4><<<blocks, threads, smem, s>>>(X, ld, n, C, k, labels, mind); return true;
    case 8: assign_small_kernel<8><<<blocks, threads, smem, s>>>(X, ld, n, C, k, labels, mind); return true;
    case 16: assign_small_kernel<16><<<blocks, threads, smem, s>>>(X, ld, n, C, k, labels, mind); return true;
    case 32: assign_small_kernel<32><<<blocks, threads, smem, s>>>(X, ld, n, C, k, labels, mind); return true;
    default: return false;
  }
}


__global__ void __launch_bounds__(1024, 1) mstep_kernel(MStepArgs a) {
  pdl_launch_dependents();
  pdl_wait();  // the E-step's labels, deltas and counters
  FitState* st = a.st;
  const unsigned int nb = gridDim.x;
  const long long ks = (long long)a.k * a.ld;
  const long long* dcnt = a.D + ks;
  const int done = st->done;  // uniform: `done` is only written at the very end
  const unsigned long long changed_now = *a.changed;  // cleared at the end
  const int bulk = st->bulk;  // D holds the sums of all rows (replace S), not deltas
  if (done) return;
  extern __shared__ __align__(16) long long dyn_smem[];
  if (bulk && !a.bulk_external) {
    bulk_pass(a.X, a.ld, a.n, a.labels, a.k, a.D, st, reinterpret_cast<unsigned char*>(dyn_smem),
              mstep_smem_bytes(a.k, a.ld), &st->error);
    if (!grid_barrier(st, nb)) return;
  }
  // 1. empty clusters of the new assignment; every block computes the same answer
  const int n_empty = find_empty_clusters(a, bulk);

  if (n_empty == 0) {
    // ---------------- fast path: no relocation. One warp per cluster folds
    // its sums (S + D; bulk: D) and writes its centre; the last block to
    // finish folds the counts, totals the shifts in the canonical order and
    // sets the loop flags.
    const double inv_scale = st->inv_scale;
    const float cs = ldexpf(1.0f, st->xexp);  // centres are bounded by max |x|
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    long long* S = const_cast<long long*>(a.S);
    long long* cnt = const_cast<long long*>(a.counts);
    double* dsq_c = a.shift_partial;  // k entries
    for (int c = blockIdx.x * nwarps + warp; c < a.k; c += nb * nwarps) {
      const long long dcc = __ldcg(&dcnt[c]);
      const long long cnew = (bulk ? 0 : __ldcg(&cnt[c])) + dcc;
      double dsq, nrm;
      warp_centre_from_sums(c, a.ld, a.d, S, a.D, bulk, cnew, inv_scale, a.C_old, cs, a.cimg, CentreImage{}, S,
                            a.C_new, a.D, &dsq, &nrm);
      if (lane == 0) {
        dsq_c[c] = dsq;
        if (a.shift_out) a.shift_out[c] = (float)sqrt(dsq);
        if (a.bias) a.bias[c] = (float)nrm;
      }
    }
    // the last block to get here folds the counts (every block has read them
    // in find_empty_clusters by now), totals the shifts and finishes the
    // iteration
    __shared__ int last_s;
    block_sync();
    if (threadIdx.x == 0) {
      __threadfence();
      last_s = atomicAdd(&st->ticket, 1u) == nb - 1;
    }
    block_sync();
    if (!last_s) return;
    __threadfence();
    for (int c = threadIdx.x; c < a.k; c += blockDim.x) {
      const long long dcc = __ldcg(&dcnt[c]);
      const long long cnew = (bulk ? 0 : __ldcg(&cnt[c])) + dcc;
      cnt[c] = cnew;
      a.cnt_adj[c] = cnew;
      if (dcc != 0) a.D[ks + c] = 0;
    }
    if (threadIdx.x >= 32) return;
    const double tot = warp_ordered_sum(dsq_c, a.k);
    if (threadIdx.x == 0) {
      st->ticket = 0;
      st->n_empty = 0;
      st->relocated = 0;
      finish_iteration(a, st, changed_now, tot);
    }
    return;
  }

  relocation_path(a, n_empty, bulk, changed_now);
}

// Multi-GPU fits, between the E-step and the all-reduce of the payload
// [D | one candidate slot per rank]: the bulk pass of a bulk iteration; the
// rank's own cluster counts; and, when one of them is empty after this
// iteration, the rank's farthest rows as relocation candidates in its slot.
// A cluster can only be empty globally if it is empty on every rank, so every
// rank then supplies its min(local empties, cap) farthest rows, which contain
// its share of the global farthest rows. The other ranks' slots are zeroed
// here, so the integer all-reduce delivers each rank's slot unchanged.
__global__ void __launch_bounds__(1024, 1) shard_prep_kernel(MStepArgs a, long long* local_counts, int rank) {
  FitState* st = a.st;
  const unsigned int nb = gridDim.x;
  const size_t cb = cand_block_bytes(a.cand_cap, a.ld);
  unsigned char* slots = const_cast<unsigned char*>(a.cand);
  unsigned char* mine = slots + (size_t)rank * cb;
  // every slot starts at zero (the payload's other parts are D)
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < cb * a.cand_ranks / 8;
       i += (size_t)nb * blockDim.x)
    reinterpret_cast<long long*>(slots)[i] = 0;
  if (st->done) return;
  const int bulk = st->bulk;
  extern __shared__ __align__(16) long long dyn_smem[];
  if (bulk)
    bulk_pass(a.X, a.ld, a.n, a.labels, a.k, a.D, st, reinterpret_cast<unsigned char*>(dyn_smem),
              mstep_smem_bytes(a.k, a.ld), &st->error);
  if (!grid_barrier(st, nb)) return;
  // local counts after this iteration, and how many clusters this rank has empty
  const long long* dcnt = a.D + (long long)a.k * a.ld;
  int n_local_empty = 0;
  for (int c0 = 0; c0 < a.k; c0 += blockDim.x) {
    const int c = c0 + threadIdx.x;
    long long v = 0;
    if (c < a.k) v = (bulk ? 0 : local_counts[c]) + dcnt[c];
    __syncwarp();
    n_local_empty += __syncthreads_count(c < a.k && v == 0);
    if (blockIdx.x == 0 && c < a.k) a.cnt_adj[c] = v;  // staged: written back after the barrier
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) st->sel_count = 0;
  if (!grid_barrier(st, nb)) return;
  if (blockIdx.x == 0)
    for (int c = threadIdx.x; c < a.k; c += blockDim.x) local_counts[c] = a.cnt_adj[c];
  if (n_local_empty == 0) return;  // the slot's count stays 0
  const int m = (int)min((long long)min(n_local_empty, a.cand_cap), a.n);
  rows_dist_to_old_centres(a, nb);
  if (!grid_barrier(st, nb)) return;
  if (!select_farthest(a.mind, a.n, a.row_base, m, st, a.hist, a.sel, nb)) return;
  if (blockIdx.x == 0) {
    const int cap = a.cand_cap;
    float* dist = reinterpret_cast<float*>(mine + cand_dist_off(cap));
    long long* row = reinterpret_cast<long long*>(mine + cand_row_off(cap));
    int* label = reinterpret_cast<int*>(mine + cand_label_off(cap));
    float* x = reinterpret_cast<float*>(mine + cand_x_off(cap));
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
      const long long r = a.sel[i];
      dist[i] = a.mind[r];
      row[i] = a.row_base + r;
      label[i] = a.labels[r];
      for (int j = 0; j < a.ld; ++j) x[(long long)i * a.ld + j] = a.X[xblk_index(r, j, a.ld)];
    }
    if (threadIdx.x == 0) *reinterpret_cast<int*>(mine) = m;
  }
}

__global__ void counts_to_float_kernel(const long long* __restrict__ c, int k, float* __restrict__ out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < k; i += gridDim.x * blockDim.x) out[i] = (float)c[i];
}

// bias[c] = ||c||^2 (float64 sum, rounded) and the centre image of C for the
// tensor-core E-step, scaled by 2^cexp with cexp = split_exp(max |C|) (stored
// in st->cexp). One block (the initial centres of a fit, k x d is small).
__global__ void centre_prep_kernel(const float* __restrict__ C, int k, int ld, int d, float* __restrict__ bias,
                                   CentreImage ci, FitState* st) {
  if (st->done || blockIdx.x != 0) return;
  __shared__ unsigned int mx_s;
  if (threadIdx.x == 0) mx_s = 0;
  block_sync();
  unsigned int m = 0;
  for (long long i = threadIdx.x; i < (long long)k * ld; i += blockDim.x)
    if ((int)(i % ld) < d) m = max(m, __float_as_uint(C[i]) & 0x7fffffffu);
  m = min(m, 0x7f800000u);
  atomicMax(&mx_s, m);
  block_sync();
  const int cexp = split_exp(mx_s);
  const float cs = ldexpf(1.0f, cexp);
  if (threadIdx.x == 0) st->cexp = cexp;
  const int lane = threadIdx.x & 31;
  for (int c = threadIdx.x >> 5; c < k; c += blockDim.x >> 5) {
    double acc = 0.0;
    for (int j = lane; j < d; j += 32) {
      const float v = C[(long long)c * ld + j];
      acc += (double)v * v;
      if (ci.img) cimg_put(ci, c, j, v, cs);
    }
    acc = warp_sum(acc);
    if (lane == 0 && bias) bias[c] = (float)acc;
  }
}

// ---------------------------------------------------------------------------
// outputs: inertia, per-row distance to the assigned centre, transform
// ---------------------------------------------------------------------------

// Per-block float64 partial of sum_r ||x_r - c_{l_r}||^2 over a fixed
// assignment of rows to blocks (deterministic for a given grid).
// Row-major X: warp per row, lanes over columns. Blocked X: lane per row of
// a 32-row group, walking the quads (coalesced 512-byte warp loads).
__global__ void inertia_partial_kernel(const float* __restrict__ X, int ld, long long n, int d,
                                       const float* __restrict__ C, const int32_t* __restrict__ labels,
                                       double* __restrict__ partial, int blocked, const float* __restrict__ w) {
  __shared__ double scratch[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  double acc = 0.0;
  if (blocked) {
    const long long items = (n + 31) / 32;
    const float4* X4 = reinterpret_cast<const float4*>(X);
    for (long long it = (long long)blockIdx.x * nw + warp; it < items; it += (long long)gridDim.x * nw) {
      const long long r = it * 32 + lane;
      if (r >= n) continue;
      const float4* xp = X4 + (r >> 7) * (32LL * ld) + (r & 127);
      const float4* cr = reinterpret_cast<const float4*>(C + (long long)labels[r] * ld);  // ld % 4 == 0
      // four quads' loads in flight per lane; the sum stays in quad order
      double rs = 0.0;  // the row's sum, times its weight in weighted fits
#pragma unroll 4
      for (int q = 0; q < (ld >> 2); ++q) {
        const float4 v = __ldcs(xp + (long long)q * 128);
        const float4 c = __ldg(cr + q);
        const double t0 = (double)v.x - c.x, t1 = (double)v.y - c.y;
        const double t2 = (double)v.z - c.z, t3 = (double)v.w - c.w;
        rs += t0 * t0 + t1 * t1 + t2 * t2 + t3 * t3;  // padding columns are zero in X and C
      }
      acc += w ? (double)w[r] * rs : rs;
    }
  } else {
    for (long long r = (long long)blockIdx.x * nw + warp; r < n; r += (long long)gridDim.x * nw) {
      const float* xr = X + r * ld;
      const float* cr = C + (long long)labels[r] * ld;
      const double wr = w ? (double)w[r] : 1.0;
      for (int j = lane; j < d; j += 32) {
        const double t = (double)__ldcs(xr + j) - (double)cr[j];
        acc += w ? wr * (t * t) : t * t;
      }
    }
  }
  acc = block_sum_f64(acc, scratch);
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

// out = sum of partial[0..m) in a fixed order (one warp: strided lane sums,
// then a fixed butterfly)
// The labels present among n: a shared-memory bitmap per block (k bits), ORed
// into the global one word by word at the end (the distinct-cluster count of
// scikit-learn's fit, _kmeans.py:1545-1552, without a host pass over n labels).
__global__ void label_bitmap_kernel(const int32_t* __restrict__ labels, long long n, int k, unsigned int* bitmap) {
  __shared__ unsigned int sb[kLabelBitmapMaxK / 32];
  const int words = (k + 31) >> 5;
  for (int i = threadIdx.x; i < words; i += blockDim.x) sb[i] = 0;
  __syncthreads();
  for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < n; r += (long long)gridDim.x * blockDim.x) {
    const int c = labels[r];
    if ((unsigned)c < (unsigned)k) atomicOr(&sb[c >> 5], 1u << (c & 31));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < words; i += blockDim.x)
    if (sb[i]) atomicOr(&bitmap[i], sb[i]);
}

__global__ void ordered_sum_kernel(const double* __restrict__ partial, int m, double* __restrict__ out) {
  if (blockIdx.x != 0 || threadIdx.x >= 32) return;
  double t = 0.0;
  for (int i = threadIdx.x; i < m; i += 32) t += partial[i];
  t = warp_sum(t);
  if (threadIdx.x == 0) *out = t;
}

__global__ void mindist_kernel(const float* __restrict__ X, int ld, long long n, int d,
                               const float* __restrict__ C, const int32_t* __restrict__ labels,
                               float* __restrict__ out) {
  for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < n;
       r += (long long)gridDim.x * blockDim.x) {
    const float* xr = X + r * ld;
    const float* cr = C + (long long)labels[r] * ld;
    float s = 0.0f;
    for (int j = 0; j < d; ++j) {
      const float t = xr[j] - cr[j];
      s = fmaf(t, t, s);
    }
    out[r] = s;
  }
}

// D[r][c] = sqrt(sum_j (x_rj - c_cj)^2), accumulated in float64
__global__ void transform_kernel(const float* __restrict__ X, int ld, long long n, int d,
                                 const float* __restrict__ C, int k, float* __restrict__ D) {
  const long long total = n * (long long)k;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / k;
    const int c = (int)(i % k);
    const float* xr = X + r * ld;
    const float* cr = C + (long long)c * ld;
    double s = 0.0;
    for (int j = 0; j < d; ++j) {
      const double t = (double)xr[j] - (double)cr[j];
      s += t * t;
    }
    D[i] = (float)sqrt(s);
  }
}

__global__ void add_mean_kernel(const float* __restrict__ C, int k, int ld, int d, const float* __restrict__ mean,
                                float* __restrict__ out) {
  const int total = k * d;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int c = i / d, j = i % d;
    const float v = C[(long long)c * ld + j];
    out[i] = mean ? v + mean[j] : v;
  }
}

}  // namespace skm
