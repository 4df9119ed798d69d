// Device code of the M-step shared by the stand-alone cooperative M-step
// (kernels.cu) and the persistent Lloyd loop kernel (loop_tc.cu): grid
// barrier, fixed-order reductions, the bulk fixed-point sums, the radix
// selection of far rows and the relocation path.
//
// Data written by other blocks of the same launch is only read after a grid
// barrier; the barrier's release/acquire fences make it visible.
#pragma once

#include "device_util.cuh"
#include "kernels.cuh"

namespace skm {

// ---------------------------------------------------------------------------
// helpers
// ---------------------------------------------------------------------------

// Bounded software grid barrier for cooperative launches: arrival is an
// acq_rel add on a counter, the last arrival resets it and releases a
// generation number the others poll with acquire loads. Returns false (and
// records error 1001 in the fit state) if the other blocks do not arrive
// within 2 s, so that a broken launch ends instead of hanging the GPU.
static __device__ bool grid_barrier(FitState* st, unsigned int nblocks) {
  __shared__ int ok_s;
  block_sync();
  if (threadIdx.x == 0) {
    int ok = 1;
    unsigned int gen, arrived;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(gen) : "l"(&st->barrier_gen) : "memory");
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(arrived) : "l"(&st->barrier_count) : "memory");
    if (arrived + 1u == nblocks) {
      // the last arrival resets the count for the next barrier, then releases
      // the generation (the release orders the reset before it)
      asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(&st->barrier_count) : "memory");
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&st->barrier_gen) : "memory");
    } else {
      const unsigned long long t0 = globaltimer();
      for (unsigned int it = 1;; ++it) {
        unsigned int g;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(g) : "l"(&st->barrier_gen) : "memory");
        if (g != gen) break;
        if ((it & 255) == 0 && globaltimer() - t0 > 2000000000ull) {
          atomicExch(&st->error, 1001);
          ok = 0;
          break;
        }
      }
    }
    ok_s = ok;
  }
  block_sync();
  return ok_s != 0;
}

template <typename T>
static __device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Deterministic block sum (fixed tree); result valid in thread 0.
static __device__ double block_sum_f64(double v, double* scratch /* >= 32 */) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) scratch[warp] = v;
  block_sync();
  double r = 0.0;
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    r = lane < nw ? scratch[lane] : 0.0;
    r = warp_sum(r);
  }
  block_sync();
  return r;
}

// ---------------------------------------------------------------------------
// bulk fixed-point sums from the labels into the delta buffer D (zero on entry)
// ---------------------------------------------------------------------------

// Fixed-point sums and counts of all rows by label, added into
// D = [dS (k x ld) | dcount (k)], which must be zero. Integer additions are
// exact, so the result does not depend on the order of the additions or the
// grid. A warp takes 8 consecutive rows at a time; lane (rsub,
// qsub) = (lane % 8, lane / 8) reads column quad 4 m + qsub of row rsub, so
// each load instruction fetches four whole 128-byte lines of the blocked
// layout (8 rows x 16 bytes per quad) and uses them at once. With `acc`
// (shared, k*ld + k int64) the block accumulates privately in the layout
// [u][c][q] (column 4q + u of cluster c) with one shared atomic per element
// and adds its non-zero entries to D at the end; without, it adds to D
// directly.
static __device__ void bulk_pass_atomic(const float* __restrict__ X, int ld, long long n,
                                        const int32_t* __restrict__ labels, int k, long long* __restrict__ D,
                                        const FitState* st, long long* acc) {
  const double scale = st->scale;
  const float* __restrict__ w = st->w;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int rsub = lane & 7, qsub = lane >> 3;
  const int nq = ld >> 2;
  const long long ks = (long long)k * ld;
  if (acc) {
    for (long long i = threadIdx.x; i < ks + k; i += blockDim.x) acc[i] = 0;
    block_sync();
  }
  const float4* X4 = reinterpret_cast<const float4*>(X);
  const long long blocks8 = (n + 7) / 8;
  for (long long b = (long long)blockIdx.x * nw + warp; b < blocks8; b += (long long)gridDim.x * nw) {
    const long long r = b * 8 + rsub;
    const bool valid = r < n;
    const int c = valid ? labels[r] : 0;
    const float wr = (valid && w) ? w[r] : 1.0f;
    const float4* xr = X4 + (r >> 7) * (32LL * ld) + (r & 127);  // quad q of row r at xr[128 q]
    for (int q0 = 0; q0 < nq; q0 += 4) {
      const int q = q0 + qsub;
      if (!valid || q >= nq) continue;
      const float4 v = __ldcs(xr + (long long)q * 128);
      const long long f[4] = {to_fixed(v.x * wr, scale), to_fixed(v.y * wr, scale), to_fixed(v.z * wr, scale),
                              to_fixed(v.w * wr, scale)};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (f[u] == 0) continue;
        if (acc)
          atomicAdd(reinterpret_cast<unsigned long long*>(&acc[((long long)u * k + c) * nq + q]),
                    static_cast<unsigned long long>(f[u]));
        else
          red_add_s64(D + (long long)c * ld + 4 * q + u, f[u]);
      }
    }
    if (valid && qsub == 0) {
      const long long cw = w ? to_fixed(wr, st->wscale) : 1;
      if (acc)
        atomicAdd(reinterpret_cast<unsigned long long*>(&acc[ks + c]), static_cast<unsigned long long>(cw));
      else
        red_add_s64(D + ks + c, cw);
    }
  }
  if (acc) {
    block_sync();
    for (long long i = threadIdx.x; i < ks + k; i += blockDim.x) {
      const long long v = acc[i];
      if (v == 0) continue;
      long long dst = i;
      if (i < ks) {  // i = (u * k + c) * nq + q
        const long long q = i % nq, uc = i / nq;
        const long long c = uc % k, u = uc / k;
        dst = c * ld + 4 * q + u;
      }
      red_add_s64(D + dst, v);
    }
  }
}


// Tiled variant (bulk_tiles_ok): block b takes the tiles b, b + B, ... of 128
// rows. Warp 0 copies each tile's quad blocks and labels into shared memory
// with bulk copies, one per lane (two tiles in flight, completion on one
// mbarrier per buffer). Warps 1-4 turn the tile's labels into row masks, one
// 32-bit word per (cluster, 32-row group) (__match_any_sync: the lowest lane
// of each label writes its group's mask), and thread t, owner of the
// (cluster, column quad) pairs t, t + T, ... (pair p = cluster p / nq, quad
// p % nq, so that a warp's lanes mostly share a cluster and read consecutive
// quads of one row), adds the quad of every row in its cluster's masks in
// registers. Two block barriers per tile; the masks alternate between two
// sets, the one not in use cleared by the other warps. The block adds its
// totals to D once at the end: no per-element atomics. Waits are bounded
// (error 1004 in *err; the pass then stops).
static __device__ void bulk_pass_tiles(const float* __restrict__ X, int ld, long long n,
                                       const int32_t* __restrict__ labels, int k, long long* __restrict__ D,
                                       const FitState* st, unsigned char* ws, int* err) {
  constexpr int TR = kBulkTileRows;
  const double scale = st->scale;
  const float* __restrict__ w = st->w;
  const double wscale = st->wscale;
  const int nq = ld >> 2;
  const size_t tb = bulk_tile_bytes(ld);
  unsigned char* tile_s[2] = {ws, ws + tb};
  const int* lab_s[2] = {reinterpret_cast<const int*>(ws + (size_t)nq * kBulkQuadStride),
                         reinterpret_cast<const int*>(ws + tb + (size_t)nq * kBulkQuadStride)};
  uint64_t* bars = reinterpret_cast<uint64_t*>(ws + 2 * tb);
  unsigned int* masks = reinterpret_cast<unsigned int*>(bars + 2);  // 2 sets x k clusters x 4 groups
  __shared__ int stop_sh;
  volatile int& stop_s = stop_sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = blockDim.x;
  const int pairs = k * nq;
  const long long n_tiles = (n + TR - 1) / TR;
  const uint32_t tx = (uint32_t)nq * 2048u + (w ? 8u : 4u) * TR;
  long long acc[kBulkMaxPairsPerThread][4];
  long long cnt_acc[kBulkMaxPairsPerThread];
#pragma unroll
  for (int m = 0; m < kBulkMaxPairsPerThread; ++m) {
    cnt_acc[m] = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[m][u] = 0;
  }
  // warp 0: copy tile t into buffer b (lane q < nq the quad block q, lane nq
  // the labels; lane 0 announces the bytes first)
  auto issue = [&](long long t, int b) {
    const uint32_t bar = smem_u32(bars + b);
    if (lane == 0) mbar_expect_tx(bar, tx);
    __syncwarp();
    const char* src = reinterpret_cast<const char*>(X + t * TR * ld);
    const uint32_t dst = smem_u32(tile_s[b]);
    for (int q = lane; q <= nq + 1; q += 32) {
      if (q < nq) bulk_load(dst + (uint32_t)q * kBulkQuadStride, src + (size_t)q * 2048, 2048u, bar);
      else if (q == nq) bulk_load(smem_u32(lab_s[b]), labels + t * TR, 4u * TR, bar);
      else if (w) bulk_load(smem_u32(lab_s[b] + TR), w + t * TR, 4u * TR, bar);  // weights after the labels
    }
  };
  if (tid == 0) {
    mbar_init(smem_u32(bars), 1);
    mbar_init(smem_u32(bars + 1), 1);
    stop_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the buffers held other data
  }
  for (int i = tid; i < 8 * k; i += T) masks[i] = 0;
  block_sync();
  const long long t0 = blockIdx.x;
  if (warp == 0) {
    if (t0 < n_tiles) issue(t0, 0);
    if (t0 + gridDim.x < n_tiles) issue(t0 + gridDim.x, 1);
  }
  int i = 0;
  for (long long t = t0; t < n_tiles; t += gridDim.x, ++i) {
    const int b = i & 1;
    unsigned int* mk = masks + b * 4 * k;
    const unsigned char* cb = tile_s[b];
    // wait for the tile (bounded)
    {
      const uint32_t bar = smem_u32(bars + b);
      const uint32_t par = (uint32_t)(i >> 1) & 1u;
      if (!mbar_try_wait(bar, par)) {
        const unsigned long long w0 = globaltimer();
        for (uint32_t it = 1; !mbar_try_wait(bar, par); ++it) {
          if ((it & 63) == 0 && (stop_s || globaltimer() - w0 > 2000000000ull)) {
            stop_s = 1;
            atomicCAS(err, 0, 1004);
            break;
          }
        }
      }
    }
    if (warp >= 1 && warp <= TR / 32) {  // masks of this tile: labels in [0, k), -1 past n
      const int g = warp - 1;
      const int c = lab_s[b][g * 32 + lane];
      const unsigned int same = __match_any_sync(0xffffffffu, c);
      if ((unsigned)c < (unsigned)k && (__ffs(same) - 1) == lane) mk[c * 4 + g] = same;
    } else {  // the other set: read by the previous tile only (before its last barrier)
      unsigned int* other = masks + (b ^ 1) * 4 * k;
      const int w = warp == 0 ? 0 : warp - TR / 32;
      const int nw_clear = (T >> 5) - TR / 32;
      for (int j = w * 32 + lane; j < 4 * k; j += nw_clear * 32) other[j] = 0;
    }
    block_sync();
    if (stop_s) break;
#pragma unroll
    for (int m = 0; m < kBulkMaxPairsPerThread; ++m) {
      const int p = tid + m * T;
      if (p >= pairs) break;
      const int c = p / nq, q = p - c * nq;
      const unsigned char* qb = cb + (size_t)q * kBulkQuadStride;
      const uint4 w4 = *reinterpret_cast<const uint4*>(mk + c * 4);
      const unsigned int wv[4] = {w4.x, w4.y, w4.z, w4.w};
      const float* wt = reinterpret_cast<const float*>(lab_s[b] + TR);  // the tile's weights (weighted fits)
      if (q == 0 && !w) cnt_acc[m] += __popc(wv[0]) + __popc(wv[1]) + __popc(wv[2]) + __popc(wv[3]);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        for (unsigned int bits = wv[g]; bits; bits &= bits - 1) {
          const int r = g * 32 + __ffs(bits) - 1;
          const float4 v = *reinterpret_cast<const float4*>(qb + r * 16);
          const float wr = w ? wt[r] : 1.0f;
          acc[m][0] += to_fixed(v.x * wr, scale);
          acc[m][1] += to_fixed(v.y * wr, scale);
          acc[m][2] += to_fixed(v.z * wr, scale);
          acc[m][3] += to_fixed(v.w * wr, scale);
          if (q == 0 && w) cnt_acc[m] += to_fixed(wr, wscale);
        }
      }
    }
    // the buffer is read; the next copy into it goes through the async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    block_sync();
    if (warp == 0 && t + 2 * (long long)gridDim.x < n_tiles) issue(t + 2 * (long long)gridDim.x, b);
  }
  // a stopped pass (at tile index i) lets its copies land before the
  // workspace is reused: tile i in buffer i & 1 and, if it exists, tile i + 1
  // in the other buffer (bounded)
  if (tid == 0 && stop_s) {
    for (int u = i; u <= i + 1; ++u) {
      if (t0 + (long long)u * gridDim.x >= n_tiles) break;
      const uint32_t bar = smem_u32(bars + (u & 1)), par = (uint32_t)(u >> 1) & 1u;
      const unsigned long long w0 = globaltimer();
      while (!mbar_try_wait(bar, par) && globaltimer() - w0 < 2000000000ull) {
      }
    }
  }
  const long long ks = (long long)k * ld;
#pragma unroll
  for (int m = 0; m < kBulkMaxPairsPerThread; ++m) {
    const int p = tid + m * T;
    if (p < pairs) {
      const int c = p / nq, q = p - c * nq;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (acc[m][u] != 0) red_add_s64(D + (long long)c * ld + 4 * q + u, acc[m][u]);
      if (q == 0 && cnt_acc[m] != 0) red_add_s64(D + ks + c, cnt_acc[m]);
    }
  }
  block_sync();  // the workspace (and its barriers) may be reused after this
}

// The bulk pass with `ws_bytes` of shared workspace `ws` (16-byte aligned):
// the tiled variant when it fits, else the atomic one with a shared
// accumulator when that fits, else straight to global memory. Every thread
// of every block calls it; `err` receives a code if a wait times out.
static __device__ __forceinline__ void bulk_pass(const float* __restrict__ X, int ld, long long n,
                                                 const int32_t* __restrict__ labels, int k, long long* __restrict__ D,
                                                 const FitState* st, unsigned char* ws, size_t ws_bytes, int* err) {
  if (bulk_tiles_ok(k, ld, blockDim.x, ws_bytes))
    bulk_pass_tiles(X, ld, n, labels, k, D, st, ws, err);
  else
    bulk_pass_atomic(X, ld, n, labels, k, D, st,
                     bulk_acc_bytes(k, ld, ws_bytes) ? reinterpret_cast<long long*>(ws) : nullptr);
}

// ---------------------------------------------------------------------------
// M-step (cooperative): empty clusters, relocation, averaging, shift, flags
// ---------------------------------------------------------------------------

static __device__ __forceinline__ unsigned long long reloc_key(float dist, long long row) {
  unsigned int b = __float_as_uint(dist);
  if (b & 0x80000000u) b = 0;  // -0.0 and (impossible) negatives sort as zero
  return ((unsigned long long)b << 32) | (unsigned long long)(0xffffffffu - (unsigned int)row);
}

// Selection of the m rows farthest from their assigned centre (largest
// (distance, -row) keys) by an exact 8-pass radix select over 64-bit keys
// (one maximum pass when m = 1). Keys are unique, so exactly m rows are
// collected. Runs inside the cooperative M-step; `hist` holds 2 x 256
// counters (8-byte aligned), zero on entry and on return.
static __device__ bool select_farthest(const float* __restrict__ mind, long long n, long long row_base, int m,
                                FitState* st, unsigned int* hist, long long* sel, unsigned int nblocks) {
  if (m == 1) {
    // one row: the largest key (keys are unique), by a block maximum and a
    // 64-bit atomicMax on the first two histogram words (zero on entry; the
    // same row as the radix select)
    __shared__ unsigned long long wmax_s[32];
    unsigned long long* top = reinterpret_cast<unsigned long long*>(hist);
    unsigned long long best = 0;
    for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < n; r += (long long)nblocks * blockDim.x)
      best = max(best, reloc_key(mind[r], row_base + r));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) wmax_s[threadIdx.x >> 5] = best;
    block_sync();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = max(best, wmax_s[w]);
      if (best) atomicMax(top, best);
    }
    if (!grid_barrier(st, nblocks)) return false;
    const unsigned long long k1 = *reinterpret_cast<volatile unsigned long long*>(top);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      // low 32 bits: 0xffffffff - global row (reloc_key)
      const long long g = (long long)(0xffffffffu - (unsigned int)(k1 & 0xffffffffull));
      sel[0] = g - row_base;
      st->sel_count = 1;
    }
    if (!grid_barrier(st, nblocks)) return false;
    if (blockIdx.x == 0 && threadIdx.x == 0) *top = 0;  // read by nobody until the next selection
    return true;
  }

  __shared__ unsigned int h[256];
  __shared__ unsigned long long prefix_s, mask_s;
  __shared__ int remaining_s, whole_s;
  unsigned long long prefix = 0, mask = 0;
  int remaining = m;
  int pass = 0;
  for (; pass < 8; ++pass) {
    const int shift = 56 - 8 * pass;
    unsigned int* gh = hist + (pass & 1) * 256;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) h[i] = 0;
    block_sync();
    for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < n; r += (long long)nblocks * blockDim.x) {
      const unsigned long long key = reloc_key(mind[r], row_base + r);
      if ((key & mask) == prefix) atomicAdd(&h[(key >> shift) & 255u], 1u);
    }
    block_sync();
    for (int i = threadIdx.x; i < 256; i += blockDim.x)
      if (h[i]) atomicAdd(&gh[i], h[i]);
    if (!grid_barrier(st, nblocks)) return false;
    if (threadIdx.x == 0) {
      // every block computes the same choice from the same global histogram
      int cum = 0, digit = 0, c = 0;
      for (int dgt = 255; dgt >= 0; --dgt) {
        c = (int)gh[dgt];
        if (cum + c >= remaining) { digit = dgt; break; }
        cum += c;
      }
      prefix_s = prefix | ((unsigned long long)digit << shift);
      mask_s = mask | (255ull << shift);
      remaining_s = remaining - cum;
      // the bucket is taken whole: the keys >= prefix (lower bits zero) are
      // exactly the m largest, no further digit is needed
      whole_s = cum + c == remaining;
    }
    block_sync();
    prefix = prefix_s;
    mask = mask_s;
    remaining = remaining_s;
    // clear the other histogram for the next pass (nobody reads it until the
    // next barrier)
    if (blockIdx.x == 0) {
      unsigned int* oh = hist + ((pass + 1) & 1) * 256;
      for (int i = threadIdx.x; i < 256; i += blockDim.x) oh[i] = 0;
    }
    if (!grid_barrier(st, nblocks)) return false;
    if (whole_s) break;  // uniform: every block read the same histogram
  }
  // after an early exit the last pass's histogram still holds counts; the
  // next selection starts from both halves zero (read by nobody until then)
  if (pass < 8 && blockIdx.x == 0) {
    unsigned int* gh = hist + (pass & 1) * 256;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) gh[i] = 0;
  }
  // keys >= prefix are exactly the m largest: the m-th largest key itself
  // after eight digits, or a whole bucket's lower bound after an early exit
  for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < n; r += (long long)nblocks * blockDim.x) {
    const unsigned long long key = reloc_key(mind[r], row_base + r);
    if (key >= prefix) {
      const int slot = atomicAdd(&st->sel_count, 1);
      if (slot < m) sel[slot] = r;
    }
  }
  return grid_barrier(st, nblocks);
}

// Averaged centre value of a non-empty cluster c (after relocation), column j.
// A relocated row carries its weighted values and its weight (weighted fits;
// unit weights otherwise, where a cluster that receives a row is that row).
static __device__ __forceinline__ float centre_value(const MStepArgs& a, int c, int j, int n_reloc) {
  const bool weighted = a.st->w != nullptr;
  for (int i = 0; i < n_reloc; ++i)
    if (a.empty_ids[i] == c) {
      if (!weighted) return a.reloc_x[(long long)i * a.ld + j];  // exactly the far row
      const long long s1 = to_fixed(a.reloc_x[(long long)i * a.ld + j] * a.reloc_w[i], a.st->scale);
      return centre_from_sum(s1, centre_factor(a.st->inv_scale, a.cnt_adj[c]));
    }
  long long s = a.S[(long long)c * a.ld + j];
  for (int i = 0; i < n_reloc; ++i)
    if (a.reloc_label[i] == c) s -= to_fixed(a.reloc_x[(long long)i * a.ld + j] * a.reloc_w[i], a.st->scale);
  return centre_from_sum(s, centre_factor(a.st->inv_scale, a.cnt_adj[c]));
}

// One centre (cluster c, columns strided over the calling warp's lanes):
// writes C_new, its centre-image entries and returns (shift^2, ||c||^2)
// summed in a fixed order (lane partials, then a fixed butterfly).
static __device__ __forceinline__ void warp_centre(const MStepArgs& a, int c, int src, int n_reloc, double* dsq_out,
                                            double* nrm_out) {
  const int lane = threadIdx.x & 31;
  const float cs = ldexpf(1.0f, a.st->xexp);  // centres are bounded by max |x|
  double dsq = 0.0, nrm = 0.0;
  for (int j = lane; j < a.ld; j += 32) {
    float v = 0.0f;
    if (j < a.d) {
      v = centre_value(a, src, j, n_reloc);
      const double df = (double)v - (double)a.C_old[(long long)c * a.ld + j];
      dsq += df * df;
      nrm += (double)v * v;
      if (a.cimg.img) cimg_put(a.cimg, c, j, v, cs);
    }
    a.C_new[(long long)c * a.ld + j] = v;
  }
  *dsq_out = warp_sum(dsq);
  *nrm_out = warp_sum(nrm);
}

// New centres when no cluster is empty. Column j of cluster c's fixed-point
// sum is (bulk ? 0 : S_in[j]) + D[j] and its centre value
// centre_from_sum(sum, 2^-F / count). One warp handles a cluster, lane l its
// column quads q = l, l + 32, ...; the squared shift against C_old and the
// squared norm are accumulated by each lane in column order and then combined
// by the xor butterfly of warp_sum. Every path of the library uses this
// order, so all blocks, both loop drivers and every GPU count reach
// bit-identical values. All arrays are k x ld with ld a multiple of 4 and
// 16-byte aligned rows.
struct QuadSums {
  long long s[4];  // folded sums of the quad's columns
  float4 old;      // previous centre values
  bool dnz;        // some delta of the quad is non-zero
};

__device__ __forceinline__ QuadSums quad_load(const long long* S_in, const long long* D, const float* C_old,
                                              long long i, int bulk) {
  QuadSums r;
  const longlong2 d01 = __ldcg(reinterpret_cast<const longlong2*>(D + i));
  const longlong2 d23 = __ldcg(reinterpret_cast<const longlong2*>(D + i + 2));
  longlong2 s01 = make_longlong2(0, 0), s23 = make_longlong2(0, 0);
  if (!bulk) {
    s01 = __ldcg(reinterpret_cast<const longlong2*>(S_in + i));
    s23 = __ldcg(reinterpret_cast<const longlong2*>(S_in + i + 2));
  }
  r.old = __ldcg(reinterpret_cast<const float4*>(C_old + i));
  r.s[0] = s01.x + d01.x;
  r.s[1] = s01.y + d01.y;
  r.s[2] = s23.x + d23.x;
  r.s[3] = s23.y + d23.y;
  r.dnz = (d01.x | d01.y | d23.x | d23.y) != 0;
  return r;
}

// Centre values of quad q (columns 4q .. 4q + 3) of cluster c from its loaded
// sums; adds the shift and norm terms of the columns < d in order; writes the
// optional outputs (null to skip): centre image entries (img1, img2), folded
// sums S_out, centre values C_new, and zeros over the non-zero deltas in
// D_clear.
__device__ __forceinline__ void quad_finish(const QuadSums& r, int c, int q, long long i, int d, double fct, float cs,
                                            const CentreImage& img1, const CentreImage& img2, long long* S_out,
                                            float* C_new, long long* D_clear, double& dsq, double& nrm) {
  const float old[4] = {r.old.x, r.old.y, r.old.z, r.old.w};
  float v[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int j = 4 * q + u;
    v[u] = 0.0f;
    if (j < d) {
      v[u] = centre_from_sum(r.s[u], fct);
      const double df = (double)v[u] - (double)old[u];
      dsq += df * df;
      nrm += (double)v[u] * v[u];
    }
  }
  // image entries of columns >= d are zero, as are v[u] there
  if (img1.img) cimg_put4(img1, c, q, v, cs);
  if (img2.img) cimg_put4(img2, c, q, v, cs);
  if (S_out) {
    *reinterpret_cast<longlong2*>(S_out + i) = make_longlong2(r.s[0], r.s[1]);
    *reinterpret_cast<longlong2*>(S_out + i + 2) = make_longlong2(r.s[2], r.s[3]);
  }
  if (C_new) *reinterpret_cast<float4*>(C_new + i) = make_float4(v[0], v[1], v[2], v[3]);
  if (D_clear && r.dnz) {
    *reinterpret_cast<longlong2*>(D_clear + i) = make_longlong2(0, 0);
    *reinterpret_cast<longlong2*>(D_clear + i + 2) = make_longlong2(0, 0);
  }
}

// One cluster, any ld (one warp; see above).
static __device__ __forceinline__ void warp_centre_from_sums(int c, int ld, int d, const long long* S_in,
                                                             const long long* D, int bulk, long long cnew,
                                                             double inv_scale, const float* C_old, float cs,
                                                             const CentreImage& img1, const CentreImage& img2,
                                                             long long* S_out, float* C_new, long long* D_clear,
                                                             double* dsq_out, double* nrm_out) {
  const int lane = threadIdx.x & 31;
  const double fct = centre_factor(inv_scale, cnew);
  double dsq = 0.0, nrm = 0.0;
  for (int q = lane; q < (ld >> 2); q += 32) {
    const long long i = (long long)c * ld + 4 * q;
    const QuadSums r = quad_load(S_in, D, C_old, i, bulk);
    quad_finish(r, c, q, i, d, fct, cs, img1, img2, S_out, C_new, D_clear, dsq, nrm);
  }
  *dsq_out = warp_sum(dsq);
  *nrm_out = warp_sum(nrm);
}

// Sum of v[0, n) in the canonical order (lane l adds v[l], v[l + 32], ... in
// order, then the xor butterfly); every lane of the calling warp gets it. v
// may be in global or shared memory.
static __device__ __forceinline__ double warp_ordered_sum(const double* v, int n) {
  double t = 0.0;
  for (int i = threadIdx.x & 31; i < n; i += 32) t += v[i];
  return warp_sum(t);
}

// Convergence bookkeeping (_kmeans.py:723-741) from the per-cluster squared
// shifts summed in a fixed order; one thread. The centre image now holds
// centres scaled by 2^xexp.
static __device__ void finish_iteration(const MStepArgs& a, FitState* st, unsigned long long changed_now, double tot) {
  st->cexp = st->xexp;
  st->bulk = st->bulk_always || changed_now > (unsigned long long)st->bulk_threshold;
  st->shift_tot = tot;
  st->iter += 1;
  if (changed_now == 0) {
    st->strict = 1;
    st->done = 1;
  } else if (tot <= st->tol) {
    st->done = 1;
  }
  if (st->iter >= st->max_iter) st->done = 1;
  *const_cast<unsigned long long*>(a.changed) = 0;
  if (a.host_done) *a.host_done = st->done ? st->iter : 0;
}

// Direct float32 squared distance of every local row to its (new) label's old
// centre, ((X - centers_old[labels])**2).sum(axis=1) (_k_means_common.pyx:185),
// into a.mind. Blocked X: lane per row of a 32-row group, columns in order.
static __device__ void rows_dist_to_old_centres(const MStepArgs& a, unsigned int nb) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  float* mind = const_cast<float*>(a.mind);
  const long long items = (a.n + 31) / 32;
  const float4* X4 = reinterpret_cast<const float4*>(a.X);
  for (long long it = blockIdx.x * (long long)nwarps + warp; it < items; it += (long long)nb * nwarps) {
    const long long r = it * 32 + lane;
    if (r >= a.n) continue;
    const float4* xp = X4 + (r >> 7) * (32LL * a.ld) + (r & 127);
    const float* cr = a.C_old + (long long)a.labels[r] * a.ld;
    float s = 0.0f;
    for (int q = 0; q < (a.ld >> 2); ++q) {
      const float4 v = xp[(long long)q * 128];
      float t = v.x - cr[4 * q];
      s = fmaf(t, t, s);
      t = v.y - cr[4 * q + 1];
      s = fmaf(t, t, s);
      t = v.z - cr[4 * q + 2];
      s = fmaf(t, t, s);
      t = v.w - cr[4 * q + 3];
      s = fmaf(t, t, s);
    }
    mind[r] = s;
  }
}

// Empty clusters after this iteration's sums (counts + deltas; bulk
// iterations: the deltas alone, which then hold the sums of all rows), in
// ascending id order. Block 0 writes their ids (up to kMaxEmptyCap) to
// a.empty_ids; every block returns the same count.
static __device__ int find_empty_clusters(const MStepArgs& a, int bulk) {
  __shared__ int n_empty_s;
  __shared__ int wcount[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const long long* dcnt = a.D + (long long)a.k * a.ld;
  if (threadIdx.x == 0) n_empty_s = 0;
  block_sync();
  for (int c0 = 0; c0 < a.k; c0 += blockDim.x) {
    const int c = c0 + threadIdx.x;
    const bool e = c < a.k && (bulk ? 0 : __ldcg(&a.counts[c])) + __ldcg(&dcnt[c]) == 0;
    const unsigned int b = __ballot_sync(0xffffffffu, e);
    if (lane == 0) wcount[warp] = __popc(b);
    block_sync();
    int base = n_empty_s;
    for (int w = 0; w < warp; ++w) base += wcount[w];
    const int pos = base + __popc(b & ((1u << lane) - 1u));
    if (e && blockIdx.x == 0 && pos < kMaxEmptyCap) a.empty_ids[pos] = c;
    block_sync();
    if (threadIdx.x == 0) {
      int t = 0;
      for (int w = 0; w < nwarps; ++w) t += wcount[w];
      n_empty_s += t;
    }
    block_sync();
  }
  const int n_empty = n_empty_s;
  block_sync();
  return n_empty;
}

// Relocation path of the M-step (cooperative, every block of the grid): folds
// this iteration's sums, relocates the empty clusters to the rows farthest
// from their centre, computes the new centres, shifts and the centre image,
// and has block 0 finish the iteration. Returns false (every block alike)
// when a grid barrier timed out or the relocation could not be done (the
// error is recorded in the fit state).
static __device__ bool relocation_path(const MStepArgs& a, int n_empty, int bulk, unsigned long long changed_now) {
  FitState* st = a.st;
  const unsigned int nb = gridDim.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const long long ks = (long long)a.k * a.ld;
  __shared__ long long hv_cnt[32];
  __shared__ int hv_idx[32];

  // ---------------- relocation path (cooperative, all blocks)
  // 0. S += dS, counts += dcount (bulk: S = dS, counts = dcount); clear the
  //    deltas (all but `changed`)
  {
    long long* S = const_cast<long long*>(a.S);
    long long* cnt = const_cast<long long*>(a.counts);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < ks + a.k;
         i += (long long)nb * blockDim.x) {
      const long long v = a.D[i];
      if (bulk) {
        if (i < ks) S[i] = v;
        else cnt[i - ks] = v;
        if (v != 0) a.D[i] = 0;
      } else if (v != 0) {
        if (i < ks) S[i] += v;
        else cnt[i - ks] += v;
        a.D[i] = 0;
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    st->n_empty = n_empty;
    st->sel_count = 0;
    if (n_empty > kMaxEmptyCap) atomicExch(&st->error, 1002);
  }
  if (n_empty > kMaxEmptyCap) return false;  // uniform
  if (!grid_barrier(st, nb)) return false;

  // 2. the n_empty rows farthest from their centre, paired in decreasing
  //    (distance, -row) order with the ascending empty ids
  if (a.cand == nullptr) {
    rows_dist_to_old_centres(a, nb);
    if (!grid_barrier(st, nb)) return false;
    if (!select_farthest(a.mind, a.n, a.row_base, n_empty, st, a.hist, a.sel, nb)) return false;
    if (blockIdx.x == 0) {
      for (int i = threadIdx.x; i < n_empty; i += blockDim.x) {
        const float di = a.mind[a.sel[i]];
        const unsigned long long ki = reloc_key(di, a.row_base + a.sel[i]);
        int rank = 0;
        for (int j = 0; j < n_empty; ++j)
          if (reloc_key(a.mind[a.sel[j]], a.row_base + a.sel[j]) > ki) ++rank;
        const long long r = a.sel[i];
        a.reloc_dist[rank] = di;
        a.reloc_label[rank] = a.labels[r];
        a.reloc_w[rank] = st->w ? st->w[r] : 1.0f;
        for (int j = 0; j < a.ld; ++j) a.reloc_x[(long long)rank * a.ld + j] = a.X[xblk_index(r, j, a.ld)];
      }
    }
  } else {
    // candidates of every rank (the same bytes on every rank): rank r's block
    // at cand + r * cand_block_bytes; its first `count` entries are valid
    const size_t cb = cand_block_bytes(a.cand_cap, a.ld);
    const int total = a.cand_ranks * a.cand_cap;
    int valid_total = 0, overflow = 0;
    for (int r = 0; r < a.cand_ranks; ++r) {
      const int cnt = *reinterpret_cast<const int*>(a.cand + r * cb);
      if (cnt < 0) overflow = 1;
      else valid_total += cnt;
    }
    if (overflow || n_empty > a.cand_cap || valid_total < n_empty) {  // uniform over blocks and ranks
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(&st->error, 1003);
      return false;
    }
    if (blockIdx.x == 0) {
      for (int t = threadIdx.x; t < total; t += blockDim.x) {
        const int r = t / a.cand_cap, i = t % a.cand_cap;
        const unsigned char* blk = a.cand + r * cb;
        if (i >= *reinterpret_cast<const int*>(blk)) continue;
        const float di = reinterpret_cast<const float*>(blk + cand_dist_off(a.cand_cap))[i];
        const long long gi = reinterpret_cast<const long long*>(blk + cand_row_off(a.cand_cap))[i];
        const unsigned long long ki = reloc_key(di, gi);
        int rank = 0;
        for (int u = 0; u < total; ++u) {
          const int r2 = u / a.cand_cap, i2 = u % a.cand_cap;
          const unsigned char* b2 = a.cand + r2 * cb;
          if (i2 >= *reinterpret_cast<const int*>(b2)) continue;
          const float dj = reinterpret_cast<const float*>(b2 + cand_dist_off(a.cand_cap))[i2];
          const long long gj = reinterpret_cast<const long long*>(b2 + cand_row_off(a.cand_cap))[i2];
          if (reloc_key(dj, gj) > ki) ++rank;
        }
        if (rank < n_empty) {
          a.reloc_dist[rank] = di;
          a.reloc_label[rank] = reinterpret_cast<const int*>(blk + cand_label_off(a.cand_cap))[i];
          a.reloc_w[rank] = 1.0f;  // sharded fits have unit weights
          const float* xs = reinterpret_cast<const float*>(blk + cand_x_off(a.cand_cap)) + (long long)i * a.ld;
          for (int j = 0; j < a.ld; ++j) a.reloc_x[(long long)rank * a.ld + j] = xs[j];
        }
      }
    }
  }
  if (!grid_barrier(st, nb)) return false;
  // no relocation when every distance is zero (_k_means_common.pyx:192-194)
  const int n_reloc = a.reloc_dist[0] > 0.0f ? n_empty : 0;

  // 3. counts after relocation (block 0), then the heaviest cluster (first max)
  if (blockIdx.x == 0) {
    for (int c = threadIdx.x; c < a.k; c += blockDim.x) a.cnt_adj[c] = a.counts[c];
    block_sync();
    if (threadIdx.x == 0) {
      for (int i = 0; i < n_reloc; ++i) {
        const long long cw = st->w ? to_fixed(a.reloc_w[i], st->wscale) : 1;
        a.cnt_adj[a.reloc_label[i]] -= cw;
        a.cnt_adj[a.empty_ids[i]] += cw;
      }
      st->relocated = n_reloc;
    }
  }
  if (!grid_barrier(st, nb)) return false;
  long long bc = -1;
  int bi = 0;
  for (int c = threadIdx.x; c < a.k; c += blockDim.x) {
    const long long v = a.cnt_adj[c];
    if (v > bc) { bc = v; bi = c; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long ov = __shfl_xor_sync(0xffffffffu, bc, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bc || (ov == bc && oi < bi)) { bc = ov; bi = oi; }
  }
  if (lane == 0) { hv_cnt[warp] = bc; hv_idx[warp] = bi; }
  block_sync();
  if (threadIdx.x == 0) {
    for (int w = 1; w < nwarps; ++w)
      if (hv_cnt[w] > hv_cnt[0] || (hv_cnt[w] == hv_cnt[0] && hv_idx[w] < hv_idx[0])) {
        hv_cnt[0] = hv_cnt[w];
        hv_idx[0] = hv_idx[w];
      }
  }
  block_sync();
  const int heavy = hv_idx[0];

  // 4. new centres (one warp per cluster) and their squared shifts
  double* dsq_s = a.shift_partial;
  for (int c = blockIdx.x * nwarps + warp; c < a.k; c += nb * nwarps) {
    double dsq, nrm;
    warp_centre(a, c, a.cnt_adj[c] > 0 ? c : heavy, n_reloc, &dsq, &nrm);
    if (lane == 0) {
      dsq_s[c] = dsq;
      if (a.shift_out) a.shift_out[c] = (float)sqrt(dsq);
      if (a.bias) a.bias[c] = (float)nrm;
    }
  }
  if (!grid_barrier(st, nb)) return false;

  // 5. convergence bookkeeping
  if (blockIdx.x == 0 && threadIdx.x < 32) {
    const double tot = warp_ordered_sum(dsq_s, a.k);
    if (threadIdx.x == 0) finish_iteration(a, st, changed_now, tot);
  }
  return true;
}

}  // namespace skm
