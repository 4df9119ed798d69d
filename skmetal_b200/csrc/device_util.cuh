// Device helpers shared by the kernel translation units.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "skm.cuh"

namespace skm {

// ---------------------------------------------------------------------------
// Blocked ("tile-major") layout of the fit's working copy of X.
// Rows are grouped in tiles of 128; inside a tile, columns are grouped in
// quads of 4 floats; quad q of tile t is a contiguous [128 rows][4 floats]
// block (2 KB) and the quads of a tile follow each other. Element (r, j) is
//   t * 128 * ld + (j / 4) * 512 + (r % 128) * 4 + j % 4      (floats)
// with ld = round_up(d, 4). A tile is therefore one contiguous region of
// 512 * ld bytes holding exactly the tile's data, and pairs of quads are the
// canonical no-swizzle K-major layout of the tensor core (8-row core matrices
// of 16-byte rows, 128 bytes apart; the two K halves of an 8-column chunk
// 2048 bytes apart), so a tile moves HBM -> shared memory with one bulk copy
// and shared memory -> tensor memory with tcgen05.cp. The buffer holds
// round_up(n, 128) rows; padding rows and columns are zero.
// ---------------------------------------------------------------------------
constexpr int kTileRows = 128;

__host__ __device__ __forceinline__ long long xblk_index(long long r, int j, int ld) {
  return (r >> 7) * (128LL * ld) + (long long)(j >> 2) * 512 + (r & 127) * 4 + (j & 3);
}

// value * 2^F rounded to the nearest integer, ties to even (2^F = scale, a
// power of two). When 2^F is a normal float the product v * 2^F is exact in
// float32 (or below 2^-126, where it rounds to 0 either way) and the float32
// conversion, twice the throughput of the float64 one, gives the same
// integer; otherwise the product is formed in float64, where it is exact.
__device__ __forceinline__ long long to_fixed(float v, double scale) {
  const float fs = static_cast<float>(scale);
  if (fs >= 1.17549435e-38f && fs <= 1.70141183e38f) return __float2ll_rn(v * fs);  // 2^-126 .. 2^127
  return __double2ll_rn(static_cast<double>(v) * scale);
}

// Centres from exact fixed-point sums: c = s * (2^-F / count), the factor
// computed once per cluster (one float64 division per cluster, not per
// element).
__device__ __forceinline__ double centre_factor(double inv_scale, long long count) {
  return inv_scale / (double)count;
}
__device__ __forceinline__ float centre_from_sum(long long s, double factor) { return (float)((double)s * factor); }

// ---------------------------------------------------------------------------
// shared-memory barriers (mbarrier) and bulk copies (cp.async.bulk, the TMA
// engine's untiled form), single-thread wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(reinterpret_cast<unsigned long long>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// L2 policy for data read once per pass (the tiles of X): evicted first, so
// that streaming X through L2 does not push out the small state the M-step
// reads back every iteration.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// L2 policy for small data every CTA re-reads many times in a pass (the
// centre units of the k > 256 E-step): kept in L2 in preference to the
// streamed tiles.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Prefetch of `bytes` (a multiple of 16) at a 16-byte-aligned global address
// into L2; no shared memory, no completion to wait for.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_load_hint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                               uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(dst), "l"(reinterpret_cast<unsigned long long>(src)), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}

// Programmatic dependent launch (kernels launched with the programmatic
// stream-serialization attribute): allow the next kernel of the stream to be
// scheduled now, and wait until every write of the previous kernel is
// visible. Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Block barrier for code in which lanes of a warp may arrive separately
// (warp-specialised roles where one elected lane runs a loop, or
// `if (threadIdx.x == 0) { ... }` sections with loops and early exits):
// bar.sync is the .aligned form, which a diverged warp must not execute, so
// the warp first reconverges on __syncwarp.
__device__ __forceinline__ void block_sync() {
  __syncwarp();
  __syncthreads();
}

__device__ __forceinline__ void red_add_s64(long long* p, long long v) {
  atomicAdd(reinterpret_cast<unsigned long long*>(p), static_cast<unsigned long long>(v));
}

// ---------------------------------------------------------------------------
// incremental update: a row whose label moved from `old` to `neu` adds its
// fixed-point coordinates to cluster `neu` and removes them from `old` in the
// delta buffer D = [dS (k x ld) | dcount (k) | changed]. In the blocked layout
// a row's column quads are 16-byte pieces 2 KB apart, so lane q loads quad q
// (one float4) and a warp fetches a whole row (ld <= 128) in one round trip.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void quad_delta(const float4& v, int q, int d, long long* __restrict__ dn,
                                           long long* __restrict__ dold, double scale, float wr) {
  const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int j = 4 * q + u;
    const long long f = to_fixed(x[u] * wr, scale);  // the float32 product, as the reference's sums take it
    if (j < d && f != 0) {
      red_add_s64(dn + j, f);
      if (dold) red_add_s64(dold + j, -f);
    }
  }
}

__device__ __forceinline__ void count_delta(int k, int ld, int old, int neu, long long* __restrict__ D,
                                            long long cw) {
  long long* cnt = D + (long long)k * ld;
  red_add_s64(cnt + neu, cw);
  if (old >= 0) red_add_s64(cnt + old, -cw);
}

// For every lane of the calling warp whose row changed label, apply its delta
// (weighted fits: the row's values times its weight, and its fixed-point
// weight instead of a count of 1). Rows are taken two at a time so that both
// rows' loads are in flight together.
__device__ __forceinline__ void warp_apply_changed(const float* __restrict__ X, int ld, int d, int k, long long row,
                                                   int old, int neu, bool changed, long long* __restrict__ D,
                                                   const FitState* st) {
  const int lane = threadIdx.x & 31;
  const int nq = ld >> 2;
  const double scale = st->scale;
  const float* w = st->w;
  unsigned int m = __ballot_sync(0xffffffffu, changed);
  while (m) {
    const int s1 = __ffs(m) - 1;
    m &= m - 1;
    const int s2 = m ? __ffs(m) - 1 : s1;
    if (m) m &= m - 1;
    const bool two = s2 != s1;
    const long long r1 = __shfl_sync(0xffffffffu, row, s1), r2 = __shfl_sync(0xffffffffu, row, s2);
    const int o1 = __shfl_sync(0xffffffffu, old, s1), o2 = __shfl_sync(0xffffffffu, old, s2);
    const int n1 = __shfl_sync(0xffffffffu, neu, s1), n2 = __shfl_sync(0xffffffffu, neu, s2);
    const float4* x1 = reinterpret_cast<const float4*>(X + xblk_index(r1, 0, ld));  // quad q at x1[128 q]
    const float4* x2 = reinterpret_cast<const float4*>(X + xblk_index(r2, 0, ld));
    long long* dn1 = D + (long long)n1 * ld;
    long long* do1 = o1 >= 0 ? D + (long long)o1 * ld : nullptr;
    long long* dn2 = D + (long long)n2 * ld;
    long long* do2 = o2 >= 0 ? D + (long long)o2 * ld : nullptr;
    const float w1 = w ? __ldg(w + r1) : 1.0f, w2 = w ? __ldg(w + r2) : 1.0f;
    for (int q = lane; q < nq; q += 32) {
      const float4 v1 = __ldg(x1 + (long long)q * 128);
      const float4 v2 = two ? __ldg(x2 + (long long)q * 128) : v1;
      quad_delta(v1, q, d, dn1, do1, scale, w1);
      if (two) quad_delta(v2, q, d, dn2, do2, scale, w2);
    }
    if (lane == 0) {
      count_delta(k, ld, o1, n1, D, w ? to_fixed(w1, st->wscale) : 1);
      if (two) count_delta(k, ld, o2, n2, D, w ? to_fixed(w2, st->wscale) : 1);
    }
  }
}

// ---------------------------------------------------------------------------
// Split-fp16 operands of the tensor-core E-step.
// x . c is computed as x_hi.c_hi + x_lo.c_hi + x_hi.c_lo with fp16 parts of
// power-of-two scaled values (v * 2^e = v_hi + v_lo, v_hi = fp16(v * 2^e),
// v_lo = fp16(v * 2^e - v_hi)) multiplied exactly and accumulated in fp32 by
// the tensor core. fp16 keeps 11 significant bits, as many as tf32, so this is
// 3xTF32 with the exponent range fixed by the scale; the dropped x_lo.c_lo
// term is below 2^-22 of |x||c|.
// ---------------------------------------------------------------------------

// The split of 8 consecutive columns of one row (two fp32 column quads a, b)
// scaled by s: hi = fp16 of the 8 scaled values, lo = fp16 of their remainders,
// each packed as 8 halves (16 bytes), element e at bytes 2e.
__device__ __forceinline__ void split8(const float4& a, const float4& b, float s, uint4* hi, uint4* lo) {
  const float v[8] = {a.x * s, a.y * s, a.z * s, a.w * s, b.x * s, b.y * s, b.z * s, b.w * s};
  uint32_t h[4], l[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    __half2 hh = __floats2half2_rn(v[2 * p], v[2 * p + 1]);
    const float2 hf = __half22float2(hh);
    __half2 ll = __floats2half2_rn(v[2 * p] - hf.x, v[2 * p + 1] - hf.y);
    h[p] = *reinterpret_cast<uint32_t*>(&hh);
    l[p] = *reinterpret_cast<uint32_t*>(&ll);
  }
  *hi = make_uint4(h[0], h[1], h[2], h[3]);
  *lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Split working copy of X for the tensor-core E-step: tile t (128 rows) at
// t * nk * 4096 bytes; its 8-column chunk c at c * 4096 holds x_hi of the
// chunk's 8 columns for rows 0..127 (2 KB, 16 bytes per row) then x_lo (2 KB):
// exactly one K = 16 slice of the kind::f16 A operand in the canonical
// no-swizzle K-major layout (8-row groups 128 bytes apart, K halves 2048 bytes
// apart). Columns past d and rows past n are zero.
// Half last chunk (stacked layout, ld = 4 mod 8): the last chunk has four
// columns and is stored in 2 KB, x_hi of its four columns in K 0..3 and x_lo
// in K 4..7 of the first K half, so a tile takes nk * 4096 - 2048 bytes; the
// second K half, read by the MMA from the shared-memory stage, is the stage's
// zeroed padding, and the centre image moves the matching c_hi copy to
// K 4..7 (cimg_put4).

// Scale exponent for values bounded by the float whose bits are given: with
// max |v| < 2^E, v * 2^(14 - E) < 2^14 (fp16 reaches 65504, so centres may be
// up to 4x larger than the bound). Clamped so that 2^(1 - 2e) stays a normal
// float; zero or non-finite bounds give 0.
__device__ __forceinline__ int split_exp(unsigned int maxabs_bits) {
  const float mx = __uint_as_float(maxabs_bits);
  if (!(mx > 0.0f) || mx > 3.0e38f) return 0;
  int E = 0;
  frexpf(mx, &E);
  return max(-50, min(63, 14 - E));
}

// Centre image: the exact shared-memory bytes of the E-step's B operand (fp16,
// K-major, no swizzle: core matrices of 8 rows x 16 bytes, 8-row groups 128
// bytes apart, the two 8-element K halves N * 16 bytes apart), K chunk c (8
// columns) at c * N * 32 bytes. Its K half 0 multiplies x_hi, half 1 x_lo.
//  stacked (2 k_pad <= 256): N = 2 k_pad; rows j < k_pad hold (c_hi | c_hi),
//    rows k_pad + j hold (c_lo | 0), so acc[j] + acc[k_pad + j] = x . c_j.
//  otherwise: N = k_pad; segment 1 holds (c_hi | c_hi) per chunk, segment 2
//    (after nk chunks) holds c_lo of chunk pairs (2m | 2m + 1), multiplied by
//    x_hi of the same pair; both accumulate into one accumulator.
//  blocked (kCimgBlocked, k > 256): the clusters in blocks of nbs (<= 256, a
//    multiple of 16); for block b and column pair m (columns 16m .. 16m + 15)
//    one unit of nbs * 64 bytes at ((b * npairs + m) * nbs * 32) halves, with
//    npairs = (nk + 1) / 2: c_hi of the pair (nbs rows x 16 halves, K-major,
//    K halves nbs * 16 bytes apart) then c_lo of the pair (same layout). One
//    unit is the B operand of three MMAs of N = nbs, K = 16: x_hi.c_hi,
//    x_lo.c_hi and x_hi.c_lo of the pair.
// Entries of padding rows and columns are zero.
constexpr int kCimgTwoSegment = 0, kCimgStacked = 1, kCimgBlocked = 2;
struct CentreImage {
  uint16_t* img;  // fp16 bit patterns; null when the tensor-core path is off
  int k_pad;      // clusters padded to 16 (blocked: nbs * blocks)
  int nk;         // K chunks of 8 columns
  int stacked;    // layout: kCimgTwoSegment, kCimgStacked or kCimgBlocked
  int nbs;        // blocked: clusters per block
  int half_last;  // stacked: the last chunk is a half chunk (the split copy's layout note)
};

__host__ __device__ inline size_t cimg_halves(int k_pad, int nk, int stacked) {
  if (stacked == kCimgBlocked) return (size_t)k_pad * ((nk + 1) / 2) * 32;
  return stacked ? (size_t)nk * 2 * k_pad * 16 : (size_t)nk * k_pad * 16 + (size_t)((nk + 1) / 2) * k_pad * 16;
}

// Offset (halves) of centre c, column e of pair m in the blocked layout, and
// that of its c_lo entry (one c_hi slice further).
__host__ __device__ __forceinline__ size_t cimg_blocked_off(const CentreImage& ci, int c, int m, int e) {
  const int b = c / ci.nbs, cl = c - b * ci.nbs;
  const size_t unit = ((size_t)b * ((ci.nk + 1) >> 1) + m) * (size_t)ci.nbs * 32;
  return unit + (size_t)(e >> 3) * ci.nbs * 8 + (size_t)(cl >> 3) * 64 + (size_t)(cl & 7) * 8 + (e & 7);
}

// Writes centre c, columns 4q .. 4q + 3 (values v[0..3], scale s = 2^e) into
// the image: the quad's entries are 4 consecutive halves in every segment
// (8-byte aligned), so three 8-byte stores write them.
__device__ __forceinline__ void cimg_put4(const CentreImage& ci, int c, int q, const float* v, float s) {
  uint32_t h[2], l[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const __half2 hh = __floats2half2_rn(v[2 * p] * s, v[2 * p + 1] * s);
    const float2 hf = __half22float2(hh);
    const __half2 ll = __floats2half2_rn(v[2 * p] * s - hf.x, v[2 * p + 1] * s - hf.y);
    h[p] = *reinterpret_cast<const uint32_t*>(&hh);
    l[p] = *reinterpret_cast<const uint32_t*>(&ll);
  }
  const uint2 hv = make_uint2(h[0], h[1]), lv = make_uint2(l[0], l[1]);
  if (ci.stacked == kCimgBlocked) {  // quad q = columns 4 (q & 3) .. + 3 of pair q / 4
    const size_t o = cimg_blocked_off(ci, c, q >> 2, (q & 3) * 4);
    *reinterpret_cast<uint2*>(ci.img + o) = hv;
    *reinterpret_cast<uint2*>(ci.img + o + (size_t)ci.nbs * 16) = lv;
    return;
  }
  const int chunk = q >> 1, e = (q & 1) * 4;
  const int N = ci.stacked ? 2 * ci.k_pad : ci.k_pad;
  const size_t base = (size_t)chunk * N * 16;
  const size_t r = (size_t)(c >> 3) * 64 + (size_t)(c & 7) * 8 + e;
  *reinterpret_cast<uint2*>(ci.img + base + r) = hv;
  // the copy of c_hi that multiplies x_lo: K half 1, or K 4..7 of a half chunk
  const bool half = ci.stacked == kCimgStacked && ci.half_last && chunk == ci.nk - 1;
  *reinterpret_cast<uint2*>(ci.img + base + (half ? (size_t)4 : (size_t)N * 8) + r) = hv;
  if (ci.stacked) {
    const int cl = ci.k_pad + c;
    *reinterpret_cast<uint2*>(ci.img + base + (size_t)(cl >> 3) * 64 + (size_t)(cl & 7) * 8 + e) = lv;
  } else {
    const size_t seg2 = (size_t)ci.nk * ci.k_pad * 16;
    *reinterpret_cast<uint2*>(ci.img + seg2 + (size_t)(chunk >> 1) * ci.k_pad * 16 + (size_t)(chunk & 1) * ci.k_pad * 8 +
                              r) = lv;
  }
}

// Writes centre c, column j (value v, scale s = 2^e) into the image.
__device__ __forceinline__ void cimg_put(const CentreImage& ci, int c, int j, float v, float s) {
  const float vs = v * s;
  const __half hi = __float2half_rn(vs);
  const __half lo = __float2half_rn(vs - __half2float(hi));
  const uint16_t hb = __half_as_ushort(hi), lb = __half_as_ushort(lo);
  if (ci.stacked == kCimgBlocked) {
    const size_t o = cimg_blocked_off(ci, c, j >> 4, j & 15);
    ci.img[o] = hb;
    ci.img[o + (size_t)ci.nbs * 16] = lb;
    return;
  }
  const int chunk = j >> 3, e = j & 7;
  const int N = ci.stacked ? 2 * ci.k_pad : ci.k_pad;
  const size_t base = (size_t)chunk * N * 16;
  const size_t r = (size_t)(c >> 3) * 64 + (size_t)(c & 7) * 8 + e;
  ci.img[base + r] = hb;
  const bool half = ci.stacked == kCimgStacked && ci.half_last && chunk == ci.nk - 1;
  ci.img[base + (half ? (size_t)4 : (size_t)N * 8) + r] = hb;
  if (ci.stacked) {
    const int cl = ci.k_pad + c;
    ci.img[base + (size_t)(cl >> 3) * 64 + (size_t)(cl & 7) * 8 + e] = lb;
  } else {
    const size_t seg2 = (size_t)ci.nk * ci.k_pad * 16;
    ci.img[seg2 + (size_t)(chunk >> 1) * ci.k_pad * 16 + (size_t)(chunk & 1) * ci.k_pad * 8 + r] = lb;
  }
}

}  // namespace skm
