// Device helpers shared by the kernel translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

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

// value * 2^F rounded to the nearest integer (2^F = scale, a power of two, so
// the product is exact in float64)
__device__ __forceinline__ long long to_fixed(float v, double scale) {
  return __double2ll_rn(static_cast<double>(v) * scale);
}

__device__ __forceinline__ void red_add_s64(long long* p, long long v) {
  atomicAdd(reinterpret_cast<unsigned long long*>(p), static_cast<unsigned long long>(v));
}

// ---------------------------------------------------------------------------
// incremental update: a row whose label moved from `old` to `neu` adds its
// fixed-point coordinates to cluster `neu` and removes them from `old` in the
// delta buffer D = [dS (k x ld) | dcount (k) | changed]. Called by all 32
// lanes of a warp with the row index and labels of one lane (`src_lane`);
// lanes stride over the columns, so loads and reductions are coalesced.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void warp_apply_delta(const float* __restrict__ X, int ld, int d, int k, long long row, int old, int neu,
                                 long long* __restrict__ D, double scale) {
  const int lane = threadIdx.x & 31;
  const float* xr = X + xblk_index(row, 0, ld);  // X is blocked: column j at xr[(j/4)*512 + j%4]
  long long* dn = D + (long long)neu * ld;
  long long* dold = old >= 0 ? D + (long long)old * ld : nullptr;
  for (int j = lane; j < d; j += 32) {
    const long long v = to_fixed(__ldg(xr + (j >> 2) * 512 + (j & 3)), scale);
    if (v != 0) {
      red_add_s64(dn + j, v);
      if (dold) red_add_s64(dold + j, -v);
    }
  }
  if (lane == 0) {
    long long* cnt = D + (long long)k * ld;
    red_add_s64(cnt + neu, 1);
    if (old >= 0) red_add_s64(cnt + old, -1);
  }
}

// For every lane of the calling warp whose row changed label, apply its delta.
__device__ __forceinline__ void warp_apply_changed(const float* __restrict__ X, int ld, int d, int k, long long row, int old, int neu,
                                   bool changed, long long* __restrict__ D, double scale) {
  unsigned int m = __ballot_sync(0xffffffffu, changed);
  while (m) {
    const int src = __ffs(m) - 1;
    m &= m - 1;
    const long long r = __shfl_sync(0xffffffffu, row, src);
    const int o = __shfl_sync(0xffffffffu, old, src);
    const int nn = __shfl_sync(0xffffffffu, neu, src);
    warp_apply_delta(X, ld, d, k, r, o, nn, D, scale);
  }
}

}  // namespace skm
