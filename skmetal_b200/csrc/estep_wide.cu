// Tensor-core E-step for more than 256 clusters (sm_100a): the codebook shape
// (k = 1024, d = 128) of the large-k workload. labels[i] = argmin_j
// (||c_j||^2 - 2 x_i . c_j) with strict '<' and the lowest index first
// (sklearn/cluster/_k_means_lloyd.pyx:205-213), as the k <= 256 pipeline of
// estep_dev.cuh, whose MMA, TMEM and barrier wrappers it uses.
//
// One MMA covers at most N = 256 clusters and the whole centre image no
// longer fits in shared memory (k = 1024, d = 128: 512 KB), so:
//   * the clusters are split into blocks of nbs <= 256 (kCimgBlocked layout
//     of CentreImage): for every block b and column pair m one unit of
//     nbs * 64 bytes (c_hi then c_lo of the pair's 16 columns) is, byte for
//     byte, the B operand of three MMAs (M = 128, N = nbs, K = 16):
//         acc += x_hi . c_hi,  acc += x_lo . c_hi,  acc += x_hi . c_lo
//     (the 3xTF32 split of device_util.cuh; A = the pair's x_hi or x_lo
//     halves of the split copy's two chunks, 4096 bytes apart);
//   * a second producer thread streams the units, which stay in L2 (an
//     evict-last policy; every CTA re-reads them for every tile), through a
//     ring of shared-memory stages while the first streams the X tiles from
//     HBM (evict-first);
//   * the block's dot products land in one of two TMEM accumulators of nbs
//     columns, so the MMAs of block b + 1 run while the epilogue reads block
//     b;
//   * epilogue group a (4 warps, one per TMEM lane quarter) reads every
//     block whose sequence number has parity a, keeping a running argmin per
//     row; at the end of a tile group 1 hands its partial minimum to group 0
//     through shared memory (two mbarriers per tile parity), which merges the
//     two in index order, writes the label, counts the change and queues a
//     changed row in the deferred-delta ring (delta_ring.cuh), whose
//     fixed-point deltas warp 3 adds; the previous labels are loaded one
//     tile ahead.
// The n x k distance matrix never leaves the SM, and X is read from HBM once
// per launch.
//
// Warp roles (384 threads): 0 X producer, 1 TMEM owner and MMA issuer (the
// whole warp runs the issuing loop on warp-uniform values, one elected lane
// issues each MMA), 2 centre-unit producer, 3 delta drainer, 4-7 epilogue group 0,
// 8-11 epilogue group 1.
//
// Every wait is bounded (2 s); on a timeout the CTA records an error code,
// sets its abort flag (every role then stops issuing work), each producer
// waits (bounded) for its copies in flight, the MMA issuer for its MMAs, and
// the CTA frees its tensor memory and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "delta_ring.cuh"
#include "device_util.cuh"
#include "driver.h"
#include "estep_dev.cuh"
#include "estep_tc.h"

namespace skm {

namespace tcw {

using tc::BM;
using tc::CHUNK_BYTES;

constexpr int THREADS = 384;
constexpr int MAX_XST = 4;    // X stages
constexpr int MAX_RING = 8;   // centre-unit stages
constexpr int MAX_NBS = 256;  // clusters per block (one UMMA N)
constexpr int MAX_K = 4096;
static_assert(MAX_K <= DQ_MAX_LABEL, "ring entries hold every label");
constexpr int PROD_X_W = 0, MMA_W = 1, PROD_C_W = 2, IDLE_W = 3, EPI_W0 = 4;
static_assert((EPI_W0 + 8) * 32 == THREADS, "two epilogue groups of four warps end the block");

struct Params {
  int n_tiles;
  long long n;
  int k, k_pad, nbs, nblk, nk, npairs;
  int xst, ring, tmem_cols;
  uint32_t stage_bytes, tile_bytes, unit_bytes;
  const unsigned char* Xs;  // split working copy (tile t at t * tile_bytes)
  const uint16_t* img;      // centre image, kCimgBlocked layout
  const int* sexp;          // {xexp, cexp}
  const float* bias;        // ||c||^2, k entries
  int32_t* labels;
  unsigned long long* changed;  // nullable
  long long* D;                 // nullable: fixed-point deltas (needs st)
  const float* X;               // fp32 blocked copy (the deltas read exact values)
  int ld, d;
  const FitState* st;  // nullable
  int* err;
};

// barrier indices
__host__ __device__ constexpr int XF(int s) { return s; }
__host__ __device__ constexpr int XE(int s) { return MAX_XST + s; }
__host__ __device__ constexpr int CF(int r) { return 2 * MAX_XST + r; }
__host__ __device__ constexpr int CE(int r) { return 2 * MAX_XST + MAX_RING + r; }
__host__ __device__ constexpr int AF(int a) { return 2 * MAX_XST + 2 * MAX_RING + a; }
__host__ __device__ constexpr int AE(int a) { return 2 * MAX_XST + 2 * MAX_RING + 2 + a; }
__host__ __device__ constexpr int PF(int p) { return 2 * MAX_XST + 2 * MAX_RING + 4 + p; }
__host__ __device__ constexpr int PE(int p) { return 2 * MAX_XST + 2 * MAX_RING + 6 + p; }
constexpr int B_DONE = 2 * MAX_XST + 2 * MAX_RING + 8;
constexpr int NUM_BARS = B_DONE + 1;

struct Layout {
  uint32_t ring, bias, part, bars, misc, dq, total;
};

__host__ __device__ inline Layout layout(uint32_t stage_bytes, int xst, uint32_t unit_bytes, int ring, int k_pad) {
  Layout L;
  uint32_t off = (uint32_t)xst * stage_bytes;  // stages and units are multiples of 1 KB
  L.ring = off;
  off += (uint32_t)ring * unit_bytes;
  L.bias = off;
  off += (uint32_t)k_pad * 4;
  L.part = off;  // 2 tile parities x 128 rows x {float distance, int index}
  off += 2 * BM * 8;
  L.bars = off;
  off += NUM_BARS * 8;
  L.misc = off;  // [0] tensor-memory base, [1] abort flag
  off += 16;
  L.dq = off;  // deferred-delta ring (delta_ring.cuh)
  off += dq_bytes();
  L.total = off + 1024;  // slack for aligning the base to 1024
  return L;
}

// A producer's copies still in flight land before the CTA exits: the last
// min(issued, stages) uses of its stages, each armed once (bounded). A copy
// is issued only after the previous use of its stage was consumed, so only
// those can still be in flight; waiting on a use that already completed
// returns at once (no later use of the stage follows it).
__device__ __forceinline__ void drain_copies(uint32_t bar0, int full0, long long issued, int stages, int* err,
                                             int code) {
  volatile int no_abort = 0;
  for (long long v = (issued > stages ? issued - stages : 0); v < issued; ++v)
    tc::mbar_wait(bar0 + 8u * (uint32_t)(full0 + (int)(v % stages)), (uint32_t)((v / stages) & 1), &no_abort, err,
                  code);
}

// Bounded wait of a whole warp (every lane waits) with one outcome for all
// lanes: the .sync.aligned TMEM loads and the warp votes that follow need the
// warp converged, even if the wait ends at its time limit on some lanes only.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err, int code) {
  const bool ok = tc::mbar_wait(bar, parity, abort_flag, err, code);
  return __all_sync(0xffffffffu, ok);
}

__global__ void __launch_bounds__(THREADS, 1) estep_wide_kernel(Params p) {
  pdl_launch_dependents();
  pdl_wait();
  if (p.st && p.st->done) return;
  long long* const deltas = (p.st && p.st->bulk) ? nullptr : p.D;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = layout(p.stage_bytes, p.xst, p.unit_bytes, p.ring, p.k_pad);
  const uint32_t sbase = smem_u32(base);
  const uint32_t bar0 = sbase + L.bars;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(base + L.misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  float* bias_s = reinterpret_cast<float*>(base + L.bias);
  float* part_d = reinterpret_cast<float*>(base + L.part);        // [parity][row]
  int* part_i = reinterpret_cast<int*>(base + L.part + 2 * BM * 4);  // [parity][row]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int my_tiles = (p.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < MAX_XST; ++s) {
      mbar_init(bar(XF(s)), 1);
      mbar_init(bar(XE(s)), 1);
    }
    for (int r = 0; r < MAX_RING; ++r) {
      mbar_init(bar(CF(r)), 1);
      mbar_init(bar(CE(r)), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar(AF(a)), 1);
      mbar_init(bar(AE(a)), 4);      // the four warps of the accumulator's epilogue group
      // one arrival per warp, after __syncwarp (which orders the warp's
      // shared-memory accesses before its lane 0's arrival)
      mbar_init(bar(PF(a)), 4);      // the four warps of group 1
      mbar_init(bar(PE(a)), 4);      // the four warps of group 0
    }
    mbar_init(bar(B_DONE), 1);
    misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_W) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + L.misc),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  for (int j = threadIdx.x; j < p.k_pad; j += blockDim.x) bias_s[j] = j < p.k ? __ldcg(p.bias + j) : INFINITY;
  const DeltaRing ring = dq_ring(base + L.dq);
  dq_init(ring);
  // the extra chunk of an odd nk (the x_hi / x_lo K half of the last pair)
  // is zero in every stage; the bulk copies write only tile_bytes
  if (p.tile_bytes < p.stage_bytes)
    for (int s = 0; s < p.xst; ++s)
      for (uint32_t o = p.tile_bytes + 16u * threadIdx.x; o < p.stage_bytes; o += 16u * blockDim.x)
        *reinterpret_cast<uint4*>(base + (uint32_t)s * p.stage_bytes + o) = make_uint4(0, 0, 0, 0);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc::tc_fence_before();
  block_sync();
  tc::tc_fence_after();
  const uint32_t tmem_base = misc[0];
  const float negscale = -ldexpf(1.0f, 1 - __ldcg(p.sexp) - __ldcg(p.sexp + 1));
  const unsigned long long s2 = tc::pack_pair(__float_as_uint(negscale), __float_as_uint(negscale));

  if (warp == PROD_X_W) {
    // ------------------------------------------------------------ X tiles
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int issued = 0;
      for (int i = 0; i < my_tiles; ++i) {
        const int s = i % p.xst;
        if (!tc::mbar_wait(bar(XE(s)), (uint32_t)((i / p.xst) & 1) ^ 1u, abort_flag, p.err, 2601)) break;
        const int tile = (int)blockIdx.x + i * (int)gridDim.x;
        mbar_expect_tx(bar(XF(s)), p.tile_bytes);
        bulk_load_hint(sbase + (uint32_t)s * p.stage_bytes, p.Xs + (size_t)tile * p.tile_bytes, p.tile_bytes,
                       bar(XF(s)), pol);
        issued = i + 1;
      }
      drain_copies(bar0, XF(0), issued, p.xst, p.err, 2611);
    }
  } else if (warp == PROD_C_W) {
    // ------------------------------------------------------- centre units
    if (lane == 0) {
      const uint64_t pol = l2_evict_last_policy();
      const int per_tile = p.nblk * p.npairs;
      const long long total = (long long)my_tiles * per_tile;
      const unsigned char* img = reinterpret_cast<const unsigned char*>(p.img);
      long long issued = 0;
      for (long long v = 0; v < total; ++v) {
        const int r = (int)(v % p.ring);
        if (!tc::mbar_wait(bar(CE(r)), (uint32_t)((v / p.ring) & 1) ^ 1u, abort_flag, p.err, 2602)) break;
        const int u = (int)(v % per_tile);  // unit (b, m) = (u / npairs, u % npairs), stored in that order
        mbar_expect_tx(bar(CF(r)), p.unit_bytes);
        bulk_load_hint(sbase + L.ring + (uint32_t)r * p.unit_bytes, img + (size_t)u * p.unit_bytes, p.unit_bytes,
                       bar(CF(r)), pol);
        issued = v + 1;
      }
      drain_copies(bar0, CF(0), issued, p.ring, p.err, 2612);
    }
  } else if (warp == MMA_W) {
    // ------------------------------------------------------------- MMAs
    // the whole warp runs this loop (every value in it is warp-uniform); one
    // elected lane issues each MMA and commit
    const uint32_t idesc = tc::idesc_f16(p.nbs);
    long long v = 0;
    bool ok = true;
    for (int i = 0; ok && i < my_tiles; ++i) {
      const int s = i % p.xst;
      if (!warp_wait(bar(XF(s)), (uint32_t)(i / p.xst) & 1u, abort_flag, p.err, 2603)) break;
      tc::tc_fence_after();
      const uint32_t stage = sbase + (uint32_t)s * p.stage_bytes;
      // A: x_hi of the pair's two chunks (K halves 4096 bytes apart), x_lo 2048 bytes further
      const tc::SmemDesc ahi0 = tc::kmajor_desc(stage, (uint32_t)CHUNK_BYTES, 128u);
      const tc::SmemDesc alo0 = tc::kmajor_desc(stage + 2048u, (uint32_t)CHUNK_BYTES, 128u);
      for (int b = 0; ok && b < p.nblk; ++b) {
        const int u = i * p.nblk + b, a = u & 1;
        if (!warp_wait(bar(AE(a)), (uint32_t)((u >> 1) & 1) ^ 1u, abort_flag, p.err, 2604)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t tacc = tmem_base + (uint32_t)(a * p.nbs);
        for (int m = 0; m < p.npairs; ++m, ++v) {
          const int r = (int)(v % p.ring);
          if (!warp_wait(bar(CF(r)), (uint32_t)((v / p.ring) & 1), abort_flag, p.err, 2605)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t unit = sbase + L.ring + (uint32_t)r * p.unit_bytes;
          const tc::SmemDesc bhi = tc::kmajor_desc(unit, (uint32_t)(p.nbs * 16), 128u);
          const tc::SmemDesc blo = tc::kmajor_desc(unit + (uint32_t)(p.nbs * 32), (uint32_t)(p.nbs * 16), 128u);
          const tc::SmemDesc ahi = tc::desc_advance(ahi0, (uint32_t)(2 * m) * CHUNK_BYTES);
          const tc::SmemDesc alo = tc::desc_advance(alo0, (uint32_t)(2 * m) * CHUNK_BYTES);
          tc::mma_f16_elect(tacc, ahi, bhi, idesc, m > 0 ? 1u : 0u);
          tc::mma_f16_elect(tacc, alo, bhi, idesc, 1u);
          tc::mma_f16_elect(tacc, ahi, blo, idesc, 1u);
          tc::tc_commit_elect(bar(CE(r)));  // the unit is no longer read by the tensor core
        }
        if (!ok) break;
        tc::tc_commit_elect(bar(AF(a)));
      }
      if (!ok) break;
      tc::tc_commit_elect(bar(XE(s)));
    }
    // every tcgen05 operation issued by this warp is complete once DONE fires
    tc::tc_commit_elect(bar(B_DONE));
    volatile int no_abort = 0;
    warp_wait(bar(B_DONE), 0u, &no_abort, p.err, 2606);
  } else if (warp >= EPI_W0) {
    // -------------------------------------------------------------- epilogue
    const int g = (warp - EPI_W0) >> 2;
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const bool finisher = g == 0;
    // the finisher loads each tile's previous labels one tile ahead
    int old_next = -1;
    if (finisher && p.changed && my_tiles > 0) {
      const long long g0 = (long long)blockIdx.x * BM + row;
      old_next = g0 < p.n ? p.labels[g0] : -1;
    }
    bool ok = true;
    for (int i = 0; ok && i < my_tiles; ++i) {
      const long long grow = (long long)((int)blockIdx.x + i * (int)gridDim.x) * BM + row;
      const int old = old_next;
      if (finisher && p.changed && i + 1 < my_tiles) {
        const long long g1 = grow + (long long)gridDim.x * BM;
        old_next = g1 < p.n ? p.labels[g1] : -1;
      }
      float best = INFINITY;
      int bl = 0x7fffffff;
      for (int b = 0; b < p.nblk; ++b) {
        const int u = i * p.nblk + b, a = u & 1;
        if (a != g) continue;
        if (!warp_wait(bar(AF(a)), (uint32_t)(u >> 1) & 1u, abort_flag, p.err, 2607)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t taddr = tmem_base + lane_off + (uint32_t)(a * p.nbs);
        const float* bias_b = bias_s + b * p.nbs;
        float bb;
        int bj;
        tc::scan_row4_n(p.nbs >> 4, taddr, bias_b, s2, bb, bj);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(AE(a)));
        if (bj != 0x7fffffff && tc::better(bb, b * p.nbs + bj, best, bl)) {
          best = bb;
          bl = b * p.nbs + bj;
        }
      }
      if (!ok) break;
      // merge the two groups' minima of this tile (index order: better())
      const int par = i & 1;
      const uint32_t use = (uint32_t)(i >> 1) & 1u;
      if (g == 1) {
        if (!warp_wait(bar(PE(par)), use ^ 1u, abort_flag, p.err, 2608)) break;
        part_d[par * BM + row] = best;
        part_i[par * BM + row] = bl;
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(PF(par)));
      } else {
        if (!warp_wait(bar(PF(par)), use, abort_flag, p.err, 2609)) break;
        const float ob = part_d[par * BM + row];
        const int oi = part_i[par * BM + row];
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(PE(par)));
        if (tc::better(ob, oi, best, bl)) {
          best = ob;
          bl = oi;
        }
        if (bl >= p.k) bl = 0;  // only reachable when every distance is +inf or NaN
        bool ch = false;
        if (grow < p.n) {
          ch = p.changed && old != bl;
          p.labels[grow] = bl;
        }
        if (p.changed) {
          const unsigned int mk = __ballot_sync(0xffffffffu, ch);
          if (lane == 0 && mk) atomicAdd(p.changed, (unsigned long long)__popc(mk));
          // the deltas are applied by warp IDLE_W (delta_ring.cuh)
          if (deltas) dq_push(ring, abort_flag, p.err, grow, old, bl, ch);
        }
      }
    }
    if (finisher && p.changed && deltas) dq_close(ring);
  } else if (warp == IDLE_W && p.changed && deltas) {
    // ---------------------------------------------------- delta drainer
    dq_drain(ring, 4u, abort_flag, p.err, p.X, p.ld, p.d, p.k, p.st, deltas);
  }
  // the single-lane roles leave warps 0-2 diverged: reconverge before the
  // block barrier
  __syncwarp();
  tc::tc_fence_before();
  block_sync();
  if (warp == MMA_W) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.tmem_cols));
  }
}

}  // namespace tcw

// ---------------------------------------------------------------------------
// probe: the blocked image layout and the three-MMA sequence on exact values
// ---------------------------------------------------------------------------
// The k <= 256 probe's operands (estep_tc.cu): a 128 x 16 tile split by
// split8 and 32 centres written by cimg_put into a blocked image of two
// 16-cluster blocks (one column pair); block b's three MMAs (N = 16) land in
// TMEM columns 16 b .. 16 b + 15. out: [0, 4096) x.c row-major 128 x 32
// (float bits); [4096] error code.
namespace tcw {

constexpr int PROBE_K = 32, PROBE_NBS = 16, PROBE_NK = 2;

__global__ void __launch_bounds__(128, 1) tc_probe_wide_kernel(uint16_t* img_g, uint32_t* out) {
  constexpr uint32_t TILE = PROBE_NK * CHUNK_BYTES;         // 8 KB
  constexpr uint32_t UNIT = PROBE_NBS * 64;                 // 1 KB
  constexpr uint32_t IMG = (PROBE_K / PROBE_NBS) * UNIT;    // 2 KB
  __shared__ __align__(1024) unsigned char sm[TILE + IMG + 64];
  const uint32_t sa = smem_u32(sm), sb = sa + TILE, sbar = sb + IMG;
  uint32_t* misc = reinterpret_cast<uint32_t*>(sm + TILE + IMG + 16);
  const uint32_t smisc = smem_u32(misc);
  int* err = reinterpret_cast<int*>(out + 4096);
  const int tid = threadIdx.x, warp = tid >> 5;
  for (int j = 0; j < PROBE_NK * tc::KC; ++j)
    *reinterpret_cast<float*>(sm + (j >> 2) * 2048 + tid * 16 + (j & 3) * 4) = tc::probe_x(tid, j);
  for (int c = 0; c < PROBE_NK; ++c) {
    uint4* q0 = reinterpret_cast<uint4*>(sm + (2 * c) * 2048 + tid * 16);
    uint4* q1 = reinterpret_cast<uint4*>(sm + (2 * c + 1) * 2048 + tid * 16);
    const float4 a = *reinterpret_cast<const float4*>(q0), b = *reinterpret_cast<const float4*>(q1);
    split8(a, b, 1.0f, q0, q1);
  }
  const CentreImage ci{img_g, PROBE_K, PROBE_NK, kCimgBlocked, PROBE_NBS};
  for (int e = tid; e < PROBE_K * PROBE_NK * tc::KC; e += blockDim.x) {
    const int c = e / (PROBE_NK * tc::KC), j = e % (PROBE_NK * tc::KC);
    cimg_put(ci, c, j, tc::probe_c(c, j), 1.0f);
  }
  block_sync();
  for (uint32_t o = tid * 2; o < IMG / 2; o += 2 * blockDim.x)
    *reinterpret_cast<uint32_t*>(sm + TILE + o * 2) = *reinterpret_cast<const uint32_t*>(img_g + o);
  if (tid == 0) {
    mbar_init(sbar, 1);
    misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smisc), "r"(32));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc::tc_fence_before();
  block_sync();
  tc::tc_fence_after();
  const uint32_t tb = misc[0];
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  if (tid == 0) {
    const uint32_t idesc = tc::idesc_f16(PROBE_NBS);
    const tc::SmemDesc ahi = tc::kmajor_desc(sa, (uint32_t)CHUNK_BYTES, 128u);
    const tc::SmemDesc alo = tc::kmajor_desc(sa + 2048u, (uint32_t)CHUNK_BYTES, 128u);
    for (int b = 0; b < PROBE_K / PROBE_NBS; ++b) {
      const uint32_t unit = sb + (uint32_t)b * UNIT;
      const tc::SmemDesc bhi = tc::kmajor_desc(unit, PROBE_NBS * 16u, 128u);
      const tc::SmemDesc blo = tc::kmajor_desc(unit + PROBE_NBS * 32u, PROBE_NBS * 16u, 128u);
      const uint32_t tacc = tb + (uint32_t)(b * PROBE_NBS);
      tc::mma_f16(tacc, ahi, bhi, idesc, 0u);
      tc::mma_f16(tacc, alo, bhi, idesc, 1u);
      tc::mma_f16(tacc, ahi, blo, idesc, 1u);
    }
    tc::tc_commit(sbar);
  }
  __syncwarp();
  tc::mbar_wait(sbar, 0, abort_flag, err, 2651);
  tc::tc_fence_after();
  const uint32_t lo = (uint32_t)(warp * 32) << 16;
  uint32_t v[16], w[16];
  tc::tmem_ld16(tb + lo, v);
  tc::tmem_ld16(tb + lo + 16, w);
  tc::tmem_ld_wait16(v);
  tc::reg_pin16(w);
  for (int j = 0; j < 16; ++j) {
    out[tid * PROBE_K + j] = v[j];
    out[tid * PROBE_K + 16 + j] = w[j];
  }
  tc::tc_fence_before();
  block_sync();
  if (warp == 0) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tb), "r"(32));
  }
}

}  // namespace tcw

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static int g_probe_wide[64];
static bool g_probe_wide_init = false;

int tc_probe_wide(int* mode_out, uint32_t* raw_out) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (!g_probe_wide_init) {
    for (int& m : g_probe_wide) m = -2;
    g_probe_wide_init = true;
  }
  if (dev < 64 && g_probe_wide[dev] != -2 && !raw_out) {
    *mode_out = g_probe_wide[dev];
    return OK;
  }
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  const size_t out_words = 4097;
  const size_t img_halves = cimg_halves(tcw::PROBE_K, tcw::PROBE_NK, kCimgBlocked);
  DevBuffers buf(s);
  uint32_t* d_out = nullptr;
  uint16_t* d_img = nullptr;
  SKM_TRY(buf.alloc_n(&d_out, out_words));
  SKM_TRY(buf.alloc_n(&d_img, img_halves));
  SKM_CUDA(cudaMemsetAsync(d_out, 0, out_words * 4, s));
  SKM_CUDA(cudaMemsetAsync(d_img, 0, img_halves * 2, s));
  tcw::tc_probe_wide_kernel<<<1, 128, 0, s>>>(d_img, d_out);
  SKM_TRY(check_launch("tc_probe_wide_kernel"));
  std::vector<uint32_t> h(out_words, 0);
  SKM_CUDA(cudaMemcpyAsync(h.data(), d_out, out_words * 4, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  if (raw_out) memcpy(raw_out, h.data(), 4096 * 4);
  int mode = h[4096] == 0 ? 0 : -1;
  for (int m = 0; m < tc::BM && mode == 0; ++m)
    for (int c = 0; c < tcw::PROBE_K; ++c) {
      double t = 0.0;  // x_hi.c_hi + x_lo.c_hi + x_hi.c_lo, exact in double
      for (int j = 0; j < tcw::PROBE_NK * tc::KC; ++j) {
        const double x = tc::probe_x(m, j), cc = tc::probe_c(c, j);
        const double xh = std::nearbyint(x), ch = std::nearbyint(cc);
        t += xh * ch + (x - xh) * ch + xh * (cc - ch);
      }
      float got;
      memcpy(&got, &h[m * tcw::PROBE_K + c], 4);
      if (got != (float)t) {
        mode = -1;
        break;
      }
    }
  if (dev < 64) g_probe_wide[dev] = mode;
  *mode_out = mode;
  return OK;
}

// Plan of the k > 256 E-step (estep_wide_kernel) for d <= 128, k <= 4096.
int tc_plan_wide(const float* X, int ld, long long n, int d, int k, int optin, TcPlan* plan) {
  plan->supported = false;
  if (k <= tc::MAX_KPAD || k > tcw::MAX_K || d > tc::MAX_NK * tc::KC) return OK;
  int mode = -1;
  SKM_TRY(tc_probe_wide(&mode, nullptr));
  if (mode < 0) return OK;  // unexpected tensor-core behaviour: SIMT E-step
  plan->X = X;
  plan->ld = ld;
  plan->n = n;
  plan->d = d;
  plan->k = k;
  plan->wide = 1;
  plan->nblk = (k + tcw::MAX_NBS - 1) / tcw::MAX_NBS;
  plan->nbs = (int)round_up((size_t)((k + plan->nblk - 1) / plan->nblk), 16);
  plan->k_pad = plan->nbs * plan->nblk;
  plan->k_steps = (ld + tc::KC - 1) / tc::KC;
  const int npairs = (plan->k_steps + 1) / 2;
  plan->stacked = kCimgBlocked;
  plan->stage_bytes = (uint32_t)(2 * npairs) * tc::CHUNK_BYTES;  // an odd nk's extra chunk stays zero
  plan->unit_bytes = (uint32_t)plan->nbs * 64;
  plan->img_bytes = (uint32_t)(cimg_halves(plan->k_pad, plan->k_steps, kCimgBlocked) * 2);
  // at least 2 X stages and 4 centre units; then up to 4 X stages, then up to 8 units
  plan->stages = 0;
  int best_x = 0, best_r = 0;
  for (int xs = 2; xs <= tcw::MAX_XST; ++xs)
    for (int r = 4; r <= tcw::MAX_RING; ++r) {
      const tcw::Layout L = tcw::layout(plan->stage_bytes, xs, plan->unit_bytes, r, plan->k_pad);
      if ((int)L.total > optin) continue;
      // prefer the centre ring up to 5 units, then X stages, then more units
      const int score = std::min(r, 5) * 100 + xs * 10 + r;
      if (score > std::min(best_r, 5) * 100 + best_x * 10 + best_r) {
        best_x = xs;
        best_r = r;
      }
    }
  if (best_x == 0) return OK;
  plan->stages = best_x;
  plan->ring = best_r;
  // more than half of a CTA's shared memory: one CTA per SM, so its 512-column
  // TMEM allocation never waits for another CTA's
  plan->smem = std::max<size_t>(tcw::layout(plan->stage_bytes, best_x, plan->unit_bytes, best_r, plan->k_pad).total,
                                (size_t)optin / 2 + 1024);
  plan->acc_cols = plan->nbs;
  plan->nacc = 2;
  int tcols = 32;
  while (tcols < 2 * plan->nbs) tcols *= 2;
  plan->tmem_cols = tcols;
  const int n_tiles = (int)((n + tc::BM - 1) / tc::BM);
  plan->grid = std::min(n_tiles, sm_count());
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    SKM_CUDA(cudaFuncSetAttribute(tcw::estep_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
    attr_dev = dev;
  }
  plan->supported = true;
  return OK;
}

int tc_estep_wide(const TcPlan& plan, const uint16_t* img, const int* sexp, const float* bias, int32_t* labels,
                  unsigned long long* changed, long long* D, const FitState* st, int* err, cudaStream_t s, bool pdl) {
  tcw::Params p{};
  p.n_tiles = (int)((plan.n + tc::BM - 1) / tc::BM);
  p.n = plan.n;
  p.k = plan.k;
  p.k_pad = plan.k_pad;
  p.nbs = plan.nbs;
  p.nblk = plan.nblk;
  p.nk = plan.k_steps;
  p.npairs = (plan.k_steps + 1) / 2;
  p.xst = plan.stages;
  p.ring = plan.ring;
  p.tmem_cols = plan.tmem_cols;
  p.stage_bytes = plan.stage_bytes;
  p.tile_bytes = (uint32_t)(plan.k_steps * tc::CHUNK_BYTES);
  p.unit_bytes = plan.unit_bytes;
  p.Xs = plan.Xs;
  p.img = img;
  p.sexp = sexp;
  p.bias = bias;
  p.labels = labels;
  p.changed = changed;
  p.D = D;
  p.X = plan.X;
  p.ld = plan.ld;
  p.d = plan.d;
  p.st = st;
  p.err = err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(tcw::THREADS);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  SKM_CUDA(cudaLaunchKernelEx(&cfg, tcw::estep_wide_kernel, p));
  return check_launch("estep_wide_kernel");
}

}  // namespace skm

extern "C" int skmetal_debug_tc_probe_wide(int* mode, uint32_t* raw4096) { return skm::tc_probe_wide(mode, raw4096); }
