// Tensor-core E-step for sm_100a: labels[i] = argmin_j (||c_j||^2 - 2 x_i . c_j)
// over 128-row tiles of X, with the dot products computed by tcgen05.mma in
// split-fp16 precision (x_hi.c_hi + x_lo.c_hi + x_hi.c_lo, the 3xTF32 scheme
// with fp16 parts of power-of-two scaled values; see CentreImage) and
// accumulated in fp32 in tensor memory (TMEM). The n x k distance matrix never
// leaves the SM: the epilogue reads each row's accumulators from TMEM and keeps
// a running argmin in registers (strict '<', lowest index first, as
// sklearn/cluster/_k_means_lloyd.pyx:205-213). Rows whose label changed add
// their exact fixed-point deltas to the centroid sums (the incremental M-step
// input).
//
// Operands: the fit keeps a split working copy of X (split_x_kernel, once per
// fit) whose 128-row tiles are, byte for byte, the kind::f16 A operand
// (x_hi | x_lo per 8-column chunk, canonical no-swizzle K-major layout), and a
// centre image written by the M-step in exactly the B operand's shared-memory
// layout. A tile therefore goes HBM -> shared memory in bulk copies and
// straight into the MMAs; the image is loaded once per CTA.
//
// Data path of one tile (all asynchronous, one persistent CTA per SM):
//   producer   : HBM --bulk copy--> smem stage
//   MMA thread : acc = A . B   (one MMA per 8-column chunk)
//   epilogue   : TMEM acc --tcgen05.ld--> argmin --> labels, deltas
// X is read from HBM once per iteration (4 bytes per element, as fp32).
//
// Warp roles (640 threads): 0 bulk-copy producer, 1 TMEM owner + MMA issuer
// of even tiles, 2 MMA issuer of odd tiles, 3 idle, 4-19 epilogue. One thread
// issues tcgen05.mma at roughly one instruction per ~120 cycles whatever N is,
// while issuers on different SM sub-partitions overlap, so tiles alternate
// between two issuing warps. Warp w reads TMEM lanes 32*(w%4) .. +31 (= tile
// rows); the epilogue warps form up to four groups of one warp per lane
// quarter, group g taking the tiles of accumulator g.
//
// Every mbarrier wait is bounded in time; on timeout the CTA records an error
// code, stops issuing work, waits (bounded) for its own in-flight copies and
// tensor-core operations, frees its tensor memory and returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "device_util.cuh"
#include "driver.h"
#include "estep_tc.h"

namespace skm {

namespace tc {

constexpr int BM = 128;                   // rows per tile (UMMA M)
constexpr int KC = 8;                     // fp32 columns per K chunk (one kind::f16 MMA, K = 16)
constexpr int CHUNK_BYTES = BM * KC * 4;  // 4096
constexpr int MAX_NK = 16;                // d <= 128
constexpr int MAX_KPAD = 256;             // k <= 256 (one UMMA N)
constexpr int THREADS = 640;
constexpr int MAX_STAGES = 4;
constexpr int MAX_ACC = 4;
constexpr unsigned long long TIMEOUT_NS = 2000000000ull;  // 2 s per wait

struct Params {
  int n_tiles;
  long long n;
  int k;
  int k_pad;
  int nk;         // K chunks of 8 columns
  int stacked;    // centre image layout (CentreImage)
  int stages;     // X stages in shared memory
  int nacc;       // accumulators in TMEM (1, 2 or 4)
  int acc_cols;   // TMEM columns of one accumulator
  int tmem_cols;
  uint32_t stage_bytes;  // >= tile_bytes (an even number of chunks when not stacked)
  uint32_t tile_bytes;   // nk * 4096: one tile of the split copy
  uint32_t img_bytes;
  const unsigned char* Xs;  // split working copy
  const uint16_t* img;      // centre image
  const int* sexp;          // {xexp, cexp}: operand scales 2^xexp, 2^cexp
  const float* bias;        // ||c||^2, k entries
  int32_t* labels;
  unsigned long long* changed;
  long long* D;     // nullable: incremental deltas of rows that changed label
  const float* X;   // fp32 blocked copy (the deltas read exact values from it)
  int ld;
  int d;
  const FitState* st;   // nullable: skip when st->done; scale for D
  int* err;
};

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

// Bounded wait: false on timeout (after recording `code`) or when another
// thread of the CTA aborted.
__device__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > TIMEOUT_NS) {
        *abort_flag = 1;
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(reinterpret_cast<unsigned long long>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// K-major no-swizzle shared-memory matrix descriptor: core matrices of 8 rows
// x 16 bytes; `lbo` = bytes between the two K halves of a K = 16 slice, `sbo`
// = bytes between 8-row groups; descriptor version 1, layout type 0.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

// kind::f16 instruction descriptor: D fp32, A/B fp16, both K-major, M = 128, N.
__host__ __device__ constexpr uint32_t idesc_f16(int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// D[tmem] (+)= A[smem] . B[smem]^T
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// The MMAs of one tile: A = stage (split copy of X), B = centre image in smem.
// The start address sits in the low 14 bits of a descriptor (address / 16,
// shared memory < 256 KB), so later chunks advance a descriptor by addition.
__device__ __forceinline__ void issue_tile_mmas(uint32_t tacc, uint32_t stage, uint32_t img, int nk, int k_pad,
                                                int stacked) {
  const uint64_t a0 = kmajor_desc(stage, 2048u, 128u);
  const uint64_t a_step = CHUNK_BYTES >> 4;
  if (stacked) {
    const int N = 2 * k_pad;
    const uint32_t idesc = idesc_f16(N);
    const uint64_t b0 = kmajor_desc(img, (uint32_t)(N * 16), 128u);
    const uint64_t b_step = (uint64_t)(N * 32) >> 4;
    for (int c = 0; c < nk; ++c) mma_f16(tacc, a0 + c * a_step, b0 + c * b_step, idesc, c > 0 ? 1u : 0u);
  } else {
    const uint32_t idesc = idesc_f16(k_pad);
    const uint64_t b0 = kmajor_desc(img, (uint32_t)(k_pad * 16), 128u);
    const uint64_t b_step = (uint64_t)(k_pad * 32) >> 4;
    for (int c = 0; c < nk; ++c) mma_f16(tacc, a0 + c * a_step, b0 + c * b_step, idesc, c > 0 ? 1u : 0u);
    // x_hi of chunk pairs (2m | 2m + 1) times c_lo of the same pair
    const uint64_t p0 = kmajor_desc(stage, (uint32_t)CHUNK_BYTES, 128u);
    const uint64_t q0 = kmajor_desc(img + (uint32_t)(nk * k_pad * 32), (uint32_t)(k_pad * 16), 128u);
    for (int m = 0; 2 * m < nk; ++m) mma_f16(tacc, p0 + 2 * m * a_step, q0 + m * b_step, idesc, 1u);
  }
}

// stages at s * stage_bytes from 0, then the centre image, bias, barriers and
// misc words
struct Smem {
  uint32_t c, bias, bars, misc, total;
};

// barrier indices
__host__ __device__ constexpr int B_FULL(int s) { return s; }               // stage loaded
__host__ __device__ constexpr int B_EMPTY(int s) { return MAX_STAGES + s; }  // stage consumed by the MMAs
__host__ __device__ constexpr int B_ACC_FULL(int a) { return 2 * MAX_STAGES + a; }
__host__ __device__ constexpr int B_ACC_EMPTY(int a) { return 2 * MAX_STAGES + MAX_ACC + a; }
constexpr int B_C_FULL = 2 * MAX_STAGES + 2 * MAX_ACC;
__host__ __device__ constexpr int B_DONE(int t) { return B_C_FULL + 1 + t; }  // drain of MMA issuer t
constexpr int NUM_BARS = B_C_FULL + 3;

constexpr int MMA_W0 = 1, MMA_W1 = 2;
constexpr int EPI_W0 = 4;
constexpr int EPI_GROUPS = 4;  // one warp per TMEM lane quarter each
static_assert((EPI_W0 + 4 * EPI_GROUPS) * 32 == THREADS, "warp roles must fill the block");

__host__ __device__ inline Smem smem_layout(uint32_t stage_bytes, uint32_t img_bytes, int k_pad, int stages) {
  Smem s;
  uint32_t off = (uint32_t)stages * stage_bytes;
  s.c = off;
  off += img_bytes;
  s.bias = off;
  off += (uint32_t)k_pad * 4;
  off = (off + 15) & ~15u;
  s.bars = off;
  off += NUM_BARS * 8;
  s.misc = off;
  off += 16;             // [0] tmem base, [1] abort flag
  s.total = off + 1024;  // slack for aligning the base to 1024
  return s;
}

__device__ __forceinline__ bool better(float d, int i, float bd, int bi) { return d < bd || (d == bd && i < bi); }

__global__ void __launch_bounds__(THREADS, 1) estep_tc_kernel(Params p) {
  // the M-step that follows may be scheduled as soon as SMs free up; the
  // previous M-step's centres, bias, image and flags must be visible first
  pdl_launch_dependents();
  pdl_wait();
  if (p.st && p.st->done) return;
  // bulk iterations rebuild the sums from all rows in the M-step
  long long* const deltas = (p.st && p.st->bulk) ? nullptr : p.D;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Smem L = smem_layout(p.stage_bytes, p.img_bytes, p.k_pad, p.stages);
  const uint32_t sbase = smem_u32(base);
  const uint32_t bar0 = sbase + L.bars;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(base + L.misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  float* bias_s = reinterpret_cast<float*>(base + L.bias);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int my_tiles = (p.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  // issuer t owns the accumulators a = t mod n_iss and epilogue group g those
  // with a = g mod n_grp (n_iss and n_grp divide nacc), so each accumulator
  // barrier has exactly one producer and one consumer
  const int n_iss = p.nacc >= 2 ? 2 : 1;
  const int n_grp = p.nacc;

  if (threadIdx.x == 0) {
    for (int s = 0; s < MAX_STAGES; ++s) {
      mbar_init(bar(B_FULL(s)), 1);
      mbar_init(bar(B_EMPTY(s)), 1);
    }
    for (int a = 0; a < MAX_ACC; ++a) {
      mbar_init(bar(B_ACC_FULL(a)), 1);
      mbar_init(bar(B_ACC_EMPTY(a)), 4);  // the four warps of one epilogue group
    }
    mbar_init(bar(B_C_FULL), 1);
    mbar_init(bar(B_DONE(0)), 1);
    mbar_init(bar(B_DONE(1)), 1);
    misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_W0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + L.misc),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  for (int j = threadIdx.x; j < p.k_pad; j += blockDim.x) bias_s[j] = j < p.k ? p.bias[j] : INFINITY;
  if (p.tile_bytes < p.stage_bytes) {
    // the extra chunk of an odd nk (read as x_hi by the last pair MMA): zero
    for (int s = 0; s < p.stages; ++s)
      for (uint32_t o = p.tile_bytes + 16u * threadIdx.x; o < p.stage_bytes; o += 16u * blockDim.x)
        *reinterpret_cast<uint4*>(base + (uint32_t)s * p.stage_bytes + o) = make_uint4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = misc[0];

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      mbar_expect_tx(bar(B_C_FULL), p.img_bytes);
      for (uint32_t o = 0; o < p.img_bytes; o += 8192u)
        bulk_load(sbase + L.c + o, reinterpret_cast<const char*>(p.img) + o, min(8192u, p.img_bytes - o),
                  bar(B_C_FULL));
      int armed = 0;
      for (int i = 0; i < my_tiles; ++i) {
        const int s = i % p.stages;
        if (!mbar_wait(bar(B_EMPTY(s)), ((i / p.stages) & 1) ^ 1, abort_flag, p.err, 2101)) break;
        const int tile = (int)blockIdx.x + i * (int)gridDim.x;
        const unsigned char* src = p.Xs + (size_t)tile * p.tile_bytes;
        mbar_expect_tx(bar(B_FULL(s)), p.tile_bytes);
        for (uint32_t o = 0; o < p.tile_bytes; o += 8192u)
          bulk_load(sbase + (uint32_t)s * p.stage_bytes + o, src + o, min(8192u, p.tile_bytes - o), bar(B_FULL(s)));
        armed = i + 1;
      }
      // our own copies must land before the CTA may exit
      volatile int no_abort = 0;
      mbar_wait(bar(B_C_FULL), 0, &no_abort, p.err, 2102);
      for (int i = (armed > p.stages ? armed - p.stages : 0); i < armed; ++i)
        mbar_wait(bar(B_FULL(i % p.stages)), (i / p.stages) & 1, &no_abort, p.err, 2103);
    }
  } else if (warp == MMA_W0 || warp == MMA_W1) {
    // ---------------------------------------------------------- MMA issuers
    const int t = warp == MMA_W0 ? 0 : 1;
    if (lane == 0 && t < n_iss) {
      bool ok = mbar_wait(bar(B_C_FULL), 0, abort_flag, p.err, 2201);
      for (int i = t; ok && i < my_tiles; i += n_iss) {
        const int s = i % p.stages, a = i % p.nacc;
        if (!mbar_wait(bar(B_ACC_EMPTY(a)), ((i / p.nacc) & 1) ^ 1, abort_flag, p.err, 2203)) break;
        // A parity wait is only exact while the waiter is at most one phase
        // away from the barrier. With two issuers and an odd number of stages,
        // the previous use of stage s belongs to the other issuer, and copies
        // can land out of order, so FULL(s) alone could still show the phase
        // of use u - 2. Waiting first for the previous use to be consumed
        // (EMPTY(s), phase u - 1, as the producer does; this issuer's own MMAs
        // of use u - 2 completed before its accumulator of tile i was freed)
        // pins FULL(s) to phase u - 1 or u.
        if (!mbar_wait(bar(B_EMPTY(s)), ((i / p.stages) & 1) ^ 1, abort_flag, p.err, 2204)) break;
        if (!mbar_wait(bar(B_FULL(s)), (i / p.stages) & 1, abort_flag, p.err, 2202)) break;
        tc_fence_after();
        issue_tile_mmas(tmem_base + (uint32_t)(a * p.acc_cols), sbase + (uint32_t)s * p.stage_bytes, sbase + L.c, p.nk, p.k_pad,
                        p.stacked);
        tc_commit(bar(B_EMPTY(s)));  // the stage is no longer read by the tensor core
        tc_commit(bar(B_ACC_FULL(a)));
      }
      // every tcgen05 operation issued by this thread is complete once DONE fires
      tc_commit(bar(B_DONE(t)));
      volatile int no_abort = 0;
      mbar_wait(bar(B_DONE(t)), 0, &no_abort, p.err, 2206);
    }
  } else if (warp >= EPI_W0) {
    // ----------------------------------------------------------------- epilogue
    // groups of four warps (one per TMEM lane quarter) take the tiles of their
    // accumulator; each warp scans all clusters of its 32 rows
    const int q = warp & 3;
    const int g = (warp - EPI_W0) >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    // dist = ||c||^2 - 2 x.c with x.c = acc * 2^-(xexp + cexp)
    const float negscale = -ldexpf(1.0f, 1 - p.sexp[0] - p.sexp[1]);
    int old_next = -1;
    if (g < n_grp && p.changed && g < my_tiles) {
      const long long g0 = (long long)((int)blockIdx.x + g * (int)gridDim.x) * BM + row;
      old_next = g0 < p.n ? p.labels[g0] : -1;
    }
    for (int i = g; g < n_grp && i < my_tiles; i += n_grp) {
      const int a = i % p.nacc;
      const long long grow = (long long)((int)blockIdx.x + i * (int)gridDim.x) * BM + row;
      const int old = old_next;
      if (p.changed && i + n_grp < my_tiles) {  // prefetch the next tile's previous labels
        const long long g1 = grow + (long long)n_grp * gridDim.x * BM;
        old_next = g1 < p.n ? p.labels[g1] : -1;
      }
      if (!mbar_wait(bar(B_ACC_FULL(a)), (i / p.nacc) & 1, abort_flag, p.err, 2401)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + lane_off + (uint32_t)(a * p.acc_cols);
      // four independent running minima (columns j = 4m + u), merged in index order
      float bd[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
      int bi[4] = {0x7fffffff, 0x7fffffff, 0x7fffffff, 0x7fffffff};
      for (int jb = 0; jb < p.k_pad; jb += 16) {
        uint32_t v[16], w[16];
        tmem_ld16(taddr + (uint32_t)jb, v);
        if (p.stacked) tmem_ld16(taddr + (uint32_t)(p.k_pad + jb), w);
        tmem_ld_wait();
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int j = jb + jj;
          float dot = __uint_as_float(v[jj]);
          if (p.stacked) dot += __uint_as_float(w[jj]);
          const float dist = fmaf(dot, negscale, bias_s[j]);
          if (dist < bd[jj & 3]) {
            bd[jj & 3] = dist;
            bi[jj & 3] = j;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_ACC_EMPTY(a)));
      float best = bd[0];
      int bl = bi[0];
#pragma unroll
      for (int u = 1; u < 4; ++u)
        if (better(bd[u], bi[u], best, bl)) {
          best = bd[u];
          bl = bi[u];
        }
      if (bl >= p.k) bl = 0;  // only reachable when every distance is +inf or NaN
      bool ch = false;
      if (grow < p.n) {
        ch = p.changed && old != bl;
        p.labels[grow] = bl;
      }
      if (p.changed) {
        const unsigned int m = __ballot_sync(0xffffffffu, ch);
        if (lane == 0 && m) atomicAdd(p.changed, (unsigned long long)__popc(m));
        if (deltas) warp_apply_changed(p.X, p.ld, p.d, p.k, grow, old, bl, ch, deltas, p.st->scale);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_W0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.tmem_cols));
  }
}

// ---------------------------------------------------------------------------
// split working copy of X (see the layout note at split8)
// ---------------------------------------------------------------------------
// One thread per (tile, chunk, row): reads the row's two fp32 column quads of
// the chunk from the blocked copy and writes its x_hi and x_lo (16 bytes each)
// at the same row position of the chunk's two halves; consecutive threads take
// consecutive rows, so reads and writes are coalesced 512-byte runs per warp.
__global__ void split_x_kernel(const float* __restrict__ X, int ld, int nk, long long n_tiles,
                               const int* __restrict__ sexp, uint4* __restrict__ Xs) {
  const float s = ldexpf(1.0f, sexp[0]);
  const int nq = ld >> 2;
  const long long total = n_tiles * nk * BM;
  const float4* X4 = reinterpret_cast<const float4*>(X);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)(i & (BM - 1));
    const long long tc = i >> 7;  // tile * nk + chunk
    const long long t = tc / nk;
    const int c = (int)(tc - t * nk);
    const float4* xt = X4 + t * (32LL * ld);  // tile t of the blocked copy: quad j at xt[128 j]
    const float4 a = xt[(long long)(2 * c) * 128 + row];
    const float4 b = (2 * c + 1 < nq) ? xt[(long long)(2 * c + 1) * 128 + row] : make_float4(0.f, 0.f, 0.f, 0.f);
    uint4 hi, lo;
    split8(a, b, s, &hi, &lo);
    uint4* dst = Xs + tc * (CHUNK_BYTES / 16);
    dst[row] = hi;
    dst[BM + row] = lo;
  }
}

// ---------------------------------------------------------------------------
// probe: operand layouts of the split-fp16 path, checked on exact values
// ---------------------------------------------------------------------------
// A 128 x 16 tile (two chunks) and 16 centres whose fp16 splits are exact
// (x = p + q 2^-12, c = r + s 2^-12 with |p|, |r| in [8, 16), |q|, |s| <= 8),
// so that x_hi.c_hi + x_lo.c_hi + x_hi.c_lo is exact in fp32. The tile goes
// through split8 and the centres through cimg_put, as in the fit;
// the stacked (N = 32) and two-segment (N = 16) MMA sequences then run on
// them. out: [0, 2048) stacked x.c (acc[j] + acc[16 + j]), [2048, 4096)
// two-segment x.c, row-major 128 x 16; [4096] error code.
constexpr int PROBE_K = 16, PROBE_NK = 2;

__host__ __device__ inline float probe_x(int m, int j) {
  const int p = 8 + ((m * 7 + j * 3) % 8);
  const int q = ((m * 5 + j * 11) % 17) - 8;
  return (float)(((m + j) & 1) ? -p : p) + (float)q * (1.0f / 4096.0f);
}

__host__ __device__ inline float probe_c(int c, int j) {
  const int r = 8 + ((c * 3 + j * 5) % 8);
  const int s = ((c * 13 + j * 7) % 17) - 8;
  return (float)(((c + 2 * j) % 3 == 0) ? -r : r) + (float)s * (1.0f / 4096.0f);
}

__global__ void __launch_bounds__(128, 1) tc_probe_kernel(uint16_t* img_st, uint16_t* img_2s, uint32_t* out) {
  constexpr uint32_t TILE = PROBE_NK * CHUNK_BYTES;                 // 8 KB
  constexpr uint32_t IMG_ST = PROBE_NK * 2 * PROBE_K * 32;          // 2 KB
  constexpr uint32_t IMG_2S = PROBE_NK * PROBE_K * 32 + PROBE_K * 32;  // 1.5 KB
  __shared__ __align__(1024) unsigned char sm[TILE + IMG_ST + IMG_2S + 64];
  const uint32_t sa = smem_u32(sm), sb1 = sa + TILE, sb2 = sb1 + IMG_ST, sbar = sb2 + IMG_2S;
  uint32_t* misc = reinterpret_cast<uint32_t*>(sm + TILE + IMG_ST + IMG_2S + 16);
  const uint32_t smisc = smem_u32(misc);
  int* err = reinterpret_cast<int*>(out + 4096);
  const int tid = threadIdx.x, warp = tid >> 5;
  // fp32 tile in the blocked layout, split in place
  for (int j = 0; j < PROBE_NK * KC; ++j)
    *reinterpret_cast<float*>(sm + (j >> 2) * 2048 + tid * 16 + (j & 3) * 4) = probe_x(tid, j);
  for (int c = 0; c < PROBE_NK; ++c) {
    uint4* q0 = reinterpret_cast<uint4*>(sm + (2 * c) * 2048 + tid * 16);
    uint4* q1 = reinterpret_cast<uint4*>(sm + (2 * c + 1) * 2048 + tid * 16);
    const float4 a = *reinterpret_cast<const float4*>(q0), b = *reinterpret_cast<const float4*>(q1);
    split8(a, b, 1.0f, q0, q1);
  }
  // centre images: built in global memory by cimg_put, copied to smem
  const CentreImage st{img_st, PROBE_K, PROBE_NK, 1}, two{img_2s, PROBE_K, PROBE_NK, 0};
  for (int e = tid; e < PROBE_K * PROBE_NK * KC; e += blockDim.x) {
    const int c = e / (PROBE_NK * KC), j = e % (PROBE_NK * KC);
    cimg_put(st, c, j, probe_c(c, j), 1.0f);
    cimg_put(two, c, j, probe_c(c, j), 1.0f);
  }
  __syncthreads();
  for (uint32_t o = tid * 2; o < IMG_ST / 2; o += 2 * blockDim.x)
    *reinterpret_cast<uint32_t*>(sm + TILE + o * 2) = *reinterpret_cast<const uint32_t*>(img_st + o);
  for (uint32_t o = tid * 2; o < IMG_2S / 2; o += 2 * blockDim.x)
    *reinterpret_cast<uint32_t*>(sm + TILE + IMG_ST + o * 2) = *reinterpret_cast<const uint32_t*>(img_2s + o);
  if (tid == 0) {
    mbar_init(sbar, 1);
    misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smisc), "r"(64));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = misc[0];
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  // TMEM columns: [0, 32) stacked accumulator, [32, 48) two-segment accumulator
  if (tid == 0) {
    issue_tile_mmas(tb, sa, sb1, PROBE_NK, PROBE_K, 1);
    issue_tile_mmas(tb + 32, sa, sb2, PROBE_NK, PROBE_K, 0);
    tc_commit(sbar);
  }
  __syncwarp();
  mbar_wait(sbar, 0, abort_flag, err, 2501);
  tc_fence_after();
  const uint32_t lo = (uint32_t)(warp * 32) << 16;
  uint32_t v[16], w[16], u[16];
  tmem_ld16(tb + lo, v);
  tmem_ld16(tb + lo + 16, w);
  tmem_ld16(tb + lo + 32, u);
  tmem_ld_wait();
  for (int j = 0; j < PROBE_K; ++j) {
    out[tid * PROBE_K + j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
    out[2048 + tid * PROBE_K + j] = u[j];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tb), "r"(64));
  }
}

}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

// Per-device probe result: -2 not run, -1 unusable, 0 exact.
static int g_probe_mode[64];
static bool g_probe_init = false;

// Exact value of x_hi.c_hi + x_lo.c_hi + x_hi.c_lo for the probe operands
// (p r + q r 2^-12 + p s 2^-12 summed over 16 columns, exact in double).
static double probe_expected(int m, int c) {
  double t = 0.0;
  for (int j = 0; j < tc::PROBE_NK * tc::KC; ++j) {
    const double x = tc::probe_x(m, j), cc = tc::probe_c(c, j);
    const double xh = std::nearbyint(x), ch = std::nearbyint(cc);
    t += xh * ch + (x - xh) * ch + xh * (cc - ch);
  }
  return t;
}

int tc_probe(int* mode_out, uint32_t* raw_out) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (!g_probe_init) {
    for (int& m : g_probe_mode) m = -2;
    g_probe_init = true;
  }
  if (dev < 64 && g_probe_mode[dev] != -2 && !raw_out) {
    *mode_out = g_probe_mode[dev];
    return OK;
  }
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  const size_t out_words = 4097;
  const size_t img_halves = cimg_halves(tc::PROBE_K, tc::PROBE_NK, 1) + cimg_halves(tc::PROBE_K, tc::PROBE_NK, 0);
  uint32_t* d_out = nullptr;
  uint16_t* d_img = nullptr;
  SKM_CUDA(cudaMallocAsync(&d_out, out_words * 4, s));
  int rc = OK;
  if (cudaMallocAsync(&d_img, img_halves * 2, s) != cudaSuccess) {
    cudaGetLastError();
    rc = ERR_OOM;
  }
  if (rc == OK && (cudaMemsetAsync(d_out, 0, out_words * 4, s) != cudaSuccess ||
                   cudaMemsetAsync(d_img, 0, img_halves * 2, s) != cudaSuccess))
    rc = ERR_CUDA;
  if (rc == OK) {
    tc::tc_probe_kernel<<<1, 128, 0, s>>>(d_img, d_img + cimg_halves(tc::PROBE_K, tc::PROBE_NK, 1), d_out);
    rc = check_launch("tc_probe_kernel");
  }
  std::vector<uint32_t> h(out_words, 0);
  if (rc == OK) {
    cudaMemcpyAsync(h.data(), d_out, out_words * 4, cudaMemcpyDeviceToHost, s);
    if (cudaStreamSynchronize(s) != cudaSuccess) rc = ERR_CUDA;
  }
  cudaFreeAsync(d_out, s);
  if (d_img) cudaFreeAsync(d_img, s);
  if (rc != OK) {
    set_error(rc, "tensor-core probe failed to run");
    return rc;
  }
  if (raw_out) memcpy(raw_out, h.data(), 4096 * 4);
  int mode = h[4096] == 0 ? 0 : -1;
  for (int m = 0; m < tc::BM && mode == 0; ++m)
    for (int c = 0; c < tc::PROBE_K; ++c) {
      const float want = (float)probe_expected(m, c);
      float a, b;
      memcpy(&a, &h[m * tc::PROBE_K + c], 4);
      memcpy(&b, &h[2048 + m * tc::PROBE_K + c], 4);
      if (a != want || b != want) {
        mode = -1;
        break;
      }
    }
  if (dev < 64) g_probe_mode[dev] = mode;
  *mode_out = mode;
  return OK;
}

int tc_plan(const float* X, int ld, long long n, int d, int k, TcPlan* plan) {
  plan->supported = false;
  if (getenv("SKMETAL_DISABLE_TC")) return OK;
  if (d > tc::MAX_NK * tc::KC || k > tc::MAX_KPAD || n < 1) return OK;
  if ((reinterpret_cast<uintptr_t>(X) & 15) || ((ld * 4) & 15)) return OK;
  int dev = 0, optin = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return OK;
  int mode = -1;
  SKM_TRY(tc_probe(&mode, nullptr));
  if (mode < 0) return OK;  // unexpected tensor-core behaviour: use the SIMT E-step
  plan->X = X;
  plan->ld = ld;
  plan->n = n;
  plan->d = d;
  plan->k = k;
  plan->k_pad = (int)round_up((size_t)k, 16);
  plan->k_steps = (ld + tc::KC - 1) / tc::KC;
  // prefer one stacked operand (one MMA per chunk); both layouts need >= 2 stages
  plan->stages = 0;
  for (int stacked = (2 * plan->k_pad <= 256) ? 1 : 0; stacked >= 0 && plan->stages == 0; --stacked) {
    const int nkx = stacked ? plan->k_steps : (plan->k_steps + 1) & ~1;
    const uint32_t stage_bytes = (uint32_t)nkx * tc::CHUNK_BYTES;
    const uint32_t img_bytes = (uint32_t)(cimg_halves(plan->k_pad, plan->k_steps, stacked) * 2);
    for (int st = tc::MAX_STAGES; st >= 2; --st) {
      const tc::Smem L = tc::smem_layout(stage_bytes, img_bytes, plan->k_pad, st);
      if ((int)L.total <= optin) {
        plan->stacked = stacked;
        plan->stages = st;
        plan->stage_bytes = stage_bytes;
        plan->img_bytes = img_bytes;
        plan->smem = L.total;
        break;
      }
    }
  }
  if (plan->stages == 0) return OK;
  plan->acc_cols = plan->stacked ? 2 * plan->k_pad : plan->k_pad;
  // 4, 2 or 1 accumulators (see the issuer / epilogue pairing in the kernel)
  plan->nacc = 4 * plan->acc_cols <= 512 ? 4 : (2 * plan->acc_cols <= 512 ? 2 : 1);
  int tcols = 32;
  while (tcols < plan->nacc * plan->acc_cols) tcols *= 2;
  plan->tmem_cols = tcols;
  const int n_tiles = (int)((n + tc::BM - 1) / tc::BM);
  plan->grid = std::min(n_tiles, sm_count());
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(tc::estep_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    attr = true;
  }
  plan->supported = true;
  return OK;
}

size_t tc_split_bytes(const TcPlan& plan) {
  return (size_t)((plan.n + tc::BM - 1) / tc::BM) * plan.k_steps * tc::CHUNK_BYTES;
}

int tc_split_x(TcPlan* plan, void* Xs, const int* sexp, cudaStream_t s) {
  const long long n_tiles = (plan->n + tc::BM - 1) / tc::BM;
  const long long work = n_tiles * plan->k_steps * tc::BM;
  const int blocks = (int)std::max(1LL, std::min((work + 255) / 256, (long long)sm_count() * 8));
  tc::split_x_kernel<<<blocks, 256, 0, s>>>(plan->X, plan->ld, plan->k_steps, n_tiles, sexp,
                                            reinterpret_cast<uint4*>(Xs));
  SKM_TRY(check_launch("split_x_kernel"));
  plan->Xs = static_cast<const unsigned char*>(Xs);
  return OK;
}

CentreImage tc_centre_image(const TcPlan& plan, uint16_t* img) {
  return CentreImage{img, plan.k_pad, plan.k_steps, plan.stacked};
}

int tc_estep(const TcPlan& plan, const uint16_t* img, const int* sexp, const float* bias, int32_t* labels,
             unsigned long long* changed, long long* D, const FitState* st, int* err, cudaStream_t s, bool pdl) {
  tc::Params p;
  p.n_tiles = (int)((plan.n + tc::BM - 1) / tc::BM);
  p.n = plan.n;
  p.k = plan.k;
  p.k_pad = plan.k_pad;
  p.nk = plan.k_steps;
  p.stacked = plan.stacked;
  p.stages = plan.stages;
  p.nacc = plan.nacc;
  p.acc_cols = plan.acc_cols;
  p.tmem_cols = plan.tmem_cols;
  p.stage_bytes = plan.stage_bytes;
  p.img_bytes = plan.img_bytes;
  p.tile_bytes = (uint32_t)(plan.k_steps * tc::CHUNK_BYTES);
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
  if (pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(tc::THREADS);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SKM_CUDA(cudaLaunchKernelEx(&cfg, tc::estep_tc_kernel, p));
  } else {
    tc::estep_tc_kernel<<<plan.grid, tc::THREADS, plan.smem, s>>>(p);
  }
  return check_launch("estep_tc_kernel");
}

}  // namespace skm

extern "C" int skmetal_debug_tc_probe(int* mode, uint32_t* raw4096) { return skm::tc_probe(mode, raw4096); }
