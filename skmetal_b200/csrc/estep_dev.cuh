// Device code of the tensor-core E-step pipeline (sm_100a), shared by the
// stand-alone E-step kernel (estep_tc.cu) and the persistent Lloyd loop
// kernel (loop_tc.cu): mbarrier / bulk-copy / tcgen05 wrappers, the shared
// memory layout, and one pass of the warp-specialised pipeline over a CTA's
// tiles (estep_pass), which a persistent kernel may run once per iteration.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "device_util.cuh"
#include "estep_tc.h"
#include "skm.cuh"

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
constexpr int L2_AHEAD = 8;  // tiles of the next pass prefetched into L2 beyond the stages
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
  uint32_t tile_bytes;   // one tile of the split copy: nk * 4096, less 2048 with a half last chunk
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

// Bounded wait: false on timeout (after recording `code`) or when another
// thread of the CTA aborted.
static __device__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err, int code) {
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

// Bounded wait of a whole warp (every lane waits) with one outcome for all
// lanes, so that the warp stays converged for the .sync.aligned TMEM loads,
// votes and per-warp arrivals that follow, even if the wait ends at its time
// limit on some lanes only.
static __device__ __forceinline__ bool warp_wait_all(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err,
                                                     int code) {
  const bool ok = mbar_wait(bar, parity, abort_flag, err, code);
  return __all_sync(0xffffffffu, ok);
}

// K-major no-swizzle shared-memory matrix descriptor: core matrices of 8 rows
// x 16 bytes; `lbo` = bytes between the two K halves of a K = 16 slice, `sbo`
// = bytes between 8-row groups; descriptor version 1, layout type 0. Kept as
// two 32-bit words: lo = start address >> 4 (bits 0-13) | lbo >> 4 (bits
// 16-29), hi = sbo >> 4 (bits 32-45) | version (bit 46). Only lo changes
// along K, and the MMA wrapper joins the words in PTX.
struct SmemDesc {
  uint32_t lo, hi;
};
__device__ __forceinline__ SmemDesc kmajor_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  SmemDesc d;
  d.lo = ((saddr >> 4) & 0x3FFFu) | (((lbo >> 4) & 0x3FFFu) << 16);
  d.hi = ((sbo >> 4) & 0x3FFFu) | (1u << 14);
  return d;
}
// the descriptor of the matrix `bytes` further along (start address field)
__device__ __forceinline__ SmemDesc desc_advance(SmemDesc d, uint32_t bytes) {
  d.lo += bytes >> 4;
  return d;
}

// kind::f16 instruction descriptor: D fp32, A/B fp16, both K-major, M = 128, N.
__host__ __device__ constexpr uint32_t idesc_f16(int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// D[tmem] (+)= A[smem] . B[smem]^T
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, SmemDesc a, SmemDesc b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 ad, bd;\n\t"
      "mov.b64 ad, {%1, %2};\n\t"
      "mov.b64 bd, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %5, p;\n\t}"
      ::"r"(tmem_d), "r"(a.lo), "r"(a.hi), "r"(b.lo), "r"(b.hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same MMA issued by one elected lane of a converged warp. The whole warp
// runs the issuing loop with warp-uniform operands (descriptors, addresses,
// predicates), so they stay uniform values; elect.sync picks the one lane
// that issues, as tcgen05.mma is issued by a single thread.
__device__ __forceinline__ void mma_f16_elect(uint32_t tmem_d, SmemDesc a, SmemDesc b, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b64 ad, bd;\n\t"
      "mov.b64 ad, {%1, %2};\n\t"
      "mov.b64 bd, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %5, p;\n\t}"
      ::"r"(tmem_d), "r"(a.lo), "r"(a.hi), "r"(b.lo), "r"(b.hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// tcgen05.commit by one elected lane of a converged warp.
__device__ __forceinline__ void tc_commit_elect(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
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

// tcgen05.ld is asynchronous: its destination registers hold the data only
// after tcgen05.wait::ld. The wait takes the registers of a load as in/out
// operands, so the compiler cannot schedule their uses before it.
__device__ __forceinline__ void tmem_ld_wait16(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// Orders the uses of r after the preceding volatile asm (a second load's
// registers after tmem_ld_wait16 of the first).
__device__ __forceinline__ void reg_pin16(uint32_t* r) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// The MMAs of one tile: A = stage (split copy of X), B = centre image in smem.
// The start address sits in the low 14 bits of a descriptor (address / 16,
// shared memory < 256 KB), so later chunks advance a descriptor by addition.
__device__ __forceinline__ void issue_tile_mmas(uint32_t tacc, uint32_t stage, uint32_t img, int nk, int k_pad,
                                                int stacked) {
  const SmemDesc a0 = kmajor_desc(stage, 2048u, 128u);
  if (stacked) {
    const int N = 2 * k_pad;
    const uint32_t idesc = idesc_f16(N);
    const SmemDesc b0 = kmajor_desc(img, (uint32_t)(N * 16), 128u);
    for (int c = 0; c < nk; ++c)
      mma_f16(tacc, desc_advance(a0, (uint32_t)c * CHUNK_BYTES), desc_advance(b0, (uint32_t)(c * N * 32)), idesc,
              c > 0 ? 1u : 0u);
  } else {
    const uint32_t idesc = idesc_f16(k_pad);
    const SmemDesc b0 = kmajor_desc(img, (uint32_t)(k_pad * 16), 128u);
    for (int c = 0; c < nk; ++c)
      mma_f16(tacc, desc_advance(a0, (uint32_t)c * CHUNK_BYTES), desc_advance(b0, (uint32_t)(c * k_pad * 32)), idesc,
              c > 0 ? 1u : 0u);
    // x_hi of chunk pairs (2m | 2m + 1) times c_lo of the same pair
    const SmemDesc p0 = kmajor_desc(stage, (uint32_t)CHUNK_BYTES, 128u);
    const SmemDesc q0 = kmajor_desc(img + (uint32_t)(nk * k_pad * 32), (uint32_t)(k_pad * 16), 128u);
    for (int m = 0; 2 * m < nk; ++m)
      mma_f16(tacc, desc_advance(p0, (uint32_t)(2 * m) * CHUNK_BYTES), desc_advance(q0, (uint32_t)(m * k_pad * 32)),
              idesc, 1u);
  }
}

// stages at s * stage_bytes from 0, then the centre image, bias, the split
// epilogue's partial minima, barriers and misc words
struct Smem {
  uint32_t c, bias, part, bars, misc, total;
};

// barrier indices
__host__ __device__ constexpr int B_FULL(int s) { return s; }               // stage loaded
__host__ __device__ constexpr int B_EMPTY(int s) { return MAX_STAGES + s; }  // stage consumed by the MMAs
__host__ __device__ constexpr int B_ACC_FULL(int a) { return 2 * MAX_STAGES + a; }
__host__ __device__ constexpr int B_ACC_EMPTY(int a) { return 2 * MAX_STAGES + MAX_ACC + a; }
constexpr int B_C_FULL = 2 * MAX_STAGES + 2 * MAX_ACC;
__host__ __device__ constexpr int B_DONE(int t) { return B_C_FULL + 1 + t; }  // drain of MMA issuer t
// split epilogue (groups sharing every tile): partial minima of accumulator
// a's use slot s (use count mod 2) written / consumed
__host__ __device__ constexpr int B_PART_FULL(int a, int s) { return B_C_FULL + 3 + 2 * a + s; }
__host__ __device__ constexpr int B_PART_EMPTY(int a, int s) { return B_C_FULL + 7 + 2 * a + s; }
constexpr int NUM_BARS = B_C_FULL + 11;

constexpr int MMA_W0 = 1, MMA_W1 = 2;
constexpr int IDLE_W = 3;  // no role in the pipeline (callers give it side work)
constexpr int EPI_W0 = 4;
constexpr int EPI_GROUPS = 4;  // one warp per TMEM lane quarter each
static_assert((EPI_W0 + 4 * EPI_GROUPS) * 32 == THREADS, "warp roles must fill the block");

// With fewer accumulators than epilogue groups (two: tc_plan keeps an
// accumulator within 256 columns), every group takes every tile and scans one
// quarter of its clusters, and groups 1-3 hand their partial minima to group
// 0 through shared memory. All sixteen epilogue warps then work on the tile
// of one accumulator while the MMAs fill the other; with two groups per
// accumulator both accumulators' epilogues ran together and the tensor core
// waited for them.
__host__ __device__ constexpr int epi_split(int nacc) { return nacc >= EPI_GROUPS ? 1 : EPI_GROUPS; }
__host__ __device__ constexpr uint32_t part_bytes(int nacc) {
  // 2 accumulators x 2 slots x (split - 1) parts x 128 rows x {float, int}
  return epi_split(nacc) > 1 ? (uint32_t)(2 * 2 * (epi_split(nacc) - 1) * BM * 8) : 0u;
}

__host__ __device__ inline Smem smem_layout(uint32_t stage_bytes, uint32_t img_bytes, int k_pad, int stages,
                                            int nacc) {
  Smem s;
  uint32_t off = (uint32_t)stages * stage_bytes;
  s.c = off;
  off += img_bytes;
  s.bias = off;
  off += (uint32_t)k_pad * 4;
  off = (off + 15) & ~15u;
  s.part = off;
  off += part_bytes(nacc);
  s.bars = off;
  off += NUM_BARS * 8;
  s.misc = off;
  off += 16;             // [0] tmem base, [1] abort flag
  s.total = off + 1024;  // slack for aligning the base to 1024
  return s;
}

__device__ __forceinline__ bool better(float d, int i, float bd, int bi) { return d < bd || (d == bd && i < bi); }
__host__ __device__ constexpr int round_up_dev(int a, int b) { return (a + b - 1) / b * b; }

// ---------------------------------------------------------------------------
// Row scan of the epilogue: the first column of smallest distance, with
// dist = fmaf(dot, negscale, bias) in float32 and strict '<' (a NaN distance
// never wins, ties keep the lower column). Columns are taken in pairs: one
// fma.rn.f32x2 forms both distances (each half rounds exactly as fmaf), one
// three-input min folds both into a running minimum, and the pair's first
// column wins when it equals the new minimum. Four chains of pairs run
// independently and are merged in (distance, column) order.
// ---------------------------------------------------------------------------

// {a + b} on float pairs (add.rn.f32x2)
__device__ __forceinline__ unsigned long long add_pair(uint32_t a0, uint32_t a1, uint32_t b0, uint32_t b1) {
  unsigned long long a, b, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "r"(a0), "r"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "r"(b0), "r"(b1));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// the distances of a column pair from the packed dot products: dot * s + bias
__device__ __forceinline__ void dist_pair(unsigned long long dot, unsigned long long s2, float b0, float b1,
                                          float& d0, float& d1) {
  unsigned long long c, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(c) : "f"(b0), "f"(b1));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(dot), "l"(s2), "l"(c));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

__device__ __forceinline__ unsigned long long pack_pair(uint32_t a0, uint32_t a1) {
  unsigned long long a;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "r"(a0), "r"(a1));
  return a;
}

// running minimum (bd, bi) of one chain after the pair (d0 at column j, d1 at j + 1)
__device__ __forceinline__ void pair_step(float& bd, int& bi, float d0, float d1, int j) {
  float m;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(bd), "f"(d0), "f"(d1));
  const int jm = d0 == m ? j : j + 1;
  bi = m < bd ? jm : bi;
  bd = m;
}

// Scan of NB16 x 16 columns of one TMEM accumulator row (columns local to
// `taddr`; stacked: column j's dot product is acc[j] + acc[koff + j]); bias
// points at the bias of local column 0 (16-byte aligned). LPW 16-column loads
// go out before each wait (wait::ld waits for every load of the thread, so
// loads are batched; stacked: one block and its second half). Returns the
// local column in `bl` (INT_MAX when no distance is below +inf).
template <int NB16, bool STACKED, int LPW = 2>
__device__ __forceinline__ void scan_row(uint32_t taddr, uint32_t koff, const float* __restrict__ bias,
                                         unsigned long long s2, float& best, int& bl) {
  float bd[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
  int bi[4] = {0x7fffffff, 0x7fffffff, 0x7fffffff, 0x7fffffff};
  constexpr int PER = STACKED ? 1 : LPW;  // 16-column blocks per wave
  constexpr int WAVES = (NB16 + PER - 1) / PER;
#pragma unroll
  for (int w = 0; w < WAVES; ++w) {
    uint32_t v[STACKED ? 2 : LPW][16];
    // tcgen05.ld / wait::ld are .sync.aligned: the warp reconverges first
    __syncwarp();
    if (STACKED) {
      tmem_ld16(taddr + (uint32_t)(16 * w), v[0]);
      tmem_ld16(taddr + koff + (uint32_t)(16 * w), v[1]);
    } else {
#pragma unroll
      for (int t = 0; t < PER; ++t)
        if (PER * w + t < NB16) tmem_ld16(taddr + (uint32_t)(16 * (PER * w + t)), v[t]);
    }
    tmem_ld_wait16(v[0]);
#pragma unroll
    for (int t = 1; t < (STACKED ? 2 : LPW); ++t) reg_pin16(v[t]);
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      if (PER * w + t >= NB16) break;
      const int cb = 16 * (PER * w + t);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 b4 = *reinterpret_cast<const float4*>(bias + cb + 4 * u);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int jj = 4 * u + 2 * e;
          const unsigned long long dot = STACKED ? add_pair(v[0][jj], v[0][jj + 1], v[1][jj], v[1][jj + 1])
                                                 : pack_pair(v[t][jj], v[t][jj + 1]);
          float d0, d1;
          dist_pair(dot, s2, e ? b4.z : b4.x, e ? b4.w : b4.y, d0, d1);
          pair_step(bd[(jj >> 1) & 3], bi[(jj >> 1) & 3], d0, d1, cb + jj);
        }
      }
    }
  }
  best = bd[0];
  bl = bi[0];
#pragma unroll
  for (int u = 1; u < 4; ++u)
    if (better(bd[u], bi[u], best, bl)) {
      best = bd[u];
      bl = bi[u];
    }
}

// scan_row of 1..16 unstacked 16-column blocks with four loads per wait
// (kernels with registers to spare: 64 columns in flight)
__device__ __forceinline__ void scan_row4_n(int nb16, uint32_t taddr, const float* __restrict__ bias,
                                            unsigned long long s2, float& best, int& bl) {
#define SKM_SCAN4_CASE(N)                                    \
  case N:                                                    \
    scan_row<N, false, 4>(taddr, 0u, bias, s2, best, bl);    \
    return;
  best = INFINITY;
  bl = 0x7fffffff;
  switch (nb16) {
    SKM_SCAN4_CASE(1) SKM_SCAN4_CASE(2) SKM_SCAN4_CASE(3) SKM_SCAN4_CASE(4) SKM_SCAN4_CASE(5)
    SKM_SCAN4_CASE(6) SKM_SCAN4_CASE(7) SKM_SCAN4_CASE(8) SKM_SCAN4_CASE(9) SKM_SCAN4_CASE(10)
    SKM_SCAN4_CASE(11) SKM_SCAN4_CASE(12) SKM_SCAN4_CASE(13) SKM_SCAN4_CASE(14) SKM_SCAN4_CASE(15)
    SKM_SCAN4_CASE(16)
    default: return;
  }
#undef SKM_SCAN4_CASE
}

// scan_row for a run-time count of 16-column blocks (1..16; stacked 1..8)
__device__ __forceinline__ void scan_row_n(int nb16, bool stacked, uint32_t taddr, uint32_t koff,
                                           const float* __restrict__ bias, unsigned long long s2, float& best,
                                           int& bl) {
#define SKM_SCAN_CASE(N, ST)                                \
  case N:                                                   \
    scan_row<N, ST>(taddr, koff, bias, s2, best, bl);       \
    return;
  best = INFINITY;
  bl = 0x7fffffff;
  if (stacked) {
    switch (nb16) {
      SKM_SCAN_CASE(1, true) SKM_SCAN_CASE(2, true) SKM_SCAN_CASE(3, true) SKM_SCAN_CASE(4, true)
      SKM_SCAN_CASE(5, true) SKM_SCAN_CASE(6, true) SKM_SCAN_CASE(7, true) SKM_SCAN_CASE(8, true)
      default: return;
    }
  }
  switch (nb16) {
    SKM_SCAN_CASE(1, false) SKM_SCAN_CASE(2, false) SKM_SCAN_CASE(3, false) SKM_SCAN_CASE(4, false)
    SKM_SCAN_CASE(5, false) SKM_SCAN_CASE(6, false) SKM_SCAN_CASE(7, false) SKM_SCAN_CASE(8, false)
    SKM_SCAN_CASE(9, false) SKM_SCAN_CASE(10, false) SKM_SCAN_CASE(11, false) SKM_SCAN_CASE(12, false)
    SKM_SCAN_CASE(13, false) SKM_SCAN_CASE(14, false) SKM_SCAN_CASE(15, false) SKM_SCAN_CASE(16, false)
    default: return;
  }
#undef SKM_SCAN_CASE
}

// Per-CTA view of a launch's shared memory, barriers and tensor memory.
struct Cta {
  unsigned char* base;  // dynamic shared memory, aligned to 1024
  uint32_t sbase;
  Smem L;
  uint32_t bar0;
  uint32_t* misc;  // [0] tensor-memory base, [1] abort flag
  volatile int* abort_flag;
  float* bias_s;  // ||c||^2, k_pad entries (+inf beyond k)
  uint32_t tmem_base;
  int my_tiles;  // tiles blockIdx.x + i * gridDim.x, i < my_tiles
  int n_iss;     // MMA issuers (1 or 2)
  int n_grp;     // epilogue group sets (= accumulators); a set is epi_split(nacc) groups
  int issued;    // producer thread: tiles of the CTA's sequence whose copies it issued
  __device__ __forceinline__ uint32_t bar(int i) const { return bar0 + 8u * (uint32_t)i; }
};

// One pass of the pipeline (see estep_pass).
struct Pass {
  int ig0;       // tiles this CTA processed in earlier passes of the launch
  int par;       // parity of the pass (the issuers' drain barriers complete once per pass)
  int pre;       // tiles of this pass whose copies the previous pass already issued
  int pre_next;  // tiles of the next pass to issue at the end of this one
  int load_image;  // the producer issues the copy of the centre image from global memory
  int wait_image;  // the pass waits for an image copy (issued by the producer or earlier by the caller)
  int img_par;     // parity of that image copy
  float negscale;  // -2^(1 - xexp - cexp): dot products to distances
  long long* deltas;            // nullable: fixed-point deltas of rows that change label
  unsigned long long* changed;  // nullable: count of rows that change label
};

// The extra chunk of an odd nk (read as x_hi by the last pair MMA of the
// two-segment layout) is zero in every stage. All threads; the caller
// synchronises the block before the next bulk copy into the stages.
__device__ __forceinline__ void zero_stage_padding(const Params& p, const Cta& c) {
  if (p.tile_bytes < p.stage_bytes) {
    for (int s = 0; s < p.stages; ++s)
      for (uint32_t o = p.tile_bytes + 16u * threadIdx.x; o < p.stage_bytes; o += 16u * blockDim.x)
        *reinterpret_cast<uint4*>(c.base + (uint32_t)s * p.stage_bytes + o) = make_uint4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
}

// ||c||^2 into shared memory (+inf for the padding clusters). All threads.
__device__ __forceinline__ void load_bias(const Params& p, const Cta& c, const float* bias) {
  for (int j = threadIdx.x; j < p.k_pad; j += blockDim.x) c.bias_s[j] = j < p.k ? __ldcg(bias + j) : INFINITY;
}

// All threads, once per launch: layout, barriers, tensor-memory allocation
// (warp MMA_W0), bias (nullable), zeroed stage padding; ends with a block
// barrier after which c.tmem_base is valid.
__device__ __forceinline__ void cta_setup(const Params& p, unsigned char* smem_raw, const float* bias, Cta& c) {
  c.base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  c.L = smem_layout(p.stage_bytes, p.img_bytes, p.k_pad, p.stages, p.nacc);
  c.sbase = smem_u32(c.base);
  c.bar0 = c.sbase + c.L.bars;
  c.misc = reinterpret_cast<uint32_t*>(c.base + c.L.misc);
  c.abort_flag = reinterpret_cast<volatile int*>(c.misc + 1);
  c.bias_s = reinterpret_cast<float*>(c.base + c.L.bias);
  c.my_tiles = (p.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  // issuer t owns the accumulators a = t mod n_iss and epilogue group g those
  // with a = g mod n_grp (n_iss and n_grp divide nacc), so each accumulator
  // barrier has exactly one producer and one consumer
  c.n_iss = p.nacc >= 2 ? 2 : 1;
  c.n_grp = EPI_GROUPS / epi_split(p.nacc);
  c.issued = 0;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < MAX_STAGES; ++s) {
      mbar_init(c.bar(B_FULL(s)), 1);
      mbar_init(c.bar(B_EMPTY(s)), 1);
    }
    for (int a = 0; a < MAX_ACC; ++a) {
      mbar_init(c.bar(B_ACC_FULL(a)), 1);
      // the four warps of each epilogue group reading the accumulator
      mbar_init(c.bar(B_ACC_EMPTY(a)), 4 * epi_split(p.nacc));
    }
    for (int a = 0; a < 2; ++a)
      for (int sl = 0; sl < 2; ++sl) {
        // every thread of the partner groups (unused without a split)
        // one arrival per warp (after __syncwarp, which orders the warp's
        // shared-memory accesses before its lane 0's arrival): the partner
        // groups' warps, and the finishing group's four
        mbar_init(c.bar(B_PART_FULL(a, sl)), 4 * (epi_split(p.nacc) > 1 ? epi_split(p.nacc) - 1 : 1));
        mbar_init(c.bar(B_PART_EMPTY(a, sl)), 4);
      }
    mbar_init(c.bar(B_C_FULL), 1);
    mbar_init(c.bar(B_DONE(0)), 1);
    mbar_init(c.bar(B_DONE(1)), 1);
    c.misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_W0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(c.sbase + c.L.misc),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (bias) load_bias(p, c, bias);
  zero_stage_padding(p, c);
  tc_fence_before();
  block_sync();
  tc_fence_after();
  c.tmem_base = c.misc[0];
}

// All threads, once per launch, after the last pass: frees the tensor memory.
__device__ __forceinline__ void cta_teardown(const Params& p, const Cta& c) {
  if (threadIdx.x == 0) {
    // copies still in flight (prefetched for a pass that did not run, or
    // left by an abort) land before the CTA exits; at most `stages` are
    // outstanding and each stage barrier is armed once per use
    volatile int no_abort = 0;
    for (int ig = (c.issued > p.stages ? c.issued - p.stages : 0); ig < c.issued; ++ig)
      mbar_wait(c.bar(B_FULL(ig % p.stages)), (ig / p.stages) & 1, &no_abort, p.err, 2103);
  }
  tc_fence_before();
  block_sync();
  if ((threadIdx.x >> 5) == MMA_W0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(c.tmem_base), "r"(p.tmem_cols));
  }
}

// One thread: copies the centre image from global memory into the CTA's
// image region, completing on B_C_FULL.
__device__ __forceinline__ void issue_image_copy(const Params& p, const Cta& c) {
  mbar_expect_tx(c.bar(B_C_FULL), p.img_bytes);  // < 1 MB: one copy, one transaction count
  bulk_load(c.sbase + c.L.c, p.img, p.img_bytes, c.bar(B_C_FULL));
}

// One pass of the pipeline over this CTA's tiles, every thread in its warp
// role: the producer copies the centre image (P.load_image; the MMAs wait for
// a copy when P.wait_image, which the caller may also have issued) and the
// tiles,
// the issuers run the MMAs, the epilogue writes labels, counts changed rows
// into P.changed and, with P.deltas non-null, adds their fixed-point deltas.
// P.ig0 = tiles this CTA processed in earlier passes of the launch: stage and
// accumulator phases continue from there, so consecutive passes need no
// barrier re-initialisation. The copies of the first P.pre tiles were issued
// by the previous pass; at its end the producer issues the first P.pre_next
// tiles of the next pass (X does not change between passes), which then land
// while the caller runs other work that must leave the stages alone. Without
// a copied image the caller has written it in place before the pass (then
// fenced for the async proxy and synchronised the block). No block barrier at
// the end. On a timeout the CTA's abort flag is set and every role stops
// issuing work; the producer's copies are drained at teardown.
__device__ __forceinline__ void estep_pass(const Params& p, Cta& c, const Pass& P) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int my_tiles = c.my_tiles;
  const int ig0 = P.ig0;
  long long* const deltas = P.deltas;
  unsigned long long* const changed = P.changed;
  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      if (P.load_image) issue_image_copy(p, c);
      // tiles i of this pass (i >= pre), then tiles i < pre_next of the next
      const int n_issue = my_tiles - P.pre + min(P.pre_next, my_tiles);
      const uint64_t pol = l2_evict_first_policy();
      for (int q = 0; q < n_issue; ++q) {
        const int ig = c.issued;
        const int i = ig - ig0 < my_tiles ? ig - ig0 : ig - ig0 - my_tiles;
        const int s = ig % p.stages;
        if (!mbar_wait(c.bar(B_EMPTY(s)), ((ig / p.stages) & 1) ^ 1, c.abort_flag, p.err, 2101)) break;
        const int tile = (int)blockIdx.x + i * (int)gridDim.x;
        const unsigned char* src = p.Xs + (size_t)tile * p.tile_bytes;
        mbar_expect_tx(c.bar(B_FULL(s)), p.tile_bytes);  // <= 64 KB: one copy per tile
        bulk_load_hint(c.sbase + (uint32_t)s * p.stage_bytes, src, p.tile_bytes, c.bar(B_FULL(s)), pol);
        c.issued = ig + 1;
      }
      // the next pass's tiles after those copied into the stages go to L2
      // now, so HBM keeps streaming while the caller's work between passes
      // runs and the next pass's first MMAs wait for their centre image
      if (P.pre_next > 0 && !*c.abort_flag)
        for (int i = P.pre_next; i < min(my_tiles, P.pre_next + L2_AHEAD); ++i)
          bulk_prefetch_l2(p.Xs + (size_t)((int)blockIdx.x + i * (int)gridDim.x) * p.tile_bytes, p.tile_bytes);
      if (P.wait_image) {  // the image copy lands before the pass ends
        volatile int no_abort = 0;
        mbar_wait(c.bar(B_C_FULL), P.img_par, &no_abort, p.err, 2102);
      }
    }
  } else if (warp == MMA_W0 || warp == MMA_W1) {
    // ---------------------------------------------------------- MMA issuers
    const int t = warp == MMA_W0 ? 0 : 1;
    if (lane == 0 && t < c.n_iss) {
      bool ok = !P.wait_image || mbar_wait(c.bar(B_C_FULL), P.img_par, c.abort_flag, p.err, 2201);
      for (int i = (t - ig0 % c.n_iss + c.n_iss) % c.n_iss; ok && i < my_tiles; i += c.n_iss) {
        const int ig = ig0 + i;
        const int s = ig % p.stages, a = ig % p.nacc;
        if (!mbar_wait(c.bar(B_ACC_EMPTY(a)), ((ig / p.nacc) & 1) ^ 1, c.abort_flag, p.err, 2203)) break;
        // A parity wait is only exact while the waiter is at most one phase
        // away from the barrier. With two issuers and an odd number of stages,
        // the previous use of stage s belongs to the other issuer, and copies
        // can land out of order, so FULL(s) alone could still show the phase
        // of use u - 2. Waiting first for the previous use to be consumed
        // (EMPTY(s), phase u - 1, as the producer does; this issuer's own MMAs
        // of use u - 2 completed before its accumulator of tile i was freed)
        // pins FULL(s) to phase u - 1 or u.
        if (!mbar_wait(c.bar(B_EMPTY(s)), ((ig / p.stages) & 1) ^ 1, c.abort_flag, p.err, 2204)) break;
        if (!mbar_wait(c.bar(B_FULL(s)), (ig / p.stages) & 1, c.abort_flag, p.err, 2202)) break;
        tc_fence_after();
        issue_tile_mmas(c.tmem_base + (uint32_t)(a * p.acc_cols), c.sbase + (uint32_t)s * p.stage_bytes,
                        c.sbase + c.L.c, p.nk, p.k_pad, p.stacked);
        tc_commit(c.bar(B_EMPTY(s)));  // the stage is no longer read by the tensor core
        tc_commit(c.bar(B_ACC_FULL(a)));
      }
      // every tcgen05 operation issued by this thread is complete once DONE fires
      tc_commit(c.bar(B_DONE(t)));
      volatile int no_abort = 0;
      mbar_wait(c.bar(B_DONE(t)), P.par, &no_abort, p.err, 2206);
    }
  } else if (warp >= EPI_W0) {
    // ----------------------------------------------------------------- epilogue
    // groups of four warps (one per TMEM lane quarter). With four
    // accumulators group g takes the tiles of accumulator g and scans every
    // cluster of its 32 rows; with two, every group takes every tile and
    // scans part h = g of the clusters, and groups 1-3 hand their partial
    // minima to group 0 (the finisher) through shared memory
    const int q = warp & 3;
    const int g = (warp - EPI_W0) >> 2;
    const int split = epi_split(p.nacc);
    const int ga = g % c.n_grp;  // accumulator set whose tiles this group takes
    const int h = g / c.n_grp;   // part of the clusters
    const int jpart = (int)round_up_dev((p.k_pad + split - 1) / split, 16);
    const int jlo = min(p.k_pad, h * jpart);
    const int jhi = min(p.k_pad, (h + 1) * jpart);
    const bool finisher = h == 0;
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const int np = split > 1 ? split - 1 : 1;  // partial slots per (accumulator, use slot)
    float* part_d = reinterpret_cast<float*>(c.base + c.L.part);  // [a][slot][part][row]
    int* part_i = reinterpret_cast<int*>(c.base + c.L.part + 2 * 2 * np * BM * 4);
    // dist = ||c||^2 - 2 x.c with x.c = acc * 2^-(xexp + cexp)
    const float negscale = P.negscale;
    const unsigned long long s2 = pack_pair(__float_as_uint(negscale), __float_as_uint(negscale));
    const int i0 = (g < c.n_grp * split) ? (ga - ig0 % c.n_grp + c.n_grp) % c.n_grp : my_tiles;
    int old_next = -1;
    if (finisher && changed && i0 < my_tiles) {
      const long long g0 = (long long)((int)blockIdx.x + i0 * (int)gridDim.x) * BM + row;
      old_next = g0 < p.n ? p.labels[g0] : -1;
    }
    for (int i = i0; i < my_tiles; i += c.n_grp) {
      const int ig = ig0 + i;
      const int a = ig % p.nacc;
      const int use = ig / p.nacc;  // uses of accumulator a so far in the launch
      const long long grow = (long long)((int)blockIdx.x + i * (int)gridDim.x) * BM + row;
      const int old = old_next;
      if (finisher && changed && i + c.n_grp < my_tiles) {  // prefetch the next tile's previous labels
        const long long g1 = grow + (long long)c.n_grp * gridDim.x * BM;
        old_next = g1 < p.n ? p.labels[g1] : -1;
      }
      if (!warp_wait_all(c.bar(B_ACC_FULL(a)), use & 1, c.abort_flag, p.err, 2401)) break;
      tc_fence_after();
      const uint32_t taddr = c.tmem_base + lane_off + (uint32_t)(a * p.acc_cols);
      float best;
      int bl;
      scan_row_n((jhi - jlo) >> 4, p.stacked != 0, taddr + (uint32_t)jlo, (uint32_t)p.k_pad, c.bias_s + jlo, s2,
                 best, bl);
      if (bl != 0x7fffffff) bl += jlo;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(c.bar(B_ACC_EMPTY(a)));
      if (split > 1) {
        // partial minima of the parts meet in slot use mod 2 of accumulator a
        const int sl = use & 1;
        const uint32_t ph = (uint32_t)(use >> 1) & 1u;
        const int o = (a * 2 + sl) * np * BM + row;
        if (!finisher) {
          if (!warp_wait_all(c.bar(B_PART_EMPTY(a, sl)), ph ^ 1u, c.abort_flag, p.err, 2402)) break;
          part_d[o + (h - 1) * BM] = best;
          part_i[o + (h - 1) * BM] = bl;
          __syncwarp();
          if (lane == 0) mbar_arrive(c.bar(B_PART_FULL(a, sl)));
          continue;
        }
        if (!warp_wait_all(c.bar(B_PART_FULL(a, sl)), ph, c.abort_flag, p.err, 2403)) break;
        float ob[EPI_GROUPS - 1];
        int oi[EPI_GROUPS - 1];
#pragma unroll
        for (int u = 0; u < EPI_GROUPS - 1; ++u) {
          if (u < split - 1) {
            ob[u] = part_d[o + u * BM];
            oi[u] = part_i[o + u * BM];
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(c.bar(B_PART_EMPTY(a, sl)));
#pragma unroll
        for (int u = 0; u < EPI_GROUPS - 1; ++u)
          if (u < split - 1 && better(ob[u], oi[u], best, bl)) {
            best = ob[u];
            bl = oi[u];
          }
      }
      if (bl >= p.k) bl = 0;  // only reachable when every distance is +inf or NaN
      bool ch = false;
      if (grow < p.n) {
        ch = changed && old != bl;
        p.labels[grow] = bl;
      }
      if (changed) {
        const unsigned int m = __ballot_sync(0xffffffffu, ch);
        if (lane == 0 && m) atomicAdd(changed, (unsigned long long)__popc(m));
        if (deltas) warp_apply_changed(p.X, p.ld, p.d, p.k, grow, old, bl, ch, deltas, p.st);
      }
    }
  }
  // the single-lane roles leave warps 0-2 diverged: reconverge before the
  // caller's block barriers
  __syncwarp();
}


// Operands of the tensor-core probes (estep_tc.cu, estep_wide.cu): x and c
// values whose fp16 splits are exact (x = p + q 2^-12, c = r + s 2^-12 with
// |p|, |r| in [8, 16), |q|, |s| <= 8), so that x_hi.c_hi + x_lo.c_hi +
// x_hi.c_lo is exact in fp32 for 16 columns.
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

// Launch parameters of a plan; the per-launch operands (image, scales, bias,
// labels, changed, D, fit state, error word) are filled in by the caller.
inline Params make_params(const TcPlan& plan) {
  Params p{};
  p.n_tiles = (int)((plan.n + BM - 1) / BM);
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
  p.tile_bytes = tc_tile_bytes(plan);
  p.Xs = plan.Xs;
  p.X = plan.X;
  p.ld = plan.ld;
  p.d = plan.d;
  return p;
}

}  // namespace tc

}  // namespace skm
