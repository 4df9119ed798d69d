// Tensor-core E-step for sm_100a: labels[i] = argmin_j (||c_j||^2 - 2 x_i . c_j)
// over 128-row tiles of X, with the dot products computed by tcgen05.mma in
// 3xTF32 split precision and accumulated in fp32 in tensor memory (TMEM):
//     x . c  ~=  T(x).T(c) + T(x).c_lo + x_lo.T(c)
// where T is the tensor core's own fp32 -> tf32 conversion (measured once per
// device by tc_probe), x_lo = x - T(x) and c_lo = c - T(c). The n x k
// distance matrix never leaves the SM: the epilogue reads each row's k
// accumulators from TMEM and keeps a running argmin in registers (strict '<',
// lowest index first, as sklearn/cluster/_k_means_lloyd.pyx:205-213). Rows
// whose label changed add their exact fixed-point deltas to the centroid sums
// (the incremental M-step input).
//
// Data path of one tile (all asynchronous, one CTA per SM, persistent):
//   HBM --bulk copy--> smem stage (x, the A operand of the first MMAs)
//   MMA thread : acc  = x.[C_hi | C_lo]     (A = smem stage, B = smem; one MMA
//                                            per K chunk with N = 2k, or two)
//   converter  : smem stage --> x_lo = x - T(x) --tcgen05.st--> TMEM (2 buffers)
//   MMA thread : acc += x_lo.C_hi           (A = TMEM, B = smem)
//   epilogue   : TMEM acc --tcgen05.ld--> argmin --> labels, deltas
// X is read from HBM exactly once per iteration.
//
// X is the fit's blocked working copy (xblk_index): a 128-row tile is one
// contiguous region already in the tensor core's canonical no-swizzle K-major
// layout (8-column chunk c = 4 KB at c * 4096: two 2 KB halves of 4 columns,
// 8-row core matrices of 16-byte rows 128 bytes apart), so one bulk copy per
// tile lands it ready for the MMAs. The centres (B operand) are loaded once
// per CTA by TMA in the SWIZZLE_32B layout, C_hi and C_lo of chunk c side by
// side so that [C_hi | C_lo] is one 2k-row operand.
//
// Warp roles (608 threads): 0 bulk-copy producer, 1 TMEM owner + MMA issuer
// of even tiles, 18 MMA issuer of odd tiles, 2-9 converter, 10-17 epilogue.
// A single thread issues tcgen05.mma at roughly one instruction per ~120
// cycles whatever N is, while issuers on different SM sub-partitions overlap,
// so tiles alternate between two issuing warps (each with its own
// accumulator and x_lo buffer). Warp w owns TMEM lanes 32*(w%4) .. +31 (= tile
// rows); the two converter (epilogue) warps of a lane quarter split the K
// chunks (the clusters) between them.
//
// Every mbarrier wait is bounded in time; on timeout the CTA records an error
// code, stops issuing work, waits (bounded) for its own in-flight copies and
// tensor-core operations, frees its tensor memory and returns.
#include <cuda.h>
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
constexpr int KC = 8;                     // fp32 columns per K chunk (UMMA K for tf32)
constexpr int CHUNK_BYTES = BM * KC * 4;  // 4096
constexpr int MAX_NK = 16;                // d <= 128
constexpr int MAX_KPAD = 256;             // k <= 256 (one UMMA N)
constexpr int THREADS = 608;
constexpr int MAX_STAGES = 4;
constexpr unsigned long long TIMEOUT_NS = 2000000000ull;  // 2 s per wait

struct Params {
  int n_tiles;
  long long n;
  int k;
  int k_pad;
  int nk;      // K chunks of 8 columns
  int stages;  // X stages in shared memory
  int nbl;     // x_lo buffers in TMEM (1 or 2)
  int nba;     // accumulator buffers in TMEM (1 or 2)
  int xcols;   // TMEM columns of one x_lo buffer (>= 8 nk, multiple of 32)
  int tmem_cols;
  int round_mode;  // fp32->tf32 conversion of the tensor core: 0 truncate, 1 nearest-even
  const float* bias;  // ||c||^2, k entries
  int32_t* labels;
  unsigned long long* changed;
  long long* D;  // nullable: incremental deltas of rows that changed label
  const float* X;  // blocked layout
  int ld;
  int d;
  uint32_t tile_bytes;  // 512 * ld: one tile of blocked X
  const FitState* st;  // nullable: skip when st->done
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

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<unsigned long long>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(reinterpret_cast<unsigned long long>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// K-major no-swizzle shared-memory matrix descriptor for one 128 x 8 fp32
// chunk of a blocked tile: core matrices of 8 rows x 16 bytes, 8-row groups
// 128 bytes apart (stride byte offset), the two 4-column halves 2048 bytes
// apart (leading byte offset), descriptor version 1, layout type 0.
__device__ __forceinline__ uint64_t blk_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(2048u >> 4) << 16;
  d |= (uint64_t)(128u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

// K-major SWIZZLE_32B shared-memory matrix descriptor: rows of 32 bytes,
// 8-row atoms of 256 bytes (stride byte offset), leading byte offset unused
// (1), descriptor version 1 (sm_100), layout type 6 (SWIZZLE_32B).
__device__ __forceinline__ uint64_t sw32_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(256u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)6u << 61;
  return d;
}

// kind::tf32 instruction descriptor: D fp32, A/B tf32, both K-major, M=128, N.
__host__ __device__ constexpr uint32_t idesc_tf32(int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// D[tmem] (+)= A[smem] . B[smem]^T
__device__ __forceinline__ void mma_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem]^T
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 128 rows x 8 fp32 (one chunk) from shared memory into TMEM lanes 0..127
__device__ __forceinline__ void tmem_cp_chunk(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
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
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// The tensor core's fp32 -> tf32 conversion: 0 = truncate the low 13 mantissa
// bits, 1 = round to nearest even at bit 13 (finite inputs).
__host__ __device__ __forceinline__ uint32_t to_tf32_bits(uint32_t u, int mode) {
  if (mode == 0) return u & 0xffffe000u;
  const uint32_t lsb = (u >> 13) & 1u;
  return (u + 0x0fffu + lsb) & 0xffffe000u;
}

struct Smem {
  uint32_t x[MAX_STAGES], c, bias, ep, bars, misc, total;
};

// barrier indices
__host__ __device__ constexpr int B_FULL(int s) { return s; }
__host__ __device__ constexpr int B_EMPTY(int s) { return MAX_STAGES + s; }
__host__ __device__ constexpr int B_XLO_FULL(int b) { return 2 * MAX_STAGES + b; }
__host__ __device__ constexpr int B_XLO_FREE(int b) { return 2 * MAX_STAGES + 2 + b; }
__host__ __device__ constexpr int B_ACC_FULL(int a) { return 2 * MAX_STAGES + 4 + a; }
__host__ __device__ constexpr int B_ACC_EMPTY(int a) { return 2 * MAX_STAGES + 6 + a; }
constexpr int B_C_FULL = 2 * MAX_STAGES + 8;
__host__ __device__ constexpr int B_DONE(int t) { return 2 * MAX_STAGES + 9 + t; }  // drain of MMA issuer t
constexpr int NUM_BARS = 2 * MAX_STAGES + 11;
constexpr int MMA_W1 = 18;  // second MMA issuer warp (sub-partition 2)

constexpr int CONV_WARPS = 8;
constexpr int EPI_WARPS = 8;
constexpr int CONV_W0 = 2;
constexpr int EPI_W0 = CONV_W0 + CONV_WARPS;

__host__ __device__ inline Smem smem_layout(int nk, int k_pad, int stages) {
  Smem s;
  uint32_t off = 0;
  const uint32_t stage = (uint32_t)nk * CHUNK_BYTES;
  for (int i = 0; i < MAX_STAGES; ++i) {
    s.x[i] = off;
    if (i < stages) off += stage;
  }
  s.c = off;  // chunk c: C_hi (k_pad rows) then C_lo (k_pad rows), 32 bytes each
  off += (uint32_t)nk * 2 * k_pad * 32;
  s.bias = off;
  off += (uint32_t)k_pad * 4;
  s.ep = off;  // epilogue pair exchange: [2 parities][128 rows] (float, int)
  off += 2 * BM * 8;
  off = (off + 15) & ~15u;
  s.bars = off;
  off += NUM_BARS * 8;
  s.misc = off;
  off += 16;             // [0] tmem base, [1] abort flag
  s.total = off + 1024;  // slack for aligning the base to 1024
  return s;
}

__device__ __forceinline__ bool better(float d, int i, float bd, int bi) { return d < bd || (d == bd && i < bi); }

__global__ void __launch_bounds__(THREADS, 1)
estep_tc_kernel(const __grid_constant__ CUtensorMap tmap_chi, const __grid_constant__ CUtensorMap tmap_clo,
                Params p) {
  if (p.st && p.st->done) return;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Smem L = smem_layout(p.nk, p.k_pad, p.stages);
  const uint32_t sbase = smem_u32(base);
  const uint32_t bar0 = sbase + L.bars;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(base + L.misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  float* bias_s = reinterpret_cast<float*>(base + L.bias);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int my_tiles = (p.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const uint32_t stage_bytes = (uint32_t)p.nk * CHUNK_BYTES;
  const uint32_t cstride = (uint32_t)(2 * p.k_pad * 32);  // bytes per K chunk of [C_hi | C_lo]
  const bool stacked = 2 * p.k_pad <= 256;
  const int acc_cols = stacked ? 2 * p.k_pad : p.k_pad;

  if (threadIdx.x == 0) {
    for (int s = 0; s < MAX_STAGES; ++s) {
      mbar_init(bar(B_FULL(s)), 1);
      mbar_init(bar(B_EMPTY(s)), 1 + CONV_WARPS);  // first MMAs done + every converter warp
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(B_XLO_FULL(b)), 32 * CONV_WARPS);
      mbar_init(bar(B_XLO_FREE(b)), 1);
      mbar_init(bar(B_ACC_FULL(b)), 1);
      mbar_init(bar(B_ACC_EMPTY(b)), 32 * EPI_WARPS);
    }
    mbar_init(bar(B_C_FULL), 1);
    mbar_init(bar(B_DONE(0)), 1);
    mbar_init(bar(B_DONE(1)), 1);
    misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + L.misc),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  for (int j = threadIdx.x; j < p.k_pad; j += blockDim.x) bias_s[j] = j < p.k ? p.bias[j] : INFINITY;
  if (p.tile_bytes < stage_bytes) {
    // 4-column tail of the last chunk (d % 8 in 1..4): never copied, must be zero
    for (int s = 0; s < p.stages; ++s)
      for (uint32_t o = p.tile_bytes + 16u * threadIdx.x; o < stage_bytes; o += 16u * blockDim.x)
        *reinterpret_cast<uint4*>(base + L.x[s] + o) = make_uint4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = misc[0];
  // TMEM column map: acc[0..nba) | x_lo[0..nbl)
  const uint32_t col_xlo = (uint32_t)(p.nba * acc_cols);

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      mbar_expect_tx(bar(B_C_FULL), 2u * (uint32_t)p.nk * p.k_pad * 32u);
      for (int c = 0; c < p.nk; ++c) {
        tma_load_2d(sbase + L.c + (uint32_t)c * cstride, &tmap_chi, c * KC, 0, bar(B_C_FULL));
        tma_load_2d(sbase + L.c + (uint32_t)c * cstride + (uint32_t)p.k_pad * 32, &tmap_clo, c * KC, 0,
                    bar(B_C_FULL));
      }
      int armed = 0;
      for (int i = 0; i < my_tiles; ++i) {
        const int s = i % p.stages;
        if (!mbar_wait(bar(B_EMPTY(s)), ((i / p.stages) & 1) ^ 1, abort_flag, p.err, 2101)) break;
        const int tile = (int)blockIdx.x + i * (int)gridDim.x;
        const char* src = reinterpret_cast<const char*>(p.X) + (size_t)tile * p.tile_bytes;
        mbar_expect_tx(bar(B_FULL(s)), p.tile_bytes);
        for (uint32_t o = 0; o < p.tile_bytes; o += 8192u)
          bulk_load(sbase + L.x[s] + o, src + o, min(8192u, p.tile_bytes - o), bar(B_FULL(s)));
        armed = i + 1;
      }
      // our own copies must land before the CTA may exit
      volatile int no_abort = 0;
      mbar_wait(bar(B_C_FULL), 0, &no_abort, p.err, 2102);
      for (int i = (armed > p.stages ? armed - p.stages : 0); i < armed; ++i)
        mbar_wait(bar(B_FULL(i % p.stages)), (i / p.stages) & 1, &no_abort, p.err, 2103);
    }
  } else if (warp == 1 || warp == MMA_W1) {
    // ---------------------------------------------------------- MMA issuers
    // two issuers when every tile has its own accumulator and x_lo buffer
    // (nba == nbl == 2), else warp 1 issues everything
    const int n_iss = (p.nba == 2 && p.nbl == 2) ? 2 : 1;
    const int t = warp == 1 ? 0 : 1;
    if (lane == 0 && t < n_iss) {
      const uint32_t idesc_k = idesc_tf32(p.k_pad);
      const uint32_t idesc_2k = idesc_tf32(stacked ? 2 * p.k_pad : p.k_pad);
      bool ok = mbar_wait(bar(B_C_FULL), 0, abort_flag, p.err, 2201);
      for (int i = t; ok && i < my_tiles; i += n_iss) {
        const int s = i % p.stages, a = i % p.nba, b = i % p.nbl;
        if (!mbar_wait(bar(B_ACC_EMPTY(a)), ((i / p.nba) & 1) ^ 1, abort_flag, p.err, 2203)) break;
        if (!mbar_wait(bar(B_FULL(s)), (i / p.stages) & 1, abort_flag, p.err, 2202)) break;
        tc_fence_after();
        const uint32_t tacc = tmem_base + (uint32_t)(a * acc_cols);
        for (int c = 0; c < p.nk; ++c) {
          const uint64_t a_desc = blk_desc(sbase + L.x[s] + (uint32_t)c * CHUNK_BYTES);
          const uint32_t cb = sbase + L.c + (uint32_t)c * cstride;
          if (stacked) {
            mma_ss(tacc, a_desc, sw32_desc(cb), idesc_2k, c > 0 ? 1u : 0u);
          } else {
            mma_ss(tacc, a_desc, sw32_desc(cb + (uint32_t)p.k_pad * 32), idesc_k, c > 0 ? 1u : 0u);
            mma_ss(tacc, a_desc, sw32_desc(cb), idesc_k, 1u);
          }
        }
        tc_commit(bar(B_EMPTY(s)));  // the stage is no longer read by the tensor core
        if (!mbar_wait(bar(B_XLO_FULL(b)), (i / p.nbl) & 1, abort_flag, p.err, 2204)) break;
        tc_fence_after();
        const uint32_t txl = tmem_base + col_xlo + (uint32_t)(b * p.xcols);
        for (int c = 0; c < p.nk; ++c)
          mma_ts(tacc, txl + (uint32_t)(c * KC), sw32_desc(sbase + L.c + (uint32_t)c * cstride), idesc_k, 1u);
        tc_commit(bar(B_ACC_FULL(a)));
        tc_commit(bar(B_XLO_FREE(b)));
      }
      // every tcgen05 operation issued by this thread is complete once DONE fires
      tc_commit(bar(B_DONE(t)));
      volatile int no_abort = 0;
      mbar_wait(bar(B_DONE(t)), 0, &no_abort, p.err, 2206);
    }
  } else if (warp >= CONV_W0 && warp < EPI_W0) {
    // ---------------------------------------------------------------- converter
    // thread = tile row: reads its row's 16-byte quads of its K chunks from the
    // shared-memory stage (a warp reads 512 contiguous bytes per quad) and
    // writes x - T(x) to its TMEM lane
    const int q = warp & 3;
    const int h = (warp - CONV_W0) >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const int half = (p.nk + 1) >> 1;
    const int c0 = h ? half : 0, c1 = h ? p.nk : half;
    for (int i = 0; i < my_tiles; ++i) {
      const int s = i % p.stages, b = i % p.nbl;
      if (!mbar_wait(bar(B_FULL(s)), (i / p.stages) & 1, abort_flag, p.err, 2301)) break;
      if (!mbar_wait(bar(B_XLO_FREE(b)), ((i / p.nbl) & 1) ^ 1, abort_flag, p.err, 2302)) break;
      tc_fence_after();
      const float4* stg = reinterpret_cast<const float4*>(base + L.x[s]) + row;  // quad j at stg[128 j]
      const uint32_t tl = tmem_base + lane_off + col_xlo + (uint32_t)(b * p.xcols);
#pragma unroll 2
      for (int c = c0; c < c1; ++c) {
        const float4 a0 = stg[(2 * c) * 128];
        const float4 a1 = stg[(2 * c + 1) * 128];  // zero past the last column (stage tail is zero)
        const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        uint32_t r[8];
#pragma unroll
        for (int e2 = 0; e2 < 8; ++e2)
          r[e2] = __float_as_uint(v[e2] - __uint_as_float(to_tf32_bits(__float_as_uint(v[e2]), p.round_mode)));
        tmem_st8(tl + (uint32_t)(c * KC), r);
      }
      // the stage may be refilled once the first MMAs and all converter warps are done
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_EMPTY(s)));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(B_XLO_FULL(b)));
    }
  } else if (warp >= EPI_W0 && warp < EPI_W0 + EPI_WARPS) {
    // ----------------------------------------------------------------- epilogue
    // the two warps of a lane quarter take the clusters [0, k/2) and
    // [k/2, k); the upper warp hands its (min, index) to the lower one
    const int q = warp & 3;
    const int h = (warp - EPI_W0) >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    // split at a multiple of 16 (the TMEM load width): [0, kh0) and [kh0, k_pad)
    const int kh0 = ((p.k_pad >> 1) + 15) & ~15;
    const int j0 = h ? kh0 : 0;
    const int kh = h ? p.k_pad - kh0 : kh0;
    float* ep_best = reinterpret_cast<float*>(base + L.ep);
    int* ep_idx = reinterpret_cast<int*>(base + L.ep + 2 * BM * 4);
    int old_next = -1;
    if (h == 0 && p.changed && my_tiles > 0) {
      const long long g0 = (long long)blockIdx.x * BM + row;
      old_next = g0 < p.n ? p.labels[g0] : -1;
    }
    for (int i = 0; i < my_tiles; ++i) {
      const int a = i % p.nba;
      const long long grow = (long long)((int)blockIdx.x + i * (int)gridDim.x) * BM + row;
      const int old = old_next;
      if (h == 0 && p.changed && i + 1 < my_tiles) {  // prefetch the next tile's previous labels
        const long long g1 = grow + (long long)gridDim.x * BM;
        old_next = g1 < p.n ? p.labels[g1] : -1;
      }
      if (!mbar_wait(bar(B_ACC_FULL(a)), (i / p.nba) & 1, abort_flag, p.err, 2401)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + lane_off + (uint32_t)(a * acc_cols);
      // four independent running minima (columns j = 4m + u), merged in index order
      float bd[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
      int bi[4] = {0x7fffffff, 0x7fffffff, 0x7fffffff, 0x7fffffff};
      for (int jb = 0; jb < kh; jb += 16) {
        uint32_t v[16], w[16];
        tmem_ld16(taddr + (uint32_t)(j0 + jb), v);
        if (stacked) tmem_ld16(taddr + (uint32_t)(p.k_pad + j0 + jb), w);
        tmem_ld_wait();
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int j = j0 + jb + jj;
          float dot = __uint_as_float(v[jj]);
          if (stacked) dot += __uint_as_float(w[jj]);
          const float dist = fmaf(-2.0f, dot, bias_s[j]);
          if (dist < bd[jj & 3]) {
            bd[jj & 3] = dist;
            bi[jj & 3] = j;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(bar(B_ACC_EMPTY(a)));
      float best = bd[0];
      int bl = bi[0];
#pragma unroll
      for (int u = 1; u < 4; ++u)
        if (better(bd[u], bi[u], best, bl)) {
          best = bd[u];
          bl = bi[u];
        }
      const int slot = (i & 1) * BM + row;
      if (h == 1) {
        ep_best[slot] = best;
        ep_idx[slot] = bl;
        named_bar(1 + q, 64);
        continue;
      }
      named_bar(1 + q, 64);
      if (better(ep_best[slot], ep_idx[slot], best, bl)) {
        best = ep_best[slot];
        bl = ep_idx[slot];
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
        if (p.D) warp_apply_changed(p.X, p.ld, p.d, p.k, grow, old, bl, ch, p.D, p.st->scale);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.tmem_cols));
  }
}

// ---------------------------------------------------------------------------
// probe: tcgen05.cp layout and the tensor core's fp32 -> tf32 conversion
// ---------------------------------------------------------------------------
// A (128 x 8) holds fp32 values whose dropped mantissa bits distinguish
// truncation from rounding (rows 64..127 negative); B (16 x 8) is the identity
// on its first 8 rows, so D[m][n] = tf32(A[m][n]) for n < 8. out: [0,1024) the
// TMEM copy of A made by tcgen05.cp, [1024,2048) D with A read from TMEM,
// [2048,3072) D with A read from shared memory, [3072] error code.
__host__ __device__ __forceinline__ uint32_t probe_bits(int m, int k) {
  const uint32_t low = 0x1000u | ((uint32_t)(m * 8 + k) & 0x0fffu);
  return 0x3f800000u | ((uint32_t)k << 13) | low | (m >= 64 ? 0x80000000u : 0u);
}

__global__ void __launch_bounds__(128, 1) tc_probe_kernel(uint32_t* out) {
  __shared__ __align__(1024) unsigned char sm[CHUNK_BYTES + 512 + 64];
  const uint32_t sa = smem_u32(sm), sb = sa + CHUNK_BYTES, sbar = sb + 512;
  uint32_t* misc = reinterpret_cast<uint32_t*>(sm + CHUNK_BYTES + 512 + 16);
  const uint32_t smisc = smem_u32(misc);
  int* err = reinterpret_cast<int*>(out + 3072);
  const int tid = threadIdx.x, warp = tid >> 5;
  // A in the blocked no-swizzle layout (column quad q at q * 2048, row m at
  // m * 16); B in SWIZZLE_32B (bit 4 of the byte offset XORed with bit 7)
  auto sw32 = [](uint32_t off) { return off ^ (((off >> 7) & 1u) << 4); };
  for (int k = 0; k < 8; ++k)
    *reinterpret_cast<uint32_t*>(sm + (uint32_t)((k >> 2) * 2048 + tid * 16 + (k & 3) * 4)) = probe_bits(tid, k);
  if (tid < 16)
    for (int k = 0; k < 8; ++k)
      *reinterpret_cast<float*>(sm + CHUNK_BYTES + sw32((uint32_t)(tid * 32 + k * 4))) = (tid == k) ? 1.0f : 0.0f;
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = misc[0];
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  // TMEM columns: [0,8) copy of A, [8,24) D (A from TMEM); then [16,32) D (A from smem)
  if (tid == 0) {
    const uint32_t idesc = idesc_tf32(16);
    tmem_cp_chunk(tb, blk_desc(sa));
    mma_ts(tb + 8, tb, sw32_desc(sb), idesc, 0u);
    tc_commit(sbar);
  }
  __syncwarp();
  mbar_wait(sbar, 0, abort_flag, err, 2501);
  tc_fence_after();
  const uint32_t lo = (uint32_t)(warp * 32) << 16;
  uint32_t r[8];
  tmem_ld8(tb + lo, r);
  tmem_ld_wait();
  for (int e = 0; e < 8; ++e) out[tid * 8 + e] = r[e];
  tmem_ld8(tb + lo + 8, r);
  tmem_ld_wait();
  for (int e = 0; e < 8; ++e) out[1024 + tid * 8 + e] = r[e];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
    const uint32_t idesc = idesc_tf32(16);
    mma_ss(tb + 16, blk_desc(sa), sw32_desc(sb), idesc, 0u);
    tc_commit(sbar);
  }
  __syncwarp();
  mbar_wait(sbar, 1, abort_flag, err, 2502);
  tc_fence_after();
  tmem_ld8(tb + lo + 16, r);
  tmem_ld_wait();
  for (int e = 0; e < 8; ++e) out[2048 + tid * 8 + e] = r[e];
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tb), "r"(32));
  }
}

}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D fp32 tensor map over a rows x ld matrix, box = 8 columns x box_rows rows,
// 32-byte swizzle, out-of-bounds elements read as zero.
static int make_map(CUtensorMap* m, const float* ptr, int ld, long long rows, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error(ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    return ERR_UNSUPPORTED;
  }
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)tc::KC, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) ld=%d rows=%lld box_rows=%d", (int)r, ld, rows,
              box_rows);
    return ERR_CUDA;
  }
  return OK;
}

// Per-device probe result: -2 not run, -1 unusable, 0 truncation, 1 rounding.
static int g_probe_mode[64];
static bool g_probe_init = false;

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
  uint32_t* d_out = nullptr;
  SKM_CUDA(cudaMallocAsync(&d_out, 3073 * 4, s));
  SKM_CUDA(cudaMemsetAsync(d_out, 0, 3073 * 4, s));
  tc::tc_probe_kernel<<<1, 128, 0, s>>>(d_out);
  int rc = check_launch("tc_probe_kernel");
  std::vector<uint32_t> h(3073, 0);
  if (rc == OK) {
    cudaMemcpyAsync(h.data(), d_out, 3073 * 4, cudaMemcpyDeviceToHost, s);
    if (cudaStreamSynchronize(s) != cudaSuccess) rc = ERR_CUDA;
  }
  cudaFreeAsync(d_out, s);
  if (rc != OK) {
    set_error(ERR_CUDA, "tensor-core probe failed to run");
    return rc;
  }
  if (raw_out) memcpy(raw_out, h.data(), 3072 * 4);
  int mode = -1;
  bool copy_ok = h[3072] == 0;
  for (int m = 0; m < 128 && copy_ok; ++m)
    for (int k = 0; k < 8; ++k)
      if (h[m * 8 + k] != tc::probe_bits(m, k)) copy_ok = false;
  if (copy_ok) {
    for (int cand = 0; cand < 2 && mode < 0; ++cand) {
      bool ok = true;
      for (int m = 0; m < 128 && ok; ++m)
        for (int k = 0; k < 8; ++k) {
          const uint32_t want = tc::to_tf32_bits(h[m * 8 + k], cand);
          if (h[1024 + m * 8 + k] != want || h[2048 + m * 8 + k] != want) {
            ok = false;
            break;
          }
        }
      if (ok) mode = cand;
    }
  }
  if (dev < 64) g_probe_mode[dev] = mode;
  *mode_out = mode;
  return OK;
}

int tc_plan(const float* X, int ld, long long n, int d, int k, TcPlan* plan) {
  plan->supported = false;
  if (getenv("SKMETAL_DISABLE_TC")) return OK;
  if (!encode_fn()) return OK;
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
  plan->round_mode = mode;
  plan->X = X;
  plan->ld = ld;
  plan->n = n;
  plan->d = d;
  plan->k = k;
  plan->k_pad = (int)round_up((size_t)k, 16);
  plan->k_steps = (ld + tc::KC - 1) / tc::KC;
  // TMEM: accumulators (2k columns when [C_hi | C_lo] is one N <= 256 operand,
  // else k) and x_lo buffers (32-column aligned); double-buffer what fits
  plan->xcols = (int)round_up((size_t)plan->k_steps * tc::KC, 32);
  const int acc_cols = 2 * plan->k_pad <= 256 ? 2 * plan->k_pad : plan->k_pad;
  plan->nbl = 2;
  plan->nba = 2;
  auto cols = [&]() { return plan->nba * acc_cols + plan->nbl * plan->xcols; };
  if (cols() > 512) plan->nba = 1;
  if (cols() > 512) plan->nbl = 1;
  if (cols() > 512) return OK;
  int tcols = 32;
  while (tcols < cols()) tcols *= 2;
  plan->tmem_cols = tcols;
  // shared memory: as many X stages as fit (2..4)
  plan->stages = 0;
  for (int st = tc::MAX_STAGES; st >= 2; --st) {
    const tc::Smem L = tc::smem_layout(plan->k_steps, plan->k_pad, st);
    if ((int)L.total <= optin) {
      plan->stages = st;
      plan->smem = L.total;
      break;
    }
  }
  if (plan->stages == 0) return OK;
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

int tc_set_centres(TcPlan* plan, const float* Chi, const float* Clo) {
  SKM_TRY(make_map(&plan->tmap_chi, Chi, plan->ld, plan->k, plan->k_pad));
  SKM_TRY(make_map(&plan->tmap_clo, Clo, plan->ld, plan->k, plan->k_pad));
  return OK;
}

int tc_estep(const TcPlan& plan, const float* bias, int32_t* labels, unsigned long long* changed, long long* D,
             const FitState* st, int* err, cudaStream_t s) {
  tc::Params p;
  p.n_tiles = (int)((plan.n + tc::BM - 1) / tc::BM);
  p.n = plan.n;
  p.k = plan.k;
  p.k_pad = plan.k_pad;
  p.nk = plan.k_steps;
  p.stages = plan.stages;
  p.nbl = plan.nbl;
  p.nba = plan.nba;
  p.xcols = plan.xcols;
  p.tmem_cols = plan.tmem_cols;
  p.round_mode = plan.round_mode;
  p.bias = bias;
  p.labels = labels;
  p.changed = changed;
  p.D = D;
  p.X = plan.X;
  p.ld = plan.ld;
  p.d = plan.d;
  p.tile_bytes = (uint32_t)(512 * plan.ld);
  p.st = st;
  p.err = err;
  tc::estep_tc_kernel<<<plan.grid, tc::THREADS, plan.smem, s>>>(plan.tmap_chi, plan.tmap_clo, p);
  return check_launch("estep_tc_kernel");
}

}  // namespace skm

extern "C" int skmetal_debug_tc_probe(int* mode, uint32_t* raw3072) { return skm::tc_probe(mode, raw3072); }
