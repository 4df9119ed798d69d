// Tensor-core E-step for sm_100a: labels[i] = argmin_j (||c_j||^2 - 2 x_i . c_j)
// for 128-row tiles of X, with the dot products computed by tcgen05.mma in
// 3xTF32 (x = x_hi + x_lo, c = c_hi + c_lo; x_hi.c_hi + x_hi.c_lo + x_lo.c_hi,
// accumulated in fp32 in tensor memory). The n x k distance matrix never
// leaves the SM: the epilogue reads each row's k accumulators from TMEM and
// keeps a running argmin in registers (strict '<', lowest index first, as
// sklearn/cluster/_k_means_lloyd.pyx:205-213).
//
// CTA = 6 warps, persistent over row tiles (tile t handled by CTA t % grid):
//   warp 0      TMA producer: X tiles (2-stage ring), centre tiles once
//   warp 1      TMEM owner + MMA issuer (one elected lane)
//   warps 2..5  per tile: split X into tf32 hi (in place) / lo and compute
//               ||x||^2 (converter), then read the accumulators of the
//               previous tile and take the argmin (epilogue); thread r of the
//               group owns TMEM lane / tile row r.
// Shared-memory layout of a tile: K is cut into 8-column chunks (32 bytes
// per row); chunk c of a 128-row tile occupies 4 KB in the canonical
// K-major SWIZZLE_32B layout that TMA writes and UMMA reads (8-row atoms of
// 256 bytes). Columns past d are zero (TMA out-of-bounds fill).
//
// Every mbarrier wait is bounded in time; on timeout the CTA records an error
// code, stops issuing work, waits for its own in-flight copies and MMAs,
// frees its tensor memory and returns.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "device_util.cuh"
#include "driver.h"
#include "estep_tc.h"

namespace skm {

namespace tc {

constexpr int BM = 128;          // rows per tile (UMMA M)
constexpr int KC = 8;            // fp32 columns per K chunk (UMMA K for tf32)
constexpr int CHUNK_BYTES = BM * KC * 4;  // 4096
constexpr int MAX_NK = 16;       // d <= 128
constexpr int MAX_KPAD = 256;    // k <= 256 (one UMMA N)
constexpr int THREADS = 192;
constexpr int NUM_BARS = 12;
constexpr unsigned long long TIMEOUT_NS = 2000000000ull;  // 2 s per wait

enum Bar { FULL0 = 0, FULL1, EMPTY0, EMPTY1, LO_FULL, LO_EMPTY, ACC_FULL0, ACC_FULL1, ACC_EMPTY0, ACC_EMPTY1,
           C_FULL, MMA_DONE };

struct Params {
  int n_tiles;
  long long n;
  int k;
  int k_pad;
  int nk;         // K chunks
  const float* bias;   // ||c||^2, k entries
  int32_t* labels;
  float* mind;    // ||x||^2 + min_j (||c_j||^2 - 2 x.c_j)
  unsigned long long* changed;
  long long* D;        // nullable: incremental deltas of rows that changed label
  const float* X;      // rows (global) for the deltas
  int ld;
  int d;
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

// Bounded wait: returns false on timeout or when another thread aborted.
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

// K-major SWIZZLE_32B UMMA shared-memory descriptor: rows of 32 bytes, 8-row
// atoms of 256 bytes (stride byte offset), leading byte offset unused (1),
// descriptor version 1 (sm_100), layout type 6 (SWIZZLE_32B).
__device__ __forceinline__ uint64_t sw32_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;                 // LBO (unused for swizzled K-major)
  d |= (uint64_t)(256u >> 4) << 32;        // SBO = 256 B
  d |= (uint64_t)1u << 46;                 // version
  d |= (uint64_t)6u << 61;                 // SWIZZLE_32B
  return d;
}

// kind::tf32 instruction descriptor: D fp32, A/B tf32, both K-major, M=128, N.
__host__ __device__ constexpr uint32_t idesc_tf32(int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }

struct Smem {
  // byte offsets from the 1024-aligned dynamic smem base
  uint32_t x[2], xlo, chi, clo, bias, nx, bars, misc;
  uint32_t total;
};

__host__ __device__ inline Smem smem_layout(int nk, int k_pad) {
  Smem s;
  uint32_t off = 0;
  const uint32_t stage = (uint32_t)nk * CHUNK_BYTES;
  s.x[0] = off; off += stage;
  s.x[1] = off; off += stage;
  s.xlo = off; off += stage;
  s.chi = off; off += (uint32_t)nk * k_pad * 32;
  s.clo = off; off += (uint32_t)nk * k_pad * 32;
  s.bias = off; off += (uint32_t)k_pad * 4;
  s.nx = off; off += 2 * BM * 4;
  off = (off + 15) & ~15u;
  s.bars = off; off += NUM_BARS * 8;
  s.misc = off; off += 16;  // [0] tmem base, [1] abort flag
  s.total = off + 1024;     // slack for aligning the base to 1024
  return s;
}

__global__ void __launch_bounds__(THREADS, 1)
estep_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_chi,
                const __grid_constant__ CUtensorMap tmap_clo, Params p) {
  if (p.st && p.st->done) return;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Smem L = smem_layout(p.nk, p.k_pad);
  const uint32_t sbase = smem_u32(base);
  const uint32_t bar0 = sbase + L.bars;
  auto bar = [&](int i) { return bar0 + 8u * (uint32_t)i; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(base + L.misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  float* bias_s = reinterpret_cast<float*>(base + L.bias);
  float* nx_s = reinterpret_cast<float*>(base + L.nx);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int my_tiles = (p.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const uint32_t stage_bytes = (uint32_t)p.nk * CHUNK_BYTES;
  const uint32_t cbytes = (uint32_t)p.nk * p.k_pad * 32;
  const int tmem_cols_alloc = (2 * p.k_pad <= 32) ? 32 : (2 * p.k_pad <= 64) ? 64 : (2 * p.k_pad <= 128) ? 128
                              : (2 * p.k_pad <= 256) ? 256 : 512;

  if (threadIdx.x == 0) {
    mbar_init(bar(FULL0), 1);
    mbar_init(bar(FULL1), 1);
    mbar_init(bar(EMPTY0), 1);
    mbar_init(bar(EMPTY1), 1);
    mbar_init(bar(LO_FULL), 128);
    mbar_init(bar(LO_EMPTY), 1);
    mbar_init(bar(ACC_FULL0), 1);
    mbar_init(bar(ACC_FULL1), 1);
    mbar_init(bar(ACC_EMPTY0), 128);
    mbar_init(bar(ACC_EMPTY1), 128);
    mbar_init(bar(C_FULL), 1);
    mbar_init(bar(MMA_DONE), 1);
    misc[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sbase + L.misc),
                 "r"(tmem_cols_alloc));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  for (int j = threadIdx.x; j < p.k_pad; j += blockDim.x) bias_s[j] = j < p.k ? p.bias[j] : INFINITY;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = misc[0];

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_expect_tx(bar(C_FULL), 2 * cbytes);
      for (int c = 0; c < p.nk; ++c) {
        tma_load_2d(sbase + L.chi + (uint32_t)c * p.k_pad * 32, &tmap_chi, c * KC, 0, bar(C_FULL));
        tma_load_2d(sbase + L.clo + (uint32_t)c * p.k_pad * 32, &tmap_clo, c * KC, 0, bar(C_FULL));
      }
      int armed = 0;
      for (int i = 0; i < my_tiles; ++i) {
        const int s = i & 1;
        if (!mbar_wait(bar(EMPTY0 + s), ((i >> 1) & 1) ^ 1, abort_flag, p.err, 2101)) break;
        const int tile = (int)blockIdx.x + i * (int)gridDim.x;
        mbar_expect_tx(bar(FULL0 + s), stage_bytes);
        for (int c = 0; c < p.nk; ++c)
          tma_load_2d(sbase + L.x[s] + (uint32_t)c * CHUNK_BYTES, &tmap_x, c * KC, tile * BM, bar(FULL0 + s));
        armed = i + 1;
      }
      // drain: wait for our own copies before the CTA can exit
      volatile int no_abort = 0;
      mbar_wait(bar(C_FULL), 0, &no_abort, p.err, 2102);
      for (int i = (armed > 2 ? armed - 2 : 0); i < armed; ++i)
        mbar_wait(bar(FULL0 + (i & 1)), (i >> 1) & 1, &no_abort, p.err, 2103);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32(p.k_pad);
      bool ok = mbar_wait(bar(C_FULL), 0, abort_flag, p.err, 2201);
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int s = i & 1, b = i & 1;
        if (!mbar_wait(bar(FULL0 + s), (i >> 1) & 1, abort_flag, p.err, 2202)) break;
        if (!mbar_wait(bar(LO_FULL), i & 1, abort_flag, p.err, 2203)) break;
        if (!mbar_wait(bar(ACC_EMPTY0 + b), ((i >> 1) & 1) ^ 1, abort_flag, p.err, 2204)) break;
        tc_fence_after();
        const uint32_t tacc = tmem_base + (uint32_t)(b * p.k_pad);
        for (int c = 0; c < p.nk; ++c) {
          const uint64_t a_hi = sw32_desc(sbase + L.x[s] + (uint32_t)c * CHUNK_BYTES);
          const uint64_t a_lo = sw32_desc(sbase + L.xlo + (uint32_t)c * CHUNK_BYTES);
          const uint64_t b_hi = sw32_desc(sbase + L.chi + (uint32_t)c * p.k_pad * 32);
          const uint64_t b_lo = sw32_desc(sbase + L.clo + (uint32_t)c * p.k_pad * 32);
          mma_tf32(tacc, a_lo, b_hi, idesc, c > 0 ? 1u : 0u);
          mma_tf32(tacc, a_hi, b_lo, idesc, 1u);
          mma_tf32(tacc, a_hi, b_hi, idesc, 1u);
        }
        mma_commit(bar(ACC_FULL0 + b));
        mma_commit(bar(EMPTY0 + s));
        mma_commit(bar(LO_EMPTY));
      }
      // all MMAs issued by this thread are complete once MMA_DONE fires
      mma_commit(bar(MMA_DONE));
      volatile int no_abort = 0;
      mbar_wait(bar(MMA_DONE), 0, &no_abort, p.err, 2205);
    }
  } else {
    // ------------------------------------------------ converter + epilogue
    const int q = warp & 3;            // TMEM lane quarter of this warp
    const int row = q * 32 + lane;     // tile row owned in the epilogue
    const int ct = threadIdx.x - 64;   // 0..127 within the group
    bool ok = true;
    for (int i = 0; i <= my_tiles; ++i) {
      // ---- converter for tile i
      if (ok && i < my_tiles) {
        const int s = i & 1;
        ok = mbar_wait(bar(FULL0 + s), (i >> 1) & 1, abort_flag, p.err, 2301) &&
             mbar_wait(bar(LO_EMPTY), (i & 1) ^ 1, abort_flag, p.err, 2302);
        if (ok) {
          // flat pass over the tile: float4 index f = ct + 128*j covers rows
          // (ct>>1) and (ct>>1)+64 of every chunk, half (ct&1) of each row
          float4* xs = reinterpret_cast<float4*>(base + L.x[s]);
          float4* xl = reinterpret_cast<float4*>(base + L.xlo);
          float na = 0.f, nb = 0.f;
          const int nf4 = p.nk * (CHUNK_BYTES / 16);
          for (int f = ct, j = 0; f < nf4; f += 128, ++j) {
            float4 v = xs[f];
            float4 h = make_float4(tf32_trunc(v.x), tf32_trunc(v.y), tf32_trunc(v.z), tf32_trunc(v.w));
            xs[f] = h;
            xl[f] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
            const float sq = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            if (j & 1) nb += sq; else na += sq;
          }
          na += __shfl_xor_sync(0xffffffffu, na, 1);
          nb += __shfl_xor_sync(0xffffffffu, nb, 1);
          if ((ct & 1) == 0) {
            nx_s[(i & 1) * BM + (ct >> 1)] = na;
            nx_s[(i & 1) * BM + (ct >> 1) + 64] = nb;
          }
          fence_async_smem();
          mbar_arrive(bar(LO_FULL));
        }
      }
      named_bar(1, 128);  // nx of tile i visible; epilogue of tile i-1 may read nx[(i-1)&1]
      // ---- epilogue for tile i-1
      if (ok && i > 0) {
        const int t = i - 1, b = t & 1;
        ok = mbar_wait(bar(ACC_FULL0 + b), (t >> 1) & 1, abort_flag, p.err, 2303);
        if (ok) {
          tc_fence_after();
          const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * p.k_pad);
          float best = INFINITY;
          int bl = 0;
          for (int j0 = 0; j0 < p.k_pad; j0 += 16) {
            float v[16];
            tmem_ld16(taddr + (uint32_t)j0, v);
            tmem_ld_wait();
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const float dist = fmaf(-2.0f, v[jj], bias_s[j0 + jj]);
              if (dist < best) {
                best = dist;
                bl = j0 + jj;
              }
            }
          }
          tc_fence_before();
          mbar_arrive(bar(ACC_EMPTY0 + b));
          const long long grow = (long long)((int)blockIdx.x + t * (int)gridDim.x) * BM + row;
          bool ch = false;
          int old = -1;
          if (grow < p.n) {
            if (p.changed) {
              old = p.labels[grow];
              ch = old != bl;
            }
            p.labels[grow] = bl;
            if (p.mind) p.mind[grow] = best + nx_s[b * BM + row];
          }
          if (p.changed) {
            const unsigned int m = __ballot_sync(0xffffffffu, ch);
            if (lane == 0 && m) atomicAdd(p.changed, (unsigned long long)__popc(m));
            if (p.D) warp_apply_changed(p.X, p.ld, p.d, p.k, grow, old, bl, ch, p.D, p.st->scale);
          }
        }
      }
      named_bar(1, 128);  // nx[(i-1)&1] consumed before tile i+1 overwrites it
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols_alloc));
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

int tc_plan(const float* X, int ld, long long n, int d, int k, TcPlan* plan) {
  plan->supported = false;
  if (!encode_fn()) return OK;
  if (d > tc::MAX_NK * tc::KC || k > tc::MAX_KPAD || n < 1) return OK;
  if ((reinterpret_cast<uintptr_t>(X) & 15) || ((ld * 4) & 15)) return OK;
  int dev = 0, optin = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return OK;
  plan->X = X;
  plan->ld = ld;
  plan->n = n;
  plan->d = d;
  plan->k = k;
  plan->k_pad = (int)round_up((size_t)k, 16);
  plan->k_steps = (ld + tc::KC - 1) / tc::KC;
  const tc::Smem L = tc::smem_layout(plan->k_steps, plan->k_pad);
  plan->smem = L.total;
  if ((int)plan->smem > optin) return OK;
  const int n_tiles = (int)((n + tc::BM - 1) / tc::BM);
  plan->grid = std::min(n_tiles, sm_count());
  SKM_TRY(make_map(&plan->tmap_x, X, ld, n, tc::BM));
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(tc::estep_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    attr = true;
  }
  plan->supported = true;
  return OK;
}

int tc_estep(const TcPlan& plan, const float* Chi, const float* Clo, const float* bias, int32_t* labels, float* mind,
             unsigned long long* changed, long long* D, const FitState* st, int* err, cudaStream_t s) {
  CUtensorMap mhi, mlo;
  SKM_TRY(make_map(&mhi, Chi, plan.ld, plan.k, plan.k_pad));
  SKM_TRY(make_map(&mlo, Clo, plan.ld, plan.k, plan.k_pad));
  tc::Params p;
  p.n_tiles = (int)((plan.n + tc::BM - 1) / tc::BM);
  p.n = plan.n;
  p.k = plan.k;
  p.k_pad = plan.k_pad;
  p.nk = plan.k_steps;
  p.bias = bias;
  p.labels = labels;
  p.mind = mind;
  p.changed = changed;
  p.D = D;
  p.X = plan.X;
  p.ld = plan.ld;
  p.d = plan.d;
  p.st = st;
  p.err = err;
  tc::estep_tc_kernel<<<plan.grid, tc::THREADS, plan.smem, s>>>(plan.tmap_x, mhi, mlo, p);
  return check_launch("estep_tc_kernel");
}

}  // namespace skm
