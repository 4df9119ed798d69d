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
#include "estep_dev.cuh"
#include "estep_tc.h"
#include "loop_tc.h"

namespace skm {

namespace tc {

__global__ void __launch_bounds__(THREADS, 1) estep_tc_kernel(Params p) {
  // the M-step that follows may be scheduled as soon as SMs free up; the
  // previous M-step's centres, bias, image and flags must be visible first
  pdl_launch_dependents();
  pdl_wait();
  if (p.st && p.st->done) return;
  // bulk iterations rebuild the sums from all rows in the M-step
  long long* const deltas = (p.st && p.st->bulk) ? nullptr : p.D;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Cta c;
  cta_setup(p, smem_raw, p.bias, c);
  Pass P{};
  P.load_image = 1;
  P.wait_image = 1;
  P.negscale = -ldexpf(1.0f, 1 - __ldcg(p.sexp) - __ldcg(p.sexp + 1));
  P.deltas = deltas;
  P.changed = p.changed;
  estep_pass(p, c, P);
  cta_teardown(p, c);
}

// ---------------------------------------------------------------------------
// split working copy of X (see the layout note at split8)
// ---------------------------------------------------------------------------
// One thread per (tile, chunk, row): reads the row's two fp32 column quads of
// the chunk from the blocked copy and writes its x_hi and x_lo (16 bytes each)
// at the same row position of the chunk's two halves; consecutive threads take
// consecutive rows, so reads and writes are coalesced 512-byte runs per warp.
__global__ void split_x_kernel(const float* __restrict__ X, int ld, int nk, long long n_tiles,
                               const int* __restrict__ sexp, uint4* __restrict__ Xs, uint32_t tile_bytes,
                               int half_last) {
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
    uint4* dst = Xs + (t * tile_bytes + (size_t)c * CHUNK_BYTES) / 16;
    if (half_last && c == nk - 1) {  // x_hi of the four columns, then their x_lo
      dst[row] = make_uint4(hi.x, hi.y, lo.x, lo.y);
    } else {
      dst[row] = hi;
      dst[BM + row] = lo;
    }
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
  block_sync();
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
  block_sync();
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
  tmem_ld_wait16(v);
  reg_pin16(w);
  reg_pin16(u);
  for (int j = 0; j < PROBE_K; ++j) {
    out[tid * PROBE_K + j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
    out[2048 + tid * PROBE_K + j] = u[j];
  }
  tc_fence_before();
  block_sync();
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
  plan->half_last = 0;
  if (getenv("SKMETAL_DISABLE_TC")) return OK;
  if (d > tc::MAX_NK * tc::KC || n < 1) return OK;
  if ((reinterpret_cast<uintptr_t>(X) & 15) || ((ld * 4) & 15)) return OK;
  int dev = 0, optin = 0, major = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return OK;
  if (k > tc::MAX_KPAD) return tc_plan_wide(X, ld, n, d, k, optin, plan);
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
  // prefer one stacked operand (one MMA per chunk); both layouts need >= 2 stages;
  // the persistent loop kernel's static shared memory stays free
  const int avail = optin - (int)tc_loop_static_smem();
  plan->stages = 0;
  for (int stacked = (2 * plan->k_pad <= 256) ? 1 : 0; stacked >= 0 && plan->stages == 0; --stacked) {
    const int nkx = stacked ? plan->k_steps : (plan->k_steps + 1) & ~1;
    const uint32_t stage_bytes = (uint32_t)nkx * tc::CHUNK_BYTES;
    const uint32_t img_bytes = (uint32_t)(cimg_halves(plan->k_pad, plan->k_steps, stacked) * 2);
    const int acc_cols = stacked ? 2 * plan->k_pad : plan->k_pad;
    const int nacc = 4 * acc_cols <= 512 ? 4 : (2 * acc_cols <= 512 ? 2 : 1);
    for (int st = tc::MAX_STAGES; st >= 2; --st) {
      const tc::Smem L = tc::smem_layout(stage_bytes, img_bytes, plan->k_pad, st, nacc);
      if ((int)L.total <= avail) {
        plan->stacked = stacked;
        plan->half_last = stacked && (ld % tc::KC) == 4;
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

uint32_t tc_tile_bytes(const TcPlan& plan) {
  return (uint32_t)(plan.k_steps * tc::CHUNK_BYTES) - (plan.half_last ? (uint32_t)tc::CHUNK_BYTES / 2 : 0u);
}

size_t tc_split_bytes(const TcPlan& plan) {
  return (size_t)((plan.n + tc::BM - 1) / tc::BM) * tc_tile_bytes(plan);
}

int tc_split_x(TcPlan* plan, void* Xs, const int* sexp, cudaStream_t s) {
  const long long n_tiles = (plan->n + tc::BM - 1) / tc::BM;
  const long long work = n_tiles * plan->k_steps * tc::BM;
  const int blocks = (int)std::max(1LL, std::min((work + 255) / 256, (long long)sm_count() * 8));
  tc::split_x_kernel<<<blocks, 256, 0, s>>>(plan->X, plan->ld, plan->k_steps, n_tiles, sexp,
                                            reinterpret_cast<uint4*>(Xs), tc_tile_bytes(*plan), plan->half_last);
  SKM_TRY(check_launch("split_x_kernel"));
  plan->Xs = static_cast<const unsigned char*>(Xs);
  return OK;
}

CentreImage tc_centre_image(const TcPlan& plan, uint16_t* img) {
  return CentreImage{img, plan.k_pad, plan.k_steps, plan.stacked, plan.nbs, plan.half_last};
}

int tc_estep(const TcPlan& plan, const uint16_t* img, const int* sexp, const float* bias, int32_t* labels,
             unsigned long long* changed, long long* D, const FitState* st, int* err, cudaStream_t s, bool pdl) {
  if (plan.wide) return tc_estep_wide(plan, img, sexp, bias, labels, changed, D, st, err, s, pdl);
  tc::Params p = tc::make_params(plan);
  p.img = img;
  p.sexp = sexp;
  p.bias = bias;
  p.labels = labels;
  p.changed = changed;
  p.D = D;
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
