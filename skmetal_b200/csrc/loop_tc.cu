// Persistent Lloyd loop for one GPU: a single cooperative launch of one CTA
// per SM runs all iterations of a fit,
//
//   E-step   the tensor-core pipeline of estep_dev.cuh over the CTA's tiles
//            (labels, changed count, fixed-point deltas of changed rows)
//   barrier
//   M-step   [bulk iterations: fixed-point sums of all rows, barrier]
//            empty clusters; fast path: (cluster, column part) units fold
//            the sums and write the new centres, their image and partial
//            shifts; relocation path: relocation_path of mstep_dev.cuh
//   barrier
//   every CTA reduces the unit partials in the same fixed order, so all of
//   them reach the same convergence decision and refresh their ||c||^2
//
// which is the work of the E-step / M-step kernel pair of the multi-launch
// loop, with the same arithmetic in the same order: both loops give
// bit-identical fits. What the persistent loop removes is two kernel launches
// per iteration, the pipeline's per-launch set-up (barrier initialisation,
// tensor-memory allocation) and the host's polling of the done flag.
//
// Buffers whose readers and writers would overlap across the iteration
// boundary alternate by iteration parity: the delta buffer D (the next E-step
// adds into the other one while this iteration's counts part is cleared), the
// counts (units read the old, write the new) and the centres (as in the
// multi-launch loop). The centre image is written by the units of iteration t
// between the two barriers and read by the E-step of t + 1 after the second
// one.
//
// Every wait is bounded: mbarrier waits (estep_dev.cuh) and grid barriers
// record an error code in the fit state and the CTAs leave the loop together
// after the next grid barrier.
#include <cuda_runtime.h>

#include <algorithm>

#include "driver.h"
#include "estep_dev.cuh"
#include "loop_tc.h"
#include "mstep_dev.cuh"

namespace skm {

namespace {

struct LoopArgs {
  tc::Params p;
  MStepArgs m;
  long long* D[2];
  long long* cnt[2];
  float* C[2];
  unsigned long long* prof;
};

__device__ __forceinline__ void proxy_fence_all() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Profile stamps (block 0, thread 0): per iteration t, [4t] start, [4t + 1]
// E-step done (after the barrier), [4t + 2] bulk sums and empty clusters
// done, [4t + 3] centres done (after the barrier); [4 T] the end.
__device__ __forceinline__ void stamp(unsigned long long* prof, int i) {
  if (prof && blockIdx.x == 0 && threadIdx.x == 0) prof[i] = tc::globaltimer();
}

__global__ void __launch_bounds__(tc::THREADS, 1) lloyd_loop_kernel(LoopArgs la) {
  using namespace tc;
  const Params& p = la.p;
  FitState* st = la.m.st;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ double dsq_s[MAX_KPAD];
  __shared__ double red[32];
  __shared__ int flags_s[2];
  Cta c;
  cta_setup(p, smem_raw, p.bias, c);

  const unsigned int nb = gridDim.x;
  const int k = p.k, ld = p.ld;
  const long long ks = (long long)k * ld;
  const double inv_scale = st->inv_scale;
  const float cs = ldexpf(1.0f, st->xexp);  // centres are bounded by max |x|
  const int nq = ld >> 2;
  const int parts = max(1, min(nq, (int)nb / k));
  const int units = k * parts;
  long long* S = const_cast<long long*>(la.m.S);
  int bulk = st->bulk;
  int done = st->done;
  int t = 0;
  for (; !done; ++t) {
    const int par = t & 1;
    long long* Dp = la.D[par];
    long long* dcnt = Dp + ks;
    unsigned long long* chg = reinterpret_cast<unsigned long long*>(Dp + ks + k);
    const long long* cnt_in = la.cnt[par];
    long long* cnt_out = la.cnt[par ^ 1];
    const float* C_old = la.C[par];
    float* C_new = la.C[par ^ 1];
    stamp(la.prof, 4 * t);
    // the centre image written by other CTAs' generic stores is next read by
    // this CTA's bulk copies (async proxy)
    if (t > 0) proxy_fence_all();

    // ---------------------------------------------------------------- E-step
    estep_pass(p, c, t * c.my_tiles, par, bulk ? nullptr : Dp, chg);
    proxy_fence_all();
    if (!grid_barrier(st, nb)) break;
    if (__ldcg(&st->error)) break;  // uniform: read after the barrier
    stamp(la.prof, 4 * t + 1);
    const unsigned long long changed_now = __ldcg(chg);

    // ---------------------------------------------------------------- M-step
    MStepArgs a = la.m;
    a.D = Dp;
    a.changed = chg;
    a.counts = cnt_in;
    a.C_old = C_old;
    a.C_new = C_new;
    a.host_done = nullptr;
    if (bulk) {
      bulk_pass(p.X, ld, p.n, p.labels, k, Dp, st->scale,
                bulk_acc_bytes(k, ld, c.L.bars) ? reinterpret_cast<long long*>(c.base) : nullptr);
      zero_stage_padding(p, c);
      proxy_fence_all();
      if (!grid_barrier(st, nb)) break;
    }
    const int n_empty = find_empty_clusters(a, bulk);
    stamp(la.prof, 4 * t + 2);
    if (n_empty == 0) {
      // fast path: units of (cluster, column part) over the blocks
      if (blockIdx.x == 0 && threadIdx.x == 0) st->cexp = st->xexp;  // read by the next E-step only
      for (int u = blockIdx.x; u < units; u += nb) {
        const int cl = u / parts, pt = u % parts;
        const int q0 = (int)((long long)nq * pt / parts), q1 = (int)((long long)nq * (pt + 1) / parts);
        const int j0 = 4 * q0, j1 = 4 * q1;
        const long long cnew = (bulk ? 0 : __ldcg(&cnt_in[cl])) + __ldcg(&dcnt[cl]);
        const double fct = centre_factor(inv_scale, cnew);
        double dsq = 0.0, nrm = 0.0;
        for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
          const long long i = (long long)cl * ld + j;
          const long long dv = __ldcg(&Dp[i]);
          const long long sum = (bulk ? 0 : __ldcg(&S[i])) + dv;
          const float old = __ldcg(&C_old[i]);
          S[i] = sum;
          if (dv != 0) Dp[i] = 0;
          float v = 0.0f;
          if (j < p.d) {
            v = centre_from_sum(sum, fct);
            const double df = (double)v - (double)old;
            dsq += df * df;
            nrm += (double)v * v;
            cimg_put(a.cimg, cl, j, v, cs);
          }
          C_new[i] = v;
        }
        // one column per thread (ld <= 128 < blockDim): the block tree then
        // sums the same terms in the same order as the 1024-thread M-step
        dsq = block_sum_f64(dsq, red);
        nrm = block_sum_f64(nrm, red);
        if (threadIdx.x == 0) {
          a.unit_dsq[u] = dsq;
          a.unit_nrm[u] = nrm;
          if (pt == 0) cnt_out[cl] = cnew;
        }
        block_sync();
      }
      proxy_fence_all();
      if (!grid_barrier(st, nb)) break;
      stamp(la.prof, 4 * t + 3);
      // every CTA: per-cluster shift and ||c||^2 from the unit partials in
      // part order, then the total in the fixed order of block_ordered_sum
      for (int cl = threadIdx.x; cl < p.k_pad; cl += blockDim.x) {
        if (cl >= k) {  // padding clusters (the bulk sums may have used this memory)
          c.bias_s[cl] = INFINITY;
          continue;
        }
        double dsq = 0.0, nrm = 0.0;
        for (int pt = 0; pt < parts; ++pt) {
          dsq += __ldcg(&a.unit_dsq[cl * parts + pt]);
          nrm += __ldcg(&a.unit_nrm[cl * parts + pt]);
        }
        dsq_s[cl] = dsq;
        c.bias_s[cl] = (float)nrm;
        if (blockIdx.x == 0) la.m.bias[cl] = (float)nrm;  // for the final E-step after the loop
      }
      block_sync();
      const double tot = block_ordered_sum(dsq_s, k, red);
      if (threadIdx.x == 0) {
        // _kmeans.py:723-741, as finish_iteration
        const int it = t + 1;
        const int strict = changed_now == 0;
        const int dn = strict || tot <= st->tol || it >= st->max_iter;
        const int bk = st->bulk_always || changed_now > (unsigned long long)st->bulk_threshold;
        flags_s[0] = dn;
        flags_s[1] = bk;
        if (blockIdx.x == 0) {
          st->shift_tot = tot;
          st->iter = it;
          st->bulk = bk;
          st->n_empty = 0;
          st->relocated = 0;
          if (strict) st->strict = 1;
          st->done = dn;
          *chg = 0;  // every CTA read it before the barrier
        }
      }
      // this iteration's count deltas: read by the units before the barrier,
      // next written by the E-step of iteration t + 2
      if (blockIdx.x == 0)
        for (int cl = threadIdx.x; cl < k; cl += blockDim.x) dcnt[cl] = 0;
      block_sync();
      done = flags_s[0];
      bulk = flags_s[1];
    } else {
      if (!relocation_path(a, n_empty, bulk, changed_now)) break;
      // the counts were folded into cnt_in (before a barrier of the path)
      if (blockIdx.x == 0)
        for (int cl = threadIdx.x; cl < k; cl += blockDim.x) cnt_out[cl] = __ldcg(&cnt_in[cl]);
      proxy_fence_all();
      if (!grid_barrier(st, nb)) break;
      stamp(la.prof, 4 * t + 3);
      load_bias(p, c, la.m.bias);
      done = *reinterpret_cast<volatile int*>(&st->done);
      bulk = *reinterpret_cast<volatile int*>(&st->bulk);
      block_sync();
    }
  }
  stamp(la.prof, 4 * t);
  cta_teardown(p, c);
}

}  // namespace

size_t tc_loop_static_smem() {
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, lloyd_loop_kernel) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return fa.sharedSizeBytes;
}

bool tc_loop_supported(const TcPlan& plan) {
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, lloyd_loop_kernel) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return plan.supported && plan.k <= tc::MAX_KPAD && fa.sharedSizeBytes + plan.smem <= (size_t)optin;
}

int tc_lloyd_loop(const TcPlan& plan, const LoopInputs& in, cudaStream_t s) {
  LoopArgs la{};
  la.p = tc::make_params(plan);
  la.p.img = in.img;
  la.p.sexp = in.sexp;
  la.p.bias = in.bias;
  la.p.labels = const_cast<int32_t*>(in.m.labels);
  la.p.st = in.m.st;
  la.p.err = &in.m.st->error;
  la.m = in.m;
  for (int i = 0; i < 2; ++i) {
    la.D[i] = in.D[i];
    la.cnt[i] = in.counts[i];
    la.C[i] = in.C[i];
  }
  la.prof = in.prof;
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa{};
    SKM_CUDA(cudaFuncGetAttributes(&fa, lloyd_loop_kernel));
    SKM_CUDA(cudaFuncSetAttribute(lloyd_loop_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  optin - (int)fa.sharedSizeBytes));
    attr_dev = dev;
  }
  void* args[] = {&la};
  SKM_CUDA(cudaLaunchCooperativeKernel((void*)lloyd_loop_kernel, dim3(plan.grid), dim3(tc::THREADS), args,
                                       plan.smem, s));
  return check_launch("lloyd_loop_kernel");
}

}  // namespace skm
