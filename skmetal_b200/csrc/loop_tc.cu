// Persistent Lloyd loop for one GPU: a single cooperative launch of one CTA
// per SM runs all iterations of a fit. Iteration t:
//
//   E-step   the tensor-core pipeline of estep_dev.cuh over the CTA's tiles
//            (labels, changed count, fixed-point deltas of changed rows); at
//            its end the producer already issues the copies of the next
//            iteration's first tiles (X does not change)
//   grid barrier
//   M-step   [bulk iterations: fixed-point sums of all rows, grid barrier]
//            the CTA owning cluster c (c mod CTAs) folds c's sums and count,
//            writes its centre, centre image entries, squared shift and
//            squared norm, or flags it empty, and clears c's deltas of
//            iteration t - 1
//   grid barrier
//            every CTA reads the k shifts, norms and flags: ||c||^2 for its
//            epilogue and, totalled in the canonical order, the same stop
//            decision as every other CTA; the next E-step copies the centre
//            image from global memory. With an empty cluster instead: the
//            cooperative relocation path of mstep_dev.cuh and a grid barrier.
//
// No kernel launches and no host round trips between iterations. The
// arithmetic is that of the multi-launch loop (E-step and M-step kernels) in
// the same order, so both give bit-identical fits.
//
// Buffers whose readers and writers overlap across iterations are rotated
// (each 16-byte aligned, rows of ld entries): the delta buffers D by t mod 3
// (written by E-step t, read by the owners in M-step t, cleared by them in
// M-step t + 1, written again by E-step t + 3), the sums, counts and centres
// by t mod 2 (the owners write the next ones while the relocation path may
// still need the current ones).
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
  long long* D[3];
  long long* S[2];
  long long* cnt[2];
  float* C[2];
  double* part;  // per cluster: squared shift [0, k), squared norm [k, 2k), empty flag [2k, 3k)
  unsigned int* bar;  // the loop's grid-barrier counter, zero at launch
  unsigned long long* prof;
};

// Grid barrier of the loop: every CTA adds 1 to a counter that only grows
// during the launch (zero at launch) and waits until it reaches nb * (number
// of barriers passed, this one included). The release add and the acquire
// polls order the CTA's earlier writes (gathered by the block barrier) before
// every other CTA's later reads. Bounded: after 2 s the CTA records error
// 1001 and returns false.
__device__ __forceinline__ bool loop_barrier(FitState* st, unsigned int* counter, unsigned int target) {
  __shared__ int ok_s;
  block_sync();
  if (threadIdx.x == 0) {
    int ok = 1;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
    if (v < target) {
      const unsigned long long t0 = globaltimer();
      for (unsigned int i = 1;; ++i) {
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
        if (v >= target) break;
        if ((i & 255) == 0 && globaltimer() - t0 > 2000000000ull) {
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

__device__ __forceinline__ void proxy_fence_all() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Profile stamps (block 0, thread 0): per iteration t, [4t] start, [4t + 1]
// E-step done (after the first barrier), [4t + 2] owners done (after the
// second), [4t + 3] M-step done; [4 T] the end.
__device__ __forceinline__ void stamp(unsigned long long* prof, int i) {
  if (prof && blockIdx.x == 0 && threadIdx.x == 0) prof[i] = globaltimer();
}

__global__ void __launch_bounds__(tc::THREADS, 1) lloyd_loop_kernel(LoopArgs la) {
  using namespace tc;
  const Params& p = la.p;
  FitState* st = la.m.st;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ int flags_s[2];
  __shared__ double dsq_s[MAX_KPAD];
  Cta c;
  cta_setup(p, smem_raw, p.bias, c);

  const unsigned int nb = gridDim.x;
  const int k = p.k, ld = p.ld, d = p.d;
  const long long ks = (long long)k * ld;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const double inv_scale = st->inv_scale;
  const int xexp = st->xexp;
  const float cs = ldexpf(1.0f, xexp);  // centres are bounded by max |x|
  // the first image (centre_prep) is scaled by 2^cexp, those of the loop by 2^xexp
  float negscale = -ldexpf(1.0f, 1 - xexp - st->cexp);
  const float negscale_loop = -ldexpf(1.0f, 1 - 2 * xexp);
  const int max_iter = st->max_iter;
  int bulk = st->bulk;
  int done = st->done;
  int img_loads = 0, pre = 0, image_issued = 0;
  unsigned int n_bar = 0;  // loop barriers passed
  int t = 0;
  for (; !done; ++t) {
    const int par = t & 1;
    long long* Dp = la.D[t % 3];
    long long* D_prev = la.D[(t + 2) % 3];
    long long* dcnt = Dp + ks;
    unsigned long long* chg = reinterpret_cast<unsigned long long*>(Dp + ks + k);
    long long* S_in = la.S[par];
    long long* S_out = la.S[par ^ 1];
    long long* cnt_in = la.cnt[par];
    long long* cnt_out = la.cnt[par ^ 1];
    const float* C_old = la.C[par];
    float* C_new = la.C[par ^ 1];
    stamp(la.prof, 4 * t);
    // an image copy issued by the producer below reads what other CTAs (or
    // the relocation path) wrote through the generic proxy
    if (t > 0) proxy_fence_all();

    // ---------------------------------------------------------------- E-step
    Pass P{};
    P.ig0 = t * c.my_tiles;
    P.par = par;
    P.pre = pre;
    // bulk iterations use the stages as the sums' workspace: nothing in flight
    P.pre_next = (bulk || t + 1 >= max_iter) ? 0 : min(p.stages, c.my_tiles);
    // the centre image of the previous M-step (or of centre_prep): after the
    // fast path the M-step already issued its copy
    P.load_image = !image_issued;
    P.wait_image = 1;
    P.img_par = img_loads & 1;
    P.negscale = negscale;
    P.deltas = bulk ? nullptr : Dp;
    P.changed = chg;
    estep_pass(p, c, P);
    ++img_loads;
    pre = P.pre_next;
    proxy_fence_all();
    if (!loop_barrier(st, la.bar, nb * ++n_bar)) break;
    if (__ldcg(&st->error)) break;  // uniform: read after the barrier
    stamp(la.prof, 4 * t + 1);
    const unsigned long long changed_now = __ldcg(chg);

    // ---------------------------------------------------------------- M-step
    MStepArgs a = la.m;
    a.S = S_in;
    a.D = Dp;
    a.changed = chg;
    a.counts = cnt_in;
    a.C_old = C_old;
    a.C_new = C_new;
    a.host_done = nullptr;
    if (bulk) {
      bulk_pass(p.X, ld, p.n, p.labels, k, Dp, st->scale, c.base, c.L.bars, &st->error);
      zero_stage_padding(p, c);
      proxy_fence_all();
      if (!loop_barrier(st, la.bar, nb * ++n_bar)) break;
    }
    // (no block touches S_in, D or the counts before the barrier above)
    // owners: cluster cl is CTA cl mod nb's, one warp per owned cluster
    {
      double* dsq_c = la.part;
      double* nrm_c = la.part + k;
      double* emp_c = la.part + 2 * k;
      const int nq = ld >> 2;  // <= 32: one column quad per lane
      for (int m = warp; blockIdx.x + (long long)m * nb < (long long)k; m += nwarps) {
        const int cl = (int)(blockIdx.x + (long long)m * nb);
        const long long i0 = (long long)cl * ld + 4 * lane;
        // the quad and the count loads go out together (one round trip)
        QuadSums r{};
        if (lane < nq) r = quad_load(S_in, Dp, C_old, i0, bulk);
        const long long cnew = (bulk ? 0 : __ldcg(cnt_in + cl)) + __ldcg(dcnt + cl);
        double dsq = 0.0, nrm = 0.0;
        if (cnew > 0 && lane < nq)  // the canonical order of warp_centre_from_sums
          quad_finish(r, cl, lane, i0, d, centre_factor(inv_scale, cnew), cs, la.m.cimg, CentreImage{}, S_out, C_new,
                      nullptr, dsq, nrm);
        dsq = warp_sum(dsq);
        nrm = warp_sum(nrm);
        // cl's deltas of iteration t - 1: their readers finished before this
        // iteration's first barrier; E-step t + 2 adds into them again
        for (int j = 4 * lane; j < ld; j += 128) {
          *reinterpret_cast<longlong2*>(D_prev + (long long)cl * ld + j) = make_longlong2(0, 0);
          *reinterpret_cast<longlong2*>(D_prev + (long long)cl * ld + j + 2) = make_longlong2(0, 0);
        }
        if (lane == 0) {
          D_prev[ks + cl] = 0;
          cnt_out[cl] = cnew;
          dsq_c[cl] = dsq;
          nrm_c[cl] = nrm;
          emp_c[cl] = cnew == 0 ? 1.0 : 0.0;
          la.m.bias[cl] = (float)nrm;  // for the final E-step after the loop
        }
      }
      if (blockIdx.x == 0 && threadIdx.x == 0) D_prev[ks + k] = 0;  // its changed counter
      proxy_fence_all();
      if (!loop_barrier(st, la.bar, nb * ++n_bar)) break;
      stamp(la.prof, 4 * t + 2);
      // every CTA: flags, ||c||^2, and the total shift in the canonical
      // order (warp_ordered_sum); one load round (k <= 256 < threads)
      const int cl_t = threadIdx.x;
      const double dsq_t = cl_t < k ? __ldcg(dsq_c + cl_t) : 0.0;
      const double nrm_t = cl_t < k ? __ldcg(nrm_c + cl_t) : 0.0;
      const double emp_t = cl_t < k ? __ldcg(emp_c + cl_t) : 0.0;
      if (cl_t < k) dsq_s[cl_t] = dsq_t;
      if (cl_t < p.k_pad) c.bias_s[cl_t] = cl_t < k ? (float)nrm_t : INFINITY;
      __syncwarp();
      const int n_empty = __syncthreads_count(emp_t != 0.0) ? 1 : 0;  // any empty cluster
      // the owners' image is complete: its copy overlaps the decision
      image_issued = n_empty == 0;
      if (image_issued && threadIdx.x == MMA_W0 * 32) {  // an otherwise idle lane
        // written by other CTAs' generic stores, read by this CTA's async proxy
        asm volatile("fence.proxy.async.global;" ::: "memory");
        issue_image_copy(p, c);
      }
      if (n_empty == 0 && warp == 0) {
        const double tot = warp_ordered_sum(dsq_s, k);
        if (lane == 0) {
          // _kmeans.py:723-741, as finish_iteration
          const int it = t + 1;
          const int strict = changed_now == 0;
          const int dn = strict || tot <= st->tol || it >= max_iter;
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
            *chg = 0;
          }
        }
      }
      block_sync();
      if (n_empty == 0) {
        done = flags_s[0];
        bulk = flags_s[1];
      } else {
        // relocation: the empty clusters again with their ids, then the
        // cooperative path, which folds this iteration's sums and counts into
        // S_in and cnt_in and writes every centre, image entry and norm
        const int ne = find_empty_clusters(a, bulk);
        if (!relocation_path(a, ne, bulk, changed_now)) break;
        for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < ks + k;
             i += (long long)nb * blockDim.x) {
          if (i < ks) S_out[i] = __ldcg(S_in + i);
          else cnt_out[i - ks] = __ldcg(cnt_in + (i - ks));
        }
        proxy_fence_all();
        if (!loop_barrier(st, la.bar, nb * ++n_bar)) break;
        load_bias(p, c, la.m.bias);
        done = *reinterpret_cast<volatile int*>(&st->done);
        bulk = *reinterpret_cast<volatile int*>(&st->bulk);
        block_sync();
      }
    }
    negscale = negscale_loop;
    stamp(la.prof, 4 * t + 3);
  }
  stamp(la.prof, 4 * t);
  if (t > 0 && blockIdx.x == 0 && threadIdx.x == 0) st->cexp = xexp;  // scale of the final image
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
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return plan.supported && plan.k <= tc::MAX_KPAD && tc_loop_static_smem() + plan.smem <= (size_t)optin;
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
  for (int i = 0; i < 3; ++i) la.D[i] = in.D[i];
  for (int i = 0; i < 2; ++i) {
    la.S[i] = in.S[i];
    la.cnt[i] = in.counts[i];
    la.C[i] = in.C[i];
  }
  la.part = in.part;
  la.bar = in.bar;
  la.prof = in.prof;
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    SKM_CUDA(cudaFuncSetAttribute(lloyd_loop_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  optin - (int)tc_loop_static_smem()));
    attr_dev = dev;
  }
  void* args[] = {&la};
  SKM_CUDA(cudaLaunchCooperativeKernel((void*)lloyd_loop_kernel, dim3(plan.grid), dim3(tc::THREADS), args,
                                       plan.smem, s));
  return check_launch("lloyd_loop_kernel");
}

}  // namespace skm
