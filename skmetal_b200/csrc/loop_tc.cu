// Persistent Lloyd loop: a single cooperative launch of one CTA per SM runs
// all iterations of a fit, on one GPU or on each rank of a sharded fit.
// Iteration t:
//
//   E-step   the tensor-core pipeline of estep_dev.cuh over the CTA's tiles
//            (labels, changed count, fixed-point deltas of changed rows); at
//            its end the producer already issues the copies of the next
//            iteration's first tiles (X does not change)
//            and, meanwhile, the idle warp clears the delta buffer that
//            E-step t + 1 adds into
//   grid barrier
//   M-step   [bulk iterations: fixed-point sums of all rows, grid barrier]
//            the CTA owning cluster c (c mod CTAs) folds c's sums and count
//            (several ranks: first pushes this rank's deltas of c into every
//            peer's inbox over NVLink and waits for every peer's push of c,
//            owner_exchange), writes its centre, centre image entries,
//            squared shift and squared norm, or flags it empty
//   grid barrier
//            every CTA reads the k shifts, norms and flags: ||c||^2 for its
//            epilogue and, totalled in the canonical order, the same stop
//            decision as every other CTA; the next E-step copies the centre
//            image from global memory. With an empty cluster instead: the
//            cooperative relocation path of mstep_dev.cuh and a grid barrier
//            (several ranks: on the global sums, with candidate rows
//            gathered from every rank, relocate_ranks).
//
// No kernel launches and no host round trips between iterations. The
// arithmetic is that of the multi-launch loop (E-step and M-step kernels) in
// the same order, so both give bit-identical fits.
//
// Buffers whose readers and writers overlap across iterations are rotated
// (each 16-byte aligned, rows of ld entries): the delta buffers D by t mod 3
// (written by E-step t, read by the owners in M-step t, cleared during
// E-step t + 2, written again by E-step t + 3), the peers' inbox rows by
// t mod 2 (a rank pushes iteration t + 2 only after every peer finished
// M-step t), the sums,
// counts and centres by t mod 2 (the owners write the next ones while the
// relocation path may still need the current ones).
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
  size_t d_clear;  // entries of a delta buffer to clear (k * ld + k + 1, rounded up to even)
  // multi-GPU (W > 1): every rank's arrival words, inbox flags, inbox rows
  // and candidate block (peer mappings; index = rank; own included), local
  // scratch for the global deltas and the gathered candidate blocks
  int W, rank;
  unsigned int* pflag[kLoopMaxRanks];
  unsigned long long* pin[kLoopMaxRanks];
  const unsigned char* pcand[kLoopMaxRanks];
  int row;  // 8-byte words of an inbox row
  long long* G;
  unsigned char* cand_all;
  size_t cand_block;
  unsigned long long peer_wait_ns;  // limit of every wait on another rank (inbox polls, rank barrier)
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

// Cross-rank barrier of the multi-GPU loop (every thread of every CTA; the
// CTAs have just passed a local grid barrier). Block 0 writes `epoch` into
// this rank's arrival word in every rank's region with a system-scope
// release (the writes that the local barrier gathered become visible to any
// rank that sees the word); thread 0 of every CTA then polls its own
// region's words with system-scope acquires until every rank's word reaches
// `epoch`. Epochs count the fit's cross-rank barriers from 1 (the words are
// zeroed before the fit's first collective). Bounded: after la.peer_wait_ns
// (5 s by default) the CTA records error 1005 and returns false.
__device__ __forceinline__ bool rank_barrier(const LoopArgs& la, FitState* st, unsigned int epoch) {
  __shared__ int ok_s;
  block_sync();
  if (blockIdx.x == 0 && threadIdx.x < la.W) {
    unsigned int* f = la.pflag[threadIdx.x] + la.rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
  }
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned long long t0 = globaltimer();
    for (int r = 0; r < la.W && ok; ++r) {
      for (unsigned int i = 1;; ++i) {
        unsigned int v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(la.pflag[la.rank] + r) : "memory");
        if (v >= epoch) break;
        if ((i & 255) == 0 && globaltimer() - t0 > la.peer_wait_ns) {
          atomicExch(&st->error, 1005);
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

// Inbox row of rank q's deltas of cluster c (iteration parity par) in the
// region of rank `dst`: 8-byte words, value j in words 2j (low half) and
// 2j + 1 (high half), each word {32 bits of the value, epoch}. A word is
// written by one 8-byte store, so a reader that sees the epoch in it sees
// its half of the value: no fence and no separate flag.
__device__ __forceinline__ unsigned long long* inbox_row(const LoopArgs& la, int dst, int par, int q, int c, int k) {
  return la.pin[dst] + (((long long)par * la.W + q) * k + c) * la.row;
}
__device__ __forceinline__ ulonglong2 ll_pack(long long v, unsigned int epoch) {
  const unsigned long long e = (unsigned long long)epoch << 32;
  return make_ulonglong2(e | (unsigned int)(unsigned long long)v, e | (unsigned int)((unsigned long long)v >> 32));
}
__device__ __forceinline__ long long ll_value(ulonglong2 w) {
  return (long long)(((w.y & 0xffffffffull) << 32) | (w.x & 0xffffffffull));
}
__device__ __forceinline__ bool ll_ready(ulonglong2 w, unsigned int epoch) {
  return (unsigned int)(w.x >> 32) == epoch && (unsigned int)(w.y >> 32) == epoch;
}
__device__ __forceinline__ void ll_store(unsigned long long* p, ulonglong2 w) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(w.x), "l"(w.y) : "memory");
}
__device__ __forceinline__ ulonglong2 ll_load(const unsigned long long* p) {
  ulonglong2 w;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
  return w;
}
// Value j of an inbox row whose epoch was already seen.
__device__ __forceinline__ long long ll_get(const unsigned long long* row, int j) {
  return ll_value(make_ulonglong2(__ldcg(row + 2 * j), __ldcg(row + 2 * j + 1)));
}

// One owner warp of the multi-GPU loop, cluster c, iteration parity par,
// after the local barrier that completed this rank's deltas: pushes the
// rank's deltas of c (lane l: column quad l), count delta and, for c = 0,
// change count into every peer's inbox row (8-byte stores over NVLink),
// then reads every peer's row of c (all peers' loads in flight together) and
// re-polls the words that did not carry this iteration's epoch yet (each lane
// its own; bounded: la.peer_wait_ns, then error 1005), and returns
// c's sums over every rank (S_in added unless bulk; as quad_load) and c's
// count delta over every rank.
__device__ __forceinline__ QuadSums owner_exchange(const LoopArgs& la, FitState* st, const long long* S_in,
                                                   const long long* Dp, const unsigned long long* chg,
                                                   const float* C_old, int c, int par, unsigned int epoch, int bulk,
                                                   long long* cnt_delta) {
  const int lane = threadIdx.x & 31;
  const int k = la.p.k, ld = la.p.ld, nq = ld >> 2;
  const long long i = (long long)c * ld + 4 * lane;
  const long long* dcnt = Dp + (long long)k * ld;
  long long o[4] = {0, 0, 0, 0};
  if (lane < nq) {
    const longlong2 o01 = __ldcg(reinterpret_cast<const longlong2*>(Dp + i));
    const longlong2 o23 = __ldcg(reinterpret_cast<const longlong2*>(Dp + i + 2));
    o[0] = o01.x;
    o[1] = o01.y;
    o[2] = o23.x;
    o[3] = o23.y;
  }
  const long long ocnt = __ldcg(dcnt + c);
  const long long ochg = c == 0 ? (long long)__ldcg(chg) : 0;
  for (int q = 0; q < la.W; ++q) {
    if (q == la.rank) continue;
    unsigned long long* dst = inbox_row(la, q, par, la.rank, c, k);
    if (lane < nq)
#pragma unroll
      for (int u = 0; u < 4; ++u) ll_store(dst + 2 * (4 * lane + u), ll_pack(o[u], epoch));
    if (lane == 0) {
      ll_store(dst + 2 * ld, ll_pack(ocnt, epoch));
      ll_store(dst + 2 * (ld + 1), ll_pack(ochg, epoch));
    }
  }
  long long s[4] = {o[0], o[1], o[2], o[3]};
  if (!bulk && lane < nq) {
    const longlong2 a01 = __ldcg(reinterpret_cast<const longlong2*>(S_in + i));
    const longlong2 a23 = __ldcg(reinterpret_cast<const longlong2*>(S_in + i + 2));
    s[0] += a01.x;
    s[1] += a01.y;
    s[2] += a23.x;
    s[3] += a23.y;
  }
  long long cnt = ocnt;
  // every peer's words go out together; a peer whose words (this lane's) do
  // not carry the epoch yet is polled again below
  unsigned int pending = 0;
#pragma unroll
  for (int q = 0; q < kLoopMaxRanks; ++q) {
    if (q >= la.W || q == la.rank) continue;
    const unsigned long long* src = inbox_row(la, la.rank, par, q, c, k);
    ulonglong2 w[4] = {};
    bool ready = true;
    if (lane < nq)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        w[u] = ll_load(src + 2 * (4 * lane + u));
        ready = ready && ll_ready(w[u], epoch);
      }
    const ulonglong2 wc = ll_load(src + 2 * ld);  // every lane: the count delta
    ready = ready && ll_ready(wc, epoch);
    if (c == 0 && lane == 0) ready = ready && ll_ready(ll_load(src + 2 * (ld + 1)), epoch);  // change count
    if (ready) {
#pragma unroll
      for (int u = 0; u < 4; ++u) s[u] += ll_value(w[u]);
      cnt += ll_value(wc);
    } else {
      pending |= 1u << q;
    }
  }
  const unsigned long long t0 = globaltimer();
  for (unsigned int it = 1; __any_sync(0xffffffffu, pending != 0); ++it) {
    if (pending) {
      const int q = __ffs(pending) - 1;
      const unsigned long long* src = inbox_row(la, la.rank, par, q, c, k);
      ulonglong2 w[4] = {};
      bool ready = true;
      if (lane < nq)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          w[u] = ll_load(src + 2 * (4 * lane + u));
          ready = ready && ll_ready(w[u], epoch);
        }
      const ulonglong2 wc = ll_load(src + 2 * ld);
      ready = ready && ll_ready(wc, epoch);
      if (c == 0 && lane == 0) ready = ready && ll_ready(ll_load(src + 2 * (ld + 1)), epoch);
      if (ready) {
#pragma unroll
        for (int u = 0; u < 4; ++u) s[u] += ll_value(w[u]);
        cnt += ll_value(wc);
        pending &= ~(1u << q);
      }
    }
    if ((it & 63) == 0) {  // the same iterations on every lane; lane 0's clock decides
      const bool late = __shfl_sync(0xffffffffu, globaltimer() - t0 > la.peer_wait_ns, 0);
      if (late) {
        if (lane == 0) atomicExch(&st->error, 1005);
        break;
      }
    }
  }
  QuadSums r;
  r.old = lane < nq ? __ldcg(reinterpret_cast<const float4*>(C_old + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int u = 0; u < 4; ++u) r.s[u] = s[u];
  r.dnz = true;
  *cnt_delta = cnt;
  return r;
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

// Multi-GPU relocation (some cluster is empty after summing every rank's
// counts): the global deltas into G; this rank's min(empties, cap, rows)
// rows farthest from their centre into its candidate block; a cross-rank
// barrier; every rank's block gathered into cand_all; then the relocation
// path on the global sums with those candidates, as the multi-launch loop
// runs it after its all-reduce. Every thread of every CTA.
__device__ bool relocate_ranks(const LoopArgs& la, MStepArgs a, const long long* Dp, int par, int bulk,
                               unsigned long long changed_now, unsigned int& n_bar, unsigned int& epoch) {
  FitState* st = a.st;
  const unsigned int nb = gridDim.x;
  const long long ks = (long long)a.k * a.ld;
  // every owner has seen every peer's push (before the last grid barrier)
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < ks + a.k + 1;
       i += (long long)nb * blockDim.x) {
    long long v = __ldcg(Dp + i);
    if (i < ks + a.k) {
      const int c = i < ks ? (int)(i / a.ld) : (int)(i - ks);
      const int j = i < ks ? (int)(i - (long long)c * a.ld) : a.ld;
      for (int q = 0; q < la.W; ++q)
        if (q != la.rank) v += ll_get(inbox_row(la, la.rank, par, q, c, a.k), j);
    } else {
      v = (long long)changed_now;
    }
    la.G[i] = v;
  }
  a.D = la.G;
  a.changed = reinterpret_cast<const unsigned long long*>(la.G + ks + a.k);
  if (blockIdx.x == 0 && threadIdx.x == 0) st->sel_count = 0;
  if (!loop_barrier(st, la.bar, nb * ++n_bar)) return false;
  const int ne = find_empty_clusters(a, bulk);
  const int m = (int)min((long long)min(ne, kCandCap), a.n);
  if (m > 0) {
    rows_dist_to_old_centres(a, nb);
    if (!loop_barrier(st, la.bar, nb * ++n_bar)) return false;
    if (!select_farthest(a.mind, a.n, a.row_base, m, st, a.hist, a.sel, nb)) return false;
  }
  if (blockIdx.x == 0) {  // this rank's candidate block (the layout of shard_prep_kernel)
    unsigned char* mine = const_cast<unsigned char*>(la.pcand[la.rank]);
    float* dist = reinterpret_cast<float*>(mine + cand_dist_off(kCandCap));
    long long* row = reinterpret_cast<long long*>(mine + cand_row_off(kCandCap));
    int* label = reinterpret_cast<int*>(mine + cand_label_off(kCandCap));
    float* x = reinterpret_cast<float*>(mine + cand_x_off(kCandCap));
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
      const long long r = a.sel[i];
      dist[i] = a.mind[r];
      row[i] = a.row_base + r;
      label[i] = a.labels[r];
      for (int j = 0; j < a.ld; ++j) x[(long long)i * a.ld + j] = a.X[xblk_index(r, j, a.ld)];
    }
    if (threadIdx.x == 0) *reinterpret_cast<int*>(mine) = m;
  }
  if (!rank_barrier(la, st, ++epoch)) return false;
  const size_t words = la.cand_block / 16;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < words * la.W; i += (size_t)nb * blockDim.x) {
    const int r = (int)(i / words);
    const size_t w = i - (size_t)r * words;
    reinterpret_cast<int4*>(la.cand_all + (size_t)r * la.cand_block)[w] =
        __ldcv(reinterpret_cast<const int4*>(la.pcand[r]) + w);
  }
  if (!loop_barrier(st, la.bar, nb * ++n_bar)) return false;
  a.cand = la.cand_all;
  a.cand_ranks = la.W;
  a.cand_cap = kCandCap;
  return relocation_path(a, ne, bulk, changed_now);
}

__global__ void __launch_bounds__(tc::THREADS, 1) lloyd_loop_kernel(LoopArgs la) {
  using namespace tc;
  const Params& p = la.p;
  FitState* st = la.m.st;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ int flags_s[2];
  __shared__ double dsq_s[MAX_KPAD];
  __shared__ unsigned long long chg_s;
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
  unsigned int epoch = 0;  // cross-rank barriers passed
  int t = 0;
  for (; !done; ++t) {
    const int par = t & 1;
    long long* Dp = la.D[t % 3];
    long long* D_next = la.D[(t + 1) % 3];
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
    if (warp == IDLE_W) {
      // the deltas E-step t + 1 adds into, idle since M-step t - 2 (their
      // readers finished before this iteration's first barrier): cleared off
      // the M-step's path; the barrier after this pass orders it before
      // E-step t + 1
      for (size_t i = 2 * ((size_t)blockIdx.x * 32 + lane); i < la.d_clear; i += 64 * (size_t)nb)
        *reinterpret_cast<longlong2*>(D_next + i) = make_longlong2(0, 0);
    }
    estep_pass(p, c, P);
    ++img_loads;        // the pass waited for its image copy
    image_issued = 0;
    pre = P.pre_next;
    proxy_fence_all();
    if (!loop_barrier(st, la.bar, nb * ++n_bar)) break;
    if (__ldcg(&st->error)) break;  // uniform: read after the barrier
    stamp(la.prof, 4 * t + 1);

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
      bulk_pass(p.X, ld, p.n, p.labels, k, Dp, st, c.base, c.L.bars, &st->error);
      zero_stage_padding(p, c);
      proxy_fence_all();
      if (!loop_barrier(st, la.bar, nb * ++n_bar)) break;
    }
    // every rank's deltas of this iteration are complete
    // one GPU: the change count, taken by the last warp (which owns no
    // cluster) while the owners work, read after the next block barrier.
    // Several ranks: it comes with the pushes of cluster 0 (below).
    if (la.W == 1 && threadIdx.x == blockDim.x - 32) chg_s = __ldcg(chg);
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
        long long cnew;
        if (la.W > 1) {  // the exchange of cl's deltas with every peer
          long long cd = 0;
          r = owner_exchange(la, st, S_in, Dp, chg, C_old, cl, par, (unsigned int)t + 1, bulk, &cd);
          cnew = (bulk ? 0 : __ldcg(cnt_in + cl)) + cd;
        } else {
          if (lane < nq) r = quad_load(S_in, Dp, C_old, i0, bulk);
          cnew = (bulk ? 0 : __ldcg(cnt_in + cl)) + __ldcg(dcnt + cl);
        }
        double dsq = 0.0, nrm = 0.0;
        if (cnew > 0 && lane < nq)  // the canonical order of warp_centre_from_sums
          quad_finish(r, cl, lane, i0, d, centre_factor(inv_scale, cnew), cs, la.m.cimg, CentreImage{}, S_out, C_new,
                      nullptr, dsq, nrm);
        dsq = warp_sum(dsq);
        nrm = warp_sum(nrm);
        if (lane == 0) {
          cnt_out[cl] = cnew;
          dsq_c[cl] = dsq;
          nrm_c[cl] = nrm;
          emp_c[cl] = cnew == 0 ? 1.0 : 0.0;
          la.m.bias[cl] = (float)nrm;  // for the final E-step after the loop
        }
      }
      proxy_fence_all();
      if (!loop_barrier(st, la.bar, nb * ++n_bar)) break;
      stamp(la.prof, 4 * t + 2);
      if (la.W > 1) {
        if (__ldcg(&st->error)) break;  // uniform: a peer's push did not arrive
        // the change count over every rank: own plus the peers' rows of
        // cluster 0 (their owner saw them arrive before the barrier)
        if (threadIdx.x == blockDim.x - 32) {
          unsigned long long v = __ldcg(chg);
          for (int q = 0; q < la.W; ++q)
            if (q != la.rank) v += (unsigned long long)ll_get(inbox_row(la, la.rank, par, q, 0, k), ld + 1);
          chg_s = v;
        }
      }
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
      const unsigned long long changed_now = chg_s;
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
            // (with several ranks other CTAs may still read it after the
            // barrier: it is cleared with its buffer, in E-step t + 2)
            if (la.W == 1) *chg = 0;
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
        if (la.W > 1) {
          if (!relocate_ranks(la, a, Dp, par, bulk, changed_now, n_bar, epoch)) break;
        } else {
          const int ne = find_empty_clusters(a, bulk);
          if (!relocation_path(a, ne, bulk, changed_now)) break;
        }
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
  // the image copy issued by the last M-step (the loop stopped after it)
  // lands before the CTA exits
  if (image_issued && threadIdx.x == MMA_W0 * 32) {
    volatile int no_abort = 0;
    mbar_wait(c.bar(B_C_FULL), img_loads & 1, &no_abort, p.err, 2106);
  }
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
  la.d_clear = ((size_t)plan.k * plan.ld + plan.k + 2) & ~(size_t)1;
  la.W = in.nranks;
  la.rank = in.rank;
  la.peer_wait_ns = in.peer_wait_ns ? in.peer_wait_ns : 5000000000ull;
  if (la.W > 1) {
    if (la.W > kLoopMaxRanks || in.rank < 0 || in.rank >= la.W || !in.G || !in.cand_all) {
      set_error(ERR_INVALID, "multi-GPU loop: bad rank layout");
      return ERR_INVALID;
    }
    const size_t ioff = region_inbox_off(la.W, plan.k), coff = region_cand_off(la.W, plan.k, plan.ld);
    for (int r = 0; r < la.W; ++r) {
      unsigned char* rg = in.region[r];
      if (!rg) {
        set_error(ERR_INVALID, "multi-GPU loop: no peer region for rank %d", r);
        return ERR_INVALID;
      }
      la.pflag[r] = reinterpret_cast<unsigned int*>(rg);
      la.pin[r] = reinterpret_cast<unsigned long long*>(rg + ioff);
      la.pcand[r] = rg + coff;
    }
    la.row = (int)region_row(plan.ld);
    la.G = in.G;
    la.cand_all = in.cand_all;
    la.cand_block = cand_block_bytes(kCandCap, plan.ld);
  }
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
