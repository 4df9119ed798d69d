// KMeans fit / predict engine and the KMeans entry points of the C ABI.
//
// A fit runs entirely on the device and follows scikit-learn's
// KMeans(algorithm="lloyd", n_init=1, init=array).fit
// (sklearn/cluster/_kmeans.py:1436-1562, loop at :705-758):
//   prep   : mean (exact fixed-point column sums), centring of X and of the
//            init centres, fixed-point scale, scaled tolerance
//   loop   : per iteration one E-step launch (labels, change count, sums),
//            [all-reduce of the sums over ranks], one cooperative M-step launch
//            (relocation, averaging, shift, convergence flags)
//   final  : E-step again when the loop did not converge strictly, inertia,
//            centres + mean.
// The host enqueues iterations in chunks and only reads the `done` flag of the
// previous chunk, so the GPU never waits for the host inside the loop.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "comm.h"
#include "driver.h"
#include "estep_tc.h"
#include "kernels.cuh"
#include "loop_tc.h"
#include "../../include/skmetal_cuda.h"

namespace skm {

// SKMETAL_FIT_PROFILE times the E-step launches of iterations 0, 10, 20, ...
// with CUDA events: one event pair per iteration costs a few microseconds of
// device time, so timing a sample keeps the measured loop representative.
constexpr int kProfileEvery = 10;

struct FitStats {
  double ms_total = 0, ms_prep = 0, ms_loop = 0, ms_final = 0;
  int estep_launches = 0;
  double estep_ms_sum = 0;
  unsigned long long launches = 0;
  int iterations = 0;
  int distinct = -1;  // labels present in the final assignment (-1: not counted)
};
static thread_local FitStats t_stats;
// globaltimer stamps of the last profiled persistent-loop fit (lloyd_loop_kernel)
static thread_local std::vector<unsigned long long> t_loop_stamps;

struct Dataset {
  int device = 0;
  float* X = nullptr;  // n x ld, raw (not centred)
  long long n = 0;
  int d = 0;
  int ld = 0;
};

struct FitParams {
  const float* X_host = nullptr;  // n x d host rows, or
  const float* X_dev = nullptr;   // n x ld device rows (raw)
  long long n = 0;
  int d = 0;
  int k = 0;
  const float* init_host = nullptr;  // k x d
  const float* w_host = nullptr;     // n sample weights (host, nullable: unit weights)
  int max_iter = 300;
  double tol = 0.0;
  bool tol_abs = false;
  bool center = true;
  bool simt = false;
  bool profile = false;
  bool distributed = false;
  bool bulk_sums = false;  // recompute sums from scratch every iteration
  long long row_base = 0;
  long long n_total = 0;
  // outputs (host, nullable)
  float* centers_out = nullptr;
  int32_t* labels_out = nullptr;
  uint32_t* labels_out_u32 = nullptr;
  double* inertia_out = nullptr;
  int32_t* n_iter_out = nullptr;
  // single Lloyd step (skmetal_kmeans_lloyd_iter)
  bool single_step = false;
  float* weight_out = nullptr;
  float* shift_out = nullptr;
};

static int validate(long long n, long long d, long long k) {
  if (n <= 0 || d <= 0 || k <= 0) {
    set_error(ERR_INVALID, "invalid shape n=%lld d=%lld k=%lld", n, d, k);
    return ERR_INVALID;
  }
  if (n >= (1LL << 31) || d > (1 << 20) || k > (1 << 20)) {
    set_error(ERR_INVALID, "shape too large n=%lld d=%lld k=%lld", n, d, k);
    return ERR_INVALID;
  }
  return OK;
}

static inline int ld_of(int d) { return (int)round_up((size_t)d, 4); }

static int blocks_for(long long work, int threads, int cap_per_sm = 8) {
  long long b = (work + threads - 1) / threads;
  long long cap = (long long)sm_count() * cap_per_sm;
  return (int)std::max(1LL, std::min(b, cap));
}

// ---------------------------------------------------------------------------
// E-step dispatch: tensor-core kernel when the shape is supported, else SIMT
// ---------------------------------------------------------------------------

struct EStepPlan {
  bool tc = false;
  TcPlan tcp;
};

static int launch_assign_simt(const float* X, int ld, long long n, int d, const float* C, int k, int32_t* labels,
                              float* mind, const FitState* st, unsigned long long* changed, long long* D,
                              int skip_if_strict, int blocked, cudaStream_t s) {
  const int chunk = std::max(1, std::min(k, kAssignSmemFloats / ld));
  const size_t smem = sizeof(float) * (size_t)chunk * ld;
  const int threads = 256;
  const int blocks = (int)((n + threads - 1) / threads);
  assign_simt_kernel<<<blocks, threads, smem, s>>>(X, ld, n, d, C, k, labels, mind, st, changed, D,
                                                   skip_if_strict, blocked);
  return check_launch("assign_simt_kernel");
}

// The cooperative M-step; with `pdl` it is launched with programmatic stream
// serialization so that its launch overlaps the E-step's tail (the kernel
// waits for the E-step's writes itself).
static int launch_mstep(MStepArgs& ma, int blocks, int threads, size_t smem, bool pdl, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  SKM_CUDA(cudaLaunchKernelEx(&cfg, mstep_kernel, ma));
  return check_launch("mstep_kernel");
}

// ---------------------------------------------------------------------------
// the fit
// ---------------------------------------------------------------------------

static int run_fit(const FitParams& p) {
  SKM_TRY(check_injected("fit"));
  SKM_TRY(validate(p.n, p.d, p.k));
  const long long n_total = p.distributed ? p.n_total : p.n;
  if (!p.distributed && p.k > p.n) {
    set_error(ERR_INVALID, "n_samples=%lld should be >= n_clusters=%d", p.n, p.k);
    return ERR_INVALID;
  }
  if (n_total >= (1LL << 32) - 1) {
    set_error(ERR_INVALID, "too many rows (%lld)", n_total);
    return ERR_INVALID;
  }
  Comm* comm = nullptr;
  if (p.distributed) {
    comm = comm_get();
    if (!comm) {
      set_error(ERR_INVALID, "distributed fit without a communicator (call skmetal_comm_init)");
      return ERR_INVALID;
    }
  }
  cudaStream_t s;
  double* pinned;
  SKM_TRY(thread_stream(&s, &pinned));
  const unsigned long long launches0 = g_launches.load();
  const long long n = p.n;
  const int d = p.d, k = p.k, ld = ld_of(d);
  const int nsm = sm_count();

  cudaEvent_t ev0, ev1, ev2, ev3;
  SKM_CUDA(cudaEventCreate(&ev0));
  SKM_CUDA(cudaEventCreate(&ev1));
  SKM_CUDA(cudaEventCreate(&ev2));
  SKM_CUDA(cudaEventCreate(&ev3));
  struct EvGuard {
    cudaEvent_t e[4];
    ~EvGuard() {
      for (auto x : e) cudaEventDestroy(x);
    }
  } evg{{ev0, ev1, ev2, ev3}};

  DevBuffers buf(s);
  float *X = nullptr, *Cb0 = nullptr, *Cb1 = nullptr, *mean = nullptr, *mind = nullptr, *init_d = nullptr;
  int32_t* labels = nullptr;
  long long *S = nullptr, *colsum = nullptr;
  FitState* st = nullptr;
  unsigned int* u32s = nullptr;  // [0] raw maxabs, [1] centred maxabs, [2..513] hist
  double* dscr = nullptr;        // scale(1) sumsq(1) partials(...)
  int* empty_ids = nullptr;
  long long *sel = nullptr, *cnt_adj = nullptr;
  int* reloc_label = nullptr;
  float *reloc_dist = nullptr, *reloc_x = nullptr, *reloc_w = nullptr;
  const int n_part = nsm * 4;
  const int reloc_rows = std::min(k, kMaxEmptyCap);

  // sample weights: finite and non-negative, not all zero; single-GPU fits
  if (p.w_host) {
    if (comm) {
      set_error(ERR_INVALID, "sample weights are supported on one GPU only");
      return ERR_INVALID;
    }
    double wsum = 0.0;
    for (long long i = 0; i < n; ++i) {
      const float wi = p.w_host[i];
      if (!(wi >= 0.0f) || !std::isfinite(wi)) {
        set_error(ERR_INVALID, "sample_weight[%lld] = %g: weights must be finite and non-negative", i, (double)wi);
        return ERR_INVALID;
      }
      wsum += wi;
    }
    if (!(wsum > 0.0)) {
      set_error(ERR_INVALID, "sample weights sum to zero");
      return ERR_INVALID;
    }
  }
  // X: the blocked working copy (round_up(n, 128) rows, see xblk_index)
  const long long n_pad = (n + 127) / 128 * 128;
  SKM_TRY(buf.alloc_n(&X, (size_t)n_pad * ld));
  SKM_TRY(buf.alloc_n(&Cb0, (size_t)k * ld));
  SKM_TRY(buf.alloc_n(&Cb1, (size_t)k * ld));
  SKM_TRY(buf.alloc_n(&mean, (size_t)ld));
  SKM_TRY(buf.alloc_n(&mind, (size_t)n));
  SKM_TRY(buf.alloc_n(&init_d, (size_t)k * d));
  // whole 128-row tiles (-1 past n): the tiled bulk pass copies them per tile
  SKM_TRY(buf.alloc_n(&labels, (size_t)n_pad));
  // persistent sums of the current labels: S (k*ld) | counts (k)
  SKM_TRY(buf.alloc_n(&S, (size_t)k * ld + k));
  long long* counts = S + (size_t)k * ld;
  // per-iteration deltas (the all-reduced payload): dS (k*ld) | dcount (k) | changed (1)
  // all-reduced payload: D = [dS (k x ld) | dcount (k) | changed], then on
  // multi-GPU fits one relocation-candidate slot per rank (16-byte aligned)
  const size_t d_len = (size_t)k * ld + k + 1;
  const size_t cand_off = (d_len + 1) & ~(size_t)1;
  const size_t cand_bytes = comm ? cand_block_bytes(kCandCap, ld) : 0;
  const size_t payload_len = comm ? cand_off + cand_bytes / 8 * (size_t)comm_nranks(comm) : d_len;
  long long* D = nullptr;
  SKM_TRY(buf.alloc_n(&D, payload_len));
  unsigned long long* changed = reinterpret_cast<unsigned long long*>(D + (size_t)k * ld + k);
  SKM_TRY(buf.alloc_n(&colsum, (size_t)ld));
  SKM_TRY(buf.alloc_n(&st, 1));
  SKM_TRY(buf.alloc_n(&u32s, 2 + 512 + 2));  // [514], [515]: max |w x|, max w (weighted fits)
  float* w_dev = nullptr;  // weighted fits: n_pad weights, 0 past n (the tiled bulk pass copies whole tiles)
  if (p.w_host) {
    SKM_TRY(buf.alloc_n(&w_dev, (size_t)n_pad));
    SKM_CUDA(cudaMemsetAsync(w_dev, 0, sizeof(float) * n_pad, s));
    SKM_CUDA(cudaMemcpyAsync(w_dev, p.w_host, sizeof(float) * n, cudaMemcpyHostToDevice, s));
  }
  SKM_TRY(buf.alloc_n(&dscr, 2 + n_part + std::max(nsm, k)));
  SKM_TRY(buf.alloc_n(&empty_ids, kMaxEmptyCap));
  SKM_TRY(buf.alloc_n(&sel, kMaxEmptyCap));
  SKM_TRY(buf.alloc_n(&cnt_adj, (size_t)k));
  SKM_TRY(buf.alloc_n(&reloc_label, kMaxEmptyCap));
  SKM_TRY(buf.alloc_n(&reloc_dist, kMaxEmptyCap));
  SKM_TRY(buf.alloc_n(&reloc_w, kMaxEmptyCap));
  SKM_TRY(buf.alloc_n(&reloc_x, (size_t)reloc_rows * ld));
  double* scale_mean = dscr;
  double* sumsq = dscr + 1;
  double* partials = dscr + 2;
  double* shift_partial = dscr + 2 + n_part;

  // Multi-GPU fits may run the persistent loop, which exchanges the deltas
  // through the ranks' peer regions: set up once per communicator
  // (collective) and zeroed here, before this fit's first collective, so no
  // peer can write into it before the zeroing (peers only write from their
  // loop kernels, which start after this fit's collectives, and the previous
  // fit's kernels ended before its last collective).
  const char* loop_env = getenv("SKMETAL_LOOP");
  const bool launches_loop = loop_env && strcmp(loop_env, "launches") == 0;
  // SKMETAL_PEER_WAIT_MS: limit of the persistent loop's waits on other ranks
  // (default 5 s); SKMETAL_DEBUG_ORPHAN_PEER=1 (tests only): a one-GPU fit
  // runs its loop as rank 0 of two ranks of which the second never starts
  const char* wait_env = getenv("SKMETAL_PEER_WAIT_MS");
  const unsigned long long peer_wait_ns = wait_env ? (unsigned long long)(atof(wait_env) * 1e6) : 0ull;
  const char* orphan_env = getenv("SKMETAL_DEBUG_ORPHAN_PEER");
  const bool orphan_peer = !comm && orphan_env && atoi(orphan_env) == 1;
  void* const* regions = nullptr;
  if (comm && !p.single_step && !launches_loop) {
    SKM_TRY(comm_peer_region(comm, s, &regions));
    const size_t rb = region_bytes(comm_nranks(comm), k, ld);
    if (regions && rb > kPeerRegionBytes) regions = nullptr;  // the same on every rank
    if (regions) SKM_CUDA(cudaMemsetAsync(regions[comm_rank(comm)], 0, rb, s));
  }

  SKM_CUDA(cudaEventRecord(ev0, s));
  // ---- data in: row-major X (host rows are staged, a dataset is used in place)
  const float* raw = p.X_dev;
  float* staged = nullptr;
  if (p.X_host) {
    SKM_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&staged), sizeof(float) * (size_t)n * ld, s));
    int rc = upload_rows(staged, ld, p.X_host, n, d, s);
    if (rc) {
      cudaFreeAsync(staged, s);
      return rc;
    }
    raw = staged;
  }
  SKM_CUDA(cudaMemcpyAsync(init_d, p.init_host, sizeof(float) * (size_t)k * d, cudaMemcpyHostToDevice, s));
  SKM_CUDA(cudaMemsetAsync(u32s, 0, sizeof(unsigned int) * (2 + 512 + 2), s));
  SKM_CUDA(cudaMemsetAsync(colsum, 0, sizeof(long long) * ld, s));
  SKM_CUDA(cudaMemsetAsync(mean, 0, sizeof(float) * ld, s));

  // ---- exact mean, then the blocked (centred) working copy -------------------
  const int ew_blocks = blocks_for(n * ld / 4, 256, 8);
  const bool tol_rel = !p.tol_abs && p.tol != 0.0;
  int prep_rc = OK;
  if (p.center) {
    maxabs_kernel<<<ew_blocks, 256, 0, s>>>(raw, ld, n, d, &u32s[0]);
    prep_rc = check_launch("maxabs_kernel");
    if (!prep_rc && comm) prep_rc = comm_allreduce_max_u32(comm, &u32s[0], 1, s);
    if (!prep_rc) {
      scale_kernel<<<1, 32, 0, s>>>(&u32s[0], (double)n_total, scale_mean);
      prep_rc = check_launch("scale_kernel");
    }
    if (!prep_rc) {
      const int q = ld / 4;
      const int threads = q <= 1024 ? q * std::max(1, 256 / q) : 1024;
      colsum_fixed_kernel<<<nsm * 2, threads, sizeof(long long) * ld, s>>>(raw, ld, n, d, scale_mean, colsum);
      prep_rc = check_launch("colsum_fixed_kernel");
    }
    if (!prep_rc && comm) prep_rc = comm_allreduce_sum_s64(comm, colsum, ld, s);
    if (!prep_rc) {
      mean_from_colsum_kernel<<<1, 256, 0, s>>>(colsum, d, scale_mean, (double)n_total, mean);
      prep_rc = check_launch("mean_from_colsum_kernel");
    }
  }
  if (!prep_rc) {
    // one pass: blocked copy (minus the mean), max |x|, sum of squares for the relative tolerance
    center_block_kernel<<<n_part, 256, 0, s>>>(raw, ld, n, d, p.center ? mean : nullptr, X, &u32s[1],
                                               tol_rel ? partials : nullptr);
    prep_rc = check_launch("center_block_kernel");
  }
  if (staged) cudaFreeAsync(staged, s);
  SKM_TRY(prep_rc);
  if (comm) SKM_TRY(comm_allreduce_max_u32(comm, &u32s[1], 1, s));
  center_init_kernel<<<std::max(1, std::min(1024, (k * ld + 255) / 256)), 256, 0, s>>>(
      init_d, d, k, p.center ? mean : nullptr, Cb0, ld);
  SKM_TRY(check_launch("center_init_kernel"));
  if (tol_rel) {
    ordered_sum_kernel<<<1, 32, 0, s>>>(partials, n_part, sumsq);
    SKM_TRY(check_launch("ordered_sum_kernel"));
    if (comm) SKM_TRY(comm_allreduce_sum_f64(comm, sumsq, 1, s));
  }
  if (w_dev) {
    weight_max_kernel<<<n_part, 256, 0, s>>>(X, ld, n, w_dev, &u32s[514]);
    SKM_TRY(check_launch("weight_max_kernel"));
  }
  init_state_kernel<<<1, 32, 0, s>>>(st, p.max_iter, p.tol, tol_rel ? 1 : 0, tol_rel ? sumsq : nullptr,
                                     (double)n_total, d, &u32s[1], p.bulk_sums ? 1 : 0, w_dev, &u32s[514],
                                     bulk_divisor(k, ld));
  SKM_TRY(check_launch("init_state_kernel"));
  SKM_CUDA(cudaMemsetAsync(labels, 0xff, sizeof(int32_t) * n_pad, s));  // label -1: every row changes in iteration 1
  SKM_CUDA(cudaMemsetAsync(S, 0, sizeof(long long) * ((size_t)k * ld + k), s));
  SKM_CUDA(cudaMemsetAsync(D, 0, sizeof(long long) * payload_len, s));

  // ---- E-step plan ---------------------------------------------------------
  EStepPlan plan;
  if (!p.simt) {
    int rc = tc_plan(X, ld, n, d, k, &plan.tcp);
    plan.tc = (rc == OK) && plan.tcp.supported;
  }
  float* bias = nullptr;
  CentreImage cimg{};
  if (plan.tc) {
    void* Xs = nullptr;
    SKM_TRY(buf.alloc(&Xs, tc_split_bytes(plan.tcp)));
    SKM_TRY(tc_split_x(&plan.tcp, Xs, &st->xexp, s));
    SKM_TRY(buf.alloc_n(&bias, (size_t)plan.tcp.k_pad));
    const size_t halves = plan.tcp.img_bytes / 2;
    uint16_t* img = nullptr;
    SKM_TRY(buf.alloc_n(&img, halves));
    SKM_CUDA(cudaMemsetAsync(img, 0, plan.tcp.img_bytes, s));  // padding entries stay zero
    cimg = tc_centre_image(plan.tcp, img);
    // operands of the first E-step; later ones come out of the M-step
    centre_prep_kernel<<<1, 1024, 0, s>>>(Cb0, k, ld, d, bias, cimg, st);
    SKM_TRY(check_launch("centre_prep_kernel"));
  }
  int* dev_err = &st->error;
  SKM_CUDA(cudaEventRecord(ev1, s));

  // ---- Lloyd loop -----------------------------------------------------------
  MStepArgs ma{};
  ma.st = st;
  ma.X = X;
  ma.ld = ld;
  ma.d = d;
  ma.n = n;
  ma.row_base = p.row_base;
  ma.labels = labels;
  ma.mind = mind;
  ma.S = S;
  ma.counts = counts;
  ma.D = D;
  ma.changed = changed;
  float* shift_dev = nullptr;
  if (p.single_step) {
    SKM_TRY(buf.alloc_n(&shift_dev, (size_t)k));
    ma.shift_out = shift_dev;
  }
  ma.k = k;
  ma.empty_ids = empty_ids;
  ma.hist = &u32s[2];
  ma.sel = sel;
  ma.cnt_adj = cnt_adj;
  ma.reloc_label = reloc_label;
  ma.reloc_dist = reloc_dist;
  ma.reloc_x = reloc_x;
  ma.reloc_w = reloc_w;
  ma.shift_partial = shift_partial;
  ma.cimg = cimg;
  ma.bias = bias;
  const int mstep_blocks = nsm;
  const int mstep_threads = 1024;
  const size_t mstep_smem = mstep_smem_bytes(k, ld);
  if (mstep_smem > 48 * 1024)
  {
    SKM_CUDA(cudaFuncSetAttribute(mstep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mstep_smem));
    SKM_CUDA(cudaFuncSetAttribute(shard_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mstep_smem));
  }

  std::vector<cudaEvent_t> prof_ev;
  if (p.profile) {
    prof_ev.resize(2 * (size_t)p.max_iter);
    for (auto& e : prof_ev) SKM_CUDA(cudaEventCreate(&e));
  }
  struct ProfGuard {
    std::vector<cudaEvent_t>* v;
    ~ProfGuard() {
      for (auto e : *v) cudaEventDestroy(e);
    }
  } pg{&prof_ev};

  // done flag written by the M-steps straight into mapped pinned memory
  volatile int* host_done = reinterpret_cast<volatile int*>(pinned);
  *host_done = 0;
  int* host_done_dev = nullptr;
  SKM_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&host_done_dev), pinned, 0));
  ma.host_done = host_done_dev;
  ma.bulk_external = comm ? 1 : 0;
  // multi-GPU: candidate slots after D, and this rank's own cluster counts
  long long* local_counts = nullptr;
  if (comm) {
    ma.cand = reinterpret_cast<const unsigned char*>(D + cand_off);
    ma.cand_ranks = comm_nranks(comm);
    ma.cand_cap = kCandCap;
    SKM_TRY(buf.alloc_n(&local_counts, (size_t)k));
    SKM_CUDA(cudaMemsetAsync(local_counts, 0, sizeof(long long) * k, s));
  }

  // One GPU with the tensor-core E-step: the persistent loop kernel runs
  // every iteration in one launch (SKMETAL_LOOP=launches selects the
  // multi-launch loop instead; both give bit-identical fits).
  const bool multi = comm && comm_nranks(comm) > 1;
  static_assert(kLoopMaxRanks == kMaxPeerRanks, "rank limits of the loop and the peer region");
  bool persistent = plan.tc && (!multi || regions) && !p.single_step && !launches_loop && tc_loop_supported(plan.tcp);
  if (multi && regions) {
    // every rank must take the same loop (a rank with an empty shard, for
    // one, has no tensor-core plan): agree with a max all-reduce
    unsigned int* w = &u32s[1];  // the centred maxabs word is no longer needed
    unsigned int not_ok = persistent ? 0u : 1u;
    SKM_CUDA(cudaMemcpyAsync(w, &not_ok, sizeof(not_ok), cudaMemcpyHostToDevice, s));
    SKM_TRY(comm_allreduce_max_u32(comm, w, 1, s));
    SKM_CUDA(cudaMemcpyAsync(&not_ok, w, sizeof(not_ok), cudaMemcpyDeviceToHost, s));
    SKM_CUDA(cudaStreamSynchronize(s));
    persistent = not_ok == 0;
  }
  std::vector<unsigned long long> prof_stamps;
  if (persistent) {
    // second and third delta buffers, second sums + counts (the loop rotates them)
    // (16-byte aligned: the loop reads and writes them as column quads)
    const size_t d_stride = round_up(d_len, 4);
    long long *D23 = nullptr, *S2 = nullptr;
    SKM_TRY(buf.alloc_n(&D23, 2 * d_stride));
    SKM_TRY(buf.alloc_n(&S2, (size_t)k * ld + k));
    SKM_CUDA(cudaMemsetAsync(D23, 0, sizeof(long long) * 2 * d_stride, s));
    SKM_CUDA(cudaMemsetAsync(S2, 0, sizeof(long long) * ((size_t)k * ld + k), s));
    unsigned long long* prof_d = nullptr;
    if (p.profile) {
      prof_stamps.assign(4 * (size_t)p.max_iter + 1, 0);
      SKM_TRY(buf.alloc_n(&prof_d, prof_stamps.size()));
      SKM_CUDA(cudaMemsetAsync(prof_d, 0, sizeof(unsigned long long) * prof_stamps.size(), s));
    }
    LoopInputs li{};
    li.img = cimg.img;
    li.sexp = &st->xexp;
    li.bias = bias;
    li.D[0] = D;
    li.D[1] = D23;
    li.D[2] = D23 + d_stride;
    li.S[0] = S;
    li.S[1] = S2;
    li.counts[0] = counts;
    li.counts[1] = S2 + (size_t)k * ld;
    li.C[0] = Cb0;
    li.C[1] = Cb1;
    li.m = ma;
    li.prof = prof_d;
    if (multi) {
      li.nranks = comm_nranks(comm);
      li.rank = comm_rank(comm);
      for (int r = 0; r < li.nranks; ++r) li.region[r] = static_cast<unsigned char*>(regions[r]);
      SKM_TRY(buf.alloc_n(&li.G, d_len));
      SKM_TRY(buf.alloc(reinterpret_cast<void**>(&li.cand_all), cand_block_bytes(kCandCap, ld) * li.nranks));
    } else if (orphan_peer) {
      // failure-path test: the loop runs as rank 0 of two whose rank 1 never
      // starts. Both regions are local, zeroed, and only this kernel touches
      // them: its pushes land in region 1, and its polls for rank 1's pushes
      // into region 0 run out after the peer-wait limit (error 1005)
      li.nranks = 2;
      li.rank = 0;
      const size_t rb = region_bytes(2, k, ld);
      for (int r = 0; r < 2; ++r) {
        SKM_TRY(buf.alloc(reinterpret_cast<void**>(&li.region[r]), rb));
        SKM_CUDA(cudaMemsetAsync(li.region[r], 0, rb, s));
      }
      SKM_TRY(buf.alloc_n(&li.G, d_len));
      SKM_TRY(buf.alloc(reinterpret_cast<void**>(&li.cand_all), cand_block_bytes(kCandCap, ld) * 2));
    }
    li.peer_wait_ns = peer_wait_ns;
    SKM_TRY(buf.alloc_n(&li.part, 3 * (size_t)k));
    SKM_TRY(buf.alloc_n(&li.bar, 1));
    SKM_CUDA(cudaMemsetAsync(li.bar, 0, sizeof(unsigned int), s));
    SKM_TRY(tc_lloyd_loop(plan.tcp, li, s));
    SKM_CUDA(cudaEventRecord(ev2, s));
    if (prof_d)
      SKM_CUDA(cudaMemcpyAsync(prof_stamps.data(), prof_d, sizeof(unsigned long long) * prof_stamps.size(),
                               cudaMemcpyDeviceToHost, s));
  } else {
    const int chunk = 8;
    int it = 0, chunk_idx = 0, pending = -1;
    bool done_seen = false;
    cudaEvent_t chunk_ev[2];
    SKM_CUDA(cudaEventCreateWithFlags(&chunk_ev[0], cudaEventDisableTiming));
    SKM_CUDA(cudaEventCreateWithFlags(&chunk_ev[1], cudaEventDisableTiming));
    struct ChunkGuard {
      cudaEvent_t* e;
      ~ChunkGuard() {
        cudaEventDestroy(e[0]);
        cudaEventDestroy(e[1]);
      }
    } cg{chunk_ev};

    auto wait_event = [&](cudaEvent_t e) -> int {
      if (!comm) {
        SKM_CUDA(cudaEventSynchronize(e));
        return OK;
      }
      return comm_wait_event(comm, e);
    };

    while (it < p.max_iter && !done_seen) {
      const int end = std::min(p.max_iter, it + chunk);
      for (; it < end; ++it) {
        const float* Cin = (it & 1) ? Cb1 : Cb0;
        float* Cout = (it & 1) ? Cb0 : Cb1;
        const bool timed = p.profile && it % kProfileEvery == 0;
        if (timed) SKM_CUDA(cudaEventRecord(prof_ev[2 * it], s));
        // Iterations flagged `bulk` on the device (the first one, and those
        // after an iteration that changed many rows) rebuild the sums from all
        // rows; the others add the deltas of the rows that changed label.
        if (plan.tc) {
          SKM_TRY(tc_estep(plan.tcp, cimg.img, &st->xexp, bias, labels, changed, D, st, dev_err, s, !comm && !timed));
        } else {
          SKM_TRY(launch_assign_simt(X, ld, n, d, Cin, k, labels, nullptr, st, changed, D, 0, 1, s));
        }
        if (timed) SKM_CUDA(cudaEventRecord(prof_ev[2 * it + 1], s));
        ma.C_old = Cin;
        ma.C_new = Cout;
        if (comm) {
          // bulk pass, local counts and relocation candidates, then one all-reduce
          int rank = comm_rank(comm);
          void* pargs[] = {&ma, &local_counts, &rank};
          SKM_CUDA(cudaLaunchCooperativeKernel((void*)shard_prep_kernel, dim3(mstep_blocks), dim3(mstep_threads), pargs,
                                               mstep_smem, s));
          SKM_TRY(check_launch("shard_prep_kernel"));
          SKM_TRY(comm_allreduce_sum_s64(comm, D, payload_len, s));
        }
        SKM_TRY(launch_mstep(ma, mstep_blocks, mstep_threads, mstep_smem, !comm && !timed, s));
      }
      SKM_CUDA(cudaEventRecord(chunk_ev[chunk_idx & 1], s));
      if (pending >= 0) {
        SKM_TRY(wait_event(chunk_ev[pending & 1]));
        // The M-steps publish the iteration count at convergence (0 while
        // running). One GPU may stop as soon as it is seen; ranks of a sharded
        // fit stop only once it falls in a chunk they have all waited for, so
        // that every rank enqueues the same collectives.
        const int at = *host_done;
        const int pending_end = std::min(p.max_iter, (pending + 1) * chunk);
        if (at > 0 && (!comm || at <= pending_end)) done_seen = true;
      }
      pending = chunk_idx++;
    }
    if (pending >= 0) SKM_TRY(wait_event(chunk_ev[pending & 1]));
    SKM_CUDA(cudaEventRecord(ev2, s));
  }

  FitState hs;
  SKM_CUDA(cudaMemcpyAsync(&hs, st, sizeof(FitState), cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  if (hs.error) {
    set_error(ERR_DEVICE, "device-side check failed in the Lloyd loop (code %d)", hs.error);
    return ERR_DEVICE;
  }
  if ((hs.maxabs_bits & 0x7fffffffu) >= 0x7f800000u) {
    set_error(ERR_INVALID, "X contains NaN or infinity");
    return ERR_INVALID;
  }
  const int iters = hs.iter;
  float* Cfin = (iters & 1) ? Cb1 : Cb0;

  if (p.single_step) {
    // outputs of one lloyd_iter: E-step labels, M-step centres, weights after
    // relocation, per-centre shifts
    float* wf = reinterpret_cast<float*>(sel);  // k floats fit in the selection scratch when k <= cap
    float* wbuf = nullptr;
    if (k > kMaxEmptyCap * 2) SKM_TRY(buf.alloc_n(&wbuf, (size_t)k));
    if (wbuf) wf = wbuf;
    counts_to_float_kernel<<<std::max(1, std::min(1024, (k + 255) / 256)), 256, 0, s>>>(cnt_adj, k, wf);
    SKM_TRY(check_launch("counts_to_float_kernel"));
    add_mean_kernel<<<std::max(1, std::min(1024, (k * d + 255) / 256)), 256, 0, s>>>(Cfin, k, ld, d, nullptr,
                                                                                    init_d);
    SKM_TRY(check_launch("add_mean_kernel"));
    if (p.centers_out)
      SKM_CUDA(cudaMemcpyAsync(p.centers_out, init_d, sizeof(float) * (size_t)k * d, cudaMemcpyDeviceToHost, s));
    if (p.labels_out)
      SKM_CUDA(cudaMemcpyAsync(p.labels_out, labels, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, s));
    if (p.weight_out) SKM_CUDA(cudaMemcpyAsync(p.weight_out, wf, sizeof(float) * k, cudaMemcpyDeviceToHost, s));
    if (p.shift_out)
      SKM_CUDA(cudaMemcpyAsync(p.shift_out, shift_dev, sizeof(float) * k, cudaMemcpyDeviceToHost, s));
    SKM_CUDA(cudaStreamSynchronize(s));
    return OK;
  }

  // ---- final E-step, inertia, outputs ----------------------------------------
  if (!hs.strict) {
    if (plan.tc) {
      // centre image and bias of the final centres were written by the last M-step
      SKM_TRY(tc_estep(plan.tcp, cimg.img, &st->xexp, bias, labels, nullptr, nullptr, nullptr, dev_err, s));
    } else {
      SKM_TRY(launch_assign_simt(X, ld, n, d, Cfin, k, labels, nullptr, nullptr, nullptr, nullptr, 0, 1, s));
    }
  }
  inertia_partial_kernel<<<n_part, 256, 0, s>>>(X, ld, n, d, Cfin, labels, partials, 1, w_dev);
  SKM_TRY(check_launch("inertia_partial_kernel"));
  // the clusters the final labels use (one GPU; sharded fits leave the count out)
  unsigned int* bitmap = nullptr;
  std::vector<unsigned int> bitmap_h;
  if (!comm && k <= kLabelBitmapMaxK) {
    const int words = (k + 31) / 32;
    SKM_TRY(buf.alloc_n(&bitmap, (size_t)words));
    SKM_CUDA(cudaMemsetAsync(bitmap, 0, sizeof(unsigned int) * words, s));
    label_bitmap_kernel<<<blocks_for(n, 256, 4), 256, 0, s>>>(labels, n, k, bitmap);
    SKM_TRY(check_launch("label_bitmap_kernel"));
    bitmap_h.resize(words);
  }
  ordered_sum_kernel<<<1, 32, 0, s>>>(partials, n_part, &dscr[1]);
  SKM_TRY(check_launch("ordered_sum_kernel"));
  if (comm) SKM_TRY(comm_allreduce_sum_f64(comm, &dscr[1], 1, s));
  float* cout_d = init_d;  // reuse: k x d
  add_mean_kernel<<<std::max(1, std::min(1024, (k * d + 255) / 256)), 256, 0, s>>>(Cfin, k, ld, d,
                                                                                  p.center ? mean : nullptr, cout_d);
  SKM_TRY(check_launch("add_mean_kernel"));
  SKM_CUDA(cudaEventRecord(ev3, s));
  double inertia = 0.0;
  SKM_CUDA(cudaMemcpyAsync(&inertia, &dscr[1], sizeof(double), cudaMemcpyDeviceToHost, s));
  if (p.centers_out)
    SKM_CUDA(cudaMemcpyAsync(p.centers_out, cout_d, sizeof(float) * (size_t)k * d, cudaMemcpyDeviceToHost, s));
  if (p.labels_out)
    SKM_CUDA(cudaMemcpyAsync(p.labels_out, labels, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, s));
  if (p.labels_out_u32)
    SKM_CUDA(cudaMemcpyAsync(p.labels_out_u32, labels, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, s));
  if (bitmap)
    SKM_CUDA(cudaMemcpyAsync(bitmap_h.data(), bitmap, sizeof(unsigned int) * bitmap_h.size(), cudaMemcpyDeviceToHost,
                             s));
  SKM_CUDA(cudaStreamSynchronize(s));
  if (p.inertia_out) *p.inertia_out = inertia;
  if (p.n_iter_out) *p.n_iter_out = iters;

  FitStats fs;
  float ms = 0;
  cudaEventElapsedTime(&ms, ev0, ev3);
  fs.ms_total = ms;
  cudaEventElapsedTime(&ms, ev0, ev1);
  fs.ms_prep = ms;
  cudaEventElapsedTime(&ms, ev1, ev2);
  fs.ms_loop = ms;
  cudaEventElapsedTime(&ms, ev2, ev3);
  fs.ms_final = ms;
  if (!(p.profile && persistent)) t_loop_stamps.clear();  // stamps describe the last profiled loop-kernel fit only
  if (p.profile && persistent) {
    // E-step phases of the persistent loop from its globaltimer stamps
    for (int i = 0; i < iters && 4 * i + 1 < (int)prof_stamps.size(); ++i) {
      if (prof_stamps[4 * i + 1] > prof_stamps[4 * i]) {
        fs.estep_ms_sum += (double)(prof_stamps[4 * i + 1] - prof_stamps[4 * i]) * 1e-6;
        fs.estep_launches += 1;
      }
    }
    prof_stamps.resize(std::min(prof_stamps.size(), 4 * (size_t)iters + 1));
    t_loop_stamps = prof_stamps;
  } else if (p.profile) {
    for (int i = 0; i < iters; i += kProfileEvery) {
      float m = 0;
      if (cudaEventElapsedTime(&m, prof_ev[2 * i], prof_ev[2 * i + 1]) == cudaSuccess) {
        fs.estep_ms_sum += m;
        fs.estep_launches += 1;
      }
    }
  }
  fs.launches = g_launches.load() - launches0;
  fs.iterations = iters;
  if (bitmap) {
    fs.distinct = 0;
    for (unsigned int wd : bitmap_h) fs.distinct += __builtin_popcount(wd);
  }
  t_stats = fs;
  return OK;
}

// ---------------------------------------------------------------------------
// predict-style helpers (no centring)
// ---------------------------------------------------------------------------

static int launch_assign_any(const float* X, int ld, long long n, int d, const float* C, int k, int32_t* labels,
                             float* mind, cudaStream_t s) {
  const bool small = k * std::max(d, 4) <= 12288 && ld == d && (d == 4 || d == 8 || d == 16 || d == 32);
  if (small) {
    const int threads = 256;
    const int blocks = blocks_for(n, threads, 16);
    const size_t smem = sizeof(float) * (size_t)k * d;
    launch_assign_small(d, blocks, threads, smem, s, X, ld, n, C, k, labels, mind);
    return check_launch("assign_small_kernel");
  }
  return launch_assign_simt(X, ld, n, d, C, k, labels, mind, nullptr, nullptr, nullptr, 0, 0, s);
}

struct Staged {
  float* X = nullptr;
  float* C = nullptr;
  int32_t* labels = nullptr;
  unsigned int* maxabs = nullptr;  // [0] max |x| bits of X, [1] of C (NaN above +inf)
  int ld = 0;
};

static int stage_xc(DevBuffers& buf, const float* X, const float* C, long long n, int d, int k, bool want_labels,
                    const uint32_t* labels_in, Staged* out, cudaStream_t s) {
  out->ld = ld_of(d);
  SKM_TRY(buf.alloc_n(&out->X, (size_t)n * out->ld));
  SKM_TRY(buf.alloc_n(&out->C, (size_t)k * out->ld));
  SKM_TRY(buf.alloc_n(&out->maxabs, 2));
  SKM_TRY(upload_rows(out->X, out->ld, X, n, d, s));
  SKM_TRY(upload_rows(out->C, out->ld, C, k, d, s));
  // non-finite inputs are detected on the device (callers need not scan X on the host)
  SKM_CUDA(cudaMemsetAsync(out->maxabs, 0, 2 * sizeof(unsigned int), s));
  maxabs_kernel<<<blocks_for(n * out->ld / 4, 256, 8), 256, 0, s>>>(out->X, out->ld, n, d, out->maxabs);
  SKM_TRY(check_launch("maxabs_kernel"));
  maxabs_kernel<<<1, 256, 0, s>>>(out->C, out->ld, k, d, out->maxabs + 1);
  SKM_TRY(check_launch("maxabs_kernel"));
  if (want_labels || labels_in) {
    SKM_TRY(buf.alloc_n(&out->labels, (size_t)n));
    if (labels_in)
      SKM_CUDA(cudaMemcpyAsync(out->labels, labels_in, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s));
  }
  return OK;
}

// After the stream has been synchronised: ERR_INVALID when X or C held NaN
// or infinity (their max |x| words, copied back into mx).
// Exact column mean of n raw rows into mean (ld entries, float32): the
// fixed-point column sums of run_fit's single-GPU prologue, so that a seeding
// centres X exactly as the fit that follows does.
static int exact_mean(const float* raw, int ld, long long n, int d, float* mean, DevBuffers& buf, cudaStream_t s) {
  unsigned int* mx = nullptr;
  double* scale = nullptr;
  long long* colsum = nullptr;
  SKM_TRY(buf.alloc_n(&mx, 1));
  SKM_TRY(buf.alloc_n(&scale, 1));
  SKM_TRY(buf.alloc_n(&colsum, (size_t)ld));
  SKM_CUDA(cudaMemsetAsync(mx, 0, sizeof(unsigned int), s));
  SKM_CUDA(cudaMemsetAsync(colsum, 0, sizeof(long long) * ld, s));
  SKM_CUDA(cudaMemsetAsync(mean, 0, sizeof(float) * ld, s));
  maxabs_kernel<<<blocks_for(n * ld / 4, 256, 8), 256, 0, s>>>(raw, ld, n, d, mx);
  SKM_TRY(check_launch("maxabs_kernel"));
  scale_kernel<<<1, 32, 0, s>>>(mx, (double)n, scale);
  SKM_TRY(check_launch("scale_kernel"));
  const int q = ld / 4;
  const int threads = q <= 1024 ? q * std::max(1, 256 / q) : 1024;
  colsum_fixed_kernel<<<sm_count() * 2, threads, sizeof(long long) * ld, s>>>(raw, ld, n, d, scale, colsum);
  SKM_TRY(check_launch("colsum_fixed_kernel"));
  mean_from_colsum_kernel<<<1, 256, 0, s>>>(colsum, d, scale, (double)n, mean);
  SKM_TRY(check_launch("mean_from_colsum_kernel"));
  return OK;
}

// k-means++ seeding of device rows (raw, stride ld): host weights (nullable)
// and uniforms ((k - 1) x T) in, host centres (k x d, raw rows) and indices out.
static int plusplus_rows(const float* Xd, int ld, long long n, int d, size_t k, const float* sample_weight,
                         int64_t first_index, const double* uniforms, size_t n_local_trials, int center,
                         float* centers_out, int64_t* indices_out, cudaStream_t s) {
  SKM_TRY(validate(n, d, (long long)k));
  if ((long long)k > n || n_local_trials < 1 || n_local_trials > 16 || first_index < 0 || first_index >= n ||
      (k > 1 && uniforms == nullptr) || centers_out == nullptr || indices_out == nullptr) {
    set_error(ERR_INVALID, "kmeans_plusplus: invalid arguments (k=%zu, n=%lld, n_local_trials=%zu, first=%lld)", k, n,
              n_local_trials, (long long)first_index);
    return ERR_INVALID;
  }
  DevBuffers buf(s);
  float* mean = nullptr;
  if (center) {
    SKM_TRY(buf.alloc_n(&mean, (size_t)ld));
    SKM_TRY(exact_mean(Xd, ld, n, d, mean, buf, s));
  }
  float* w = nullptr;
  if (sample_weight) {
    SKM_TRY(buf.alloc_n(&w, (size_t)n));
    SKM_CUDA(cudaMemcpyAsync(w, sample_weight, sizeof(float) * n, cudaMemcpyHostToDevice, s));
  }
  const int T = (int)n_local_trials;
  double* u = nullptr;
  if (k > 1) {
    SKM_TRY(buf.alloc_n(&u, (k - 1) * (size_t)T));
    SKM_CUDA(cudaMemcpyAsync(u, uniforms, sizeof(double) * (k - 1) * T, cudaMemcpyHostToDevice, s));
  }
  void* scratch = nullptr;
  SKM_TRY(buf.alloc(&scratch, kmeanspp_scratch_bytes(n, T)));
  float* cen = nullptr;
  long long* idx = nullptr;
  SKM_TRY(buf.alloc_n(&cen, k * (size_t)d));
  SKM_TRY(buf.alloc_n(&idx, k));
  SKM_TRY(kmeanspp_device(Xd, ld, n, d, (int)k, mean, w, first_index, u, T, scratch, cen, idx, s));
  SKM_CUDA(cudaMemcpyAsync(centers_out, cen, sizeof(float) * k * d, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaMemcpyAsync(indices_out, idx, sizeof(long long) * k, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  return OK;
}

static int check_finite(const unsigned int* mx, const char* what) {
  if ((mx[0] & 0x7fffffffu) >= 0x7f800000u || (mx[1] & 0x7fffffffu) >= 0x7f800000u) {
    set_error(ERR_INVALID, "%s: %s contains NaN or infinity", what,
              (mx[0] & 0x7fffffffu) >= 0x7f800000u ? "X" : "the centres");
    return ERR_INVALID;
  }
  return OK;
}

static float inertia_common(const float* X, const float* centroids, const uint32_t* labels, const float* sample_weight,
                            size_t n, size_t d, size_t k) {
  if (validate((long long)n, (long long)d, (long long)k)) return -1.0f;
  cudaStream_t s;
  if (thread_stream(&s, nullptr)) return -1.0f;
  DevBuffers buf(s);
  Staged g;
  if (stage_xc(buf, X, centroids, (long long)n, (int)d, (int)k, false, labels, &g, s)) return -1.0f;
  const int n_part = sm_count() * 4;
  double* part = nullptr;
  if (buf.alloc_n(&part, (size_t)n_part + 1)) return -1.0f;
  float* w = nullptr;
  if (sample_weight) {
    if (buf.alloc_n(&w, n)) return -1.0f;
    if (cudaMemcpyAsync(w, sample_weight, sizeof(float) * n, cudaMemcpyHostToDevice, s) != cudaSuccess) return -1.0f;
  }
  inertia_partial_kernel<<<n_part, 256, 0, s>>>(g.X, g.ld, (long long)n, (int)d, g.C, g.labels, part, 0, w);
  if (check_launch("inertia_partial_kernel")) return -1.0f;
  ordered_sum_kernel<<<1, 32, 0, s>>>(part, n_part, part + n_part);
  if (check_launch("ordered_sum_kernel")) return -1.0f;
  double v = 0;
  unsigned int mx[2];
  if (cudaMemcpyAsync(mx, g.maxabs, sizeof(mx), cudaMemcpyDeviceToHost, s) != cudaSuccess) return -1.0f;
  if (cudaMemcpyAsync(&v, part + n_part, sizeof(double), cudaMemcpyDeviceToHost, s) != cudaSuccess) return -1.0f;
  if (cudaStreamSynchronize(s) != cudaSuccess) {
    set_error(ERR_CUDA, "kmeans_inertia: %s", cudaGetErrorString(cudaGetLastError()));
    return -1.0f;
  }
  if (check_finite(mx, "kmeans_inertia")) return -1.0f;
  return (float)v;
}

}  // namespace skm

using namespace skm;

extern "C" {

int skmetal_kmeans_assign(const float* X, const float* centroids, uint32_t* labels, size_t n, size_t d, size_t k) {
  SKM_TRY(check_injected("kmeans_assign"));
  SKM_TRY(validate((long long)n, (long long)d, (long long)k));
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  DevBuffers buf(s);
  Staged g;
  SKM_TRY(stage_xc(buf, X, centroids, (long long)n, (int)d, (int)k, true, nullptr, &g, s));
  bool done = false;
  SKM_TRY(launch_assign_const(g.X, g.ld, (long long)n, (int)d, centroids, g.C, g.ld, (int)k, g.labels, s, &done));
  if (!done) SKM_TRY(launch_assign_any(g.X, g.ld, (long long)n, (int)d, g.C, (int)k, g.labels, nullptr, s));
  unsigned int mx[2];
  SKM_CUDA(cudaMemcpyAsync(mx, g.maxabs, sizeof(mx), cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaMemcpyAsync(labels, g.labels, sizeof(uint32_t) * n, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  return check_finite(mx, "kmeans_assign");
}

int skmetal_compute_mindists(const float* X, const float* centroids, const uint32_t* labels, float* dists, size_t n,
                             size_t d, size_t k) {
  SKM_TRY(check_injected("compute_mindists"));
  SKM_TRY(validate((long long)n, (long long)d, (long long)k));
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  DevBuffers buf(s);
  Staged g;
  SKM_TRY(stage_xc(buf, X, centroids, (long long)n, (int)d, (int)k, false, labels, &g, s));
  float* out = nullptr;
  SKM_TRY(buf.alloc_n(&out, n));
  mindist_kernel<<<blocks_for((long long)n, 256), 256, 0, s>>>(g.X, g.ld, (long long)n, (int)d, g.C, g.labels, out);
  SKM_TRY(check_launch("mindist_kernel"));
  unsigned int mx[2];
  SKM_CUDA(cudaMemcpyAsync(mx, g.maxabs, sizeof(mx), cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaMemcpyAsync(dists, out, sizeof(float) * n, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  return check_finite(mx, "compute_mindists");
}

float skmetal_kmeans_inertia(const float* X, const float* centroids, const uint32_t* labels, size_t n, size_t d,
                             size_t k) {
  if (check_injected("kmeans_inertia")) return -1.0f;
  return inertia_common(X, centroids, labels, nullptr, n, d, k);
}

float skmetal_kmeans_inertia_weighted(const float* X, const float* centroids, const uint32_t* labels,
                                      const float* sample_weight, size_t n, size_t d, size_t k) {
  if (check_injected("kmeans_inertia_weighted")) return -1.0f;
  return inertia_common(X, centroids, labels, sample_weight, n, d, k);
}

int skmetal_row_norm_sq(const float* X, float* norms, size_t n, size_t d) {
  SKM_TRY(check_injected("row_norm_sq"));
  SKM_TRY(validate((long long)n, (long long)d, 1));
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  DevBuffers buf(s);
  const int ld = ld_of((int)d);
  float *Xd = nullptr, *zero = nullptr, *out = nullptr;
  int32_t* lab = nullptr;
  SKM_TRY(buf.alloc_n(&Xd, n * ld));
  SKM_TRY(buf.alloc_n(&zero, (size_t)ld));
  SKM_TRY(buf.alloc_n(&out, n));
  SKM_TRY(buf.alloc_n(&lab, n));
  SKM_TRY(upload_rows(Xd, ld, X, (long long)n, (int)d, s));
  SKM_CUDA(cudaMemsetAsync(zero, 0, sizeof(float) * ld, s));
  SKM_CUDA(cudaMemsetAsync(lab, 0, sizeof(int32_t) * n, s));
  mindist_kernel<<<blocks_for((long long)n, 256), 256, 0, s>>>(Xd, ld, (long long)n, (int)d, zero, lab, out);
  SKM_TRY(check_launch("mindist_kernel"));
  SKM_CUDA(cudaMemcpyAsync(norms, out, sizeof(float) * n, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  return OK;
}

int skmetal_kmeans_transform(const float* X, const float* centroids, float* D, size_t n, size_t d, size_t k) {
  SKM_TRY(check_injected("kmeans_transform"));
  SKM_TRY(validate((long long)n, (long long)d, (long long)k));
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  DevBuffers buf(s);
  Staged g;
  SKM_TRY(stage_xc(buf, X, centroids, (long long)n, (int)d, (int)k, false, nullptr, &g, s));
  float* out = nullptr;
  SKM_TRY(buf.alloc_n(&out, n * k));
  transform_kernel<<<blocks_for((long long)n * k, 256), 256, 0, s>>>(g.X, g.ld, (long long)n, (int)d, g.C, (int)k,
                                                                   out);
  SKM_TRY(check_launch("transform_kernel"));
  unsigned int mx[2];
  SKM_CUDA(cudaMemcpyAsync(mx, g.maxabs, sizeof(mx), cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaMemcpyAsync(D, out, sizeof(float) * n * k, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  return check_finite(mx, "kmeans_transform");
}

int skmetal_kmeans_batch_fused(const float* X, float* centroids, uint32_t* labels, size_t n, size_t d, size_t k,
                               size_t num_groups, size_t max_iter, float tol, int32_t* n_iter_out) {
  (void)num_groups;
  FitParams p;
  p.X_host = X;
  p.n = (long long)n;
  p.d = (int)d;
  p.k = (int)k;
  p.init_host = centroids;
  p.max_iter = (int)std::min<size_t>(max_iter, 1 << 30);
  p.tol = tol;
  p.tol_abs = true;
  p.center = false;
  p.centers_out = centroids;
  p.labels_out_u32 = labels;
  p.n_iter_out = n_iter_out;
  return run_fit(p);
}

int skmetal_kmeans_fit(const float* X, size_t n, size_t d, size_t k, const float* init, int32_t max_iter, double tol,
                       uint32_t flags, float* centers_out, int32_t* labels_out, double* inertia_out,
                       int32_t* n_iter_out) {
  return skmetal_kmeans_fit_weighted(X, n, d, k, init, max_iter, tol, flags, nullptr, centers_out, labels_out,
                                     inertia_out, n_iter_out);
}

int skmetal_kmeans_fit_weighted(const float* X, size_t n, size_t d, size_t k, const float* init, int32_t max_iter,
                                double tol, uint32_t flags, const float* sample_weight, float* centers_out,
                                int32_t* labels_out, double* inertia_out, int32_t* n_iter_out) {
  if (flags & SKMETAL_FIT_DISTRIBUTED) {
    set_error(ERR_INVALID, "use skmetal_kmeans_fit_shard for distributed fits");
    return ERR_INVALID;
  }
  FitParams p;
  p.X_host = X;
  p.n = (long long)n;
  p.d = (int)d;
  p.k = (int)k;
  p.init_host = init;
  p.w_host = sample_weight;
  p.max_iter = max_iter;
  p.tol = tol;
  p.tol_abs = (flags & SKMETAL_FIT_TOL_ABS) != 0;
  p.center = (flags & SKMETAL_FIT_CENTER) != 0;
  p.simt = (flags & SKMETAL_FIT_SIMT) != 0;
  p.profile = (flags & SKMETAL_FIT_PROFILE) != 0;
  p.bulk_sums = (flags & SKMETAL_FIT_BULK_SUMS) != 0;
  p.centers_out = centers_out;
  p.labels_out = labels_out;
  p.inertia_out = inertia_out;
  p.n_iter_out = n_iter_out;
  return run_fit(p);
}

int skmetal_kmeans_fit_shard(const float* X, size_t n, size_t d, size_t k, const float* init, int32_t max_iter,
                             double tol, uint32_t flags, uint64_t row_base, uint64_t n_total, float* centers_out,
                             int32_t* labels_out, double* inertia_out, int32_t* n_iter_out) {
  FitParams p;
  p.X_host = X;
  p.n = (long long)n;
  p.d = (int)d;
  p.k = (int)k;
  p.init_host = init;
  p.max_iter = max_iter;
  p.tol = tol;
  p.tol_abs = (flags & SKMETAL_FIT_TOL_ABS) != 0;
  p.center = (flags & SKMETAL_FIT_CENTER) != 0;
  p.simt = (flags & SKMETAL_FIT_SIMT) != 0;
  p.profile = (flags & SKMETAL_FIT_PROFILE) != 0;
  p.bulk_sums = (flags & SKMETAL_FIT_BULK_SUMS) != 0;
  p.distributed = true;
  p.row_base = (long long)row_base;
  p.n_total = (long long)n_total;
  p.centers_out = centers_out;
  p.labels_out = labels_out;
  p.inertia_out = inertia_out;
  p.n_iter_out = n_iter_out;
  return run_fit(p);
}

int skmetal_kmeans_lloyd_iter(const float* X, const float* centers_old, float* centers_new, int32_t* labels_out,
                              float* weight_out, float* center_shift_out, size_t n, size_t d, size_t k) {
  SKM_TRY(check_injected("lloyd_iter"));
  SKM_TRY(validate((long long)n, (long long)d, (long long)k));
  // one Lloyd iteration = the fit engine with max_iter = 1, no centring, whose
  // M-step results are read back instead of running the final E-step
  FitParams p;
  p.X_host = X;
  p.n = (long long)n;
  p.d = (int)d;
  p.k = (int)k;
  p.init_host = centers_old;
  p.max_iter = 1;
  p.tol = 0.0;
  p.tol_abs = true;
  p.center = false;
  p.single_step = true;
  p.centers_out = centers_new;
  p.labels_out = labels_out;
  p.weight_out = weight_out;
  p.shift_out = center_shift_out;
  return run_fit(p);
}

int skmetal_dataset_create(const float* X, size_t n, size_t d, void** handle) {
  SKM_TRY(check_injected("dataset_create"));
  SKM_TRY(validate((long long)n, (long long)d, 1));
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  Dataset* ds = new Dataset();
  ds->n = (long long)n;
  ds->d = (int)d;
  ds->ld = ld_of((int)d);
  current_device(&ds->device);
  cudaError_t e = cudaMalloc(&ds->X, sizeof(float) * n * ds->ld);
  if (e != cudaSuccess) {
    delete ds;
    set_error(e == cudaErrorMemoryAllocation ? ERR_OOM : ERR_CUDA, "dataset allocation: %s", cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? ERR_OOM : ERR_CUDA;
  }
  int rc = upload_rows(ds->X, ds->ld, X, (long long)n, (int)d, s);
  if (rc == OK && cudaStreamSynchronize(s) != cudaSuccess) rc = ERR_CUDA;
  if (rc != OK) {
    cudaFree(ds->X);
    delete ds;
    return rc;
  }
  *handle = ds;
  return OK;
}

int skmetal_dataset_free(void* handle) {
  Dataset* ds = static_cast<Dataset*>(handle);
  if (!ds) return OK;
  cudaFree(ds->X);
  delete ds;
  return OK;
}

static int fit_dataset_common(void* handle, const float* init, size_t k, int32_t max_iter, double tol, uint32_t flags,
                              bool distributed, uint64_t row_base, uint64_t n_total, float* centers_out,
                              int32_t* labels_out, double* inertia_out, int32_t* n_iter_out,
                              const float* sample_weight = nullptr) {
  Dataset* ds = static_cast<Dataset*>(handle);
  if (!ds) {
    set_error(ERR_INVALID, "null dataset handle");
    return ERR_INVALID;
  }
  FitParams p;
  p.X_dev = ds->X;
  p.n = ds->n;
  p.d = ds->d;
  p.k = (int)k;
  p.init_host = init;
  p.w_host = sample_weight;
  p.max_iter = max_iter;
  p.tol = tol;
  p.tol_abs = (flags & SKMETAL_FIT_TOL_ABS) != 0;
  p.center = (flags & SKMETAL_FIT_CENTER) != 0;
  p.simt = (flags & SKMETAL_FIT_SIMT) != 0;
  p.profile = (flags & SKMETAL_FIT_PROFILE) != 0;
  p.bulk_sums = (flags & SKMETAL_FIT_BULK_SUMS) != 0;
  p.distributed = distributed;
  p.row_base = (long long)row_base;
  p.n_total = (long long)n_total;
  p.centers_out = centers_out;
  p.labels_out = labels_out;
  p.inertia_out = inertia_out;
  p.n_iter_out = n_iter_out;
  return run_fit(p);
}

int skmetal_kmeans_fit_dataset(void* handle, const float* init, size_t k, int32_t max_iter, double tol,
                               uint32_t flags, float* centers_out, int32_t* labels_out, double* inertia_out,
                               int32_t* n_iter_out) {
  return fit_dataset_common(handle, init, k, max_iter, tol, flags, false, 0, 0, centers_out, labels_out, inertia_out,
                            n_iter_out);
}

int skmetal_dataset_fit_weighted(void* handle, const float* init, size_t k, int32_t max_iter, double tol,
                                 uint32_t flags, const float* sample_weight, float* centers_out, int32_t* labels_out,
                                 double* inertia_out, int32_t* n_iter_out) {
  return fit_dataset_common(handle, init, k, max_iter, tol, flags, false, 0, 0, centers_out, labels_out, inertia_out,
                            n_iter_out, sample_weight);
}

int skmetal_dataset_fit_shard(void* handle, const float* init, size_t k, int32_t max_iter, double tol,
                              uint32_t flags, uint64_t row_base, uint64_t n_total, float* centers_out,
                              int32_t* labels_out, double* inertia_out, int32_t* n_iter_out) {
  return fit_dataset_common(handle, init, k, max_iter, tol, flags, true, row_base, n_total, centers_out, labels_out,
                            inertia_out, n_iter_out);
}

int skmetal_kmeans_predict_dataset(void* handle, const float* centroids, size_t k, int32_t* labels_out) {
  SKM_TRY(check_injected("predict_dataset"));
  Dataset* ds = static_cast<Dataset*>(handle);
  if (!ds) {
    set_error(ERR_INVALID, "null dataset handle");
    return ERR_INVALID;
  }
  SKM_TRY(validate(ds->n, ds->d, (long long)k));
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  const unsigned long long l0 = g_launches.load();
  cudaEvent_t e0, e1;
  SKM_CUDA(cudaEventCreate(&e0));
  SKM_CUDA(cudaEventCreate(&e1));
  DevBuffers buf(s);
  float* C = nullptr;
  int32_t* lab = nullptr;
  SKM_TRY(buf.alloc_n(&C, k * ds->ld));
  SKM_TRY(buf.alloc_n(&lab, (size_t)ds->n));
  SKM_TRY(upload_rows(C, ds->ld, centroids, (long long)k, ds->d, s));
  SKM_CUDA(cudaEventRecord(e0, s));
  bool done = false;
  SKM_TRY(launch_assign_const(ds->X, ds->ld, ds->n, ds->d, centroids, C, ds->ld, (int)k, lab, s, &done));
  if (!done) SKM_TRY(launch_assign_any(ds->X, ds->ld, ds->n, ds->d, C, (int)k, lab, nullptr, s));
  SKM_CUDA(cudaEventRecord(e1, s));
  if (labels_out) SKM_CUDA(cudaMemcpyAsync(labels_out, lab, sizeof(int32_t) * ds->n, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  FitStats fs;
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  fs.ms_total = fs.ms_loop = ms;
  fs.estep_launches = 1;
  fs.estep_ms_sum = ms;
  fs.launches = g_launches.load() - l0;
  t_stats = fs;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return OK;
}

int skmetal_kmeans_plusplus(const float* X, size_t n, size_t d, size_t k, const float* sample_weight,
                            int64_t first_index, const double* uniforms, size_t n_local_trials, int center,
                            float* centers_out, int64_t* indices_out) {
  SKM_TRY(check_injected("kmeans_plusplus"));
  SKM_TRY(validate((long long)n, (long long)d, (long long)k));
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  DevBuffers buf(s);
  const int ld = ld_of((int)d);
  float* Xd = nullptr;
  SKM_TRY(buf.alloc_n(&Xd, n * (size_t)ld));
  SKM_TRY(upload_rows(Xd, ld, X, (long long)n, (int)d, s));
  return plusplus_rows(Xd, ld, (long long)n, (int)d, k, sample_weight, first_index, uniforms, n_local_trials, center,
                       centers_out, indices_out, s);
}

int skmetal_dataset_kmeans_plusplus(void* handle, size_t k, const float* sample_weight, int64_t first_index,
                                    const double* uniforms, size_t n_local_trials, int center, float* centers_out,
                                    int64_t* indices_out) {
  SKM_TRY(check_injected("dataset_kmeans_plusplus"));
  Dataset* ds = static_cast<Dataset*>(handle);
  if (!ds) {
    set_error(ERR_INVALID, "dataset_kmeans_plusplus: null dataset");
    return ERR_INVALID;
  }
  cudaStream_t s;
  SKM_TRY(thread_stream(&s, nullptr));
  return plusplus_rows(ds->X, ds->ld, ds->n, ds->d, k, sample_weight, first_index, uniforms, n_local_trials, center,
                       centers_out, indices_out, s);
}

int skmetal_debug_loop_stamps(uint64_t* out, int cap) {
  const int n = (int)std::min((size_t)std::max(cap, 0), t_loop_stamps.size());
  for (int i = 0; i < n; ++i) out[i] = t_loop_stamps[i];
  return (int)t_loop_stamps.size();
}

int skmetal_last_fit_distinct(void) { return t_stats.distinct; }

int skmetal_last_fit_stats(double* ms_total, double* ms_prep, double* ms_loop, double* ms_final,
                           int32_t* estep_launches, double* estep_ms_sum, uint64_t* launches, int32_t* iterations) {
  const FitStats& f = t_stats;
  if (ms_total) *ms_total = f.ms_total;
  if (ms_prep) *ms_prep = f.ms_prep;
  if (ms_loop) *ms_loop = f.ms_loop;
  if (ms_final) *ms_final = f.ms_final;
  if (estep_launches) *estep_launches = f.estep_launches;
  if (estep_ms_sum) *estep_ms_sum = f.estep_ms_sum;
  if (launches) *launches = f.launches;
  if (iterations) *iterations = f.iterations;
  return OK;
}

}  // extern "C"
