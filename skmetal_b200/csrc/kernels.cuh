// Kernel declarations shared by the host driver and the kernel files.
#pragma once

#include "device_util.cuh"
#include "skm.cuh"

#include <algorithm>

namespace skm {

constexpr int kAssignSmemFloats = 12288;  // 48 KB of centres per chunk
constexpr size_t kBulkSmemBytes = 160 * 1024;  // bulk pass accumulates privately when (k*ld + k) int64 fit

// The atomic bulk pass's private accumulator: (k*ld + k) int64 when they fit
// in `avail` bytes of shared memory, else 0 (sums go straight to global
// memory).
__host__ __device__ inline size_t bulk_acc_bytes(int k, int ld, size_t avail) {
  const size_t b = sizeof(long long) * ((size_t)k * ld + k);
  return b <= avail ? b : 0;
}

// The tiled bulk pass (bulk_pass_tiles) stages tiles of 128 rows of the
// blocked X in shared memory with bulk copies, one per 2 KB column-quad block
// at a stride of 2064 bytes (so that lanes reading consecutive quads of one
// row hit distinct banks), two tiles in flight. Layout: 2 x [nq quad blocks |
// 128 labels (int32) | 128 weights (float32, copied for weighted fits)], 2
// mbarriers, then two mask sets. Usable when each thread owns at most 2
// (cluster, column quad) pairs and ld <= 128; the labels buffer (and the
// weights of a weighted fit) must hold round_up(n, 128) entries (labels -1
// past n).
constexpr int kBulkTileRows = 128;
constexpr int kBulkMaxPairsPerThread = 2;
constexpr int kBulkQuadStride = 2064;  // bytes between quad blocks of a staged tile
__host__ __device__ inline size_t bulk_tile_bytes(int ld) {
  return (size_t)(ld / 4) * kBulkQuadStride + 8 * kBulkTileRows;  // quads, then labels, then weights
}
__host__ __device__ inline size_t bulk_tiles_bytes(int k, int ld) {
  return 2 * bulk_tile_bytes(ld) + 16 + 4 * 8 * (size_t)k;  // tiles, barriers, two mask sets
}
__host__ __device__ inline bool bulk_tiles_ok(int k, int ld, int threads, size_t avail) {
  const long long pairs = (long long)k * (ld / 4);
  return ld <= 128 && threads >= 32 * (kBulkTileRows / 32 + 1) && pairs <= (long long)kBulkMaxPairsPerThread * threads &&
         bulk_tiles_bytes(k, ld) <= avail;
}

// Relocation candidates of one rank (multi-GPU fits), one slot per rank after
// D in the all-reduced payload: [count int32, 3 x int32 padding | dist
// float[cap] | global row int64[cap] | label int32[cap] | x float[cap][ld]].
// count = min(clusters this rank has empty, cap).
constexpr int kCandCap = 16;
__host__ __device__ inline size_t cand_block_bytes(int cap, int ld) {
  return (16 + (size_t)cap * 16 + (size_t)cap * ld * 4 + 15) & ~(size_t)15;
}
__host__ __device__ inline size_t cand_dist_off(int) { return 16; }
__host__ __device__ inline size_t cand_row_off(int cap) { return 16 + (size_t)cap * 4; }
__host__ __device__ inline size_t cand_label_off(int cap) { return 16 + (size_t)cap * 12; }
__host__ __device__ inline size_t cand_x_off(int cap) { return 16 + (size_t)cap * 16; }

// Above n / 10 changed rows in an iteration, per-row deltas (about 2 d
// contended reductions per row) cost more than rebuilding the sums from all
// rows, so the next iteration is a bulk one. When the bulk pass itself adds
// every element to global memory (the k x ld sums fit neither the tiled pass
// nor a shared accumulator), a delta costs two global reductions per element
// of a changed row against one per element of every row, so deltas stay
// cheaper up to n / 4 changed rows.
constexpr int kBulkDivisor = 10;
constexpr int kBulkDivisorGlobal = 4;

// Dynamic shared memory of mstep_kernel for k clusters of ld columns.
__host__ __device__ inline size_t mstep_smem_bytes(int k, int ld) {
  return bulk_tiles_ok(k, ld, 1024, kBulkSmemBytes) ? bulk_tiles_bytes(k, ld) : bulk_acc_bytes(k, ld, kBulkSmemBytes);
}


// k-means++ seeding (kmeanspp.cu)
size_t kmeanspp_scratch_bytes(long long n, int T);
int kmeanspp_device(const float* X, int ld, long long n, int d, int k, const float* mean, const float* w,
                    long long first, const double* u, int T, void* scratch, float* centers, long long* indices,
                    cudaStream_t s);

struct MStepArgs {
  FitState* st;
  const float* X;       // blocked layout (xblk_index)
  int ld;
  int d;
  long long n;          // local rows
  long long row_base;   // global index of local row 0
  const int32_t* labels;
  const float* mind;    // per-row distance to the assigned centre
  const long long* S;   // k x ld fixed-point sums of the current labels (global over ranks)
  const long long* counts;
  long long* D;         // deltas of this iteration: dS (k x ld) | dcount (k) | changed
  const unsigned long long* changed;  // = D + k*ld + k
  int k;
  const float* C_old;
  float* C_new;
  // scratch
  int* empty_ids;       // kMaxEmptyCap
  unsigned int* hist;   // 512
  long long* sel;       // kMaxEmptyCap
  long long* cnt_adj;   // k
  int* reloc_label;     // kMaxEmptyCap
  float* reloc_dist;    // kMaxEmptyCap
  float* reloc_w;       // kMaxEmptyCap: weights of the relocated rows
  float* reloc_x;       // min(k, kMaxEmptyCap) x ld
  double* shift_partial;  // max(k, gridDim.x) entries
  float* shift_out;       // per-centre shift (nullable)
  // operands of the next tensor-core E-step: the fp16 split image of C_new
  // (img nullable) and ||C_new||^2 (nullable)
  CentreImage cimg;
  float* bias;
  // mapped pinned host word (nullable): receives the iteration count once
  // the loop has converged (0 while it runs), so that the host can poll the
  // loop without a copy in the stream
  volatile int* host_done;
  // bulk iterations: the sums were already added into D before the M-step
  // (multi-GPU: before the all-reduce), so the M-step only replaces S by D
  int bulk_external;
  // relocation candidates gathered from every rank (multi-GPU); null on one
  // GPU: cand_ranks blocks of cand_block_bytes(cand_cap, ld) bytes each
  const unsigned char* cand;
  int cand_ranks;
  int cand_cap;
};

__global__ void maxabs_kernel(const float* X, int ld, long long n, int d, unsigned int* out_bits);
__global__ void colsum_fixed_kernel(const float* X, int ld, long long n, int d, const double* scale, long long* colsum);
__global__ void mean_from_colsum_kernel(const long long* colsum, int d, const double* scale, double n_total, float* mean);
__global__ void scale_kernel(const unsigned int* maxabs_bits, double n_total, double* out);
__global__ void init_state_kernel(FitState* st, int max_iter, double tol, int tol_mode, const double* sumsq,
                                  double n_total, int d, const unsigned int* maxabs_bits, int bulk_always,
                                  const float* w, const unsigned int* wmax_bits, int bulk_divisor);

// kBulkDivisorGlobal when the bulk pass of k clusters of ld columns (in the
// M-step kernel's shared memory) adds straight to global memory, else
// kBulkDivisor.
inline int bulk_divisor(int k, int ld) {
  return (bulk_tiles_ok(k, ld, 1024, kBulkSmemBytes) || bulk_acc_bytes(k, ld, kBulkSmemBytes)) ? kBulkDivisor
                                                                                              : kBulkDivisorGlobal;
}
__global__ void weight_max_kernel(const float* X, int ld, long long n, const float* w, unsigned int* out);
__global__ void center_kernel(float* X, int ld, long long n, int d, const float* mean, unsigned int* maxabs_bits,
                              double* partial);
__global__ void sumsq_partial_kernel(const float* X, int ld, long long n, int d, double* partial);
__global__ void center_block_kernel(const float* raw, int ld, long long n, int d, const float* mean, float* out,
                                    unsigned int* maxabs_bits, double* partial);
__global__ void center_init_kernel(const float* init, int d, int k, const float* mean, float* C, int ld);
__global__ void assign_simt_kernel(const float* X, int ld, long long n, int d, const float* C, int k,
                                   int32_t* labels, float* mind, const FitState* st, unsigned long long* changed,
                                   long long* D, int skip_if_strict, int blocked);
__global__ void counts_to_float_kernel(const long long* c, int k, float* out);
// Small-d assignment (d in {4, 8, 16, 32}, all centres in shared memory);
// returns false when d has no specialisation.
bool launch_assign_small(int d, int blocks, int threads, size_t smem, cudaStream_t s, const float* X, int ld,
                         long long n, const float* C, int k, int32_t* labels, float* mind);

// Small-d, small-k assignment with the centres in the kernel's parameter
// block (predict.cu): d in {4, 8, 16}, k <= 32 (16 for d = 16), ld == d.
// C_host: the k x d centres on the host; C_dev: the same on the device (k x
// ldc). *used = false when the shape has no specialisation (nothing launched).
int launch_assign_const(const float* X, int ld, long long n, int d, const float* C_host, const float* C_dev, int ldc,
                        int k, int32_t* labels, cudaStream_t s, bool* used);

__global__ void __launch_bounds__(1024, 1) mstep_kernel(MStepArgs a);
// Multi-GPU, before the all-reduce (cooperative): bulk pass, the rank's
// local counts and its relocation-candidate slot (see kernels.cu).
__global__ void __launch_bounds__(1024, 1) shard_prep_kernel(MStepArgs a, long long* local_counts, int rank);
__global__ void centre_prep_kernel(const float* C, int k, int ld, int d, float* bias, CentreImage ci, FitState* st);
__global__ void inertia_partial_kernel(const float* X, int ld, long long n, int d, const float* C,
                                       const int32_t* labels, double* partial, int blocked, const float* w);
__global__ void ordered_sum_kernel(const double* partial, int m, double* out);
// Bit c of bitmap (k <= kLabelBitmapMaxK) is set when some label equals c.
constexpr int kLabelBitmapMaxK = 4096;
__global__ void label_bitmap_kernel(const int32_t* labels, long long n, int k, unsigned int* bitmap);
__global__ void mindist_kernel(const float* X, int ld, long long n, int d, const float* C, const int32_t* labels,
                               float* out);
__global__ void transform_kernel(const float* X, int ld, long long n, int d, const float* C, int k, float* D);
__global__ void add_mean_kernel(const float* C, int k, int ld, int d, const float* mean, float* out);

}  // namespace skm
