// Persistent Lloyd loop (single GPU, tensor-core E-step): one cooperative
// launch runs every iteration of a fit, E-step and M-step alike, separated by
// grid barriers instead of kernel boundaries.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "estep_tc.h"
#include "kernels.cuh"

namespace skm {

// Multi-GPU loop (one rank per GPU, rows sharded): each rank's peer region
// (mapped into every rank) holds, at these byte offsets,
//   [0, 256)              one arrival word per rank (rank_barrier)
//   region_inbox_off      inbox rows: 2 parities x W ranks x k clusters x
//                         2 (ld + 4) words: the sender's deltas of the
//                         cluster, its count delta and (cluster 0) its change
//                         count, each int64 as two 8-byte words {32 bits of
//                         the value, the iteration's epoch}
//   region_cand_off       the rank's relocation-candidate block
//                         (cand_block_bytes(kCandCap, ld) bytes)
constexpr int kLoopMaxRanks = 8;
constexpr size_t kRegionFlags = 256;
inline size_t region_row(int ld) { return 2 * ((size_t)ld + 4); }  // 8-byte words per inbox row
inline size_t region_inbox_off(int, int) { return kRegionFlags; }
inline size_t region_cand_off(int W, int k, int ld) {
  return region_inbox_off(W, k) + 2 * (size_t)W * k * region_row(ld) * sizeof(long long);
}
inline size_t region_bytes(int W, int k, int ld) { return region_cand_off(W, k, ld) + cand_block_bytes(kCandCap, ld); }

struct LoopInputs {
  const uint16_t* img;       // centre image of the start centres (B operand)
  const int* sexp;           // {xexp, cexp} in the fit state
  float* bias;               // ||c||^2 of the start centres (k floats); kept current by the loop
  long long* D[3];           // delta buffers, rotated by iteration mod 3: dS (k x ld) | dcount (k) | changed; zero
  long long* S[2];           // fixed-point sums by iteration parity (S[0] = those of the start labels)
  long long* counts[2];      // cluster counts by iteration parity (counts[0] = those of the start labels)
  float* C[2];               // centres by iteration parity: iteration t reads C[t & 1], writes C[(t + 1) & 1]
  MStepArgs m;               // the M-step's state and scratch (D, S, counts, changed, C_old, C_new unused)
  double* part;              // 3 k doubles of per-cluster results of the owners
  unsigned int* bar;         // grid-barrier counter of the loop, zero at launch
  unsigned long long* prof;  // nullable: 4 * max_iter + 1 globaltimer stamps (see lloyd_loop_kernel)
  // multi-GPU (nranks > 1): every rank's peer region (own at [rank]), and
  // local scratch for the global deltas (k * ld + k + 1) and the gathered
  // candidate blocks
  int nranks = 1, rank = 0;
  unsigned char* region[kLoopMaxRanks] = {};
  long long* G = nullptr;
  unsigned char* cand_all = nullptr;
  // limit of every wait on another rank, in ns (0: 5 s); a rank that stops
  // leaves its peers to run out of it and report error 1005
  unsigned long long peer_wait_ns = 0;
};

// True when the plan's shared memory leaves room for the loop kernel's own.
bool tc_loop_supported(const TcPlan& plan);

// Static shared memory of the loop kernel (0 if it cannot be queried); plans
// keep this much of a CTA's shared memory free.
size_t tc_loop_static_smem();

// Launches the loop (cooperative, plan.grid CTAs); runs until the fit state
// says done. Errors of the device side are left in the fit state.
int tc_lloyd_loop(const TcPlan& plan, const LoopInputs& in, cudaStream_t s);

}  // namespace skm
