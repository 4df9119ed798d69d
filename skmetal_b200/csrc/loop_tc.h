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
//   [0, 64)                 one arrival word per rank, written by that rank
//   [kRegionD, + 3 d_stride int64)   the rank's delta buffers D[0..2]
//   region_cand_off(..)     the rank's relocation-candidate block
//                           (cand_block_bytes(kCandCap, ld) bytes)
constexpr int kLoopMaxRanks = 8;
constexpr size_t kRegionD = 256;
inline size_t region_cand_off(size_t d_stride) { return kRegionD + 3 * d_stride * sizeof(long long); }
inline size_t region_bytes(size_t d_stride, int ld) { return region_cand_off(d_stride) + cand_block_bytes(kCandCap, ld); }

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
  // multi-GPU (nranks > 1): every rank's peer region (own at [rank]; the
  // delta buffers are then this rank's region buffers, D above is ignored),
  // d_stride, and local scratch for the global deltas (k * ld + k + 1) and
  // the gathered candidate blocks
  int nranks = 1, rank = 0;
  unsigned char* region[kLoopMaxRanks] = {};
  size_t d_stride = 0;
  long long* G = nullptr;
  unsigned char* cand_all = nullptr;
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
