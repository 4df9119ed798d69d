// Tensor-core (tcgen05, sm_100a) E-step: TMA-fed X tiles, 3xTF32 distance
// tiles accumulated in tensor memory, running argmin in registers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "skm.cuh"

namespace skm {

struct TcPlan {
  bool supported = false;
  const float* X = nullptr;
  int ld = 0;
  long long n = 0;
  int d = 0;
  int k = 0;
  int k_pad = 0;      // clusters padded to the MMA N granularity
  int k_steps = 0;    // K = d padded to multiples of 8 (tf32 MMA K)
  int grid = 0;
  size_t smem = 0;
  CUtensorMap tmap_x;  // X tiles
};

int tc_plan(const float* X, int ld, long long n, int d, int k, TcPlan* plan);
// Chi / Clo: tf32 split of the centres (k x ld); bias: ||c||^2 (k floats).
// `changed` (nullable) counts rows whose label differs from labels[] on entry;
// `D` (nullable, needs `st`) receives the fixed-point deltas of those rows;
// `st` (nullable) makes the launch a no-op once st->done is set; `err`
// receives a nonzero code if a pipeline wait times out.
int tc_estep(const TcPlan& plan, const float* Chi, const float* Clo, const float* bias, int32_t* labels, float* mind,
             unsigned long long* changed, long long* D, const FitState* st, int* err, cudaStream_t s);

}  // namespace skm
