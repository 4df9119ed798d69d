// Tensor-core (tcgen05, sm_100a) E-step: bulk-copied X tiles, 3xTF32 distance
// tiles accumulated in tensor memory, running argmin in registers, incremental
// fixed-point deltas for rows that change label.
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
  int k_pad = 0;       // clusters padded to the MMA N granularity (16)
  int k_steps = 0;     // K = ld in chunks of 8 columns
  int stages = 0;      // X stages in shared memory
  int nbl = 0;         // x_lo buffers in tensor memory
  int nba = 0;         // accumulator buffers in tensor memory
  int xcols = 0;       // tensor-memory columns per x_lo buffer
  int tmem_cols = 0;   // tensor-memory allocation
  int round_mode = 0;  // tensor-core fp32->tf32 conversion (probe result)
  int grid = 0;
  size_t smem = 0;
  CUtensorMap tmap_chi;
  CUtensorMap tmap_clo;
};

// Runs (once per device) a tiny kernel that checks the tcgen05.cp layout and
// measures the tensor core's fp32 -> tf32 conversion: *mode = 0 truncation,
// 1 round-to-nearest-even, -1 neither (the tensor-core path is then unused).
// With raw3072 non-null the probe reruns and returns its raw output.
int tc_probe(int* mode, uint32_t* raw3072);

// X: the fit's blocked working copy (xblk_index), round_up(n, 128) rows.
int tc_plan(const float* X, int ld, long long n, int d, int k, TcPlan* plan);

// Chi / Clo: tf32 split of the centres (k x ld), fixed for the plan's lifetime
// (the buffers are rewritten in place between launches).
int tc_set_centres(TcPlan* plan, const float* Chi, const float* Clo);

// bias: ||c||^2 (k floats). `changed` (nullable) counts rows whose label
// differs from labels[] on entry; `D` (nullable, needs `st`) receives the
// fixed-point deltas of those rows; `st` (nullable) makes the launch a no-op
// once st->done is set; `err` receives a nonzero code if a pipeline wait
// times out.
int tc_estep(const TcPlan& plan, const float* bias, int32_t* labels, unsigned long long* changed, long long* D,
             const FitState* st, int* err, cudaStream_t s);

}  // namespace skm
