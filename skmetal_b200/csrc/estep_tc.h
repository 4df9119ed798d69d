// Tensor-core (tcgen05, sm_100a) E-step: tiles of a split-fp16 working copy
// of X bulk-copied into shared memory, distance tiles accumulated in tensor
// memory, running argmin in registers, incremental fixed-point deltas for rows
// that change label.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "device_util.cuh"
#include "skm.cuh"

namespace skm {

struct TcPlan {
  bool supported = false;
  const float* X = nullptr;
  int ld = 0;
  long long n = 0;
  int d = 0;
  int k = 0;
  int k_pad = 0;     // clusters padded to the MMA N granularity (16)
  int k_steps = 0;   // K = ld in chunks of 8 columns
  int stacked = 0;   // centre image layout (CentreImage)
  int half_last = 0; // stacked, ld = 4 mod 8: the last chunk is a half chunk (2 KB)
  int stages = 0;    // X stages in shared memory
  int nacc = 0;      // accumulators in tensor memory
  int acc_cols = 0;  // tensor-memory columns per accumulator
  int tmem_cols = 0; // tensor-memory allocation
  const unsigned char* Xs = nullptr;  // split working copy (tc_split_x)
  uint32_t stage_bytes = 0;
  uint32_t img_bytes = 0;
  int grid = 0;
  size_t smem = 0;
  // k > 256 (estep_wide.cu): the clusters in nblk blocks of nbs, centre units
  // of unit_bytes streamed through `ring` shared-memory stages
  int wide = 0;
  int nblk = 0;
  int nbs = 0;
  int ring = 0;
  uint32_t unit_bytes = 0;
};

// Runs (once per device) a tiny kernel that pushes exactly representable
// operands through the fit's split, centre-image and MMA code and compares
// the products with their exact values: *mode = 0 when they match, -1
// otherwise (the tensor-core path is then unused). With raw4096 non-null the
// probe reruns and returns its raw output.
int tc_probe(int* mode, uint32_t* raw4096);

// The same check for the k > 256 E-step's blocked centre image and MMA
// sequence (estep_wide.cu).
int tc_probe_wide(int* mode, uint32_t* raw4096);

// X: the fit's blocked working copy (xblk_index), round_up(n, 128) rows.
// k <= 256: the pipeline of estep_dev.cuh; 256 < k <= 4096: the blocked one
// of estep_wide.cu (plan.wide); d <= 128 either way.
int tc_plan(const float* X, int ld, long long n, int d, int k, TcPlan* plan);
int tc_plan_wide(const float* X, int ld, long long n, int d, int k, int optin, TcPlan* plan);

// Bytes of the split working copy of X for this plan, and the launch that
// builds it from the fp32 blocked copy with the scale 2^sexp[0] (device int);
// the plan then reads its tiles from Xs.
size_t tc_split_bytes(const TcPlan& plan);
// Bytes of one 128-row tile of the split copy.
uint32_t tc_tile_bytes(const TcPlan& plan);
int tc_split_x(TcPlan* plan, void* Xs, const int* sexp, cudaStream_t s);

// Geometry of the centre image the plan's kernel reads (img: cimg_halves(...)
// fp16 entries, zero-initialised by the caller).
CentreImage tc_centre_image(const TcPlan& plan, uint16_t* img);

// img: centre image; sexp: {xexp, cexp} operand scale exponents (device);
// bias: ||c||^2 (k floats). `changed` (nullable) counts rows whose label
// differs from labels[] on entry; `D` (nullable, needs `st`) receives the
// fixed-point deltas of those rows; `st` (nullable) makes the launch a no-op
// once st->done is set; `err` receives a nonzero code if a pipeline wait
// times out.
// `pdl`: launch with programmatic stream serialization (the kernel waits for
// the previous kernel's writes itself). In bulk iterations (st->bulk) no
// deltas are written.
int tc_estep(const TcPlan& plan, const uint16_t* img, const int* sexp, const float* bias, int32_t* labels,
             unsigned long long* changed, long long* D, const FitState* st, int* err, cudaStream_t s,
             bool pdl = false);
int tc_estep_wide(const TcPlan& plan, const uint16_t* img, const int* sexp, const float* bias, int32_t* labels,
                  unsigned long long* changed, long long* D, const FitState* st, int* err, cudaStream_t s, bool pdl);

}  // namespace skm
