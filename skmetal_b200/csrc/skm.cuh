// Shared definitions for the skmetal CUDA library (sm_100a).
//
// Layout conventions used by every kernel:
//   X       n rows x ld floats, row-major, ld = round_up(d, 4) (16-byte rows so
//           that TMA and 128-bit loads apply); columns [d, ld) are zero.
//   C       k rows x ld floats (centres), same padding.
//   labels  n int32.
//   S       k x ld int64: per-cluster coordinate sums in fixed point
//           (value * 2^F, F chosen per fit so that no sum can overflow).
//   counts  k int64.
// Fixed-point sums are exact and therefore independent of summation order,
// CTA scheduling and the number of GPUs the rows are sharded over.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

namespace skm {

enum Status : int {
  OK = 0,
  ERR_INVALID = 1,
  ERR_CUDA = 2,
  ERR_OOM = 3,
  ERR_NCCL = 4,
  ERR_TIMEOUT = 5,
  ERR_UNSUPPORTED = 6,
  ERR_DEVICE = 7,   // a kernel reported an error through the fit state
  ERR_INJECTED = 8, // host-side fault injection (tests only)
};

void set_error(int code, const char* fmt, ...);

// Device-side fit state: one per fit, lives in device memory.
struct FitState {
  int32_t iter;        // completed Lloyd iterations
  int32_t done;        // loop finished (converged or max_iter)
  int32_t strict;      // strict convergence (labels unchanged)
  int32_t max_iter;
  int32_t n_empty;     // empty clusters found in the current iteration
  int32_t relocated;   // relocations applied in the current iteration
  int32_t error;       // nonzero: a kernel detected an inconsistency
  int32_t full_update; // current iteration recomputes sums from scratch
  unsigned long long changed;      // rows whose label changed this iteration
  unsigned long long sel_prefix;   // radix-select state (64-bit keys)
  int32_t sel_remaining;
  int32_t sel_count;
  double tol;          // absolute tolerance on the sum of squared shifts
  double scale;        // 2^F: a row's value v enters the sums as round(v * w * 2^F)
  double inv_scale;    // 2^-F * wscale: centre = S * inv_scale / W
  double shift_tot;    // sum of squared centre shifts of the last M-step
  double inertia;
  unsigned int barrier_count;  // software grid barrier
  unsigned int barrier_gen;
  unsigned int ticket;         // M-step: blocks done with their clusters (the last one finishes)
  unsigned int pad_ticket;
  unsigned int maxabs_bits;    // max |x| (float bits) of centred X
  int32_t xexp;        // tensor-core operand scale of X: x * 2^xexp (split_exp)
  int32_t cexp;        // same for the centres of the current centre image
  int32_t bulk;        // this iteration rebuilds the sums from all rows (no per-row deltas)
  int32_t bulk_always; // every iteration does (diagnostic flag)
  int32_t pad0;
  long long bulk_threshold;  // changed rows above which the next iteration is a bulk one
  const float* w;      // per-row sample weights (device), null: unit weights
  double wscale;       // 2^G: a row's weight enters the cluster weights W as round(w * 2^G); 1 unweighted
};

constexpr int kMaxEmptyCap = 4096;  // upper bound on relocations per iteration

inline size_t round_up(size_t a, size_t b) { return (a + b - 1) / b * b; }

}  // namespace skm
