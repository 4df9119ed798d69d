// Deferred fixed-point deltas for an E-step epilogue (sm_100a device code).
//
// A row that changes label adds its fixed-point coordinates to its new
// cluster's delta sums and removes them from its old one. Applying that in the
// epilogue puts a dependent global load (the row's float32 values) and its
// atomics on the path of the warp that must go on to the next tile. Instead
// the finishing epilogue warps append (row, old label, new label) to a ring in
// shared memory (dq_push), and a warp without another role applies the
// entries in order (dq_drain), many rows' loads in flight at once.
//
// Ring entry (8 bytes, published by one store): bit 63 valid, bits 50..62 the
// new label, bits 37..49 the old label + 1 (0: none), bits 0..36 the row.
// Counters (monotonic 32-bit, wrapping): [0] entries reserved, [1] entries
// consumed, [2] producer warps that closed. Every wait is bounded in time; on
// a timeout the waiter sets the CTA's abort flag and records an error code.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "device_util.cuh"
#include "skm.cuh"

namespace skm {

constexpr int DQ_CAP = 256;  // entries, a power of two >= 32
constexpr unsigned long long DQ_VALID = 1ull << 63;
constexpr int DQ_MAX_LABEL = 8191;      // labels up to 13 bits
constexpr long long DQ_MAX_ROW = (1ll << 37) - 1;
constexpr int DQ_ILP = 4;               // value loads in flight per lane while draining
constexpr unsigned long long DQ_TIMEOUT_NS = 2000000000ull;

__host__ __device__ constexpr uint32_t dq_bytes() { return DQ_CAP * 8 + 16; }

struct DeltaRing {
  unsigned long long* q;  // DQ_CAP entries
  unsigned int* ctl;      // the three counters (and one spare word)
};

// `base`: dq_bytes() of shared memory, 8-byte aligned.
__device__ __forceinline__ DeltaRing dq_ring(unsigned char* base) {
  DeltaRing r;
  r.q = reinterpret_cast<unsigned long long*>(base);
  r.ctl = reinterpret_cast<unsigned int*>(base + DQ_CAP * 8);
  return r;
}

// All threads of the block, before the block barrier that precedes its use.
__device__ __forceinline__ void dq_init(DeltaRing r) {
  for (int i = threadIdx.x; i < DQ_CAP + 2; i += blockDim.x) r.q[i] = 0;
}

__device__ __forceinline__ unsigned long long dq_clock() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Warp-collective (all 32 lanes): the lanes with `ch` append their row. Lane
// 0 reserves the slots and waits until the drainer has freed them.
__device__ __forceinline__ void dq_push(DeltaRing r, volatile int* abort_flag, int* err, long long row, int old,
                                        int neu, bool ch) {
  const int lane = threadIdx.x & 31;
  const unsigned int m = __ballot_sync(0xffffffffu, ch);
  if (!m) return;
  const unsigned int cnt = __popc(m);
  unsigned int base = 0;
  if (lane == 0) {
    base = atomicAdd(r.ctl, cnt);
    const volatile unsigned int* consumed = r.ctl + 1;
    if ((int)(base + cnt - *consumed) > DQ_CAP) {
      const unsigned long long t0 = dq_clock();
      for (uint32_t i = 1; (int)(base + cnt - *consumed) > DQ_CAP; ++i) {
        if ((i & 63) == 0) {
          if (*abort_flag) break;
          if (dq_clock() - t0 > DQ_TIMEOUT_NS) {
            *abort_flag = 1;
            atomicCAS(err, 0, 2701);
            break;
          }
        }
      }
    }
    __threadfence_block();  // the slots' previous entries were cleared before `consumed` moved
  }
  base = __shfl_sync(0xffffffffu, base, 0);
  if (ch) {
    const unsigned int pos = base + __popc(m & ((1u << lane) - 1u));
    reinterpret_cast<volatile unsigned long long*>(r.q)[pos & (DQ_CAP - 1)] =
        DQ_VALID | ((unsigned long long)neu << 50) | ((unsigned long long)(old + 1) << 37) | (unsigned long long)row;
  }
}

// Warp-collective, once per pass, after the warp's last dq_push.
__device__ __forceinline__ void dq_close(DeltaRing r) {
  __threadfence_block();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) atomicAdd(r.ctl + 2, 1u);
}

// Warp-collective: applies the entries in order until `closes` producer
// closes have been seen and every reserved entry is applied. Count deltas
// are added by the entries' own lanes; value deltas are (entry, column quad)
// items spread over the lanes, DQ_ILP loads in flight per lane. X is the
// blocked float32 copy (xblk_index), D = [dS (k x ld) | dcount (k) | ...].
__device__ __forceinline__ void dq_drain(DeltaRing r, unsigned int closes, volatile int* abort_flag, int* err,
                                         const float* __restrict__ X, int ld, int d, int k, const FitState* st,
                                         long long* __restrict__ D) {
  const int lane = threadIdx.x & 31;
  volatile unsigned long long* q = reinterpret_cast<volatile unsigned long long*>(r.q);
  volatile unsigned int* ctl = r.ctl;
  unsigned int head = ctl[1];
  const int nq = ld >> 2;
  const double scale = st->scale;
  const float* w = st->w;
  unsigned long long t0 = 0;
  for (uint32_t spin = 1;; ++spin) {
    const unsigned long long e = q[(head + lane) & (DQ_CAP - 1)];
    const unsigned int vm = __ballot_sync(0xffffffffu, (e & DQ_VALID) != 0);
    const int nv = vm == 0xffffffffu ? 32 : __ffs(~vm) - 1;  // valid entries in order from head
    if (nv == 0) {
      int stop = 0;
      if (lane == 0) {
        if (ctl[2] == closes) {  // every producer closed: the reservations are final
          __threadfence_block();
          if (ctl[0] == head) stop = 1;
        }
        if (!stop && (spin & 63) == 0) {
          if (*abort_flag) {
            stop = 1;
          } else if (t0 == 0) {
            t0 = dq_clock();
          } else if (dq_clock() - t0 > DQ_TIMEOUT_NS) {
            *abort_flag = 1;
            atomicCAS(err, 0, 2702);
            stop = 1;
          }
        }
      }
      if (__shfl_sync(0xffffffffu, stop, 0)) break;
      continue;
    }
    t0 = 0;
    const long long row = (long long)(e & (unsigned long long)DQ_MAX_ROW);
    const int old = (int)((e >> 37) & 0x1FFFu) - 1;
    const int neu = (int)((e >> 50) & 0x1FFFu);
    const float wv = (lane < nv && w) ? __ldg(w + row) : 1.0f;
    if (lane < nv) count_delta(k, ld, old, neu, D, w ? to_fixed(wv, st->wscale) : 1);
    const int total = nv * nq;
    for (int b = 0; b < total; b += 32 * DQ_ILP) {
      float4 v[DQ_ILP];
      int ei[DQ_ILP];
#pragma unroll
      for (int u = 0; u < DQ_ILP; ++u) {
        const int it = b + u * 32 + lane;
        ei[u] = it < total ? it / nq : 0;
        const long long rr = __shfl_sync(0xffffffffu, row, ei[u]);
        if (it < total)
          v[u] = __ldg(reinterpret_cast<const float4*>(X + xblk_index(rr, 0, ld)) + (long long)(it - ei[u] * nq) * 128);
      }
#pragma unroll
      for (int u = 0; u < DQ_ILP; ++u) {
        const int it = b + u * 32 + lane;
        const int o = __shfl_sync(0xffffffffu, old, ei[u]);
        const int ne = __shfl_sync(0xffffffffu, neu, ei[u]);
        const float ww = __shfl_sync(0xffffffffu, wv, ei[u]);
        if (it < total)
          quad_delta(v[u], it - ei[u] * nq, d, D + (long long)ne * ld, o >= 0 ? D + (long long)o * ld : nullptr,
                     scale, ww);
      }
    }
    // free the slots, then publish the new head
    if (lane < nv) q[(head + lane) & (DQ_CAP - 1)] = 0;
    head += (unsigned int)nv;
    __threadfence_block();
    __syncwarp();
    if (lane == 0) ctl[1] = head;
  }
}

}  // namespace skm
