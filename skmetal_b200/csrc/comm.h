// Multi-GPU communicator (one process per GPU, NCCL loaded at run time).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace skm {

struct Comm;

Comm* comm_get();  // the process communicator, or null
int comm_allreduce_sum_s64(Comm* c, long long* buf, size_t count, cudaStream_t s);
int comm_allreduce_sum_f64(Comm* c, double* buf, size_t count, cudaStream_t s);
int comm_allreduce_max_u32(Comm* c, unsigned int* buf, size_t count, cudaStream_t s);
int comm_allgather_bytes(Comm* c, const void* send, void* recv, size_t bytes_per_rank, cudaStream_t s);
int comm_nranks(Comm* c);

// Peer region for kernels that exchange data over NVLink themselves: every
// rank owns kPeerRegionBytes of device memory mapped into every other rank.
// Collective (all ranks call it, with the same answer): *ptrs receives the
// region of each rank (indexed by rank, own included), or null when there is
// no peer region (one rank, more than kMaxPeerRanks, or no peer access on
// some rank).
constexpr int kMaxPeerRanks = 8;
constexpr size_t kPeerRegionBytes = 16u << 20;
int comm_peer_region(Comm* c, cudaStream_t s, void* const** ptrs);
int comm_rank(Comm* c);
// Wait for `e` while polling the communicator for asynchronous errors; aborts
// the communicator and returns ERR_TIMEOUT / ERR_NCCL when it cannot finish.
int comm_wait_event(Comm* c, cudaEvent_t e);

}  // namespace skm
