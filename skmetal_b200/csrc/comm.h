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
int comm_rank(Comm* c);
// Wait for `e` while polling the communicator for asynchronous errors; aborts
// the communicator and returns ERR_TIMEOUT / ERR_NCCL when it cannot finish.
int comm_wait_event(Comm* c, cudaEvent_t e);

}  // namespace skm
