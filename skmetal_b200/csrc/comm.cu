// Multi-GPU plumbing: one process per GPU, an NCCL communicator per process.
//
// NCCL is opened with dlopen when the first communicator is created, so the
// library loads (and runs single-GPU) without NCCL present. The library to
// open can be named by SKMETAL_NCCL_LIB (the Python layer points it at the
// NCCL that PyTorch ships, so that one process never maps two NCCL builds);
// the default is the soname libnccl.so.2.
//
// Every wait on the GPU inside a distributed fit goes through comm_wait_event,
// which polls the event and the communicator's asynchronous error state and
// aborts the communicator after SKMETAL_COMM_TIMEOUT_S seconds (default 300)
// so that a dead peer turns into an error instead of a hang.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "comm.h"
#include "driver.h"
#include "../../include/skmetal_cuda.h"

namespace skm {

struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

struct Comm {
  ncclComm_t comm = nullptr;
  int nranks = 1;
  int rank = 0;
  int device = 0;
  bool aborted = false;
  // peer region (comm_peer_region): this rank's buffer and its mappings of
  // every rank's buffer (own entry = own buffer)
  void* region = nullptr;
  std::vector<void*> region_ptrs;
  int region_state = 0;  // 0 not tried, 1 ready, -1 unavailable on some rank
};

static NcclApi g_nccl;
static std::mutex g_comm_mu;
static Comm* g_comm = nullptr;

static int load_nccl() {
  if (g_nccl.handle) return OK;
  const char* name = getenv("SKMETAL_NCCL_LIB");
  void* h = dlopen(name && *name ? name : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    set_error(ERR_NCCL, "cannot load NCCL (%s): %s", name ? name : "libnccl.so.2", dlerror());
    return ERR_NCCL;
  }
#define SKM_SYM(field, sym)                                                       \
  g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, sym));        \
  if (!g_nccl.field) {                                                            \
    set_error(ERR_NCCL, "NCCL symbol %s missing", sym);                          \
    return ERR_NCCL;                                                              \
  }
  SKM_SYM(GetUniqueId, "ncclGetUniqueId");
  SKM_SYM(CommInitRank, "ncclCommInitRank");
  SKM_SYM(AllReduce, "ncclAllReduce");
  SKM_SYM(AllGather, "ncclAllGather");
  SKM_SYM(CommDestroy, "ncclCommDestroy");
  SKM_SYM(CommAbort, "ncclCommAbort");
  SKM_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
  SKM_SYM(GetErrorString, "ncclGetErrorString");
#undef SKM_SYM
  g_nccl.handle = h;
  return OK;
}

#define SKM_NCCL(call)                                                                              \
  do {                                                                                              \
    ncclResult_t r_ = (call);                                                                       \
    if (r_ != ncclSuccess) {                                                                        \
      ::skm::set_error(::skm::ERR_NCCL, "%s failed: %s", #call, g_nccl.GetErrorString(r_));        \
      return ::skm::ERR_NCCL;                                                                       \
    }                                                                                               \
  } while (0)

Comm* comm_get() {
  std::lock_guard<std::mutex> lk(g_comm_mu);
  return g_comm;
}

int comm_nranks(Comm* c) { return c ? c->nranks : 1; }
int comm_rank(Comm* c) { return c ? c->rank : 0; }

int comm_allreduce_sum_s64(Comm* c, long long* buf, size_t count, cudaStream_t s) {
  if (c->nranks == 1) return OK;
  SKM_NCCL(g_nccl.AllReduce(buf, buf, count, ncclInt64, ncclSum, c->comm, s));
  return OK;
}

int comm_allreduce_sum_f64(Comm* c, double* buf, size_t count, cudaStream_t s) {
  if (c->nranks == 1) return OK;
  SKM_NCCL(g_nccl.AllReduce(buf, buf, count, ncclFloat64, ncclSum, c->comm, s));
  return OK;
}

int comm_allreduce_max_u32(Comm* c, unsigned int* buf, size_t count, cudaStream_t s) {
  if (c->nranks == 1) return OK;
  SKM_NCCL(g_nccl.AllReduce(buf, buf, count, ncclUint32, ncclMax, c->comm, s));
  return OK;
}

int comm_allgather_bytes(Comm* c, const void* send, void* recv, size_t bytes_per_rank, cudaStream_t s) {
  if (c->nranks == 1) {
    if (send != recv) SKM_CUDA(cudaMemcpyAsync(recv, send, bytes_per_rank, cudaMemcpyDeviceToDevice, s));
    return OK;
  }
  SKM_NCCL(g_nccl.AllGather(send, recv, bytes_per_rank, ncclUint8, c->comm, s));
  return OK;
}

static int agree_any(Comm* c, unsigned int* dev_word, unsigned int* v, cudaStream_t s) {
  SKM_CUDA(cudaMemcpyAsync(dev_word, v, sizeof(*v), cudaMemcpyHostToDevice, s));
  SKM_TRY(comm_allreduce_max_u32(c, dev_word, 1, s));
  SKM_CUDA(cudaMemcpyAsync(v, dev_word, sizeof(*v), cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  return OK;
}

static int peer_region_exchange(Comm* c, unsigned char* dev, cudaStream_t s) {
  constexpr size_t hb = sizeof(cudaIpcMemHandle_t);
  static_assert(hb == 64, "IPC handle size");
  unsigned int* word = reinterpret_cast<unsigned int*>(dev + hb * (c->nranks + 1));
  unsigned int bad = c->nranks > kMaxPeerRanks ? 1u : 0u;
  // every rank's GPU by PCI bus id (gathered into dev), mapped to this
  // process's device ordinals: a peer whose GPU this process cannot see (its
  // own CUDA_VISIBLE_DEVICES, another host) has no peer access
  constexpr size_t bid = 16;
  char mine[bid] = {};
  if (cudaDeviceGetPCIBusId(mine, (int)bid, c->device) != cudaSuccess) bad = 1;
  cudaGetLastError();
  SKM_CUDA(cudaMemcpyAsync(dev + bid * c->nranks, mine, bid, cudaMemcpyHostToDevice, s));
  SKM_TRY(comm_allgather_bytes(c, dev + bid * c->nranks, dev, bid, s));
  std::vector<char> ids(bid * c->nranks);
  SKM_CUDA(cudaMemcpyAsync(ids.data(), dev, bid * c->nranks, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  for (int r = 0; r < c->nranks && !bad; ++r) {
    if (r == c->rank) continue;
    char id[bid + 1] = {};
    memcpy(id, ids.data() + bid * r, bid);
    int dev_r = -1, can = 0;
    if (cudaDeviceGetByPCIBusId(&dev_r, id) != cudaSuccess || dev_r == c->device ||
        cudaDeviceCanAccessPeer(&can, c->device, dev_r) != cudaSuccess || !can)
      bad = 1;
  }
  cudaIpcMemHandle_t h{};
  if (!bad && cudaMalloc(&c->region, kPeerRegionBytes) != cudaSuccess) bad = 1;
  if (!bad && cudaIpcGetMemHandle(&h, c->region) != cudaSuccess) bad = 1;
  cudaGetLastError();
  SKM_TRY(agree_any(c, word, &bad, s));  // nobody opens a handle that does not exist
  if (bad) return OK;
  SKM_CUDA(cudaMemcpyAsync(dev + hb * c->nranks, &h, hb, cudaMemcpyHostToDevice, s));
  SKM_TRY(comm_allgather_bytes(c, dev + hb * c->nranks, dev, hb, s));
  std::vector<unsigned char> all(hb * c->nranks);
  SKM_CUDA(cudaMemcpyAsync(all.data(), dev, hb * c->nranks, cudaMemcpyDeviceToHost, s));
  SKM_CUDA(cudaStreamSynchronize(s));
  c->region_ptrs.assign(c->nranks, nullptr);
  c->region_ptrs[c->rank] = c->region;
  for (int r = 0; r < c->nranks && !bad; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t hr;
    memcpy(&hr, all.data() + hb * r, hb);
    if (cudaIpcOpenMemHandle(&c->region_ptrs[r], hr, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      c->region_ptrs[r] = nullptr;
      bad = 1;
    }
  }
  cudaGetLastError();
  SKM_TRY(agree_any(c, word, &bad, s));
  if (!bad) c->region_state = 1;
  return OK;
}

// The peer region: kPeerRegionBytes of device memory per rank, mapped into
// every other rank's address space with CUDA IPC (handles exchanged with an
// NCCL all-gather). Kernels of one fit read their peers' buffers over
// NVLink and write into their arrival words. Collective: every rank calls
// it; a failure on any rank (no peer access, IPC refused) is agreed on with
// max all-reduces, so all ranks get the same answer, and it is remembered.
static int peer_region_setup(Comm* c, cudaStream_t s) {
  unsigned char* dev = nullptr;
  SKM_CUDA(cudaMalloc(reinterpret_cast<void**>(&dev), sizeof(cudaIpcMemHandle_t) * (c->nranks + 1) + 16));
  c->region_state = -1;
  const int rc = peer_region_exchange(c, dev, s);
  cudaFree(dev);
  return rc;
}

int comm_peer_region(Comm* c, cudaStream_t s, void* const** ptrs) {
  *ptrs = nullptr;
  if (!c || c->nranks < 2 || c->aborted) return OK;
  if (c->region_state == 0) SKM_TRY(peer_region_setup(c, s));
  if (c->region_state == 1) *ptrs = c->region_ptrs.data();
  return OK;
}

// Unmaps the peers' regions, waits (all-reduce, under the watchdog) for every
// rank to have done the same, then frees this rank's. Collective whenever the
// region was set up (region_state is the same on every rank); the wait is
// skipped after an abort.
static void peer_region_release(Comm* c) {
  for (int r = 0; r < (int)c->region_ptrs.size(); ++r)
    if (r != c->rank && c->region_ptrs[r]) cudaIpcCloseMemHandle(c->region_ptrs[r]);
  c->region_ptrs.clear();
  if (c->region_state != 0 && !c->aborted && c->comm) {
    cudaStream_t s = nullptr;
    cudaEvent_t e = nullptr;
    unsigned int* w = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess &&
        cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess &&
        cudaMalloc(reinterpret_cast<void**>(&w), sizeof(unsigned int)) == cudaSuccess &&
        cudaMemsetAsync(w, 0, sizeof(unsigned int), s) == cudaSuccess &&
        g_nccl.AllReduce(w, w, 1, ncclUint32, ncclMax, c->comm, s) == ncclSuccess &&
        cudaEventRecord(e, s) == cudaSuccess)
      comm_wait_event(c, e);
    if (w) cudaFree(w);
    if (e) cudaEventDestroy(e);
    if (s) cudaStreamDestroy(s);
  }
  if (c->region) cudaFree(c->region);
  c->region = nullptr;
  c->region_state = 0;
  cudaGetLastError();
}

static double timeout_s() {
  const char* t = getenv("SKMETAL_COMM_TIMEOUT_S");
  double v = t ? atof(t) : 300.0;
  return v > 0 ? v : 300.0;
}

int comm_wait_event(Comm* c, cudaEvent_t e) {
  const auto t0 = std::chrono::steady_clock::now();
  const double limit = timeout_s();
  for (;;) {
    cudaError_t q = cudaEventQuery(e);
    if (q == cudaSuccess) return OK;
    if (q != cudaErrorNotReady) {
      set_error(ERR_CUDA, "event query: %s", cudaGetErrorString(q));
      return ERR_CUDA;
    }
    if (c && c->comm && !c->aborted) {
      ncclResult_t ae = ncclSuccess;
      if (g_nccl.CommGetAsyncError(c->comm, &ae) == ncclSuccess && ae != ncclSuccess && ae != ncclInProgress) {
        g_nccl.CommAbort(c->comm);
        c->aborted = true;
        set_error(ERR_NCCL, "NCCL asynchronous error: %s (communicator aborted)", g_nccl.GetErrorString(ae));
        return ERR_NCCL;
      }
    }
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > limit) {
      if (c && c->comm && !c->aborted) {
        g_nccl.CommAbort(c->comm);
        c->aborted = true;
      }
      set_error(ERR_TIMEOUT, "GPU work did not finish within %.0f s (communicator aborted)", limit);
      return ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(el < 0.01 ? 2 : 200));
  }
}

}  // namespace skm

using namespace skm;

extern "C" {

int skmetal_comm_unique_id(uint8_t* id128) {
  SKM_TRY(check_injected("comm_unique_id"));
  SKM_TRY(load_nccl());
  ncclUniqueId id;
  SKM_NCCL(g_nccl.GetUniqueId(&id));
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
  memcpy(id128, &id, 128);
  return OK;
}

int skmetal_comm_init(const uint8_t* id128, int nranks, int rank) {
  SKM_TRY(check_injected("comm_init"));
  if (nranks < 1 || rank < 0 || rank >= nranks) {
    set_error(ERR_INVALID, "invalid rank %d of %d", rank, nranks);
    return ERR_INVALID;
  }
  std::lock_guard<std::mutex> lk(g_comm_mu);
  if (g_comm) {
    set_error(ERR_INVALID, "a communicator already exists (call skmetal_comm_destroy first)");
    return ERR_INVALID;
  }
  Comm* c = new Comm();
  c->nranks = nranks;
  c->rank = rank;
  cudaGetDevice(&c->device);
  if (nranks > 1) {
    int rc = load_nccl();
    if (rc) {
      delete c;
      return rc;
    }
    ncclUniqueId id;
    memcpy(&id, id128, 128);
    ncclResult_t r = g_nccl.CommInitRank(&c->comm, nranks, id, rank);
    if (r != ncclSuccess) {
      set_error(ERR_NCCL, "ncclCommInitRank: %s", g_nccl.GetErrorString(r));
      delete c;
      return ERR_NCCL;
    }
  }
  g_comm = c;
  return OK;
}

int skmetal_comm_destroy(void) {
  std::lock_guard<std::mutex> lk(g_comm_mu);
  if (!g_comm) return OK;
  if (g_comm->region_state != 0 || g_comm->region) peer_region_release(g_comm);
  if (g_comm->comm) {
    if (g_comm->aborted) {
      // already torn down by the watchdog
    } else {
      g_nccl.CommDestroy(g_comm->comm);
    }
  }
  delete g_comm;
  g_comm = nullptr;
  return OK;
}

}  // extern "C"
