/*
 * skmetal_cuda.h -- C ABI of libskmetal_cuda.so, the B200 (sm_100a) KMeans
 * Lloyd library that replaces the reference's libSkMetalBridge.dylib for the
 * KMeans path.
 *
 * Conventions (kept from the reference bridge, skmetal/_bridge.py:78-103):
 *   - every entry point is synchronous and returns an int status, 0 = success
 *     (skmetal_kmeans_inertia returns the value itself, -1.0f on error, as the
 *     reference does);
 *   - matrices are host pointers to C-contiguous row-major float32 arrays;
 *     sizes are size_t; labels are 4-byte integers;
 *   - a failing call returns a nonzero code; skmetal_last_error() gives the
 *     message of the calling thread's last failure.
 * Status codes: 1 invalid argument, 2 CUDA error, 3 out of device memory,
 * 4 NCCL error, 5 timeout, 6 unsupported, 7 device-side check failed,
 * 8 injected failure (tests).
 *
 * All arithmetic runs on the GPU; there is no CPU fallback.
 */
#ifndef SKMETAL_CUDA_H
#define SKMETAL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- flags for the fit entry points ------------------------------------ */
#define SKMETAL_FIT_CENTER      0x1u  /* centre X and init by the column mean (KMeans.fit semantics) */
#define SKMETAL_FIT_SIMT        0x2u  /* force the SIMT E-step instead of the tensor-core one */
#define SKMETAL_FIT_PROFILE     0x4u  /* time the E-step launches of every 10th iteration with CUDA events (see fit stats) */
#define SKMETAL_FIT_DISTRIBUTED 0x8u  /* X is this rank's shard; sums are summed over the communicator's ranks */
#define SKMETAL_FIT_TOL_ABS     0x10u /* tol is the absolute threshold on the sum of squared centre shifts */
#define SKMETAL_FIT_BULK_SUMS   0x20u /* recompute the centroid sums from all rows every iteration (diagnostic) */

/* ---- device / library management --------------------------------------- */

/* Replaces skmetal_init (skmetal_bridge/Sources/SkMetalBridge/Bridge.swift:19-23). */
int skmetal_init(void);

/* Replaces skmetal_warmup (Bridge.swift:52-144): loads the kernels once. */
int skmetal_warmup(void);

/* Replaces skmetal_device_info (Bridge.swift:25-48). `has_unified_memory` is 0
 * on a discrete GPU; `recommended_working_set_size` is the device memory size. */
int skmetal_device_info(char* name, int name_capacity, size_t* max_threads, uint8_t* has_unified_memory,
                        uint64_t* recommended_working_set_size);

/* No reference counterpart (the reference drives one implicit device). */
int skmetal_device_count(int* count);
int skmetal_set_device(int device);

/* Message of the calling thread's last failure; returns its status code. */
int skmetal_last_error(char* buf, size_t capacity);

/* Number of kernel launches issued by this library since load. */
unsigned long long skmetal_launch_count(void);

/* Host-side fault injection (tests): the `after_calls`-th guarded entry
 * point from now fails with `code` before doing any GPU work. */
int skmetal_debug_inject_failure(int code, int after_calls);

/* Tensor-core self-check (no reference counterpart): pushes exactly
 * representable operands through the E-step's fp16 split, centre image and
 * tcgen05.mma sequences on the current device and compares the products with
 * their exact values. *mode = 0 when they match, -1 otherwise (the library
 * then uses its SIMT E-step). raw4096, if not NULL, receives the products
 * (float bits): 128 x 16 for the stacked layout, then 128 x 16 for the
 * two-segment layout. */
int skmetal_debug_tc_probe(int* mode, uint32_t* raw4096);

/* The same self-check for the E-step of more than 256 clusters (no reference
 * counterpart): 32 centres in two blocks of 16 (the blocked centre image) and
 * its three-MMA sequence per block. raw4096 receives the 128 x 32 products
 * (float bits). */
int skmetal_debug_tc_probe_wide(int* mode, uint32_t* raw4096);

/* ---- KMeans path: reference entry points -------------------------------- */

/* Replaces skmetal_kmeans_assign (KMeansBridge.swift:138-181; bound at
 * skmetal/_bridge.py:111-119,576-578). labels[i] = argmin_j ||x_i - c_j||^2,
 * strict '<', first index wins. */
int skmetal_kmeans_assign(const float* X, const float* centroids, uint32_t* labels, size_t n, size_t d, size_t k);

/* Replaces skmetal_kmeans_batch_fused (KMeansBridge.swift:187-320; bound at
 * skmetal/_bridge.py:120-132,591-617) with scikit-learn's single Lloyd run
 * (sklearn/cluster/_kmeans.py:628-758) on X as given (no centring):
 * `centroids` holds the initial centres on entry and the final ones on exit,
 * `labels` the final labels; `tol` is the absolute threshold on the sum of
 * squared centre shifts; iterations stop on strict convergence, on the
 * tolerance or at max_iter; *n_iter_out follows scikit-learn's i+1 count.
 * `num_groups` is accepted for ABI compatibility and ignored. */
int skmetal_kmeans_batch_fused(const float* X, float* centroids, uint32_t* labels, size_t n, size_t d, size_t k,
                               size_t num_groups, size_t max_iter, float tol, int32_t* n_iter_out);

/* Replaces skmetal_compute_mindists (KMeansBridge.swift:89-134; bound at
 * skmetal/_bridge.py:133-142,620-624): dists[i] = ||x_i - c_{labels[i]}||^2. */
int skmetal_compute_mindists(const float* X, const float* centroids, const uint32_t* labels, float* dists, size_t n,
                             size_t d, size_t k);

/* Replaces skmetal_kmeans_inertia (KMeansBridge.swift:324-373; bound at
 * skmetal/_bridge.py:627-639): sum_i ||x_i - c_{labels[i]}||^2 accumulated in
 * float64 in a fixed order; returns -1.0f on error. */
float skmetal_kmeans_inertia(const float* X, const float* centroids, const uint32_t* labels, size_t n, size_t d,
                             size_t k);

/* Declared by the reference header (skmetal_bridge/Sources/SkMetalBridgeC/
 * include/bridge.h:25), kernel row_norm_sq (DistanceKernels.metal:6-28). */
int skmetal_row_norm_sq(const float* X, float* norms, size_t n, size_t d);

/* Squared Euclidean distance matrix D[i*n + j] = max(||x_i||^2 + ||x_j||^2
 * - 2 x_i.x_j, 0) of the n rows of X, float32 (replaces skmetal_pairwise_
 * distance, skmetal_bridge/Sources/SkMetalBridge/KMeansBridge.swift:8-85,
 * bound at skmetal/_bridge.py:108 and called at skmetal/_bridge.py:566-573). */
int skmetal_pairwise_distance(const float* X, float* D, size_t n, size_t d);

/* ---- KMeans path: extended entry points ---------------------------------- */

/* Full KMeans.fit for one explicit initialisation (sklearn/cluster/
 * _kmeans.py:1436-1562 with n_init=1, algorithm="lloyd"), replacing the
 * MetalKMeans.fit orchestration (skmetal/estimators/cluster.py:20-65).
 * `tol` is scikit-learn's relative tolerance unless SKMETAL_FIT_TOL_ABS.
 * Outputs may be NULL. centers_out is k x d (mean added back). */
int skmetal_kmeans_fit(const float* X, size_t n, size_t d, size_t k, const float* init, int32_t max_iter, double tol,
                       uint32_t flags, float* centers_out, int32_t* labels_out, double* inertia_out,
                       int32_t* n_iter_out);

/* skmetal_kmeans_fit with sample weights (KMeans.fit(X, sample_weight=...),
 * reached through skmetal/estimators/cluster.py:20-65 and scikit-learn's
 * weighted Lloyd, sklearn/cluster/_k_means_lloyd.pyx _update_chunk_dense and
 * _k_means_common.pyx _relocate_empty_clusters_dense): a row adds its values
 * times its weight (float32 products) to its cluster's sum and its weight to
 * the cluster's weight, a cluster of weight zero is empty, and the inertia is
 * weighted. sample_weight: n finite, non-negative host floats (not all zero),
 * or NULL for unit weights. One GPU only. */
int skmetal_kmeans_fit_weighted(const float* X, size_t n, size_t d, size_t k, const float* init, int32_t max_iter,
                                double tol, uint32_t flags, const float* sample_weight, float* centers_out,
                                int32_t* labels_out, double* inertia_out, int32_t* n_iter_out);

/* skmetal_kmeans_inertia with sample weights: sum_i w_i ||x_i - c_{labels[i]}||^2
 * (KMeans.score(X, sample_weight=...), sklearn/cluster/_k_means_common.pyx
 * _inertia_dense); returns -1.0f on error. */
float skmetal_kmeans_inertia_weighted(const float* X, const float* centroids, const uint32_t* labels,
                                      const float* sample_weight, size_t n, size_t d, size_t k);

/* One E+M step of sklearn's lloyd_iter_chunked_dense
 * (sklearn/cluster/_k_means_lloyd.pyx:23-165, update_centers=True) on X as
 * given: labels_out gets the E-step labels against centers_old, centers_new
 * the M-step centres, weight_out the per-cluster weights after relocation,
 * center_shift_out the per-centre Euclidean shift. Outputs may be NULL. */
int skmetal_kmeans_lloyd_iter(const float* X, const float* centers_old, float* centers_new, int32_t* labels_out,
                              float* weight_out, float* center_shift_out, size_t n, size_t d, size_t k);

/* Distances of every row to every centre, D[i*k + j] = ||x_i - c_j||
 * (replaces the MetalKMeans.transform gemm route, skmetal/estimators/
 * cluster.py:135-146 and skmetal/_bridge.py:499-563). */
int skmetal_kmeans_transform(const float* X, const float* centroids, float* D, size_t n, size_t d, size_t k);

/* ---- device-resident datasets -------------------------------------------- */

/* Copy X (n x d, host) to the current device once; fits on the handle then
 * start from HBM-resident data. */
int skmetal_dataset_create(const float* X, size_t n, size_t d, void** handle);
int skmetal_dataset_free(void* handle);

/* skmetal_kmeans_fit on a resident dataset (X is not modified). */
int skmetal_kmeans_fit_dataset(void* handle, const float* init, size_t k, int32_t max_iter, double tol,
                               uint32_t flags, float* centers_out, int32_t* labels_out, double* inertia_out,
                               int32_t* n_iter_out);

/* skmetal_kmeans_fit_weighted on a resident dataset. */
int skmetal_dataset_fit_weighted(void* handle, const float* init, size_t k, int32_t max_iter, double tol,
                                 uint32_t flags, const float* sample_weight, float* centers_out, int32_t* labels_out,
                                 double* inertia_out, int32_t* n_iter_out);

/* Predict on a resident dataset: labels_out (host, may be NULL to keep the
 * labels on the device). */
int skmetal_kmeans_predict_dataset(void* handle, const float* centroids, size_t k, int32_t* labels_out);

/* k-means++ seeding of the n rows of X (scikit-learn's greedy k-means++,
 * sklearn/cluster/_kmeans.py _kmeans_plusplus, which the reference's KMeans
 * runs on this platform; the reference's own Metal seeding is k-means||,
 * skmetal/estimators/cluster.py:70-116). The caller draws from its random
 * stream what scikit-learn draws, in the same order: first_index (the first
 * centre, random_state.choice over w / sum(w)) and, for every further centre,
 * n_local_trials (1..16) uniforms in [0, 1): uniforms[(c - 1) * T + t].
 * sample_weight (n floats) may be NULL (unit weights). With center != 0 the
 * rows are centred by their exact column mean first, as the fit centres them.
 * centers_out (k x d) receives the chosen raw rows, indices_out their
 * indices. */
int skmetal_kmeans_plusplus(const float* X, size_t n, size_t d, size_t k, const float* sample_weight,
                            int64_t first_index, const double* uniforms, size_t n_local_trials, int center,
                            float* centers_out, int64_t* indices_out);

/* skmetal_kmeans_plusplus on a resident dataset. */
int skmetal_dataset_kmeans_plusplus(void* handle, size_t k, const float* sample_weight, int64_t first_index,
                                    const double* uniforms, size_t n_local_trials, int center, float* centers_out,
                                    int64_t* indices_out);

/* Statistics of the calling thread's last fit / predict: device times in
 * milliseconds measured with CUDA events on the library's stream
 * (total, preparation, Lloyd loop, final E-step + inertia), the number of
 * E-step launches timed individually (SKMETAL_FIT_PROFILE: iterations 0, 10,
 * 20, ...) and their summed duration, the kernel launches issued, and the
 * iterations run. */
/* Debug: the device timestamps (ns) of the last profiled fit that ran the
 * persistent loop kernel on this thread: per iteration t, [4t] start, [4t+1]
 * E-step done, [4t+2] bulk sums and empty clusters done, [4t+3] centres
 * done, and a final end stamp. Copies up to `cap` and returns how many there
 * are (0 when the last profiled fit used the multi-launch loop). No
 * reference counterpart. */
int skmetal_debug_loop_stamps(uint64_t* out, int cap);

int skmetal_last_fit_stats(double* ms_total, double* ms_prep, double* ms_loop, double* ms_final,
                           int32_t* estep_launches, double* estep_ms_sum, uint64_t* launches, int32_t* iterations);

/* The number of distinct labels in the final assignment of the calling
 * thread's last full one-GPU fit (skmetal_kmeans_fit*, skmetal_dataset_fit*),
 * counted on the device; -1 when it was not counted (sharded fits, single
 * Lloyd steps, k > 4096, or before any fit). scikit-learn warns when it is
 * below n_clusters (sklearn/cluster/_kmeans.py:1545-1552). */
int skmetal_last_fit_distinct(void);

/* ---- multi-GPU (one process per GPU) -------------------------------------- */

/* 128-byte NCCL unique id, produced on one rank and broadcast by the caller. */
int skmetal_comm_unique_id(uint8_t* id128);

/* Create this process's communicator on the current device. */
int skmetal_comm_init(const uint8_t* id128, int nranks, int rank);

int skmetal_comm_destroy(void);

/* Distributed fit: X is this rank's shard (rows [row_base, row_base + n) of a
 * dataset of n_total rows); all ranks pass the same init and parameters and
 * obtain the same centres, inertia and n_iter; labels_out gets the shard's
 * labels. */
int skmetal_kmeans_fit_shard(const float* X, size_t n, size_t d, size_t k, const float* init, int32_t max_iter,
                             double tol, uint32_t flags, uint64_t row_base, uint64_t n_total, float* centers_out,
                             int32_t* labels_out, double* inertia_out, int32_t* n_iter_out);

int skmetal_dataset_fit_shard(void* handle, const float* init, size_t k, int32_t max_iter, double tol,
                              uint32_t flags, uint64_t row_base, uint64_t n_total, float* centers_out,
                              int32_t* labels_out, double* inertia_out, int32_t* n_iter_out);

/* ---- no-allocation entry point -------------------------------------------- */

/* Size of the static device scratch behind skmetal_kmeans_update_centers_noalloc
 * (2 MiB, held on every device that loads the library until the process exits). */
#define SKMETAL_NOALLOC_SCRATCH_BYTES 2097152u

/* No counterpart in the reference: an addition for callers that must not
 * allocate device memory while they run -- a process whose free device memory
 * is already claimed by another allocator's pool, where a cudaMalloc would
 * fail, or a loop that cannot afford the device-wide waits that cudaMalloc and
 * cudaFree may cause. It calls no cudaMalloc, cudaFree or allocating library
 * routine; its scratch is one static device array of
 * SKMETAL_NOALLOC_SCRATCH_BYTES.
 *
 * Centroid update from given labels: for every cluster c with at least one
 * row, centers[c] = mean of the rows i with labels[i] == c, computed with the
 * fit's exact fixed-point sums, so the result is bit-identical to the
 * centres of skmetal_kmeans_lloyd_iter for the same labels when no cluster is
 * empty. Rows of empty clusters are left unchanged (no relocation). weight,
 * if not NULL, receives the per-cluster row counts.
 *
 * X (n x d row-major float32), labels (n int32 in [0, k)), centers (k x d)
 * and weight (k float32) must be device memory of the current device. The
 * work runs on `stream` (a cudaStream_t; NULL is the default stream) and the
 * call returns once it has completed. Sizes with k * (d + 1) above
 * SKMETAL_NOALLOC_SCRATCH_BYTES / 8 - 1 (262143) do not fit the scratch and
 * return 1 (invalid argument) with a message; so do labels outside [0, k) and
 * non-finite X, which leave centers and weight untouched.
 *
 * Every call looks up the scratch's device address (cudaGetSymbolAddress, with
 * the current device), so it stays valid across a cudaDeviceReset; the first
 * call on a device also loads the library's device code there, so make that
 * first call before any stream capture begins. Each call synchronises `stream`
 * before it returns. All callers on a device share the one scratch array:
 * calls on the same device that overlap in time (from several threads, or on
 * several streams) race on it and corrupt each other's results, so serialise
 * them. */
int skmetal_kmeans_update_centers_noalloc(const float* X, const int32_t* labels, size_t n, size_t d, size_t k,
                                          float* centers, float* weight, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SKMETAL_CUDA_H */
