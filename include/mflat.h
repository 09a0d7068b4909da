/* SPDX-License-Identifier: Apache-2.0 */
/* mflat.h -- C ABI of the B200 flat-search library (libmetalflat_c.so).
 *
 * Drop-in for the flat, logging and version surface of metal-flat's C ABI
 * (reference: c/include/mflat.h, c/mflat.cpp).  Same names, same values, same
 * argument checks and status codes; the engine behind it runs on NVIDIA
 * B200 (sm_100a) instead of Metal.  Every entry point below names the
 * reference declaration it replaces.  Entries marked ADDITIVE have no
 * counterpart in the reference; the ABI stays additive-only as the
 * reference's header promises (c/include/mflat.h:5-6).
 *
 * Buffer contract for every *_search (c/include/mflat.h:8-12): out_ids and
 * out_distances are caller-allocated and hold at least m * k elements.  Rows
 * are written nearest-first and PACKED at stride k_used (the number of columns
 * actually produced, returned in *out_k_used), exactly as the reference's
 * emit() does (c/mflat.cpp:42-50).  ids are -1 padded when the database holds
 * fewer than k vectors; the padding distance is +inf (L2) or -inf (IP/Cosine).
 *
 * There is no CPU fallback: when no usable CUDA device exists, create still
 * returns a handle, mflat_flat_ready() returns 0, and search returns
 * MFLAT_ERR_DEVICE.
 */
#ifndef MFLAT_H
#define MFLAT_H

#include <stdint.h>

#if defined(_WIN32)
#  define MFLAT_API
#else
#  define MFLAT_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MFLAT_VERSION_MAJOR 0       /* c/include/mflat.h:31-33 */
#define MFLAT_VERSION_MINOR 1
#define MFLAT_VERSION_PATCH 0
/* c/include/mflat.h:34 (was 64).  Raised: the exact path serves k up to 1024.
 * Requests above it are clamped with a one-time warning (FlatIndex.mm:297-305). */
#define MFLAT_MAX_K 1024

typedef enum {                      /* c/include/mflat.h:36-40, value-stable */
    MFLAT_METRIC_L2            = 0,
    MFLAT_METRIC_INNER_PRODUCT = 1,
    MFLAT_METRIC_COSINE        = 2
} mflat_metric_t;

typedef enum {                      /* c/include/mflat.h:42-49, value-stable */
    MFLAT_OK            = 0,
    MFLAT_ERR_NULL_ARG  = 1,
    MFLAT_ERR_BAD_ARG   = 2,
    MFLAT_ERR_ALLOC     = 3,        /* host or device allocation failed */
    MFLAT_ERR_NOT_READY = 4,
    MFLAT_ERR_INTERNAL  = 5,
    MFLAT_ERR_DEVICE    = 6,        /* ADDITIVE: CUDA / NCCL failure or no device */
    MFLAT_ERR_IO        = 7         /* ADDITIVE: index file unreadable / unwritable */
} mflat_status_t;

/* ADDITIVE: storage precision of the database rows on the device. */
typedef enum {
    MFLAT_STORAGE_FP32 = 0,         /* exact path: 3 x bf16 screen + fp64 re-rank */
    MFLAT_STORAGE_FP16 = 1,         /* kind::f16 tensor cores, recall path      */
    MFLAT_STORAGE_BF16 = 2
} mflat_storage_t;

MFLAT_API const char* mflat_version(void);              /* c/mflat.cpp:72  "0.1.0" */
MFLAT_API const char* mflat_status_str(mflat_status_t); /* c/mflat.cpp:86-96       */
MFLAT_API int         mflat_max_k(void);                /* c/mflat.cpp:73          */

/* ---------------- Logging (c/include/mflat.h:55-74) ------------------- */
typedef enum {
    MFLAT_LOG_INFO  = 0,
    MFLAT_LOG_WARN  = 1,
    MFLAT_LOG_ERROR = 2,
    MFLAT_LOG_OFF   = 3
} mflat_log_level_t;

typedef void (*mflat_log_handler_t)(mflat_log_level_t level, const char* msg, void* user);

MFLAT_API void              mflat_set_log_handler(mflat_log_handler_t handler, void* user); /* c/mflat.cpp:75-79 */
MFLAT_API void              mflat_set_log_level(mflat_log_level_t threshold);                /* c/mflat.cpp:80-82 */
MFLAT_API mflat_log_level_t mflat_log_level(void);                                          /* c/mflat.cpp:83-85 */

/* ---------------- FlatIndex (exact) (c/include/mflat.h:76-90) --------- */
typedef struct mflat_flat_index mflat_flat_index_t;

/* c/mflat.cpp:99-104.  dim <= 0 -> BAD_ARG and NULL; unknown metric -> L2.
 * FP32 storage on device MFLAT_DEVICE (env) or 0. */
MFLAT_API mflat_flat_index_t*
mflat_flat_create(int dim, mflat_metric_t metric, mflat_status_t* out_status);
MFLAT_API void mflat_flat_free(mflat_flat_index_t*);                       /* c/mflat.cpp:105 */

MFLAT_API int mflat_flat_ready(const mflat_flat_index_t*);  /* c/mflat.cpp:106; 1 = device ready */
MFLAT_API int mflat_flat_size (const mflat_flat_index_t*);  /* c/mflat.cpp:107 */
MFLAT_API int mflat_flat_dim  (const mflat_flat_index_t*);  /* c/mflat.cpp:108 */

/* c/mflat.cpp:110-116: NULL -> NULL_ARG; n < 0 -> BAD_ARG; n == 0 no-op. */
MFLAT_API mflat_status_t mflat_flat_add(mflat_flat_index_t*, const float* vectors, int n);
/* c/mflat.cpp:117-121 */
MFLAT_API mflat_status_t mflat_flat_reset(mflat_flat_index_t*);
/* c/mflat.cpp:122-129: NULL h/q -> NULL_ARG; m < 0 or k < 1 -> BAD_ARG;
 * outputs nullable; results packed at stride k_used. */
MFLAT_API mflat_status_t mflat_flat_search(mflat_flat_index_t*, const float* queries,
        int m, int k, int32_t* out_ids, float* out_distances, int* out_k_used);

/* ---------------- ADDITIVE entries ------------------------------------ */

/* create with an explicit storage precision and CUDA device (-1 = default). */
MFLAT_API mflat_flat_index_t*
mflat_flat_create_ex(int dim, mflat_metric_t metric, mflat_storage_t storage, int device,
                     mflat_status_t* out_status);
MFLAT_API int mflat_flat_storage(const mflat_flat_index_t*);
MFLAT_API int mflat_flat_device(const mflat_flat_index_t*);

/* Device-resident variants: every pointer is device memory on the index's
 * device; `stream` is a cudaStream_t (NULL = the legacy default stream).  The
 * call enqueues work on `stream` and returns without synchronising; results
 * are valid once `stream` reaches that point.  Exception: searches that use
 * per-query candidate buffers (k > 21 on FP32; k > 16, or a large m * n, on
 * FP16 / BF16) check status words on the host and return after the search.
 * *out_k_used is host memory. */
MFLAT_API mflat_status_t mflat_flat_add_device(mflat_flat_index_t*, const float* d_vectors,
        int n, void* stream);
MFLAT_API mflat_status_t mflat_flat_search_device(mflat_flat_index_t*, const float* d_queries,
        int m, int k, int32_t* d_out_ids, float* d_out_distances, int* out_k_used, void* stream);

/* Allocation-free search.  No counterpart in the reference: some callers cannot
 * call cudaMalloc -- a serving process whose device memory is already reserved
 * by a framework's caching allocator, or a latency-critical loop that cannot
 * afford the device-wide synchronisation of cudaMalloc / cudaFree.  Same
 * arguments and results as mflat_flat_search_device, but every per-call
 * scratch buffer lives in one fixed array inside the library
 * (MFLAT_NOALLOC_SCRATCH_BYTES per GPU, held until the process exits).
 * Limits: m <= MFLAT_NOALLOC_MAX_QUERIES, dim <= MFLAT_NOALLOC_MAX_DIM,
 * k <= MFLAT_NOALLOC_MAX_K, FP32 storage, unsharded; larger sizes return
 * MFLAT_ERR_BAD_ARG (no clamping) and log the limit.  All calls on one GPU
 * share the array: calls that overlap on the GPU (other streams, other
 * indexes) race and must be serialised by the caller.  The first call on a
 * device looks up the array's device address; make it before any stream
 * capture. */
#define MFLAT_NOALLOC_MAX_QUERIES 128
#define MFLAT_NOALLOC_MAX_DIM 128
#define MFLAT_NOALLOC_MAX_K 21
#define MFLAT_NOALLOC_SCRATCH_BYTES (4u << 20)
MFLAT_API mflat_status_t mflat_flat_search_noalloc(mflat_flat_index_t*, const float* d_queries,
        int m, int k, int32_t* d_out_ids, float* d_out_distances, int* out_k_used, void* stream);

/* Device-side timing of the most recent search (milliseconds, CUDA events
 * on the launching stream) once enabled with mflat_flat_set_timing(h, 1).
 * Searches only record their events; the times are read when asked for, so
 * timing does not hold back a stream of asynchronous searches. */
typedef struct {
    float total_ms;                 /* first to last kernel of the search          */
    float screen_ms;                /* tensor-core distance + fused top-k kernel   */
    float select_ms;                /* merge + exact re-rank kernel                */
    int   screen_launches;          /* kernels of this library in the search       */
    int   launches;
    int   fallback_queries;         /* queries that needed the exact full scan     */
} mflat_timing_t;
MFLAT_API mflat_status_t mflat_flat_set_timing(mflat_flat_index_t*, int enable);
MFLAT_API mflat_status_t mflat_flat_last_timing(const mflat_flat_index_t*, mflat_timing_t* out);
/* Additive (no counterpart in the reference): the field-wise sums over every
 * search since timing was last enabled, and their number. */
MFLAT_API mflat_status_t mflat_flat_timing_sum(const mflat_flat_index_t*, mflat_timing_t* out,
                                               int* n_searches);

/* k-means assignment step (CoarseQuantizer, reference src/Internal.h:321-359
 * and src/CoarseQuantizer.mm:122-130): out_assign[i] = argmin_c sqL2_f32(p_i, c)
 * with the reference's fp32 sequential sqL2 and strict '<' (lowest centroid
 * wins a tie), bit-exact.  Host pointers; runs on `device` (-1 = default). */
MFLAT_API mflat_status_t mflat_kmeans_assign(const float* points, int n, const float* centroids,
        int ncentroids, int dim, int32_t* out_assign, int device);
MFLAT_API mflat_status_t mflat_kmeans_assign_device(const float* d_points, int n,
        const float* d_centroids, int ncentroids, int dim, int32_t* d_out_assign,
        int device, void* stream);

/* Row sharding over several GPUs, one process (or thread) per GPU.  Every
 * rank holds rows [id_base, id_base + size) of the database in its own index;
 * after mflat_flat_set_shard, mflat_flat_search on each rank computes the
 * rank's top-k, all-gathers the (distance, id) candidates over NCCL and
 * merges them on the device, so every rank returns the global result.  All
 * ranks must call search collectively with the same queries, m and k. */
#define MFLAT_COMM_ID_BYTES 128
MFLAT_API mflat_status_t mflat_comm_unique_id(uint8_t out_id[MFLAT_COMM_ID_BYTES]);
MFLAT_API mflat_status_t mflat_flat_set_shard(mflat_flat_index_t*, int rank, int world,
        const uint8_t comm_id[MFLAT_COMM_ID_BYTES], int64_t id_base);

/* IVF coarse layer: k-means training, CSR inverted-list scaffold, cell probing.
 * The reference has this only as an internal C++ class (src/CoarseQuantizer.h:
 * 27-75, used by its IVF indexes); these entries expose the same operations
 * to FFI callers.  train: seed 12345, 256 training points per centroid,
 * `iters` iterations, all on the device (data: host, n x dim, already
 * metric-normalised); nlist is clamped to n.  csr: cell_start[nlist + 1]
 * offsets and reordered_ids[n] (point ids grouped by cell, ascending within a
 * cell); NULL outputs are skipped.  probe: nearest-first cell ids, m x nprobe,
 * nprobe <= MFLAT_MAX_K.  Calls on one handle are serialised. */
typedef struct mflat_coarse mflat_coarse_t;
MFLAT_API mflat_coarse_t* mflat_coarse_create(int dim, int device, mflat_status_t* out_status);
MFLAT_API void mflat_coarse_free(mflat_coarse_t*);
MFLAT_API mflat_status_t mflat_coarse_train(mflat_coarse_t*, const float* data, int n, int nlist,
        int iters);
MFLAT_API int mflat_coarse_nlist(const mflat_coarse_t*);
MFLAT_API int mflat_coarse_size(const mflat_coarse_t*);
MFLAT_API int mflat_coarse_dim(const mflat_coarse_t*);
MFLAT_API mflat_status_t mflat_coarse_centroids(const mflat_coarse_t*, float* out_centroids);
MFLAT_API mflat_status_t mflat_coarse_csr(const mflat_coarse_t*, int32_t* out_cell_start,
        int32_t* out_reordered_ids);
MFLAT_API mflat_status_t mflat_coarse_probe(mflat_coarse_t*, const float* queries, int m,
        int nprobe, int32_t* out_cells);
/* Sharded training over several GPUs, one process (or thread) per GPU: this
 * handle holds global rows [row_offsets[rank], row_offsets[rank + 1]) and
 * train() receives only those (n = that count); every rank calls train with
 * the same nlist and iters.  The ranks all-gather per-cell double sums and
 * counts over NCCL each iteration and add them in rank order: every rank gets
 * the same centroids and the same global CSR (reordered ids are global).
 * world = 1 turns sharding off.  row_offsets has world + 1 entries. */
MFLAT_API mflat_status_t mflat_coarse_set_shard(mflat_coarse_t*, int rank, int world,
        const uint8_t comm_id[MFLAT_COMM_ID_BYTES], const int64_t* row_offsets);

/* Persistence of a flat index (the reference persists only its graph index:
 * GraphIndex::save / load, src/GraphIndex.mm:424-452, 'MFGR' header; this is
 * the same style for the flat index).  File: int32 header {0x4d46464c 'MFFL',
 * version 1, dim, metric, storage, n, 0, 0}, then n x dim stored elements --
 * fp32, or the fp16 / bf16 bit patterns -- little-endian.  A loaded index is
 * identical to the saved one (same rows, norms and results).
 * save: NULL h / path -> NULL_ARG; I/O failure -> MFLAT_ERR_IO.
 * load: a new handle on `device` (-1 = default) with the file's dim, metric
 * and storage; NULL path -> NULL_ARG; unreadable or malformed file ->
 * MFLAT_ERR_IO (and NULL). */
MFLAT_API mflat_status_t mflat_flat_save(const mflat_flat_index_t*, const char* path);
MFLAT_API mflat_flat_index_t* mflat_flat_load(const char* path, int device,
                                              mflat_status_t* out_status);

#ifdef __cplusplus
}
#endif
#endif /* MFLAT_H */
