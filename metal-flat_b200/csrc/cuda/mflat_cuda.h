/* mflat_cuda.h -- the thin extern "C" layer between the C++ host engine
 * (FlatIndex, CoarseQuantizer) and the CUDA kernels (libmflat_cuda.so).
 *
 * Plain C types only.  Status values are the mflat_status_t codes of
 * include/mflat.h (0 ok, 2 bad argument, 3 allocation, 5 internal, 6 device).
 * Pointers flagged `on_device` are device memory on the index's device and
 * the call only enqueues on `stream`; otherwise they are host memory and the
 * call returns after the results are in host memory.
 */
#ifndef MFLAT_CUDA_H
#define MFLAT_CUDA_H

#include <stdint.h>

#if defined(_WIN32)
#  define MFLAT_CU_API
#else
#  define MFLAT_CU_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mflat_cu_index mflat_cu_index_t;

typedef struct {
    float total_ms, screen_ms, select_ms;
    int screen_launches, launches, fallback_queries;
} mflat_cu_timing_t;

/* Message of the last failure on the calling thread ("" if none). */
MFLAT_CU_API const char* mflat_cu_last_error(void);
MFLAT_CU_API int mflat_cu_device_count(void);
/* Resolve the device for a request: device >= 0 as given, else $MFLAT_DEVICE, else 0. */
MFLAT_CU_API int mflat_cu_default_device(int device);

MFLAT_CU_API int mflat_cu_index_create(int device, int dim, int metric, int storage,
                                       mflat_cu_index_t** out);
MFLAT_CU_API void mflat_cu_index_destroy(mflat_cu_index_t* ix);
MFLAT_CU_API int64_t mflat_cu_index_size(const mflat_cu_index_t* ix);
MFLAT_CU_API int mflat_cu_index_device(const mflat_cu_index_t* ix);
MFLAT_CU_API int mflat_cu_index_add(mflat_cu_index_t* ix, const float* vectors, int64_t n,
                                    int on_device, void* stream);
MFLAT_CU_API int mflat_cu_index_reset(mflat_cu_index_t* ix);
/* Persistence.  export_rows copies stored rows [start, start + count) to host
 * memory in storage precision without padding (fp32: the ingested values;
 * fp16 / bf16: the stored bit patterns, 2 bytes per element).  add_raw appends
 * host rows in that same form as they are (no Cosine normalisation), so an
 * exported index reloads to the identical device state. */
MFLAT_CU_API int mflat_cu_index_export_rows(mflat_cu_index_t* ix, int64_t start, int64_t count,
                                            void* host_out);
MFLAT_CU_API int mflat_cu_index_add_raw(mflat_cu_index_t* ix, const void* host_rows, int64_t n);
MFLAT_CU_API int mflat_cu_index_storage(const mflat_cu_index_t* ix);
/* Writes m rows of k_out (ids, distances), nearest-first, -1 / +-inf padded. */
MFLAT_CU_API int mflat_cu_index_search(mflat_cu_index_t* ix, const float* queries, int m,
                                       int k_out, int32_t* out_ids, float* out_dist,
                                       int on_device, void* stream);
/* Same search with device pointers, but every per-call scratch buffer comes
 * from one fixed per-device array inside the library (no device allocation);
 * m <= 128, dim <= 128, k <= 21, fp32 storage.  See noalloc.cu. */
MFLAT_CU_API int mflat_cu_index_search_noalloc(mflat_cu_index_t* ix, const float* d_queries, int m,
                                               int k_out, int32_t* d_ids, float* d_dist,
                                               void* stream);
MFLAT_CU_API int mflat_cu_index_set_timing(mflat_cu_index_t* ix, int enable);
MFLAT_CU_API int mflat_cu_index_last_timing(const mflat_cu_index_t* ix, mflat_cu_timing_t* out);
/* Sums of every search's timing since timing was last enabled (waits for the
 * searches still running); *n_searches = how many. */
MFLAT_CU_API int mflat_cu_index_timing_sum(const mflat_cu_index_t* ix, mflat_cu_timing_t* out,
                                           int* n_searches);

/* The on-device merge of a sharded search on its own: d_gids / d_gdist hold
 * `world` lists per query ([world][m][k], each nearest-first, ids global, -1
 * padded); writes the merged [m][k] (nearer first, then lower id).  Device
 * pointers, enqueued on `stream`.  world rounded up to a power of two times
 * k times 12 bytes must fit in 200 KB. */
MFLAT_CU_API int mflat_cu_merge_ranks(const int32_t* d_gids, const float* d_gdist, int world, int m,
                                      int k, int metric, int32_t* d_out_ids, float* d_out_dist,
                                      void* stream);

/* k-means assignment step: bit-exact argmin of the fp32 sequential sqL2. */
MFLAT_CU_API int mflat_cu_kmeans_assign(const float* points, int64_t n, const float* centroids,
                                        int ncentroids, int dim, int32_t* out_assign,
                                        int device, int on_device, void* stream);

/* k-means training session (CoarseQuantizer::train).  create uploads this
 * rank's points (or borrows device points) and gathers its training rows
 * (train_rows: local row indices, NULL when train_n == n = all rows in
 * order); the host draws the seeds, the training subset and the empty-cell
 * reseeds from its own mt19937.  Sharded training: world > 1 ranks, each with
 * a contiguous block of rows, row_offsets[world + 1] giving every rank's
 * global range, comm_id from mflat_cu_comm_unique_id; the calls marked
 * (collective) must then be made by every rank in the same order.
 *   fetch_rows (collective): global rows -> host, from their owning ranks.
 *   set_rows: centroid cells[i] = rows[i] (host data).
 *   iterate (collective): assignment of the training points + centroid means
 *     of the non-empty cells (per-rank double sums in ascending training
 *     order, added across ranks in rank order); the cells' total counts go to
 *     host_counts[nlist]; empty cells keep their centroid.
 *   finish (collective): assignment of every point + global CSR:
 *     cell_start[nlist + 1], reordered[total] (global point ids grouped by
 *     cell, ascending within a cell); host_assign gets this rank's
 *     assignments.  Output pointers may be NULL.  The CSR also stays on the
 *     device (the *_device accessors) until destroy. */
typedef struct mflat_cu_kmeans mflat_cu_kmeans_t;
MFLAT_CU_API int mflat_cu_kmeans_create(int device, int dim, const float* points, int64_t n,
                                        int on_device, const int32_t* train_rows, int64_t train_n,
                                        int nlist, int rank, int world, const uint8_t* comm_id,
                                        const int64_t* row_offsets, mflat_cu_kmeans_t** out);
MFLAT_CU_API void mflat_cu_kmeans_destroy(mflat_cu_kmeans_t* k);
MFLAT_CU_API int mflat_cu_kmeans_set_centroids(mflat_cu_kmeans_t* k, const float* host_centroids);
MFLAT_CU_API int mflat_cu_kmeans_get_centroids(mflat_cu_kmeans_t* k, float* host_out);
MFLAT_CU_API int mflat_cu_kmeans_fetch_rows(mflat_cu_kmeans_t* k, const int64_t* host_rows,
                                            int count, float* host_out);
MFLAT_CU_API int mflat_cu_kmeans_set_rows(mflat_cu_kmeans_t* k, const int32_t* host_cells,
                                          const float* host_rows, int count);
MFLAT_CU_API int mflat_cu_kmeans_iterate(mflat_cu_kmeans_t* k, int32_t* host_counts);
MFLAT_CU_API int mflat_cu_kmeans_finish(mflat_cu_kmeans_t* k, int32_t* host_assign,
                                        int32_t* host_cell_start, int32_t* host_reordered);
MFLAT_CU_API const int32_t* mflat_cu_kmeans_cell_start_device(const mflat_cu_kmeans_t* k);
MFLAT_CU_API const int32_t* mflat_cu_kmeans_reordered_device(const mflat_cu_kmeans_t* k);

/* Row sharding across ranks (NCCL). */
MFLAT_CU_API int mflat_cu_comm_unique_id(uint8_t* out_id /* 128 bytes */);
MFLAT_CU_API int mflat_cu_index_set_shard(mflat_cu_index_t* ix, int rank, int world,
                                          const uint8_t* comm_id, int64_t id_base);

#ifdef __cplusplus
}
#endif
#endif
