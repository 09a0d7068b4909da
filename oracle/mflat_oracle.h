/* mflat_oracle.h -- CPU oracle for the exact flat-search path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs use it, and only as the checker.
 *
 * It restates, in plain C, the semantics the reference's flat path is defined
 * by (metal-flat, paths relative to that project):
 *   - src/Distance.h:26-81   dot / sqL2 (float accumulation), rowSqNorms and
 *                            normalizeRows (double accumulation), score order
 *                            "larger is nearer", empty sentinels;
 *   - src/FlatIndex.mm:259-290 cpuSearch: strict '>' insertion while scanning
 *                            ids in ascending order, so among equal scores
 *                            the lowest id ranks nearer; output nearest-first;
 *   - src/FlatIndex.mm:297-330 k clamp to [1, kMaxK], empty database result;
 *   - src/CoarseQuantizer.mm:122-130 (via Distance.h:33-37) the k-means
 *                            assignment: sequential fp32 sqL2 argmin, strict
 *                            '<', ties to the lowest centroid.
 * The exact oracle evaluates the same formulas in fp64 over the stored fp32
 * vectors (ties to the lowest id).  Compiled with -ffp-contract=off so that
 * the fp32 routines never fuse a multiply and an add.
 */
#ifndef MFLAT_ORACLE_H
#define MFLAT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { MFO_L2 = 0, MFO_IP = 1, MFO_COSINE = 2 };

/* Distance.h:26-30 / :33-37 -- float accumulation, index order. */
float mfo_dot_f32(const float* a, const float* b, int dim);
float mfo_sq_l2_f32(const float* a, const float* b, int dim);

/* Distance.h:40-47 -- per-row sum of squares in double, cast to float. */
void mfo_row_sq_norms(const float* v, int64_t n, int dim, float* out);

/* Distance.h:50-60 -- in place; rows with zero norm are left untouched. */
void mfo_normalize_rows(float* v, int64_t n, int dim);

/* Exact brute force: fp64 evaluation of sqL2 (metric 0) or dot (1, 2) over
 * the given fp32 vectors.  For metric 2 the caller passes rows already
 * normalised by mfo_normalize_rows (that is what the index stores).
 * Writes m*k_used ids/distances nearest-first, ties to the lowest id, -1 /
 * (+inf for L2, -inf otherwise) padding when n < k.  k_used = min(k, kmax).
 * Returns k_used.  Multithreaded over queries (OpenMP). */
int mfo_flat_search_f64(const float* db, int64_t n, int dim, int metric,
                        const float* q, int64_t m, int k, int kmax,
                        int32_t* out_ids, float* out_dist);

/* Same selection, fp32 Distance.h::score() (FlatIndex.mm:259-290 cpuSearch).
 * Used to pin the exact oracle against the reference's own CPU semantics. */
int mfo_flat_search_cpusearch(const float* db, int64_t n, int dim, int metric,
                              const float* q, int64_t m, int k, int kmax,
                              int32_t* out_ids, float* out_dist);

/* CoarseQuantizer.mm:122-130: out[i] = argmin_c sqL2_f32(p_i, c), strict '<'
 * so the lowest centroid index wins a tie.  Multithreaded over points. */
void mfo_kmeans_assign_f32(const float* points, int64_t n, const float* cents,
                           int ncent, int dim, int32_t* out);

/* k-means training of CoarseQuantizer::train (src/Internal.h:257-359,
 * src/CoarseQuantizer.mm:104-143): seeds, 256-points-per-centroid subset,
 * `iters` (assign, double means, reseed) iterations, final assignment and CSR.
 * out_cents[nlist*dim], out_assign[n], out_cell_start[nlist+1],
 * out_reordered[n] (the last three may be NULL).  Returns nlist (clamped to
 * n) or -1 on bad arguments.  mflat_oracle_kmeans.cpp. */
int mfo_kmeans_train(const float* data, int64_t n, int dim, int nlist_req, int iters,
                     int max_points_per_centroid, float* out_cents, int32_t* out_assign,
                     int32_t* out_cell_start, int32_t* out_reordered);
/* The same over `world` row shards (rank r holds global rows
 * [offsets[r], offsets[r+1])): per-cell sums per rank, then ranks added in order. */
int mfo_kmeans_train_sharded(const float* data, int64_t n, int dim, int nlist_req, int iters,
                             int max_points_per_centroid, int world, const int64_t* offsets,
                             float* out_cents, int32_t* out_assign, int32_t* out_cell_start,
                             int32_t* out_reordered);
/* The training's seed permutation of 0..n-1 (mt19937(seed), Fisher-Yates). */
void mfo_kmeans_seed_permutation(int64_t n, uint32_t seed, int32_t* perm);

/* Merge P per-shard result lists (each m x k, nearest-first, ids already
 * global) into one m x k list with the same order and tie rule. */
void mfo_merge_shards(const int32_t* ids, const float* dist, int nshard,
                      int64_t m, int k, int metric,
                      int32_t* out_ids, float* out_dist);

/* Exact fp64 scores of listed (query, row) pairs (score order of
 * mfo_flat_search_f64; metric 2 = 1 on normalised inputs). */
void mfo_score_pairs_f64(const float* rows, int dim, int metric, const float* q,
                         const int64_t* qi, const int64_t* ri, int64_t npairs, double* out);

/* mfo_kmeans_assign_f32 over a per-point candidate list (CSR, ascending ids). */
void mfo_kmeans_assign_cand(const float* points, int64_t n, const float* cents, int dim,
                            const int64_t* cand_ptr, const int32_t* cand_ids, int32_t* out);

#ifdef __cplusplus
}
#endif
#endif
