/* mflat_oracle.c -- CPU oracle (TEST INFRASTRUCTURE ONLY; see mflat_oracle.h).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).  The fp32
 * routines must not be contracted into FMAs: the reference's Distance.h
 * contract is "multiply, round, add, round" in index order.
 */
#include "mflat_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Distance.h:26-30 */
float mfo_dot_f32(const float* a, const float* b, int dim) {
    float acc = 0.0f;
    for (int c = 0; c < dim; ++c) acc += a[c] * b[c];
    return acc;
}

/* Distance.h:33-37 */
float mfo_sq_l2_f32(const float* a, const float* b, int dim) {
    float acc = 0.0f;
    for (int c = 0; c < dim; ++c) {
        float e = a[c] - b[c];
        acc += e * e;
    }
    return acc;
}

/* Distance.h:40-47 */
void mfo_row_sq_norms(const float* v, int64_t n, int dim, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        const float* row = v + i * (int64_t)dim;
        double s = 0.0;
        for (int c = 0; c < dim; ++c) s += (double)row[c] * row[c];
        out[i] = (float)s;
    }
}

/* Distance.h:50-60 */
void mfo_normalize_rows(float* v, int64_t n, int dim) {
    for (int64_t i = 0; i < n; ++i) {
        float* row = v + i * (int64_t)dim;
        double s = 0.0;
        for (int c = 0; c < dim; ++c) s += (double)row[c] * row[c];
        if (s > 0.0) {
            const float inv = (float)(1.0 / sqrt(s));
            for (int c = 0; c < dim; ++c) row[c] *= inv;
        }
    }
}

/* fp64 evaluation of the metric formula over fp32 inputs, index order. */
static double score_f64(int metric, const float* q, const float* x, int dim) {
    double acc = 0.0;
    if (metric == MFO_L2) {
        for (int c = 0; c < dim; ++c) {
            const double e = (double)q[c] - (double)x[c];
            acc += e * e;
        }
        return -acc;                       /* larger = nearer (Distance.h:67-69) */
    }
    for (int c = 0; c < dim; ++c) acc += (double)q[c] * (double)x[c];
    return acc;
}

/* Insertion into an ascending list (index 0 = worst kept), strict '>' so a
 * later (higher) id never displaces an equal score: FlatIndex.mm:272-281. */
#define INSERT_ASC(T, best, bid, k, s, id)                                  \
    do {                                                                    \
        if ((s) > (best)[0]) {                                              \
            int pos_ = 0;                                                   \
            while (pos_ + 1 < (k) && (s) > (best)[pos_ + 1]) {              \
                (best)[pos_] = (best)[pos_ + 1];                            \
                (bid)[pos_] = (bid)[pos_ + 1];                              \
                ++pos_;                                                     \
            }                                                               \
            (best)[pos_] = (s);                                             \
            (bid)[pos_] = (id);                                             \
        }                                                                   \
    } while (0)

static int clamp_k(int k, int kmax) {
    if (k < 1) k = 1;
    if (k > kmax) k = kmax;
    return k;
}

int mfo_flat_search_f64(const float* db, int64_t n, int dim, int metric,
                        const float* q, int64_t m, int k, int kmax,
                        int32_t* out_ids, float* out_dist) {
    if (m <= 0 || dim <= 0) return 0;
    k = clamp_k(k, kmax);
    const float empty = metric == MFO_L2 ? INFINITY : -INFINITY;
#pragma omp parallel
    {
        double* best = (double*)malloc(sizeof(double) * (size_t)k);
        int32_t* bid = (int32_t*)malloc(sizeof(int32_t) * (size_t)k);
#pragma omp for schedule(dynamic, 4)
        for (int64_t qi = 0; qi < m; ++qi) {
            const float* qv = q + qi * (int64_t)dim;
            for (int i = 0; i < k; ++i) { best[i] = -INFINITY; bid[i] = -1; }
            for (int64_t j = 0; j < n; ++j) {
                const double s = score_f64(metric, qv, db + j * (int64_t)dim, dim);
                INSERT_ASC(double, best, bid, k, s, (int32_t)j);
            }
            for (int i = 0; i < k; ++i) {
                const int src = k - 1 - i;
                out_ids[qi * k + i] = bid[src];
                if (bid[src] < 0) out_dist[qi * k + i] = empty;
                else out_dist[qi * k + i] = (float)(metric == MFO_L2 ? -best[src] : best[src]);
            }
        }
        free(best);
        free(bid);
    }
    return k;
}

int mfo_flat_search_cpusearch(const float* db, int64_t n, int dim, int metric,
                              const float* q, int64_t m, int k, int kmax,
                              int32_t* out_ids, float* out_dist) {
    if (m <= 0 || dim <= 0) return 0;
    k = clamp_k(k, kmax);
#pragma omp parallel
    {
        float* best = (float*)malloc(sizeof(float) * (size_t)k);
        int32_t* bid = (int32_t*)malloc(sizeof(int32_t) * (size_t)k);
#pragma omp for schedule(dynamic, 4)
        for (int64_t qi = 0; qi < m; ++qi) {
            const float* qv = q + qi * (int64_t)dim;
            for (int i = 0; i < k; ++i) { best[i] = -INFINITY; bid[i] = -1; }
            for (int64_t j = 0; j < n; ++j) {
                const float* xv = db + j * (int64_t)dim;
                /* Distance.h:67-69 score() */
                const float s = metric == MFO_L2 ? -mfo_sq_l2_f32(qv, xv, dim)
                                                 : mfo_dot_f32(qv, xv, dim);
                INSERT_ASC(float, best, bid, k, s, (int32_t)j);
            }
            for (int i = 0; i < k; ++i) {
                const int src = k - 1 - i;
                out_ids[qi * k + i] = bid[src];
                /* Distance.h:71 scoreToValue; empty slots keep -inf -> +inf for L2 */
                out_dist[qi * k + i] = metric == MFO_L2 ? -best[src] : best[src];
            }
        }
        free(best);
        free(bid);
    }
    return k;
}

void mfo_kmeans_assign_f32(const float* points, int64_t n, const float* cents,
                           int ncent, int dim, int32_t* out) {
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t i = 0; i < n; ++i) {
        const float* v = points + i * (int64_t)dim;
        float best = INFINITY;
        int bestC = 0;
        for (int c = 0; c < ncent; ++c) {
            const float dd = mfo_sq_l2_f32(v, cents + (int64_t)c * dim, dim);
            if (dd < best) { best = dd; bestC = c; }
        }
        out[i] = bestC;
    }
}

/* Rank (dist, id) pairs: nearer first, then lower id; -1 ids last. */
static int better(int metric, float da, int32_t ia, float db, int32_t ib) {
    if (ia < 0) return 0;
    if (ib < 0) return 1;
    if (da != db) return metric == MFO_L2 ? (da < db) : (da > db);
    return ia < ib;
}

void mfo_merge_shards(const int32_t* ids, const float* dist, int nshard,
                      int64_t m, int k, int metric,
                      int32_t* out_ids, float* out_dist) {
    const float empty = metric == MFO_L2 ? INFINITY : -INFINITY;
#pragma omp parallel
    {
        int* head = (int*)malloc(sizeof(int) * (size_t)nshard);
#pragma omp for
        for (int64_t qi = 0; qi < m; ++qi) {
            for (int p = 0; p < nshard; ++p) head[p] = 0;
            for (int j = 0; j < k; ++j) {
                int bp = -1;
                for (int p = 0; p < nshard; ++p) {
                    if (head[p] >= k) continue;
                    const int64_t o = ((int64_t)p * m + qi) * k + head[p];
                    if (ids[o] < 0) continue;
                    if (bp < 0) { bp = p; continue; }
                    const int64_t ob = ((int64_t)bp * m + qi) * k + head[bp];
                    if (better(metric, dist[o], ids[o], dist[ob], ids[ob])) bp = p;
                }
                if (bp < 0) {
                    out_ids[qi * k + j] = -1;
                    out_dist[qi * k + j] = empty;
                } else {
                    const int64_t ob = ((int64_t)bp * m + qi) * k + head[bp];
                    out_ids[qi * k + j] = ids[ob];
                    out_dist[qi * k + j] = dist[ob];
                    head[bp]++;
                }
            }
        }
        free(head);
    }
}

/* Exact fp64 scores of (query, row) pairs, the same evaluation as
 * mfo_flat_search_f64: out[i] = score(q[qi[i]], rows[ri[i]]), larger = nearer
 * (-sqL2 for metric 0, dot otherwise).  Used by the screened oracle at the
 * benchmarked sizes (oracle/scale.py). */
void mfo_score_pairs_f64(const float* rows, int dim, int metric, const float* q,
                         const int64_t* qi, const int64_t* ri, int64_t npairs, double* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < npairs; ++i)
        out[i] = score_f64(metric == MFO_L2 ? MFO_L2 : MFO_IP, q + qi[i] * (int64_t)dim,
                           rows + ri[i] * (int64_t)dim, dim);
}

/* mfo_kmeans_assign_f32 restricted to a candidate list per point (ascending
 * centroid ids, CSR cand_ptr[n+1] / cand_ids): the same sequential fp32 sqL2
 * and strict '<' scan, so when every centroid that can reach the minimum is
 * listed the result equals the full scan's. */
void mfo_kmeans_assign_cand(const float* points, int64_t n, const float* cents, int dim,
                            const int64_t* cand_ptr, const int32_t* cand_ids, int32_t* out) {
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t i = 0; i < n; ++i) {
        const float* v = points + i * (int64_t)dim;
        float best = INFINITY;
        int bestC = 0;
        for (int64_t j = cand_ptr[i]; j < cand_ptr[i + 1]; ++j) {
            const int c = cand_ids[j];
            const float dd = mfo_sq_l2_f32(v, cents + (int64_t)c * dim, dim);
            if (dd < best) { best = dd; bestC = c; }
        }
        out[i] = bestC;
    }
}
