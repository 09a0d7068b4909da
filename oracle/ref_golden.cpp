// ref_golden.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Thin extern "C" shims over the reference's OWN header-only semantics
// (metal-flat src/Distance.h, compiled in place from the reference tree by
// oracle/Makefile) and its logging unit (src/Log.cpp).  The result is
// oracle/_ref/libref_golden.so, used by tests/golden/make_golden.py to emit
// golden vectors and by the tests to pin the C restatement in
// oracle/mflat_oracle.c against the reference itself.
//
// The selection loops below restate two reference loops that live in files
// which cannot compile off Apple (they are Objective-C++ with Metal):
//   - cpuSearch, src/FlatIndex.mm:259-290 (strict '>' insertion, ascending ids,
//     reversed to nearest-first);
//   - the CPU k-means assignment, src/CoarseQuantizer.mm:122-130 (strict '<').
// Every distance they use comes from the reference's Distance.h functions.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "Distance.h"          // -I <reference>/src
#include "metalflat/Log.h"     // -I <reference>/include
#include "Log_internal.h"      // -I <reference>/src

using mflat::Metric;

static Metric toMetric(int m) {
    return m == 1 ? Metric::InnerProduct : (m == 2 ? Metric::Cosine : Metric::L2);
}

extern "C" {

void ref_row_sq_norms(const float* v, int n, int dim, float* out) {
    mflat::detail::rowSqNorms(v, n, dim, out);
}

void ref_normalize_rows(float* v, int n, int dim) {
    mflat::detail::normalizeRows(v, n, dim);
}

float ref_sq_l2(const float* a, const float* b, int dim) { return mflat::detail::sqL2(a, b, dim); }
float ref_dot(const float* a, const float* b, int dim) { return mflat::detail::dot(a, b, dim); }
float ref_l2_score_from_dot(float qn, float dn, float d) {
    return mflat::detail::l2ScoreFromDot(qn, dn, d);
}
float ref_empty_value(int metric) { return mflat::detail::emptyValue(toMetric(metric)); }

// cpuSearch (FlatIndex.mm:259-290) over Distance.h::score; k already clamped.
void ref_cpu_search(const float* db, int n, int dim, int metric, const float* q, int m,
                    int k, int32_t* ids, float* dist) {
    const Metric mt = toMetric(metric);
    std::vector<float> bestScore(k);
    std::vector<int> bestId(k);
    for (int qi = 0; qi < m; ++qi) {
        const float* qv = q + static_cast<size_t>(qi) * dim;
        for (int i = 0; i < k; ++i) { bestScore[i] = -INFINITY; bestId[i] = -1; }
        for (int j = 0; j < n; ++j) {
            const float s = mflat::detail::score(mt, qv, db + static_cast<size_t>(j) * dim, dim);
            if (s > bestScore[0]) {
                int pos = 0;
                while (pos + 1 < k && s > bestScore[pos + 1]) {
                    bestScore[pos] = bestScore[pos + 1];
                    bestId[pos] = bestId[pos + 1];
                    ++pos;
                }
                bestScore[pos] = s;
                bestId[pos] = j;
            }
        }
        for (int i = 0; i < k; ++i) {
            const int src = k - 1 - i;
            ids[static_cast<size_t>(qi) * k + i] = bestId[src];
            dist[static_cast<size_t>(qi) * k + i] = mflat::detail::scoreToValue(mt, bestScore[src]);
        }
    }
}

// CoarseQuantizer.mm:122-130 over Distance.h::sqL2.
void ref_kmeans_assign(const float* pts, int n, const float* cents, int ncent, int dim,
                       int32_t* out) {
    for (int i = 0; i < n; ++i) {
        const float* v = pts + static_cast<size_t>(i) * dim;
        float best = INFINITY;
        int bestC = 0;
        for (int c = 0; c < ncent; ++c) {
            const float dd = mflat::detail::sqL2(v, cents + static_cast<size_t>(c) * dim, dim);
            if (dd < best) { best = dd; bestC = c; }
        }
        out[i] = bestC;
    }
}

// Log.cpp behaviour probes: route messages through the reference's own sink
// logic and record what a handler sees.
static std::string gLast;
static int gLastLevel = -1;
static int gCount = 0;
static void recorder(mflat::LogLevel lvl, const char* msg, void*) {
    gLast = msg;
    gLastLevel = static_cast<int>(lvl);
    ++gCount;
}
void ref_log_install_recorder(int on) { mflat::setLogHandler(on ? &recorder : nullptr, nullptr); }
void ref_log_set_level(int l) { mflat::setLogLevel(static_cast<mflat::LogLevel>(l)); }
int ref_log_level(void) { return static_cast<int>(mflat::logLevel()); }
void ref_log_emit(int l, const char* msg) {
    mflat::detail::logf(static_cast<mflat::LogLevel>(l), "%s", msg);
}
int ref_log_count(void) { return gCount; }
int ref_log_last_level(void) { return gLastLevel; }
const char* ref_log_last(void) { return gLast.c_str(); }

}  // extern "C"
