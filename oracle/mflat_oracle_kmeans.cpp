// mflat_oracle_kmeans.cpp -- TEST INFRASTRUCTURE ONLY: CPU restatement of the
// reference's k-means training for CoarseQuantizer::train, the checker of the
// device training loop.  Never linked into the product.
//
// Restates src/Internal.h:257-359 (kmeansGpu with 256 points per centroid,
// as called from src/CoarseQuantizer.mm:118-121) and its accumulateCentroids
// (src/Internal.h:52-99), with these semantics pinned down:
//   * seed permutation: mt19937(12345) and a front-to-back Fisher-Yates pass,
//     each swap offset in [0, n-1-i] drawn as the low w bits of one engine
//     output (w = bit length of the bound), redrawn while above the bound --
//     the std::shuffle of LLVM libc++, the reference's Apple toolchain.  No
//     libc++ exists in this image, so this step is not pinned against the
//     reference's own binary;
//   * assignment: argmin of the fp32 sequential sqL2 of Distance.h:33-37,
//     strict '<' (mfo_kmeans_assign_f32);
//   * means: per cell, double sum over its points in ascending point order
//     (the single-thread order; the reference's thread-chunked sum can differ
//     in the last double bits with the host's thread count), then
//     float(sum / count); sharded training (an addition of this build) sums
//     per rank over the rank's rows, then adds the ranks' sums in rank order;
//   * empty cells, in cell order: centroid = training row rng() % trainN;
//   * CSR: cellStart = prefix sums of the final all-points histogram,
//     reorderedIds = ids grouped by cell, ascending (CoarseQuantizer.mm:134-143).
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <random>
#include <vector>

#include "mflat_oracle.h"

namespace {

uint32_t bounded(std::mt19937& g, uint32_t d) {
    int w = 0;
    while (w < 32 && (d >> w) != 0) ++w;
    const uint32_t mask = w >= 32 ? 0xffffffffu : ((1u << w) - 1u);
    uint32_t u;
    do {
        u = static_cast<uint32_t>(g()) & mask;
    } while (u > d);
    return u;
}

}  // namespace

extern "C" void mfo_kmeans_seed_permutation(int64_t n, uint32_t seed, int32_t* perm) {
    for (int64_t i = 0; i < n; ++i) perm[i] = static_cast<int32_t>(i);
    std::mt19937 g(seed);
    for (int64_t i = 0; i + 1 < n; ++i) {
        const uint32_t off = bounded(g, static_cast<uint32_t>(n - 1 - i));
        if (off) std::swap(perm[i], perm[i + off]);
    }
}

extern "C" int mfo_kmeans_train_sharded(const float* data, int64_t n, int dim, int nlist_req, int iters,
                                        int max_points_per_centroid, int world, const int64_t* offsets,
                                        float* out_cents, int32_t* out_assign,
                                        int32_t* out_cell_start, int32_t* out_reordered) {
    if (n < 1 || dim < 1 || nlist_req < 1 || world < 1) return -1;
    const int nlist = static_cast<int>(std::min<int64_t>(nlist_req, n));
    const size_t row = static_cast<size_t>(dim);
    std::mt19937 rng(12345);
    std::vector<int32_t> perm(n);
    for (int64_t i = 0; i < n; ++i) perm[i] = static_cast<int32_t>(i);
    for (int64_t i = 0; i + 1 < n; ++i) {
        const uint32_t off = bounded(rng, static_cast<uint32_t>(n - 1 - i));
        if (off) std::swap(perm[i], perm[i + off]);
    }
    std::vector<float> cents(static_cast<size_t>(nlist) * row);
    for (int c = 0; c < nlist; ++c)
        std::memcpy(&cents[c * row], data + static_cast<size_t>(perm[c % n]) * row, row * sizeof(float));

    int64_t train_n = n;
    std::vector<float> train_vec;
    const float* train = data;
    if (max_points_per_centroid > 0 && static_cast<int64_t>(max_points_per_centroid) * nlist < n) {
        train_n = static_cast<int64_t>(max_points_per_centroid) * nlist;
        train_vec.resize(static_cast<size_t>(train_n) * row);
        for (int64_t i = 0; i < train_n; ++i)
            std::memcpy(&train_vec[i * row], data + static_cast<size_t>(perm[i]) * row, row * sizeof(float));
        train = train_vec.data();
    }

    // owning rank of every training row (sharded sums: per rank, then ranks in order)
    std::vector<int> owner(train_n, 0);
    for (int64_t i = 0; i < train_n; ++i) {
        const int64_t g = train_n < n ? perm[i] : i;
        int r = 0;
        while (world > 1 && g >= offsets[r + 1]) ++r;
        owner[i] = r;
    }
    std::vector<int32_t> assign(train_n);
    std::vector<double> sums(static_cast<size_t>(world) * nlist * row);
    std::vector<int64_t> counts(nlist);
    for (int it = 0; it < iters; ++it) {
        mfo_kmeans_assign_f32(train, train_n, cents.data(), nlist, dim, assign.data());
        std::fill(sums.begin(), sums.end(), 0.0);
        std::fill(counts.begin(), counts.end(), 0);
        for (int64_t i = 0; i < train_n; ++i) {
            const int c = assign[i];
            double* s = &sums[(static_cast<size_t>(owner[i]) * nlist + c) * row];
            const float* v = train + i * row;
            for (int d = 0; d < dim; ++d) s[d] += v[d];
            ++counts[c];
        }
        for (int c = 0; c < nlist; ++c)
            if (counts[c] > 0)
                for (int d = 0; d < dim; ++d) {
                    double acc = sums[c * row + d];
                    for (int r = 1; r < world; ++r) acc += sums[(static_cast<size_t>(r) * nlist + c) * row + d];
                    cents[c * row + d] = static_cast<float>(acc / static_cast<double>(counts[c]));
                }
        for (int c = 0; c < nlist; ++c) {
            if (counts[c] == 0) {
                const int64_t r = static_cast<int64_t>(rng() % static_cast<unsigned>(train_n));
                std::memcpy(&cents[c * row], train + r * row, row * sizeof(float));
            }
        }
    }
    std::memcpy(out_cents, cents.data(), cents.size() * sizeof(float));

    std::vector<int32_t> final_assign(n);
    mfo_kmeans_assign_f32(data, n, cents.data(), nlist, dim, final_assign.data());
    if (out_assign) std::memcpy(out_assign, final_assign.data(), static_cast<size_t>(n) * 4);
    std::vector<int32_t> start(static_cast<size_t>(nlist) + 1, 0);
    for (int64_t i = 0; i < n; ++i) ++start[final_assign[i] + 1];
    for (int c = 0; c < nlist; ++c) start[c + 1] += start[c];
    if (out_cell_start) std::memcpy(out_cell_start, start.data(), start.size() * 4);
    if (out_reordered) {
        std::vector<int32_t> cursor(start.begin(), start.end() - 1);
        for (int64_t i = 0; i < n; ++i) out_reordered[cursor[final_assign[i]]++] = static_cast<int32_t>(i);
    }
    return nlist;
}

extern "C" int mfo_kmeans_train(const float* data, int64_t n, int dim, int nlist_req, int iters,
                                int max_points_per_centroid, float* out_cents, int32_t* out_assign,
                                int32_t* out_cell_start, int32_t* out_reordered) {
    const int64_t offsets[2] = {0, n};
    return mfo_kmeans_train_sharded(data, n, dim, nlist_req, iters, max_points_per_centroid, 1, offsets,
                                    out_cents, out_assign, out_cell_start, out_reordered);
}
