// SPDX-License-Identifier: Apache-2.0
// CoarseQuantizer.cpp -- host engine of the IVF coarse layer.
//
// Follows the reference's CoarseQuantizer::train (src/CoarseQuantizer.mm:
// 104-159) with the kmeansGpu training loop (src/Internal.h:257-359):
//   seeds    perm = shuffle(0..n-1) with mt19937(12345); centroid c = row
//            perm[c % n] (Internal.h:262-272);
//   subset   with 256 points per centroid, the first 256 * nlist entries of
//            perm form the training set when that is fewer than n rows
//            (Internal.h:279-291);
//   loop     iters x (assignment of the training set, centroid means, empty
//            cells reseeded in cell order from row rng() % trainN) (:351-355,
//            accumulateCentroids :52-99);
//   final    assignment of all n points, CSR (CoarseQuantizer.mm:134-143) and
//            the coarse FlatIndex(dim, L2) over the centroids (:146-157).
// The per-iteration work runs on the device (kmeans_train.cu); the host keeps
// the mt19937 stream, so seeds and reseeds draw exactly as the reference's
// host code does.
#include <algorithm>
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>

#include "../cuda/mflat_cuda.h"
#include "Log_internal.h"
#include "metalflat/CoarseQuantizer.h"

namespace mflat {

namespace {

void check(int st, const char* op) {
    if (st == 0) return;
    const std::string msg = std::string(op) + ": " + mflat_cu_last_error();
    MFLAT_LOG_ERROR("%s", msg.c_str());
    if (st == 3) throw std::bad_alloc();
    if (st == 2) throw std::invalid_argument(msg);
    throw DeviceError(msg);
}

// Uniform draw in [0, d] (d >= 1) from a 32-bit engine: the low w bits of
// each output, w = bit length of d, until the value is <= d.
uint32_t draw_upto(std::mt19937& g, uint32_t d) {
    const int w = 32 - __builtin_clz(d);
    const uint32_t mask = w == 32 ? 0xffffffffu : ((1u << w) - 1u);
    for (;;) {
        const uint32_t u = static_cast<uint32_t>(g()) & mask;
        if (u <= d) return u;
    }
}

// Front-to-back Fisher-Yates: position i swaps with i + draw_upto(n - 1 - i).
void seed_shuffle(std::vector<int>& perm, std::mt19937& g) {
    const int n = static_cast<int>(perm.size());
    for (int i = 0; i + 1 < n; ++i) {
        const uint32_t j = draw_upto(g, static_cast<uint32_t>(n - 1 - i));
        if (j != 0) std::swap(perm[i], perm[i + static_cast<int>(j)]);
    }
}

constexpr int kMaxPointsPerCentroid = 256;   // faiss convention (CoarseQuantizer.mm:118-121)

}  // namespace

void kmeansSeedPermutation(int n, uint32_t seed, std::vector<int>& perm) {
    perm.resize(std::max(n, 0));
    for (int i = 0; i < n; ++i) perm[i] = i;
    std::mt19937 g(seed);
    seed_shuffle(perm, g);
}

struct CoarseQuantizer::Impl {
    int dim = 0;
    int device = -1;
    int nlist = 0;
    int dbCount = 0;
    std::vector<float> centroids;
    std::vector<int> cellStart;
    std::vector<int> reorderedIds;
    std::unique_ptr<FlatIndex> coarse;
    mflat_cu_kmeans_t* session = nullptr;   // holds the device CSR after train

    ~Impl() { mflat_cu_kmeans_destroy(session); }
};

CoarseQuantizer::CoarseQuantizer(int dim, int device) : mImpl(std::make_unique<Impl>()) {
    if (dim <= 0) throw std::invalid_argument("CoarseQuantizer: dim must be positive");
    mImpl->dim = dim;
    mImpl->device = mflat_cu_default_device(device);
}

CoarseQuantizer::~CoarseQuantizer() = default;

void CoarseQuantizer::train(const float* data, int n, int nlistReq, int iters, KmeansBackend) {
    if (!data || n <= 0) throw std::invalid_argument("CoarseQuantizer::train: no points");
    if (nlistReq <= 0) throw std::invalid_argument("CoarseQuantizer::train: nlist must be positive");
    if (iters < 0) throw std::invalid_argument("CoarseQuantizer::train: negative iteration count");
    const int dim = mImpl->dim;
    const int nlist = std::min(nlistReq, n);
    const size_t row = static_cast<size_t>(dim);

    // seeds: shuffled ids, centroid c = row perm[c % n]
    std::mt19937 rng(12345);
    std::vector<int> perm(n);
    for (int i = 0; i < n; ++i) perm[i] = i;
    seed_shuffle(perm, rng);
    std::vector<float> cents(static_cast<size_t>(nlist) * row);
    for (int c = 0; c < nlist; ++c)
        std::memcpy(&cents[c * row], data + static_cast<size_t>(perm[c % n]) * row, row * sizeof(float));

    // training subset: the first 256 * nlist shuffled ids, when fewer than n
    int64_t trainN = n;
    if (static_cast<int64_t>(kMaxPointsPerCentroid) * nlist < n)
        trainN = static_cast<int64_t>(kMaxPointsPerCentroid) * nlist;

    mflat_cu_kmeans_destroy(mImpl->session);
    mImpl->session = nullptr;
    mImpl->coarse.reset();
    mflat_cu_kmeans_t* k = nullptr;
    check(mflat_cu_kmeans_create(mImpl->device, dim, data, n, 0, trainN < n ? perm.data() : nullptr,
                                 trainN, nlist, &k),
          "kmeans create");
    mImpl->session = k;
    check(mflat_cu_kmeans_set_centroids(k, cents.data()), "kmeans seeds");

    std::vector<int32_t> counts(nlist), cells, rows;
    for (int it = 0; it < iters; ++it) {
        check(mflat_cu_kmeans_iterate(k, counts.data()), "kmeans iteration");
        cells.clear();
        rows.clear();
        for (int c = 0; c < nlist; ++c) {
            if (counts[c] == 0) {
                cells.push_back(c);
                rows.push_back(static_cast<int32_t>(rng() % static_cast<unsigned>(trainN)));
            }
        }
        check(mflat_cu_kmeans_reseed(k, cells.data(), rows.data(), static_cast<int>(cells.size())),
              "kmeans reseed");
    }
    check(mflat_cu_kmeans_get_centroids(k, cents.data()), "kmeans centroids");

    mImpl->cellStart.assign(static_cast<size_t>(nlist) + 1, 0);
    mImpl->reorderedIds.assign(n, 0);
    check(mflat_cu_kmeans_finish(k, nullptr, mImpl->cellStart.data(), mImpl->reorderedIds.data()),
          "kmeans final assignment");
    mImpl->centroids = std::move(cents);
    mImpl->nlist = nlist;
    mImpl->dbCount = n;

    mImpl->coarse = std::make_unique<FlatIndex>(dim, Metric::L2, Storage::FP32, mImpl->device);
    mImpl->coarse->add(mImpl->centroids.data(), nlist);
}

int CoarseQuantizer::dim() const { return mImpl->dim; }
int CoarseQuantizer::nlist() const { return mImpl->nlist; }
int CoarseQuantizer::size() const { return mImpl->dbCount; }
int CoarseQuantizer::device() const { return mImpl->device; }
const std::vector<float>& CoarseQuantizer::centroids() const { return mImpl->centroids; }
const std::vector<int>& CoarseQuantizer::cellStart() const { return mImpl->cellStart; }
const std::vector<int>& CoarseQuantizer::reorderedIds() const { return mImpl->reorderedIds; }
bool CoarseQuantizer::gpuReady() const { return mImpl->coarse && mImpl->coarse->ready(); }
const int32_t* CoarseQuantizer::cellBuffer() const {
    return mflat_cu_kmeans_cell_start_device(mImpl->session);
}
const int32_t* CoarseQuantizer::idBuffer() const {
    return mflat_cu_kmeans_reordered_device(mImpl->session);
}

void CoarseQuantizer::reorderPayload(const void* src, void* dst, std::size_t elemBytes) const {
    const std::vector<int>& rid = mImpl->reorderedIds;
    for (int pos = 0; pos < mImpl->dbCount; ++pos)
        std::memcpy(static_cast<char*>(dst) + static_cast<size_t>(pos) * elemBytes,
                    static_cast<const char*>(src) + static_cast<size_t>(rid[pos]) * elemBytes, elemBytes);
}

void CoarseQuantizer::probeCells(const float* queries, int m, int nprobe,
                                 std::vector<int32_t>& probed) const {
    if (!mImpl->coarse) throw std::invalid_argument("CoarseQuantizer::probeCells: not trained");
    if (nprobe < 1 || nprobe > FlatIndex::kMaxK)
        throw std::invalid_argument("CoarseQuantizer::probeCells: nprobe outside [1, 1024]");
    if (m <= 0) {
        probed.clear();
        return;
    }
    SearchResult r = mImpl->coarse->search(queries, m, nprobe);
    probed = std::move(r.ids);   // m x nprobe, nearest-first (-1 past nlist)
}

}  // namespace mflat
