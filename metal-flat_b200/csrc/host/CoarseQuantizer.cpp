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
#include <climits>
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
constexpr int MFLAT_COMM_ID_BYTES_CU = 128;   // NCCL unique id (mflat_cu_comm_unique_id)

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
    int rank = 0, world = 1;                // sharded training (setShard)
    std::vector<uint8_t> commId;
    std::vector<int64_t> rowOffsets;        // [world + 1]
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

void CoarseQuantizer::setShard(int rank, int world, const uint8_t* comm_id, const int64_t* row_offsets) {
    if (world < 1 || rank < 0 || rank >= world)
        throw std::invalid_argument("CoarseQuantizer::setShard: bad rank / world");
    if (world == 1) {
        mImpl->rank = 0;
        mImpl->world = 1;
        mImpl->commId.clear();
        mImpl->rowOffsets.clear();
        return;
    }
    if (!comm_id || !row_offsets) throw std::invalid_argument("CoarseQuantizer::setShard: null argument");
    for (int r = 0; r < world; ++r)
        if (row_offsets[r] < 0 || row_offsets[r + 1] < row_offsets[r])
            throw std::invalid_argument("CoarseQuantizer::setShard: row offsets must be non-decreasing");
    mImpl->rank = rank;
    mImpl->world = world;
    mImpl->commId.assign(comm_id, comm_id + MFLAT_COMM_ID_BYTES_CU);
    mImpl->rowOffsets.assign(row_offsets, row_offsets + world + 1);
}

void CoarseQuantizer::train(const float* data, int n, int nlistReq, int iters, KmeansBackend) {
    const bool sharded = mImpl->world > 1;
    if ((!data && n > 0) || n < 0 || (!sharded && n == 0))
        throw std::invalid_argument("CoarseQuantizer::train: no points");
    if (nlistReq <= 0) throw std::invalid_argument("CoarseQuantizer::train: nlist must be positive");
    if (iters < 0) throw std::invalid_argument("CoarseQuantizer::train: negative iteration count");
    const int64_t base = sharded ? mImpl->rowOffsets[mImpl->rank] : 0;
    const int64_t total = sharded ? mImpl->rowOffsets[mImpl->world] : n;
    if (sharded && mImpl->rowOffsets[mImpl->rank + 1] - base != n)
        throw std::invalid_argument("CoarseQuantizer::train: n differs from this rank's row range");
    if (total <= 0 || total > INT32_MAX - 256) throw std::invalid_argument("CoarseQuantizer::train: bad size");
    const int dim = mImpl->dim;
    const int nlist = static_cast<int>(std::min<int64_t>(nlistReq, total));
    const size_t row = static_cast<size_t>(dim);
    const int nt = static_cast<int>(total);

    // seeds: shuffled global ids, centroid c = row perm[c % total]
    std::mt19937 rng(12345);
    std::vector<int> perm(nt);
    for (int i = 0; i < nt; ++i) perm[i] = i;
    seed_shuffle(perm, rng);

    // training subset: the first 256 * nlist shuffled ids, when fewer than all;
    // this rank trains on the ones it holds, in shuffled order
    int64_t trainN = total;
    if (static_cast<int64_t>(kMaxPointsPerCentroid) * nlist < total)
        trainN = static_cast<int64_t>(kMaxPointsPerCentroid) * nlist;
    const bool subsampled = trainN < total;
    std::vector<int32_t> localTrain;
    if (subsampled) {
        for (int64_t i = 0; i < trainN; ++i) {
            const int64_t g = perm[i];
            if (g >= base && g < base + n) localTrain.push_back(static_cast<int32_t>(g - base));
        }
    }

    mflat_cu_kmeans_destroy(mImpl->session);
    mImpl->session = nullptr;
    mImpl->coarse.reset();
    mflat_cu_kmeans_t* k = nullptr;
    check(mflat_cu_kmeans_create(mImpl->device, dim, data, n, 0, subsampled ? localTrain.data() : nullptr,
                                 subsampled ? static_cast<int64_t>(localTrain.size()) : n, nlist,
                                 mImpl->rank, mImpl->world, sharded ? mImpl->commId.data() : nullptr,
                                 sharded ? mImpl->rowOffsets.data() : nullptr, &k),
          "kmeans create");
    mImpl->session = k;

    std::vector<float> cents(static_cast<size_t>(nlist) * row);
    if (sharded) {
        std::vector<int64_t> seedRows(nlist);
        for (int c = 0; c < nlist; ++c) seedRows[c] = perm[c % nt];
        check(mflat_cu_kmeans_fetch_rows(k, seedRows.data(), nlist, cents.data()), "kmeans seeds");
    } else {
        for (int c = 0; c < nlist; ++c)
            std::memcpy(&cents[c * row], data + static_cast<size_t>(perm[c % nt]) * row, row * sizeof(float));
    }
    check(mflat_cu_kmeans_set_centroids(k, cents.data()), "kmeans seeds");

    std::vector<int32_t> counts(nlist), cells;
    std::vector<int64_t> rows;
    std::vector<float> rowData;
    for (int it = 0; it < iters; ++it) {
        check(mflat_cu_kmeans_iterate(k, counts.data()), "kmeans iteration");
        cells.clear();
        rows.clear();
        for (int c = 0; c < nlist; ++c) {
            if (counts[c] == 0) {
                const int64_t r = static_cast<int64_t>(rng() % static_cast<unsigned>(trainN));
                cells.push_back(c);
                rows.push_back(subsampled ? perm[r] : r);   // training row r, as a global row id
            }
        }
        if (!cells.empty()) {
            rowData.resize(cells.size() * row);
            const int cnt = static_cast<int>(cells.size());
            check(mflat_cu_kmeans_fetch_rows(k, rows.data(), cnt, rowData.data()), "kmeans reseed");
            check(mflat_cu_kmeans_set_rows(k, cells.data(), rowData.data(), cnt), "kmeans reseed");
        }
    }
    check(mflat_cu_kmeans_get_centroids(k, cents.data()), "kmeans centroids");

    mImpl->cellStart.assign(static_cast<size_t>(nlist) + 1, 0);
    mImpl->reorderedIds.assign(static_cast<size_t>(total), 0);
    check(mflat_cu_kmeans_finish(k, nullptr, mImpl->cellStart.data(), mImpl->reorderedIds.data()),
          "kmeans final assignment");
    mImpl->centroids = std::move(cents);
    mImpl->nlist = nlist;
    mImpl->dbCount = nt;

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
