// SPDX-License-Identifier: Apache-2.0
// FlatIndex.cpp -- host engine of the exact flat index.
//
// Keeps the reference's FlatIndex contract (include/metalflat/FlatIndex.h:
// 37-77, src/FlatIndex.mm:191-421): argument handling, the k clamp with a
// one-time warning (:297-305), the empty-database result (:325-330) and the
// nearest-first result layout.  Everything that touches vectors runs on the
// GPU through the extern "C" CUDA layer (mflat_cuda.h); there is no CPU
// search path.
#include <algorithm>
#include <cmath>
#include <new>
#include <stdexcept>
#include <string>

#include "../cuda/mflat_cuda.h"
#include "Log_internal.h"
#include "metalflat/FlatIndex.h"

namespace mflat {

namespace {

// Map a CUDA-layer status to the exception the C ABI turns into a status code.
void raise_status(int st, const char* op) {
    if (st == 0) return;
    const std::string msg = std::string(op) + ": " + mflat_cu_last_error();
    if (st == 3) {
        MFLAT_LOG_ERROR("%s", msg.c_str());
        throw std::bad_alloc();
    }
    if (st == 2) throw std::invalid_argument(msg);
    MFLAT_LOG_ERROR("%s", msg.c_str());
    throw DeviceError(msg);
}

}  // namespace

struct FlatIndex::Impl {
    int dim = 0;
    Metric metric = Metric::L2;
    Storage storage = Storage::FP32;
    int device = -1;
    mflat_cu_index_t* dev = nullptr;
    bool warnedK = false;

    ~Impl() { mflat_cu_index_destroy(dev); }

    int clampK(int k) {
        if (k < 1) k = 1;
        if (k > kMaxK) {
            if (!warnedK) {
                MFLAT_LOG_WARN("k=%d clamped to kMaxK=%d", k, kMaxK);
                warnedK = true;
            }
            k = kMaxK;
        }
        return k;
    }

    mflat_cu_index_t* need() const {
        if (!dev) throw DeviceError("no usable CUDA device for this index");
        return dev;
    }
};

FlatIndex::FlatIndex(int dim, Metric metric) : FlatIndex(dim, metric, Storage::FP32, -1) {}

FlatIndex::FlatIndex(int dim, Metric metric, Storage storage, int device)
    : mImpl(std::make_unique<Impl>()) {
    mImpl->dim = dim;
    mImpl->metric = metric;
    mImpl->storage = storage;
    if (dim <= 0) return;
    const int st = mflat_cu_index_create(device, dim, static_cast<int>(metric),
                                         static_cast<int>(storage), &mImpl->dev);
    if (st == 2) throw std::invalid_argument(mflat_cu_last_error());
    if (st != 0) {
        mImpl->dev = nullptr;
        MFLAT_LOG_ERROR("CUDA device unavailable (%s); index is not ready", mflat_cu_last_error());
        return;
    }
    mImpl->device = mflat_cu_index_device(mImpl->dev);
}

FlatIndex::~FlatIndex() = default;

bool FlatIndex::ready() const { return mImpl->dev != nullptr; }
int FlatIndex::size() const { return mImpl->dev ? static_cast<int>(mflat_cu_index_size(mImpl->dev)) : 0; }
int FlatIndex::dim() const { return mImpl->dim; }
Metric FlatIndex::metric() const { return mImpl->metric; }
Storage FlatIndex::storage() const { return mImpl->storage; }
int FlatIndex::device() const { return mImpl->device; }

void FlatIndex::add(const float* vectors, int n) {
    if (n <= 0 || mImpl->dim <= 0) return;
    raise_status(mflat_cu_index_add(mImpl->need(), vectors, n, 0, nullptr), "add");
}

void FlatIndex::addDevice(const float* d_vectors, int n, void* stream) {
    if (n <= 0 || mImpl->dim <= 0) return;
    raise_status(mflat_cu_index_add(mImpl->need(), d_vectors, n, 1, stream), "add");
}

void FlatIndex::reset() {
    if (mImpl->dev) raise_status(mflat_cu_index_reset(mImpl->dev), "reset");
}

SearchResult FlatIndex::search(const float* queries, int m, int k) {
    SearchResult out;
    if (m <= 0 || mImpl->dim <= 0) return out;
    k = mImpl->clampK(k);
    mflat_cu_index_t* dev = mImpl->need();
    const size_t mk = static_cast<size_t>(m) * static_cast<size_t>(k);
    out.ids.resize(mk);
    out.distances.resize(mk);
    raise_status(mflat_cu_index_search(dev, queries, m, k, out.ids.data(), out.distances.data(), 0,
                                       nullptr),
                 "search");
    return out;
}

int FlatIndex::searchDevice(const float* d_queries, int m, int k, int32_t* d_ids, float* d_dist,
                            void* stream) {
    if (m <= 0 || mImpl->dim <= 0) return 0;
    k = mImpl->clampK(k);
    raise_status(mflat_cu_index_search(mImpl->need(), d_queries, m, k, d_ids, d_dist, 1, stream),
                 "search");
    return k;
}

int FlatIndex::searchDeviceNoAlloc(const float* d_queries, int m, int k, int32_t* d_ids,
                                   float* d_dist, void* stream) {
    if (m <= 0 || mImpl->dim <= 0) return 0;
    raise_status(mflat_cu_index_search_noalloc(mImpl->need(), d_queries, m, k, d_ids, d_dist, stream),
                 "search (no-alloc)");
    return k;
}

void FlatIndex::setTiming(bool enable) {
    raise_status(mflat_cu_index_set_timing(mImpl->need(), enable ? 1 : 0), "timing");
}

SearchTiming FlatIndex::lastTiming() const {
    SearchTiming t;
    mflat_cu_timing_t c{};
    if (mImpl->dev && mflat_cu_index_last_timing(mImpl->dev, &c) == 0) {
        t.total_ms = c.total_ms;
        t.screen_ms = c.screen_ms;
        t.select_ms = c.select_ms;
        t.screen_launches = c.screen_launches;
        t.launches = c.launches;
        t.fallback_queries = c.fallback_queries;
    }
    return t;
}

void FlatIndex::setShard(int rank, int world, const uint8_t* comm_id, int64_t id_base) {
    raise_status(mflat_cu_index_set_shard(mImpl->need(), rank, world, comm_id, id_base), "shard");
}

void kmeansAssign(const float* points, int n, const float* centroids, int ncentroids, int dim,
                  int32_t* out, int device) {
    if (n <= 0) return;
    raise_status(mflat_cu_kmeans_assign(points, n, centroids, ncentroids, dim, out, device, 0, nullptr),
                 "kmeans assign");
}

}  // namespace mflat
