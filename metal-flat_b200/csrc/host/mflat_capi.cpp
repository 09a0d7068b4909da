// SPDX-License-Identifier: Apache-2.0
// mflat_capi.cpp -- the C ABI (include/mflat.h) over the C++ engine.
//
// Same shell as the reference's c/mflat.cpp:1-199 for the flat, logging and
// version entries: each handle pairs the engine with a std::mutex so calls on
// one handle are serialised; every entry point maps C++ exceptions to status
// codes (bad_alloc -> ALLOC, device failure -> DEVICE (additive), anything
// else -> INTERNAL); results are copied into caller buffers packed at stride
// k_used; the C log handler reaches the C++ sink through a trampoline.
#include <atomic>
#include <cstring>
#include <mutex>
#include <new>
#include <stdexcept>
#include <vector>

#include "../../../include/mflat.h"
#include "../cuda/mflat_cuda.h"
#include "metalflat/CoarseQuantizer.h"
#include "metalflat/FlatIndex.h"
#include "metalflat/Log.h"

using mflat::DeviceError;
using mflat::FlatIndex;
using mflat::Metric;
using mflat::SearchResult;

namespace {

Metric to_metric(mflat_metric_t m) {
    switch (m) {
        case MFLAT_METRIC_INNER_PRODUCT: return Metric::InnerProduct;
        case MFLAT_METRIC_COSINE: return Metric::Cosine;
        default: return Metric::L2;
    }
}

mflat::Storage to_storage(mflat_storage_t s) {
    switch (s) {
        case MFLAT_STORAGE_FP16: return mflat::Storage::FP16;
        case MFLAT_STORAGE_BF16: return mflat::Storage::BF16;
        default: return mflat::Storage::FP32;
    }
}

mflat_status_t emit(const SearchResult& r, int m, int32_t* out_ids, float* out_dist, int* out_k_used) {
    if (m <= 0 || r.ids.empty()) {
        if (out_k_used) *out_k_used = 0;
        return MFLAT_OK;
    }
    const int k_used = static_cast<int>(r.ids.size() / static_cast<size_t>(m));
    if (out_ids) std::memcpy(out_ids, r.ids.data(), r.ids.size() * sizeof(int32_t));
    if (out_dist) std::memcpy(out_dist, r.distances.data(), r.distances.size() * sizeof(float));
    if (out_k_used) *out_k_used = k_used;
    return MFLAT_OK;
}

std::atomic<mflat_log_handler_t> g_c_handler{nullptr};
std::atomic<void*> g_c_user{nullptr};

void c_log_trampoline(mflat::LogLevel level, const char* msg, void*) {
    if (mflat_log_handler_t h = g_c_handler.load(std::memory_order_acquire))
        h(static_cast<mflat_log_level_t>(level), msg, g_c_user.load(std::memory_order_acquire));
}

// Run `fn` and translate exceptions to status codes.
template <class Fn>
mflat_status_t guarded(Fn&& fn) {
    try {
        return fn();
    } catch (const std::bad_alloc&) {
        return MFLAT_ERR_ALLOC;
    } catch (const std::invalid_argument&) {
        return MFLAT_ERR_BAD_ARG;
    } catch (const DeviceError&) {
        return MFLAT_ERR_DEVICE;
    } catch (...) {
        return MFLAT_ERR_INTERNAL;
    }
}

mflat_status_t from_cu(int st) {
    switch (st) {
        case 0: return MFLAT_OK;
        case 2: return MFLAT_ERR_BAD_ARG;
        case 3: return MFLAT_ERR_ALLOC;
        case 5: return MFLAT_ERR_INTERNAL;
        default: return MFLAT_ERR_DEVICE;
    }
}

}  // namespace

struct mflat_flat_index {
    FlatIndex idx;
    mutable std::mutex mu;
    mflat_flat_index(int d, Metric m, mflat::Storage s, int dev) : idx(d, m, s, dev) {}
};

struct mflat_coarse {
    mflat::CoarseQuantizer cq;
    mutable std::mutex mu;
    mflat_coarse(int d, int dev) : cq(d, dev) {}
};

extern "C" {

MFLAT_API const char* mflat_version(void) { return "0.1.0"; }
MFLAT_API int mflat_max_k(void) { return MFLAT_MAX_K; }

MFLAT_API void mflat_set_log_handler(mflat_log_handler_t h, void* user) {
    g_c_user.store(user, std::memory_order_release);
    g_c_handler.store(h, std::memory_order_release);
    mflat::setLogHandler(h ? &c_log_trampoline : nullptr, nullptr);
}

MFLAT_API void mflat_set_log_level(mflat_log_level_t l) {
    mflat::setLogLevel(static_cast<mflat::LogLevel>(l));
}

MFLAT_API mflat_log_level_t mflat_log_level(void) {
    return static_cast<mflat_log_level_t>(mflat::logLevel());
}

MFLAT_API const char* mflat_status_str(mflat_status_t s) {
    switch (s) {
        case MFLAT_OK: return "ok";
        case MFLAT_ERR_NULL_ARG: return "null argument";
        case MFLAT_ERR_BAD_ARG: return "bad argument";
        case MFLAT_ERR_ALLOC: return "allocation failed";
        case MFLAT_ERR_NOT_READY: return "index not built";
        case MFLAT_ERR_INTERNAL: return "internal error";
        case MFLAT_ERR_DEVICE: return "device error";
        case MFLAT_ERR_IO: return "index file error";
    }
    return "unknown";
}

MFLAT_API mflat_flat_index_t* mflat_flat_create_ex(int dim, mflat_metric_t metric,
                                                   mflat_storage_t storage, int device,
                                                   mflat_status_t* st) {
    if (dim <= 0) {
        if (st) *st = MFLAT_ERR_BAD_ARG;
        return nullptr;
    }
    try {
        auto* h = new mflat_flat_index(dim, to_metric(metric), to_storage(storage), device);
        if (st) *st = MFLAT_OK;
        return h;
    } catch (const std::bad_alloc&) {
        if (st) *st = MFLAT_ERR_ALLOC;
    } catch (const std::invalid_argument&) {
        if (st) *st = MFLAT_ERR_BAD_ARG;
    } catch (...) {
        if (st) *st = MFLAT_ERR_INTERNAL;
    }
    return nullptr;
}

MFLAT_API mflat_flat_index_t* mflat_flat_create(int dim, mflat_metric_t metric, mflat_status_t* st) {
    return mflat_flat_create_ex(dim, metric, MFLAT_STORAGE_FP32, -1, st);
}

MFLAT_API void mflat_flat_free(mflat_flat_index_t* h) { delete h; }
MFLAT_API int mflat_flat_ready(const mflat_flat_index_t* h) { return (h && h->idx.ready()) ? 1 : 0; }
MFLAT_API int mflat_flat_size(const mflat_flat_index_t* h) { return h ? h->idx.size() : 0; }
MFLAT_API int mflat_flat_dim(const mflat_flat_index_t* h) { return h ? h->idx.dim() : 0; }
MFLAT_API int mflat_flat_storage(const mflat_flat_index_t* h) {
    return h ? static_cast<int>(h->idx.storage()) : 0;
}
MFLAT_API int mflat_flat_device(const mflat_flat_index_t* h) { return h ? h->idx.device() : -1; }

MFLAT_API mflat_status_t mflat_flat_add(mflat_flat_index_t* h, const float* v, int n) {
    if (!h || !v) return MFLAT_ERR_NULL_ARG;
    if (n < 0) return MFLAT_ERR_BAD_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        h->idx.add(v, n);
        return MFLAT_OK;
    });
}

MFLAT_API mflat_status_t mflat_flat_add_device(mflat_flat_index_t* h, const float* v, int n,
                                               void* stream) {
    if (!h || !v) return MFLAT_ERR_NULL_ARG;
    if (n < 0) return MFLAT_ERR_BAD_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        h->idx.addDevice(v, n, stream);
        return MFLAT_OK;
    });
}

MFLAT_API mflat_status_t mflat_flat_reset(mflat_flat_index_t* h) {
    if (!h) return MFLAT_ERR_NULL_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        h->idx.reset();
        return MFLAT_OK;
    });
}

MFLAT_API mflat_status_t mflat_flat_search(mflat_flat_index_t* h, const float* q, int m, int k,
                                           int32_t* oi, float* od, int* ok) {
    if (!h || !q) return MFLAT_ERR_NULL_ARG;
    if (m < 0 || k < 1) return MFLAT_ERR_BAD_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        if (oi && od) {      // both outputs given: the results go straight into them
            const int used = h->idx.searchInto(q, m, k, oi, od);
            if (ok) *ok = used;
            return MFLAT_OK;
        }
        return emit(h->idx.search(q, m, k), m, oi, od, ok);
    });
}

MFLAT_API mflat_status_t mflat_flat_search_device(mflat_flat_index_t* h, const float* q, int m,
                                                  int k, int32_t* oi, float* od, int* ok,
                                                  void* stream) {
    if (!h || !q) return MFLAT_ERR_NULL_ARG;
    if (m < 0 || k < 1) return MFLAT_ERR_BAD_ARG;
    if (m > 0 && (!oi || !od)) return MFLAT_ERR_NULL_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        const int used = h->idx.searchDevice(q, m, k, oi, od, stream);
        if (ok) *ok = used;
        return MFLAT_OK;
    });
}

MFLAT_API mflat_status_t mflat_flat_search_noalloc(mflat_flat_index_t* h, const float* q, int m,
                                                   int k, int32_t* oi, float* od, int* ok,
                                                   void* stream) {
    // a null query pointer is accepted for m == 0, as the device layer does
    if (!h || (!q && m > 0)) return MFLAT_ERR_NULL_ARG;
    if (m < 0 || k < 1) return MFLAT_ERR_BAD_ARG;
    if (m > 0 && (!oi || !od)) return MFLAT_ERR_NULL_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        const int used = h->idx.searchDeviceNoAlloc(q, m, k, oi, od, stream);
        if (ok) *ok = used;
        return MFLAT_OK;
    });
}

MFLAT_API mflat_status_t mflat_flat_set_timing(mflat_flat_index_t* h, int enable) {
    if (!h) return MFLAT_ERR_NULL_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        h->idx.setTiming(enable != 0);
        return MFLAT_OK;
    });
}

MFLAT_API mflat_status_t mflat_flat_timing_sum(const mflat_flat_index_t* h, mflat_timing_t* out,
                                               int* n_searches) {
    if (!h || !out) return MFLAT_ERR_NULL_ARG;
    int n = 0;
    const mflat::SearchTiming t = h->idx.timingSum(&n);
    out->total_ms = t.total_ms;
    out->screen_ms = t.screen_ms;
    out->select_ms = t.select_ms;
    out->screen_launches = t.screen_launches;
    out->launches = t.launches;
    out->fallback_queries = t.fallback_queries;
    if (n_searches) *n_searches = n;
    return MFLAT_OK;
}

MFLAT_API mflat_status_t mflat_flat_last_timing(const mflat_flat_index_t* h, mflat_timing_t* out) {
    if (!h || !out) return MFLAT_ERR_NULL_ARG;
    const mflat::SearchTiming t = h->idx.lastTiming();
    out->total_ms = t.total_ms;
    out->screen_ms = t.screen_ms;
    out->select_ms = t.select_ms;
    out->screen_launches = t.screen_launches;
    out->launches = t.launches;
    out->fallback_queries = t.fallback_queries;
    return MFLAT_OK;
}

MFLAT_API mflat_status_t mflat_kmeans_assign(const float* points, int n, const float* centroids,
                                             int ncentroids, int dim, int32_t* out_assign,
                                             int device) {
    if (!points || !centroids || !out_assign) return MFLAT_ERR_NULL_ARG;
    if (n < 0 || ncentroids < 1 || dim < 1) return MFLAT_ERR_BAD_ARG;
    return guarded([&] {
        mflat::kmeansAssign(points, n, centroids, ncentroids, dim, out_assign, device);
        return MFLAT_OK;
    });
}

MFLAT_API mflat_status_t mflat_kmeans_assign_device(const float* points, int n,
                                                    const float* centroids, int ncentroids, int dim,
                                                    int32_t* out_assign, int device, void* stream) {
    if (!points || !centroids || !out_assign) return MFLAT_ERR_NULL_ARG;
    if (n < 0 || ncentroids < 1 || dim < 1) return MFLAT_ERR_BAD_ARG;
    return from_cu(mflat_cu_kmeans_assign(points, n, centroids, ncentroids, dim, out_assign, device,
                                          1, stream));
}

MFLAT_API mflat_status_t mflat_comm_unique_id(uint8_t out_id[MFLAT_COMM_ID_BYTES]) {
    if (!out_id) return MFLAT_ERR_NULL_ARG;
    return from_cu(mflat_cu_comm_unique_id(out_id));
}

MFLAT_API mflat_status_t mflat_flat_set_shard(mflat_flat_index_t* h, int rank, int world,
                                              const uint8_t comm_id[MFLAT_COMM_ID_BYTES],
                                              int64_t id_base) {
    if (!h) return MFLAT_ERR_NULL_ARG;
    if (world < 1 || rank < 0 || rank >= world || id_base < 0) return MFLAT_ERR_BAD_ARG;
    if (world > 1 && !comm_id) return MFLAT_ERR_NULL_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        h->idx.setShard(rank, world, comm_id, id_base);
        return MFLAT_OK;
    });
}

MFLAT_API mflat_coarse_t* mflat_coarse_create(int dim, int device, mflat_status_t* st) {
    if (dim <= 0) {
        if (st) *st = MFLAT_ERR_BAD_ARG;
        return nullptr;
    }
    mflat_coarse_t* h = nullptr;
    const mflat_status_t rc = guarded([&] {
        h = new mflat_coarse(dim, device);
        return MFLAT_OK;
    });
    if (st) *st = rc;
    return rc == MFLAT_OK ? h : nullptr;
}

MFLAT_API void mflat_coarse_free(mflat_coarse_t* h) { delete h; }

MFLAT_API mflat_status_t mflat_coarse_train(mflat_coarse_t* h, const float* data, int n, int nlist,
                                            int iters) {
    if (!h || (!data && n > 0)) return MFLAT_ERR_NULL_ARG;
    if (n < 0 || nlist <= 0 || iters < 0) return MFLAT_ERR_BAD_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        h->cq.train(data, n, nlist, iters);
        return MFLAT_OK;
    });
}

MFLAT_API int mflat_coarse_nlist(const mflat_coarse_t* h) { return h ? h->cq.nlist() : 0; }
MFLAT_API int mflat_coarse_size(const mflat_coarse_t* h) { return h ? h->cq.size() : 0; }
MFLAT_API int mflat_coarse_dim(const mflat_coarse_t* h) { return h ? h->cq.dim() : 0; }

MFLAT_API mflat_status_t mflat_coarse_centroids(const mflat_coarse_t* h, float* out) {
    if (!h || !out) return MFLAT_ERR_NULL_ARG;
    std::lock_guard<std::mutex> lk(h->mu);
    if (h->cq.nlist() == 0) return MFLAT_ERR_NOT_READY;
    const auto& c = h->cq.centroids();
    std::memcpy(out, c.data(), c.size() * sizeof(float));
    return MFLAT_OK;
}

MFLAT_API mflat_status_t mflat_coarse_csr(const mflat_coarse_t* h, int32_t* cell_start,
                                          int32_t* reordered) {
    if (!h) return MFLAT_ERR_NULL_ARG;
    std::lock_guard<std::mutex> lk(h->mu);
    if (h->cq.nlist() == 0) return MFLAT_ERR_NOT_READY;
    const auto& cs = h->cq.cellStart();
    const auto& ro = h->cq.reorderedIds();
    if (cell_start) std::memcpy(cell_start, cs.data(), cs.size() * sizeof(int32_t));
    if (reordered) std::memcpy(reordered, ro.data(), ro.size() * sizeof(int32_t));
    return MFLAT_OK;
}

MFLAT_API mflat_status_t mflat_coarse_probe(mflat_coarse_t* h, const float* queries, int m,
                                            int nprobe, int32_t* out_cells) {
    if (!h || !queries || !out_cells) return MFLAT_ERR_NULL_ARG;
    if (m < 0 || nprobe < 1 || nprobe > MFLAT_MAX_K) return MFLAT_ERR_BAD_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        if (h->cq.nlist() == 0) return MFLAT_ERR_NOT_READY;
        std::vector<int32_t> probed;
        h->cq.probeCells(queries, m, nprobe, probed);
        std::memcpy(out_cells, probed.data(), probed.size() * sizeof(int32_t));
        return MFLAT_OK;
    });
}

MFLAT_API mflat_status_t mflat_coarse_set_shard(mflat_coarse_t* h, int rank, int world,
                                                const uint8_t comm_id[MFLAT_COMM_ID_BYTES],
                                                const int64_t* row_offsets) {
    if (!h) return MFLAT_ERR_NULL_ARG;
    if (world < 1 || rank < 0 || rank >= world) return MFLAT_ERR_BAD_ARG;
    if (world > 1 && (!comm_id || !row_offsets)) return MFLAT_ERR_NULL_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        h->cq.setShard(rank, world, comm_id, row_offsets);
        return MFLAT_OK;
    });
}

MFLAT_API mflat_status_t mflat_flat_save(const mflat_flat_index_t* h, const char* path) {
    if (!h || !path) return MFLAT_ERR_NULL_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->mu);
        return h->idx.save(path) ? MFLAT_OK : MFLAT_ERR_IO;
    });
}

MFLAT_API mflat_flat_index_t* mflat_flat_load(const char* path, int device, mflat_status_t* st) {
    if (!path) {
        if (st) *st = MFLAT_ERR_NULL_ARG;
        return nullptr;
    }
    int dim = 0, n = 0;
    Metric metric = Metric::L2;
    mflat::Storage storage = mflat::Storage::FP32;
    if (!mflat::readFlatFileInfo(path, dim, metric, storage, n)) {
        if (st) *st = MFLAT_ERR_IO;
        return nullptr;
    }
    mflat_flat_index_t* h = nullptr;
    const mflat_status_t rc = guarded([&] {
        h = new mflat_flat_index(dim, metric, storage, device);
        if (!h->idx.ready()) return MFLAT_ERR_DEVICE;
        return h->idx.load(path) ? MFLAT_OK : MFLAT_ERR_IO;
    });
    if (rc != MFLAT_OK) {
        delete h;
        h = nullptr;
    }
    if (st) *st = rc;
    return h;
}

}  // extern "C"
