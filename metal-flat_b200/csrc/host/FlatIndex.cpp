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
#include <cstdio>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

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

int FlatIndex::searchInto(const float* queries, int m, int k, int32_t* ids, float* distances) {
    if (m <= 0 || mImpl->dim <= 0) return 0;
    k = mImpl->clampK(k);
    raise_status(mflat_cu_index_search(mImpl->need(), queries, m, k, ids, distances, 0, nullptr),
                 "search");
    return k;
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

SearchTiming FlatIndex::timingSum(int* n) const {
    SearchTiming t;
    mflat_cu_timing_t c{};
    int cnt = 0;
    if (mImpl->dev && mflat_cu_index_timing_sum(mImpl->dev, &c, &cnt) == 0) {
        t.total_ms = c.total_ms;
        t.screen_ms = c.screen_ms;
        t.select_ms = c.select_ms;
        t.screen_launches = c.screen_launches;
        t.launches = c.launches;
        t.fallback_queries = c.fallback_queries;
    }
    if (n) *n = cnt;
    return t;
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

namespace {

constexpr int32_t kFlatMagic = 0x4c46464d;   // the bytes "MFFL" at the start of the file (little-endian)
constexpr int32_t kFlatVersion = 1;
constexpr size_t kIoChunkBytes = size_t(64) << 20;

struct FlatFileHeader {
    int32_t magic, version, dim, metric, storage, n, reserved0, reserved1;
};

size_t elem_bytes(Storage s) { return s == Storage::FP32 ? sizeof(float) : sizeof(uint16_t); }

// Reads and checks the header; false (with a log line) on any mismatch.
bool read_header(std::FILE* f, const char* path, FlatFileHeader& h) {
    if (std::fread(&h, sizeof h, 1, f) != 1 || h.magic != kFlatMagic) {
        MFLAT_LOG_ERROR("load %s: not a flat index file", path);
        return false;
    }
    if (h.version != kFlatVersion || h.dim <= 0 || h.n < 0 || h.metric < 0 || h.metric > 2 ||
        h.storage < 0 || h.storage > 2) {
        MFLAT_LOG_ERROR("load %s: unsupported header (version %d, dim %d, n %d)", path, h.version,
                        h.dim, h.n);
        return false;
    }
    return true;
}

}  // namespace

bool FlatIndex::save(const char* path) const {
    if (!path) return false;
    mflat_cu_index_t* dev = mImpl->need();
    std::FILE* f = std::fopen(path, "wb");
    if (!f) {
        MFLAT_LOG_ERROR("save %s: cannot open for writing", path);
        return false;
    }
    const int64_t n = mflat_cu_index_size(dev);
    const FlatFileHeader h{kFlatMagic, kFlatVersion, mImpl->dim, static_cast<int32_t>(mImpl->metric),
                           static_cast<int32_t>(mImpl->storage), static_cast<int32_t>(n), 0, 0};
    bool ok = std::fwrite(&h, sizeof h, 1, f) == 1;
    const size_t row = static_cast<size_t>(mImpl->dim) * elem_bytes(mImpl->storage);
    const int64_t chunk = std::max<int64_t>(1, static_cast<int64_t>(kIoChunkBytes / row));
    std::vector<uint8_t> buf;
    for (int64_t off = 0; ok && off < n; off += chunk) {
        const int64_t cnt = std::min(chunk, n - off);
        buf.resize(static_cast<size_t>(cnt) * row);
        const int st = mflat_cu_index_export_rows(dev, off, cnt, buf.data());
        if (st != 0) {
            std::fclose(f);
            raise_status(st, "save");
        }
        ok = std::fwrite(buf.data(), 1, buf.size(), f) == buf.size();
    }
    ok = (std::fclose(f) == 0) && ok;
    if (!ok) MFLAT_LOG_ERROR("save %s: write failed", path);
    return ok;
}

bool FlatIndex::load(const char* path) {
    if (!path) return false;
    mflat_cu_index_t* dev = mImpl->need();
    std::FILE* f = std::fopen(path, "rb");
    if (!f) {
        MFLAT_LOG_ERROR("load %s: cannot open", path);
        return false;
    }
    FlatFileHeader h{};
    if (!read_header(f, path, h)) {
        std::fclose(f);
        return false;
    }
    if (h.dim != mImpl->dim || h.metric != static_cast<int32_t>(mImpl->metric) ||
        h.storage != static_cast<int32_t>(mImpl->storage)) {
        MFLAT_LOG_ERROR("load %s: file holds dim %d metric %d storage %d, index is dim %d metric %d "
                        "storage %d", path, h.dim, h.metric, h.storage, mImpl->dim,
                        static_cast<int>(mImpl->metric), static_cast<int>(mImpl->storage));
        std::fclose(f);
        return false;
    }
    const size_t row = static_cast<size_t>(h.dim) * elem_bytes(mImpl->storage);
    // A short (truncated) file is rejected before anything is replaced, so a
    // failed load leaves the index as it was.
    const long here = std::ftell(f);
    long end = -1;
    if (here >= 0 && std::fseek(f, 0, SEEK_END) == 0) end = std::ftell(f);
    if (end < 0 || std::fseek(f, here, SEEK_SET) != 0) {
        MFLAT_LOG_ERROR("load %s: cannot determine the file size", path);
        std::fclose(f);
        return false;
    }
    const unsigned long long need = static_cast<unsigned long long>(h.n) * row;
    if (static_cast<unsigned long long>(end - here) < need) {
        MFLAT_LOG_ERROR("load %s: file holds %lld of the %llu bytes of rows its header announces",
                        path, static_cast<long long>(end - here), need);
        std::fclose(f);
        return false;
    }
    raise_status(mflat_cu_index_reset(dev), "load");
    const int64_t chunk = std::max<int64_t>(1, static_cast<int64_t>(kIoChunkBytes / row));
    std::vector<uint8_t> buf;
    for (int64_t off = 0; off < h.n; off += chunk) {
        const int64_t cnt = std::min<int64_t>(chunk, h.n - off);
        buf.resize(static_cast<size_t>(cnt) * row);
        if (std::fread(buf.data(), 1, buf.size(), f) != buf.size()) {
            MFLAT_LOG_ERROR("load %s: file ends after %lld of %d rows", path,
                            static_cast<long long>(off), h.n);
            std::fclose(f);
            raise_status(mflat_cu_index_reset(dev), "load");
            return false;
        }
        const int st = mflat_cu_index_add_raw(dev, buf.data(), cnt);
        if (st != 0) {
            std::fclose(f);
            raise_status(st, "load");
        }
    }
    std::fclose(f);
    return true;
}

bool readFlatFileInfo(const char* path, int& dim, Metric& metric, Storage& storage, int& n) {
    if (!path) return false;
    std::FILE* f = std::fopen(path, "rb");
    if (!f) return false;
    FlatFileHeader h{};
    const bool ok = read_header(f, path, h);
    std::fclose(f);
    if (!ok) return false;
    dim = h.dim;
    metric = static_cast<Metric>(h.metric);
    storage = static_cast<Storage>(h.storage);
    n = h.n;
    return true;
}

std::unique_ptr<FlatIndex> FlatIndex::open(const char* path, int device) {
    if (!path) return nullptr;
    std::FILE* f = std::fopen(path, "rb");
    if (!f) {
        MFLAT_LOG_ERROR("load %s: cannot open", path);
        return nullptr;
    }
    FlatFileHeader h{};
    const bool ok = read_header(f, path, h);
    std::fclose(f);
    if (!ok) return nullptr;
    auto idx = std::make_unique<FlatIndex>(h.dim, static_cast<Metric>(h.metric),
                                           static_cast<Storage>(h.storage), device);
    if (!idx->ready()) throw DeviceError("no usable CUDA device for the loaded index");
    if (!idx->load(path)) return nullptr;
    return idx;
}

void kmeansAssign(const float* points, int n, const float* centroids, int ncentroids, int dim,
                  int32_t* out, int device) {
    if (n <= 0) return;
    raise_status(mflat_cu_kmeans_assign(points, n, centroids, ncentroids, dim, out, device, 0, nullptr),
                 "kmeans assign");
}

}  // namespace mflat
