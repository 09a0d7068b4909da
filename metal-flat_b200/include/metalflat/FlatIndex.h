// SPDX-License-Identifier: Apache-2.0
// metalflat/FlatIndex.h -- exact (brute-force) vector search on NVIDIA B200.
//
// Same class, members and result layout as the reference's
// include/metalflat/FlatIndex.h:28-77, so code written against it compiles
// unchanged.  Differences a caller can observe:
//   * kMaxK is 1024 (was 64); larger k is clamped with a one-time warning.
//   * There is no CPU fallback: when no usable CUDA device exists, ready() is
//     false and search() throws DeviceError.
//   * The database lives on the device; add() appends there directly.
// Additive members (storage precision, device pointers, timing, sharding)
// sit below the reference's.
#pragma once

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <vector>

#include "metalflat/Export.h"
#include "metalflat/Metric.h"

namespace mflat {

struct SearchResult {
    // Row-major: m rows of k.  ids[r*k + j] is the database index of query r's
    // j-th nearest neighbour (-1 when the database holds fewer than k rows);
    // distances[r*k + j] its squared L2 distance or IP / cosine similarity.
    std::vector<int32_t> ids;
    std::vector<float>   distances;
};

// Storage precision of the database on the device.
enum class Storage { FP32 = 0, FP16 = 1, BF16 = 2 };

// Thrown when the CUDA device (or NCCL) fails or is absent.
class MFLAT_CXX_API DeviceError : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};

struct SearchTiming {
    float total_ms = 0, screen_ms = 0, select_ms = 0;
    int screen_launches = 0, launches = 0, fallback_queries = 0;
};

class MFLAT_CXX_API FlatIndex {
public:
    static constexpr int kMaxK = 1024;

    FlatIndex(int dim, Metric metric);
    FlatIndex(int dim, Metric metric, Storage storage, int device = -1);
    ~FlatIndex();

    FlatIndex(const FlatIndex&)            = delete;
    FlatIndex& operator=(const FlatIndex&) = delete;

    bool ready() const;                       // usable CUDA device
    void add(const float* vectors, int n);    // n <= 0: no-op
    void reset();
    int    size() const;
    int    dim() const;
    Metric metric() const;
    // k is clamped to [1, kMaxK]; m <= 0 returns an empty result.
    SearchResult search(const float* queries, int m, int k);

    // ---- additive ----
    Storage storage() const;
    int     device() const;
    // As search, into caller-owned host buffers holding >= m * k entries
    // (page-locked ones are filled by DMA); results are nearest-first at row
    // stride k_used, the return value.  m <= 0 returns 0 and writes nothing.
    int  searchInto(const float* queries, int m, int k, int32_t* ids, float* distances);
    void addDevice(const float* d_vectors, int n, void* stream);
    // Device pointers; enqueues on `stream`; returns the k actually used
    // (outputs are written at that row stride).
    int  searchDevice(const float* d_queries, int m, int k, int32_t* d_ids, float* d_dist,
                      void* stream);
    // As searchDevice, but allocates no device memory: the scratch is a fixed
    // array inside the library (m <= 128, dim <= 128, k <= 21; no clamping --
    // larger sizes throw std::invalid_argument).  For callers that cannot call
    // cudaMalloc; calls that overlap on one GPU race on that array.
    int  searchDeviceNoAlloc(const float* d_queries, int m, int k, int32_t* d_ids, float* d_dist,
                             void* stream);
    void setTiming(bool enable);
    SearchTiming lastTiming() const;
    // Field-wise sums over every search since setTiming(true); *n = how many.
    SearchTiming timingSum(int* n) const;
    // Row sharding: this index holds global rows [id_base, id_base + size());
    // search() becomes a collective over `world` ranks returning global ids.
    void setShard(int rank, int world, const uint8_t* comm_id, int64_t id_base);

    // Persistence (in the style of the reference's GraphIndex::save / load,
    // src/GraphIndex.mm:424-452).  File: a 32-byte header (the bytes "MFFL",
    // then int32 version 1, dim, metric, storage, n, 0, 0), then n x dim stored
    // elements (fp32, or the fp16 / bf16 bit patterns).  save() returns false on an I/O failure.
    // load() replaces this index's rows; it returns false (index unchanged)
    // when the file is unreadable, shorter than its header announces, or its
    // dim / metric / storage differ.  A device failure while the rows are
    // being appended throws DeviceError.
    bool save(const char* path) const;
    bool load(const char* path);
    // A new index on `device` (-1 = default) with the file's dim, metric and
    // storage; nullptr when the file cannot be read.
    static std::unique_ptr<FlatIndex> open(const char* path, int device = -1);

private:
    struct Impl;
    std::unique_ptr<Impl> mImpl;
};

// Header of a file written by FlatIndex::save; false when the file cannot be
// read or is not a flat index file.
MFLAT_CXX_API bool readFlatFileInfo(const char* path, int& dim, Metric& metric, Storage& storage, int& n);

// k-means assignment step: out[i] = argmin_c sqL2_f32(points[i], centroids[c])
// with the reference's fp32 sequential sqL2 and lowest-index tie rule.
MFLAT_CXX_API void kmeansAssign(const float* points, int n, const float* centroids, int ncentroids, int dim,
                  int32_t* out, int device = -1);

}  // namespace mflat
