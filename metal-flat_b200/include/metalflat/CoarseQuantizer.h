// SPDX-License-Identifier: Apache-2.0
// metalflat/CoarseQuantizer.h -- the IVF coarse layer on NVIDIA B200.
//
// Same class and members as the reference's internal CoarseQuantizer
// (src/CoarseQuantizer.h:27-75): k-means training (seed 12345, 256 training
// points per centroid), point -> cell assignment, the CSR inverted-list
// scaffold (cellStart + reorderedIds), the coarse FlatIndex over the
// centroids, and device copies of the CSR.  Differences a caller can observe:
//   * the k-means loop runs on the GPU (assignment, centroid means, CSR); the
//     assignment is the bit-exact fp32 sequential-sqL2 argmin of the flat
//     kernels, the means are double sums in ascending point order;
//   * there is no CPU path: without a CUDA device train() throws DeviceError
//     (KmeansBackend is accepted for source compatibility; both values train
//     on the device);
//   * cellBuffer() / idBuffer() are device pointers instead of MTLBuffers;
//   * probeCells() takes nprobe <= FlatIndex::kMaxK (1024) and throws
//     std::invalid_argument above it; the reference's CPU-only
//     probeCellsCpu is not provided.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <vector>

#include "metalflat/Export.h"
#include "metalflat/FlatIndex.h"

namespace mflat {

class MFLAT_CXX_API CoarseQuantizer {
public:
    enum class KmeansBackend { Auto, ForceGpuAssign };

    // device -1: $MFLAT_DEVICE or 0.
    explicit CoarseQuantizer(int dim, int device = -1);
    ~CoarseQuantizer();
    CoarseQuantizer(const CoarseQuantizer&)            = delete;
    CoarseQuantizer& operator=(const CoarseQuantizer&) = delete;

    // Train (seed 12345), assign, build the CSR and the coarse FlatIndex(dim, L2).
    // `data` is row-major n x dim host memory, already metric-normalised (Cosine).
    // nlistReq is clamped to n.
    void train(const float* data, int n, int nlistReq, int iters = 12,
               KmeansBackend backend = KmeansBackend::Auto);

    int dim() const;
    int nlist() const;
    int size() const;                                   // n (all ranks' rows when sharded)
    const std::vector<float>& centroids() const;        // nlist x dim
    const std::vector<int>& cellStart() const;          // nlist + 1 (CSR offsets)
    const std::vector<int>& reorderedIds() const;       // n: slot -> original id

    // dst[pos] = src[reorderedIds[pos]] for each of the n rows (id order -> slot order).
    void reorderPayload(const void* src, void* dst, std::size_t elemBytes) const;

    // probed (resized to m * nprobe) = nearest-first cell ids of each query,
    // from the coarse FlatIndex (exact L2 over the centroids, lowest id on ties).
    void probeCells(const float* queries, int m, int nprobe, std::vector<int32_t>& probed) const;

    // Sharded training (additive; the reference trains on one device): this
    // process holds global rows [row_offsets[rank], row_offsets[rank + 1]) and
    // passes only those to train(); every rank calls train() with the same
    // nlist and iters.  Per iteration the ranks all-gather per-cell double sums
    // and counts over NCCL (comm_id: 128 bytes from mflat_comm_unique_id) and
    // add them in rank order, so all ranks end with the same centroids and the
    // same global CSR.  world = 1 turns sharding off.
    void setShard(int rank, int world, const uint8_t* comm_id, const int64_t* row_offsets);

    bool gpuReady() const;                 // coarse FlatIndex ready
    const int32_t* cellBuffer() const;     // device: cellStart (nlist + 1)
    const int32_t* idBuffer() const;       // device: reorderedIds (n)
    int device() const;

private:
    struct Impl;
    std::unique_ptr<Impl> mImpl;
};

// The seed permutation of the k-means training: 0..n-1 shuffled by a
// front-to-back Fisher-Yates pass whose swap offsets are drawn from `rng` by
// bitmask rejection (exposed for tests).
MFLAT_CXX_API void kmeansSeedPermutation(int n, uint32_t seed, std::vector<int>& perm);

}  // namespace mflat
