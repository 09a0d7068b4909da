// kmeans_train.cu -- device side of CoarseQuantizer::train: the whole k-means
// loop of the reference's kmeansGpu (src/Internal.h:257-359) on the GPU.
//
// Per iteration (Internal.h:351-355):
//   1. assignment of the training points: the bit-exact flat-kernel assignment
//      of kmeans.cu (argmin of the fp32 sequential sqL2, lowest index on ties);
//   2. centroid update (accumulateCentroids, Internal.h:52-99): per cell the
//      mean of its points, accumulated in double and rounded to float.  The
//      points are grouped by cell with a stable radix sort, so each cell is
//      summed in ascending point order -- deterministic, and the order of the
//      reference's single-thread CPU k-means (CoarseQuantizer.mm:47-55);
//   3. empty cells keep their old centroid here; the host reseeds them from
//      its mt19937 in cell order (Internal.h:90-98) through
//      mflat_cu_kmeans_reseed, because the draws continue the host's stream.
// finish() assigns every point with the final centroids and builds the CSR
// inverted-list scaffold (CoarseQuantizer.mm:134-143): cellStart = exclusive
// prefix sum of the cell histogram, reorderedIds = point ids grouped by cell,
// ascending within a cell (the stable slot permutation).
//
// Grouping uses CUB's device radix sort and scan (header library of the CUDA
// toolkit); everything else is kernels of this file.
#include <cuda_runtime.h>

#include <algorithm>
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>
#include <vector>

#include "index_impl.cuh"
#include "kernels.cuh"
#include "mflat_cuda.h"

using namespace mflat_cu;

struct mflat_cu_kmeans {
    int device = 0;
    int dim = 0;
    int64_t n = 0, train_n = 0;
    int nlist = 0;
    cudaStream_t stream = nullptr;
    const float* data = nullptr;       // n x dim (owned when copied from the host)
    float* data_owned = nullptr;
    const float* train = nullptr;      // train_n x dim (== data when not subsampled)
    float* train_owned = nullptr;
    float* cents = nullptr;            // nlist x dim
    DevBuf assign, keys_sorted, ids, ids_sorted, counts, offsets, temp, picks;
};

namespace {

__global__ void gather_rows_kernel(const float* __restrict__ src, const int32_t* __restrict__ rows,
                                   int64_t n, int dim, float* __restrict__ dst) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= n * dim) return;
    const int64_t i = e / dim;
    const int c = static_cast<int>(e - i * dim);
    dst[e] = src[static_cast<int64_t>(rows[i]) * dim + c];
}

__global__ void iota_kernel(int32_t* p, int64_t n) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) p[i] = static_cast<int32_t>(i);
}

__global__ void histogram_kernel(const int32_t* __restrict__ assign, int64_t n, int32_t* counts) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) atomicAdd(counts + assign[i], 1);
}

// One warp per cell: cents[c] = mean of the cell's points (double sums in
// ascending point order, then rounded to float); empty cells are left alone.
__global__ void cell_mean_kernel(const float* __restrict__ pts, const int32_t* __restrict__ ids_sorted,
                                 const int32_t* __restrict__ offsets, int nlist, int dim,
                                 float* __restrict__ cents) {
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (c >= nlist) return;
    const int32_t j0 = offsets[c], j1 = offsets[c + 1];
    if (j1 == j0) return;
    const double cnt = static_cast<double>(j1 - j0);
    for (int d0 = 0; d0 < dim; d0 += 32) {
        const int d = d0 + lane;
        double acc = 0.0;
        if (d < dim)
            for (int32_t j = j0; j < j1; ++j)
                acc += static_cast<double>(pts[static_cast<int64_t>(ids_sorted[j]) * dim + d]);
        if (d < dim) cents[static_cast<int64_t>(c) * dim + d] = static_cast<float>(acc / cnt);
    }
}

// cents[cells[i]] = train[rows[i]] for the reseeded (empty) cells.
__global__ void reseed_kernel(const float* __restrict__ train, const int32_t* __restrict__ picks,
                              int count, int dim, float* __restrict__ cents) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= count * dim) return;
    const int i = e / dim;
    const int d = e - i * dim;
    cents[static_cast<int64_t>(picks[2 * i]) * dim + d] =
        train[static_cast<int64_t>(picks[2 * i + 1]) * dim + d];
}

int key_bits(int nlist) {
    int b = 1;
    while ((1 << b) < nlist && b < 31) ++b;
    return b;
}

// Group `m` assignments by cell: counts, offsets (nlist + 1), ids_sorted.
int group_by_cell(mflat_cu_kmeans* k, int64_t m) {
    cudaStream_t st = k->stream;
    const int nl = k->nlist;
    CU_TRY(cudaMemsetAsync(k->counts.p, 0, static_cast<size_t>(nl) * sizeof(int32_t), st), "counts");
    histogram_kernel<<<blocks_for(m, 256), 256, 0, st>>>(k->assign.as<int32_t>(), m,
                                                          k->counts.as<int32_t>());
    CU_TRY(cudaGetLastError(), "histogram launch");
    iota_kernel<<<blocks_for(m, 256), 256, 0, st>>>(k->ids.as<int32_t>(), m);
    CU_TRY(cudaGetLastError(), "iota launch");
    size_t sort_bytes = 0, scan_bytes = 0;
    CU_TRY(cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, k->assign.as<int32_t>(),
                                           k->keys_sorted.as<int32_t>(), k->ids.as<int32_t>(),
                                           k->ids_sorted.as<int32_t>(), static_cast<int>(m), 0,
                                           key_bits(nl), st),
           "sort size");
    CU_TRY(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, k->counts.as<int32_t>(),
                                         k->offsets.as<int32_t>(), nl + 1, st),
           "scan size");
    CU_TRY(k->temp.ensure(std::max(sort_bytes, scan_bytes)), "sort scratch");
    CU_TRY(cub::DeviceRadixSort::SortPairs(k->temp.p, sort_bytes, k->assign.as<int32_t>(),
                                           k->keys_sorted.as<int32_t>(), k->ids.as<int32_t>(),
                                           k->ids_sorted.as<int32_t>(), static_cast<int>(m), 0,
                                           key_bits(nl), st),
           "sort");
    // counts has nlist + 1 entries with a zero last one, so the scan's last
    // output is the total
    CU_TRY(cub::DeviceScan::ExclusiveSum(k->temp.p, scan_bytes, k->counts.as<int32_t>(),
                                         k->offsets.as<int32_t>(), nl + 1, st),
           "scan");
    return ST_OK;
}

int assign_points(mflat_cu_kmeans* k, const float* pts, int64_t m) {
    return mflat_cu_kmeans_assign(pts, m, k->cents, k->nlist, k->dim, k->assign.as<int32_t>(),
                                  k->device, 1, k->stream);
}

}  // namespace

extern "C" {

int mflat_cu_kmeans_create(int device, int dim, const float* data, int64_t n, int on_device,
                           const int32_t* train_rows, int64_t train_n, int nlist,
                           mflat_cu_kmeans_t** out) {
    if (!out || !data || dim < 1 || n < 1 || nlist < 1 || nlist > n || train_n < 1 || train_n > n ||
        (train_n < n && !train_rows))
        return fail(ST_BAD_ARG, "kmeans: bad argument");
    if (n > INT32_MAX - kBM) return fail(ST_BAD_ARG, "kmeans: too many points");
    *out = nullptr;
    device = mflat_cu_default_device(device);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device >= ndev)
        return fail(ST_DEVICE, "kmeans: no CUDA device");
    DeviceGuard g(device);
    auto* k = new mflat_cu_kmeans();
    k->device = device;
    k->dim = dim;
    k->n = n;
    k->train_n = train_n;
    k->nlist = nlist;
    auto bail = [&](int rc) {
        mflat_cu_kmeans_destroy(k);
        return rc;
    };
    if (cudaStreamCreateWithFlags(&k->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(ST_DEVICE, "kmeans: stream"));
    const size_t row = static_cast<size_t>(dim) * sizeof(float);
    if (on_device) {
        k->data = data;
    } else {
        if (cudaMalloc(&k->data_owned, static_cast<size_t>(n) * row) != cudaSuccess)
            return bail(fail(ST_ALLOC, "kmeans: point buffer"));
        if (cudaMemcpyAsync(k->data_owned, data, static_cast<size_t>(n) * row, cudaMemcpyHostToDevice,
                            k->stream) != cudaSuccess)
            return bail(fail(ST_DEVICE, "kmeans: point upload"));
        k->data = k->data_owned;
    }
    if (train_n < n) {
        // the training rows' indices go through the reseed buffer
        if (k->picks.ensure(static_cast<size_t>(train_n) * sizeof(int32_t)) != cudaSuccess ||
            cudaMalloc(&k->train_owned, static_cast<size_t>(train_n) * row) != cudaSuccess)
            return bail(fail(ST_ALLOC, "kmeans: training buffer"));
        cudaMemcpyAsync(k->picks.p, train_rows, static_cast<size_t>(train_n) * sizeof(int32_t),
                        cudaMemcpyHostToDevice, k->stream);
        gather_rows_kernel<<<blocks_for(train_n * dim, 256), 256, 0, k->stream>>>(
            k->data, k->picks.as<int32_t>(), train_n, dim, k->train_owned);
        if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(k->stream) != cudaSuccess)
            return bail(fail(ST_DEVICE, "kmeans: gather"));
        k->train = k->train_owned;
    } else {
        k->train = k->data;
    }
    const size_t m = static_cast<size_t>(n);
    if (cudaMalloc(&k->cents, static_cast<size_t>(nlist) * row) != cudaSuccess ||
        k->assign.ensure(m * 4) != cudaSuccess || k->keys_sorted.ensure(m * 4) != cudaSuccess ||
        k->ids.ensure(m * 4) != cudaSuccess || k->ids_sorted.ensure(m * 4) != cudaSuccess ||
        k->counts.ensure((static_cast<size_t>(nlist) + 1) * 4) != cudaSuccess ||
        k->offsets.ensure((static_cast<size_t>(nlist) + 1) * 4) != cudaSuccess)
        return bail(fail(ST_ALLOC, "kmeans: work buffers"));
    if (cudaMemsetAsync(k->counts.p, 0, (static_cast<size_t>(nlist) + 1) * 4, k->stream) != cudaSuccess ||
        cudaStreamSynchronize(k->stream) != cudaSuccess)
        return bail(fail(ST_DEVICE, "kmeans: init"));
    *out = k;
    return ST_OK;
}

void mflat_cu_kmeans_destroy(mflat_cu_kmeans_t* k) {
    if (!k) return;
    DeviceGuard g(k->device);
    if (k->stream) cudaStreamSynchronize(k->stream);
    cudaFree(k->data_owned);
    cudaFree(k->train_owned);
    cudaFree(k->cents);
    for (DevBuf* b : {&k->assign, &k->keys_sorted, &k->ids, &k->ids_sorted, &k->counts, &k->offsets,
                      &k->temp, &k->picks})
        b->release();
    if (k->stream) cudaStreamDestroy(k->stream);
    delete k;
}

int mflat_cu_kmeans_set_centroids(mflat_cu_kmeans_t* k, const float* host_centroids) {
    if (!k || !host_centroids) return fail(ST_BAD_ARG, "kmeans: bad argument");
    DeviceGuard g(k->device);
    CU_TRY(cudaMemcpyAsync(k->cents, host_centroids,
                           static_cast<size_t>(k->nlist) * k->dim * sizeof(float),
                           cudaMemcpyHostToDevice, k->stream),
           "centroid upload");
    CU_TRY(cudaStreamSynchronize(k->stream), "centroid upload");
    return ST_OK;
}

int mflat_cu_kmeans_get_centroids(mflat_cu_kmeans_t* k, float* host_out) {
    if (!k || !host_out) return fail(ST_BAD_ARG, "kmeans: bad argument");
    DeviceGuard g(k->device);
    CU_TRY(cudaMemcpyAsync(host_out, k->cents, static_cast<size_t>(k->nlist) * k->dim * sizeof(float),
                           cudaMemcpyDeviceToHost, k->stream),
           "centroid download");
    CU_TRY(cudaStreamSynchronize(k->stream), "centroid download");
    return ST_OK;
}

int mflat_cu_kmeans_iterate(mflat_cu_kmeans_t* k, int32_t* host_counts) {
    if (!k || !host_counts) return fail(ST_BAD_ARG, "kmeans: bad argument");
    DeviceGuard g(k->device);
    int rc = assign_points(k, k->train, k->train_n);
    if (rc != ST_OK) return rc;
    rc = group_by_cell(k, k->train_n);
    if (rc != ST_OK) return rc;
    const int warps_per_block = 8;
    cell_mean_kernel<<<(k->nlist + warps_per_block - 1) / warps_per_block, warps_per_block * 32, 0,
                       k->stream>>>(k->train, k->ids_sorted.as<int32_t>(), k->offsets.as<int32_t>(),
                                    k->nlist, k->dim, k->cents);
    CU_TRY(cudaGetLastError(), "centroid update launch");
    CU_TRY(cudaMemcpyAsync(host_counts, k->counts.p, static_cast<size_t>(k->nlist) * sizeof(int32_t),
                           cudaMemcpyDeviceToHost, k->stream),
           "counts download");
    CU_TRY(cudaStreamSynchronize(k->stream), "k-means iteration");
    return ST_OK;
}

int mflat_cu_kmeans_reseed(mflat_cu_kmeans_t* k, const int32_t* host_cells,
                           const int32_t* host_train_rows, int count) {
    if (!k || count < 0 || (count > 0 && (!host_cells || !host_train_rows)))
        return fail(ST_BAD_ARG, "kmeans: bad argument");
    if (count == 0) return ST_OK;
    std::vector<int32_t> picks(2 * static_cast<size_t>(count));
    for (int i = 0; i < count; ++i) {
        if (host_cells[i] < 0 || host_cells[i] >= k->nlist || host_train_rows[i] < 0 ||
            host_train_rows[i] >= k->train_n)
            return fail(ST_BAD_ARG, "kmeans: reseed index out of range");
        picks[2 * i] = host_cells[i];
        picks[2 * i + 1] = host_train_rows[i];
    }
    DeviceGuard g(k->device);
    CU_TRY(k->picks.ensure(picks.size() * sizeof(int32_t)), "reseed buffer");
    CU_TRY(cudaMemcpyAsync(k->picks.p, picks.data(), picks.size() * sizeof(int32_t),
                           cudaMemcpyHostToDevice, k->stream),
           "reseed upload");
    reseed_kernel<<<blocks_for(static_cast<int64_t>(count) * k->dim, 256), 256, 0, k->stream>>>(
        k->train, k->picks.as<int32_t>(), count, k->dim, k->cents);
    CU_TRY(cudaGetLastError(), "reseed launch");
    CU_TRY(cudaStreamSynchronize(k->stream), "reseed");
    return ST_OK;
}

int mflat_cu_kmeans_finish(mflat_cu_kmeans_t* k, int32_t* host_assign, int32_t* host_cell_start,
                           int32_t* host_reordered) {
    if (!k) return fail(ST_BAD_ARG, "kmeans: bad argument");
    DeviceGuard g(k->device);
    int rc = assign_points(k, k->data, k->n);
    if (rc != ST_OK) return rc;
    rc = group_by_cell(k, k->n);
    if (rc != ST_OK) return rc;
    if (host_assign)
        CU_TRY(cudaMemcpyAsync(host_assign, k->assign.p, static_cast<size_t>(k->n) * sizeof(int32_t),
                               cudaMemcpyDeviceToHost, k->stream),
               "assignment download");
    if (host_cell_start)
        CU_TRY(cudaMemcpyAsync(host_cell_start, k->offsets.p,
                               (static_cast<size_t>(k->nlist) + 1) * sizeof(int32_t),
                               cudaMemcpyDeviceToHost, k->stream),
               "cell start download");
    if (host_reordered)
        CU_TRY(cudaMemcpyAsync(host_reordered, k->ids_sorted.p, static_cast<size_t>(k->n) * sizeof(int32_t),
                               cudaMemcpyDeviceToHost, k->stream),
               "permutation download");
    CU_TRY(cudaStreamSynchronize(k->stream), "k-means finish");
    return ST_OK;
}

const int32_t* mflat_cu_kmeans_cell_start_device(const mflat_cu_kmeans_t* k) {
    return k ? static_cast<const int32_t*>(k->offsets.p) : nullptr;
}

const int32_t* mflat_cu_kmeans_reordered_device(const mflat_cu_kmeans_t* k) {
    return k ? static_cast<const int32_t*>(k->ids_sorted.p) : nullptr;
}

}  // extern "C"
