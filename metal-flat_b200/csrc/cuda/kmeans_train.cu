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
//      mflat_cu_kmeans_fetch_rows + mflat_cu_kmeans_set_rows, because the
//      draws continue the host's stream.
// finish() assigns every point with the final centroids and builds the CSR
// inverted-list scaffold (CoarseQuantizer.mm:134-143): cellStart = exclusive
// prefix sum of the cell histogram, reorderedIds = point ids grouped by cell,
// ascending within a cell (the stable slot permutation).
//
// Sharded training (an addition; the reference trains on one device): each
// rank holds a contiguous block of the points.  Per iteration every rank
// forms per-cell double sums of its own training points (ascending training
// order), the ranks all-gather those sums and the cell counts over NCCL, and
// every rank adds the ranks' sums in rank order before dividing -- the same
// centroids on every rank, deterministic for a given sharding.  Rows named by
// global id (seeds, reseeds) are fetched from their owning rank the same way.
//
// Grouping uses CUB's device radix sort and scan (header library of the CUDA
// toolkit); everything else is kernels of this file.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
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
    int64_t n = 0, train_n = 0;        // this rank's points / training points
    int nlist = 0;
    int rank = 0, world = 1;
    std::vector<int64_t> offsets;      // [world + 1]: global row range of every rank
    void* comm = nullptr;
    cudaStream_t stream = nullptr;
    const float* data = nullptr;       // n x dim (owned when copied from the host)
    float* data_owned = nullptr;
    const float* train = nullptr;      // train_n x dim (== data when not subsampled)
    float* train_owned = nullptr;
    float* cents = nullptr;            // nlist x dim
    DevBuf assign, keys_sorted, ids, ids_sorted, counts, offsets_dev, temp, picks;
    DevBuf sums, gsums, gcounts, rows, fetch, gfetch, gids, csr_start, csr_ids;
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

__global__ void iota_kernel(int32_t* p, int64_t n, int32_t base) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) p[i] = static_cast<int32_t>(i) + base;
}

__global__ void histogram_kernel(const int32_t* __restrict__ assign, int64_t n, int32_t* counts) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) atomicAdd(counts + assign[i], 1);
}

// One warp per cell: sums[c] = double sum of the cell's points in ascending
// point order (0 for an empty cell).  ids_sorted holds local row indices.
__global__ void cell_sum_kernel(const float* __restrict__ pts, const int32_t* __restrict__ ids_sorted,
                                const int32_t* __restrict__ offsets, int nlist, int dim,
                                double* __restrict__ sums) {
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (c >= nlist) return;
    const int32_t j0 = offsets[c], j1 = offsets[c + 1];
    for (int d = lane; d < dim; d += 32) {
        double acc = 0.0;
        for (int32_t j = j0; j < j1; ++j)
            acc += static_cast<double>(pts[static_cast<int64_t>(ids_sorted[j]) * dim + d]);
        sums[static_cast<int64_t>(c) * dim + d] = acc;
    }
}

// Centroids of the non-empty cells from the ranks' sums, added in rank order;
// total counts out.  world = 1 takes the one rank's sums as they are.
__global__ void reduce_means_kernel(const double* __restrict__ gsums, const int32_t* __restrict__ gcounts,
                                    int world, int nlist, int dim, float* __restrict__ cents,
                                    int32_t* __restrict__ counts_total) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t per = static_cast<int64_t>(nlist) * dim;
    if (e >= per) return;
    const int c = static_cast<int>(e / dim);
    int64_t cnt = 0;
    for (int r = 0; r < world; ++r) cnt += gcounts[static_cast<int64_t>(r) * nlist + c];
    if (e % dim == 0) counts_total[c] = static_cast<int32_t>(cnt);
    if (cnt == 0) return;
    double acc = gsums[e];
    for (int r = 1; r < world; ++r) acc += gsums[r * per + e];
    cents[e] = static_cast<float>(acc / static_cast<double>(cnt));
}

// out[i] = global row rows[i] when this rank owns it, else zeros.
__global__ void pick_rows_kernel(const float* __restrict__ data, int64_t n_local, int64_t base,
                                 const int64_t* __restrict__ rows, int count, int dim,
                                 float* __restrict__ out) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= static_cast<int64_t>(count) * dim) return;
    const int64_t i = e / dim;
    const int d = static_cast<int>(e - i * dim);
    const int64_t r = rows[i] - base;
    out[e] = (r >= 0 && r < n_local) ? data[r * dim + d] : 0.0f;
}

__global__ void set_rows_kernel(const int32_t* __restrict__ cells, const float* __restrict__ rows,
                                int count, int dim, float* __restrict__ cents) {
    const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= static_cast<int64_t>(count) * dim) return;
    const int64_t i = e / dim;
    const int d = static_cast<int>(e - i * dim);
    cents[static_cast<int64_t>(cells[i]) * dim + d] = rows[e];
}

int key_bits(int nlist) {
    int b = 1;
    while ((1 << b) < nlist && b < 31) ++b;
    return b;
}

int sync(mflat_cu_kmeans* k, const char* what) {
    if (k->world > 1) {
        if (!k->comm) return fail(ST_DEVICE, "kmeans: communicator lost");
        return comm_wait(&k->comm, k->stream);
    }
    CU_TRY(cudaStreamSynchronize(k->stream), what);
    return ST_OK;
}

int allgather(mflat_cu_kmeans* k, const void* send, void* recv, size_t bytes) {
    if (!k->comm) return fail(ST_DEVICE, "kmeans: communicator lost");
    return comm_allgather_bytes(k->comm, send, recv, bytes, k->stream);
}

// Group `m` local assignments by cell: counts, offsets_dev (nlist + 1) and
// ids_sorted (local row index + id_base, grouped by cell, ascending).
int group_by_cell(mflat_cu_kmeans* k, int64_t m, int32_t id_base) {
    cudaStream_t st = k->stream;
    const int nl = k->nlist;
    CU_TRY(cudaMemsetAsync(k->counts.p, 0, static_cast<size_t>(nl) * sizeof(int32_t), st), "counts");
    if (m > 0) {
        histogram_kernel<<<blocks_for(m, 256), 256, 0, st>>>(k->assign.as<int32_t>(), m,
                                                              k->counts.as<int32_t>());
        CU_TRY(cudaGetLastError(), "histogram launch");
        iota_kernel<<<blocks_for(m, 256), 256, 0, st>>>(k->ids.as<int32_t>(), m, id_base);
        CU_TRY(cudaGetLastError(), "iota launch");
        size_t sort_bytes = 0;
        CU_TRY(cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, k->assign.as<int32_t>(),
                                               k->keys_sorted.as<int32_t>(), k->ids.as<int32_t>(),
                                               k->ids_sorted.as<int32_t>(), static_cast<int>(m), 0,
                                               key_bits(nl), st),
               "sort size");
        CU_TRY(k->temp.ensure(sort_bytes), "sort scratch");
        CU_TRY(cub::DeviceRadixSort::SortPairs(k->temp.p, sort_bytes, k->assign.as<int32_t>(),
                                               k->keys_sorted.as<int32_t>(), k->ids.as<int32_t>(),
                                               k->ids_sorted.as<int32_t>(), static_cast<int>(m), 0,
                                               key_bits(nl), st),
               "sort");
    }
    // counts has nlist + 1 entries with a zero last one, so the scan's last
    // output is the total
    size_t scan_bytes = 0;
    CU_TRY(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, k->counts.as<int32_t>(),
                                         k->offsets_dev.as<int32_t>(), nl + 1, st),
           "scan size");
    CU_TRY(k->temp.ensure(scan_bytes), "scan scratch");
    CU_TRY(cub::DeviceScan::ExclusiveSum(k->temp.p, scan_bytes, k->counts.as<int32_t>(),
                                         k->offsets_dev.as<int32_t>(), nl + 1, st),
           "scan");
    return ST_OK;
}

int assign_points(mflat_cu_kmeans* k, const float* pts, int64_t m) {
    if (m == 0) return ST_OK;
    return mflat_cu_kmeans_assign(pts, m, k->cents, k->nlist, k->dim, k->assign.as<int32_t>(),
                                  k->device, 1, k->stream);
}

}  // namespace

extern "C" {

int mflat_cu_kmeans_create(int device, int dim, const float* data, int64_t n, int on_device,
                           const int32_t* train_rows, int64_t train_n, int nlist, int rank,
                           int world, const uint8_t* comm_id, const int64_t* row_offsets,
                           mflat_cu_kmeans_t** out) {
    if (!out || (!data && n > 0) || dim < 1 || n < 0 || nlist < 1 || train_n < 0 || train_n > n ||
        (train_n > 0 && train_n < n && !train_rows) || world < 1 || rank < 0 || rank >= world ||
        (world > 1 && (!comm_id || !row_offsets)))
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
    k->rank = rank;
    k->world = world;
    k->offsets.assign(world + 1, 0);
    if (world > 1) {
        for (int r = 0; r <= world; ++r) k->offsets[r] = row_offsets[r];
        if (k->offsets[rank + 1] - k->offsets[rank] != n) {
            delete k;
            return fail(ST_BAD_ARG, "kmeans: row offsets disagree with this rank's point count");
        }
    } else {
        k->offsets[1] = n;
    }
    auto bail = [&](int rc) {
        mflat_cu_kmeans_destroy(k);
        return rc;
    };
    if (k->offsets[world] < nlist) return bail(fail(ST_BAD_ARG, "kmeans: fewer points than cells"));
    if (cudaStreamCreateWithFlags(&k->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(ST_DEVICE, "kmeans: stream"));
    if (world > 1) {
        const int rc = comm_create(&k->comm, rank, world, comm_id);
        if (rc != ST_OK) return bail(rc);
    }
    const size_t row = static_cast<size_t>(dim) * sizeof(float);
    if (on_device || n == 0) {
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
        if (train_n > 0) {
            if (k->picks.ensure(static_cast<size_t>(train_n) * sizeof(int32_t)) != cudaSuccess ||
                cudaMalloc(&k->train_owned, static_cast<size_t>(train_n) * row) != cudaSuccess)
                return bail(fail(ST_ALLOC, "kmeans: training buffer"));
            cudaMemcpyAsync(k->picks.p, train_rows, static_cast<size_t>(train_n) * sizeof(int32_t),
                            cudaMemcpyHostToDevice, k->stream);
            gather_rows_kernel<<<blocks_for(train_n * dim, 256), 256, 0, k->stream>>>(
                k->data, k->picks.as<int32_t>(), train_n, dim, k->train_owned);
            if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(k->stream) != cudaSuccess)
                return bail(fail(ST_DEVICE, "kmeans: gather"));
        }
        k->train = k->train_owned;
    } else {
        k->train = k->data;
    }
    // grouped ids are all-gathered at the end, padded to the largest shard:
    // size the id buffers for that up front (a later grow would drop them)
    int64_t max_n = 1;
    for (int r = 0; r < world; ++r) max_n = std::max(max_n, k->offsets[r + 1] - k->offsets[r]);
    const size_t m = static_cast<size_t>(max_n);
    const size_t per = static_cast<size_t>(nlist) * dim;
    if (cudaMalloc(&k->cents, per * sizeof(float)) != cudaSuccess ||
        k->assign.ensure(m * 4) != cudaSuccess || k->keys_sorted.ensure(m * 4) != cudaSuccess ||
        k->ids.ensure(m * 4) != cudaSuccess || k->ids_sorted.ensure(m * 4) != cudaSuccess ||
        k->counts.ensure((static_cast<size_t>(nlist) + 1) * 4) != cudaSuccess ||
        k->offsets_dev.ensure((static_cast<size_t>(nlist) + 1) * 4) != cudaSuccess ||
        k->sums.ensure(per * sizeof(double)) != cudaSuccess ||
        (world > 1 && (k->gsums.ensure(per * world * sizeof(double)) != cudaSuccess ||
                       k->gcounts.ensure(static_cast<size_t>(nlist) * world * 4) != cudaSuccess)))
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
    comm_destroy(k->comm);
    cudaFree(k->data_owned);
    cudaFree(k->train_owned);
    cudaFree(k->cents);
    for (DevBuf* b : {&k->assign, &k->keys_sorted, &k->ids, &k->ids_sorted, &k->counts, &k->offsets_dev,
                      &k->temp, &k->picks, &k->sums, &k->gsums, &k->gcounts, &k->rows, &k->fetch,
                      &k->gfetch, &k->gids, &k->csr_start, &k->csr_ids})
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

int mflat_cu_kmeans_fetch_rows(mflat_cu_kmeans_t* k, const int64_t* host_rows, int count,
                               float* host_out) {
    if (!k || count < 0 || (count > 0 && (!host_rows || !host_out)))
        return fail(ST_BAD_ARG, "kmeans: bad argument");
    const int64_t total = k->offsets[k->world];
    for (int i = 0; i < count; ++i)
        if (host_rows[i] < 0 || host_rows[i] >= total) return fail(ST_BAD_ARG, "kmeans: row out of range");
    if (count == 0) return ST_OK;
    DeviceGuard g(k->device);
    const size_t bytes = static_cast<size_t>(count) * k->dim * sizeof(float);
    CU_TRY(k->rows.ensure(static_cast<size_t>(count) * sizeof(int64_t)), "row ids");
    CU_TRY(k->fetch.ensure(bytes), "fetch buffer");
    CU_TRY(cudaMemcpyAsync(k->rows.p, host_rows, static_cast<size_t>(count) * sizeof(int64_t),
                           cudaMemcpyHostToDevice, k->stream),
           "row ids");
    pick_rows_kernel<<<blocks_for(static_cast<int64_t>(count) * k->dim, 256), 256, 0, k->stream>>>(
        k->data, k->n, k->offsets[k->rank], k->rows.as<int64_t>(), count, k->dim, k->fetch.as<float>());
    CU_TRY(cudaGetLastError(), "fetch launch");
    if (k->world == 1) {
        CU_TRY(cudaMemcpyAsync(host_out, k->fetch.p, bytes, cudaMemcpyDeviceToHost, k->stream), "fetch");
        return sync(k, "fetch");
    }
    CU_TRY(k->gfetch.ensure(bytes * k->world), "fetch gather buffer");
    int rc = allgather(k, k->fetch.p, k->gfetch.p, bytes);
    if (rc != ST_OK) return rc;
    std::vector<float> all(static_cast<size_t>(count) * k->dim * k->world);
    CU_TRY(cudaMemcpyAsync(all.data(), k->gfetch.p, bytes * k->world, cudaMemcpyDeviceToHost, k->stream),
           "fetch");
    rc = sync(k, "fetch");
    if (rc != ST_OK) return rc;
    const size_t row = static_cast<size_t>(k->dim);
    for (int i = 0; i < count; ++i) {
        int owner = 0;
        while (host_rows[i] >= k->offsets[owner + 1]) ++owner;
        std::memcpy(host_out + i * row, &all[(static_cast<size_t>(owner) * count + i) * row],
                    row * sizeof(float));
    }
    return ST_OK;
}

int mflat_cu_kmeans_set_rows(mflat_cu_kmeans_t* k, const int32_t* host_cells, const float* host_rows,
                             int count) {
    if (!k || count < 0 || (count > 0 && (!host_cells || !host_rows)))
        return fail(ST_BAD_ARG, "kmeans: bad argument");
    for (int i = 0; i < count; ++i)
        if (host_cells[i] < 0 || host_cells[i] >= k->nlist) return fail(ST_BAD_ARG, "kmeans: cell out of range");
    if (count == 0) return ST_OK;
    DeviceGuard g(k->device);
    const size_t bytes = static_cast<size_t>(count) * k->dim * sizeof(float);
    CU_TRY(k->picks.ensure(static_cast<size_t>(count) * sizeof(int32_t)), "cell ids");
    CU_TRY(k->fetch.ensure(bytes), "row buffer");
    CU_TRY(cudaMemcpyAsync(k->picks.p, host_cells, static_cast<size_t>(count) * sizeof(int32_t),
                           cudaMemcpyHostToDevice, k->stream),
           "cell ids");
    CU_TRY(cudaMemcpyAsync(k->fetch.p, host_rows, bytes, cudaMemcpyHostToDevice, k->stream), "rows");
    set_rows_kernel<<<blocks_for(static_cast<int64_t>(count) * k->dim, 256), 256, 0, k->stream>>>(
        k->picks.as<int32_t>(), k->fetch.as<float>(), count, k->dim, k->cents);
    CU_TRY(cudaGetLastError(), "set rows launch");
    CU_TRY(cudaStreamSynchronize(k->stream), "set rows");
    return ST_OK;
}

int mflat_cu_kmeans_iterate(mflat_cu_kmeans_t* k, int32_t* host_counts) {
    if (!k || !host_counts) return fail(ST_BAD_ARG, "kmeans: bad argument");
    DeviceGuard g(k->device);
    int rc = assign_points(k, k->train, k->train_n);
    if (rc != ST_OK) return rc;
    rc = group_by_cell(k, k->train_n, 0);
    if (rc != ST_OK) return rc;
    const int warps_per_block = 8;
    cell_sum_kernel<<<(k->nlist + warps_per_block - 1) / warps_per_block, warps_per_block * 32, 0,
                      k->stream>>>(k->train, k->ids_sorted.as<int32_t>(), k->offsets_dev.as<int32_t>(),
                                   k->nlist, k->dim, k->sums.as<double>());
    CU_TRY(cudaGetLastError(), "cell sum launch");
    const size_t per = static_cast<size_t>(k->nlist) * k->dim;
    const double* gs = k->sums.as<double>();
    const int32_t* gc = k->counts.as<int32_t>();
    if (k->world > 1) {
        rc = allgather(k, k->sums.p, k->gsums.p, per * sizeof(double));
        if (rc == ST_OK) rc = allgather(k, k->counts.p, k->gcounts.p, static_cast<size_t>(k->nlist) * 4);
        if (rc != ST_OK) return rc;
        gs = k->gsums.as<double>();
        gc = k->gcounts.as<int32_t>();
    }
    // the total counts land in offsets_dev (free until the next grouping)
    reduce_means_kernel<<<blocks_for(static_cast<int64_t>(per), 256), 256, 0, k->stream>>>(
        gs, gc, k->world, k->nlist, k->dim, k->cents, k->offsets_dev.as<int32_t>());
    CU_TRY(cudaGetLastError(), "centroid update launch");
    CU_TRY(cudaMemcpyAsync(host_counts, k->offsets_dev.p, static_cast<size_t>(k->nlist) * sizeof(int32_t),
                           cudaMemcpyDeviceToHost, k->stream),
           "counts download");
    return sync(k, "k-means iteration");
}

int mflat_cu_kmeans_finish(mflat_cu_kmeans_t* k, int32_t* host_assign, int32_t* host_cell_start,
                           int32_t* host_reordered) {
    if (!k) return fail(ST_BAD_ARG, "kmeans: bad argument");
    DeviceGuard g(k->device);
    int rc = assign_points(k, k->data, k->n);
    if (rc != ST_OK) return rc;
    const int32_t base = static_cast<int32_t>(k->offsets[k->rank]);
    rc = group_by_cell(k, k->n, base);
    if (rc != ST_OK) return rc;
    if (host_assign && k->n > 0)
        CU_TRY(cudaMemcpyAsync(host_assign, k->assign.p, static_cast<size_t>(k->n) * sizeof(int32_t),
                               cudaMemcpyDeviceToHost, k->stream),
               "assignment download");
    const int nl = k->nlist;
    const int64_t total = k->offsets[k->world];
    if (k->world == 1) {
        if (host_cell_start)
            CU_TRY(cudaMemcpyAsync(host_cell_start, k->offsets_dev.p, (static_cast<size_t>(nl) + 1) * 4,
                                   cudaMemcpyDeviceToHost, k->stream),
                   "cell start download");
        if (host_reordered)
            CU_TRY(cudaMemcpyAsync(host_reordered, k->ids_sorted.p, static_cast<size_t>(k->n) * 4,
                                   cudaMemcpyDeviceToHost, k->stream),
                   "permutation download");
        return sync(k, "k-means finish");
    }
    // every rank's counts and grouped ids (padded to the largest shard)
    int64_t max_n = 1;
    for (int r = 0; r < k->world; ++r) max_n = std::max(max_n, k->offsets[r + 1] - k->offsets[r]);
    CU_TRY(k->gids.ensure(static_cast<size_t>(max_n) * 4 * k->world), "id gather buffer");
    rc = allgather(k, k->counts.p, k->gcounts.p, static_cast<size_t>(nl) * 4);
    if (rc == ST_OK) rc = allgather(k, k->ids_sorted.p, k->gids.p, static_cast<size_t>(max_n) * 4);
    if (rc != ST_OK) return rc;
    std::vector<int32_t> cnt(static_cast<size_t>(nl) * k->world), ids(static_cast<size_t>(max_n) * k->world);
    CU_TRY(cudaMemcpyAsync(cnt.data(), k->gcounts.p, cnt.size() * 4, cudaMemcpyDeviceToHost, k->stream),
           "count download");
    CU_TRY(cudaMemcpyAsync(ids.data(), k->gids.p, ids.size() * 4, cudaMemcpyDeviceToHost, k->stream),
           "id download");
    rc = sync(k, "k-means finish");
    if (rc != ST_OK) return rc;
    // global CSR: cells in order, within a cell the ranks in order (= ascending id)
    std::vector<int32_t> start(static_cast<size_t>(nl) + 1, 0), reord(static_cast<size_t>(total));
    std::vector<int64_t> cursor(k->world, 0);
    for (int c = 0; c < nl; ++c) {
        int64_t pos = start[c];
        for (int r = 0; r < k->world; ++r) {
            const int32_t m = cnt[static_cast<size_t>(r) * nl + c];
            const int32_t* src = &ids[static_cast<size_t>(r) * max_n + cursor[r]];
            std::memcpy(&reord[pos], src, static_cast<size_t>(m) * 4);
            cursor[r] += m;
            pos += m;
        }
        start[c + 1] = static_cast<int32_t>(pos);
    }
    CU_TRY(k->csr_start.ensure(start.size() * 4), "CSR buffer");
    CU_TRY(k->csr_ids.ensure(std::max<size_t>(reord.size(), 1) * 4), "CSR buffer");
    CU_TRY(cudaMemcpyAsync(k->csr_start.p, start.data(), start.size() * 4, cudaMemcpyHostToDevice, k->stream),
           "CSR upload");
    CU_TRY(cudaMemcpyAsync(k->csr_ids.p, reord.data(), reord.size() * 4, cudaMemcpyHostToDevice, k->stream),
           "CSR upload");
    CU_TRY(cudaStreamSynchronize(k->stream), "CSR upload");
    if (host_cell_start) std::memcpy(host_cell_start, start.data(), start.size() * 4);
    if (host_reordered) std::memcpy(host_reordered, reord.data(), reord.size() * 4);
    return ST_OK;
}

const int32_t* mflat_cu_kmeans_cell_start_device(const mflat_cu_kmeans_t* k) {
    if (!k) return nullptr;
    return static_cast<const int32_t*>(k->world > 1 ? k->csr_start.p : k->offsets_dev.p);
}

const int32_t* mflat_cu_kmeans_reordered_device(const mflat_cu_kmeans_t* k) {
    if (!k) return nullptr;
    return static_cast<const int32_t*>(k->world > 1 ? k->csr_ids.p : k->ids_sorted.p);
}

}  // extern "C"
