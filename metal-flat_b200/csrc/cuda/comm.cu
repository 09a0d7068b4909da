// comm.cu -- database row sharding across GPUs (one process or thread per
// GPU).  The reference has no distributed layer; this adds the one exchange
// step the sharded flat search needs: each rank computes the top-k of its
// rows for every query (ids already global: id_base + local row), the ranks
// all-gather those (id, distance) lists over NCCL (NVLink / NVSwitch), and
// every rank merges the P sorted lists on the device with the same order as
// the single-GPU path: nearer first, then lower id.
//
// NCCL is loaded lazily (dlopen of libnccl.so.2, reusing the copy already in
// the process when there is one), so a single-GPU user never loads it.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>

#include "index_impl.cuh"
#include "kernels.cuh"
#include "mflat_cuda.h"
#include "ptx.cuh"

namespace mflat_cu {
namespace {

constexpr int kMaxRanks = 256;

struct NcclApi {
    bool ok = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

const NcclApi& nccl() {
    std::call_once(g_nccl_once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
#define MFLAT_SYM(field, name) g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, name))
        MFLAT_SYM(GetUniqueId, "ncclGetUniqueId");
        MFLAT_SYM(CommInitRank, "ncclCommInitRank");
        MFLAT_SYM(AllGather, "ncclAllGather");
        MFLAT_SYM(GroupStart, "ncclGroupStart");
        MFLAT_SYM(GroupEnd, "ncclGroupEnd");
        MFLAT_SYM(CommDestroy, "ncclCommDestroy");
        MFLAT_SYM(CommAbort, "ncclCommAbort");
        MFLAT_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
        MFLAT_SYM(GetErrorString, "ncclGetErrorString");
#undef MFLAT_SYM
        g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRank && g_nccl.AllGather &&
                    g_nccl.GroupStart && g_nccl.GroupEnd && g_nccl.CommDestroy &&
                    g_nccl.CommAbort && g_nccl.CommGetAsyncError && g_nccl.GetErrorString;
    });
    return g_nccl;
}

int nccl_fail(const char* what, ncclResult_t r) {
    char buf[256];
    std::snprintf(buf, sizeof buf, "%s: %s", what,
                  nccl().GetErrorString ? nccl().GetErrorString(r) : "nccl error");
    return fail(ST_DEVICE, buf);
}

// P-way merge of the gathered per-rank lists ([P][m][k], each nearest-first,
// ids global) into [m][k], one block per query, as a tree of two-way merges
// in shared memory.  Entries become 64-bit keys whose unsigned order is the
// result order (nearer first, then lower id; 0 = empty slot), so a merge is a
// plain descending merge of distinct keys.  Each output position of a
// two-way merge finds its split with a binary search along its diagonal (the
// merge-path co-rank), so every thread works independently: log2(P) levels of
// k outputs per pair.  Shared memory: 1.5 x (P rounded up to a power of two) x
// k x 8 bytes.
__device__ __forceinline__ uint64_t merge_key(float d, int32_t id, bool l2) {
    if (id < 0) return 0ull;
    return (static_cast<uint64_t>(score_key(l2 ? -d : d)) << 32) |
           static_cast<uint32_t>(~static_cast<uint32_t>(id));
}

// Output t of the top-k of descending x and y (k keys each).
__device__ __forceinline__ uint64_t merge_at(const uint64_t* x, const uint64_t* y, int k, int t) {
    int lo = t > k ? t - k : 0;
    int hi = t < k ? t : k;
    while (lo < hi) {                 // first a with x[a] not ahead of y[t - 1 - a]
        const int mid = (lo + hi) >> 1;
        if (x[mid] > y[t - 1 - mid]) lo = mid + 1;
        else hi = mid;
    }
    const uint64_t xa = lo < k ? x[lo] : 0ull;
    const uint64_t yb = t - lo < k ? y[t - lo] : 0ull;
    return xa > yb ? xa : yb;
}

__global__ void merge_ranks_kernel(const int32_t* __restrict__ gids, const float* __restrict__ gdist,
                                   int world, int p2, int m, int k, int metric,
                                   int32_t* __restrict__ out_ids, float* __restrict__ out_dist) {
    extern __shared__ uint64_t sm_keys[];
    const int qi = blockIdx.x;
    const bool l2 = metric == kL2;
    uint64_t* a = sm_keys;                                   // p2 lists
    uint64_t* b = sm_keys + static_cast<size_t>(p2) * k;     // p2 / 2 lists
    for (int e = threadIdx.x; e < p2 * k; e += blockDim.x) {
        const int p = e / k;
        uint64_t key = 0ull;
        if (p < world) {
            const int64_t o = (static_cast<int64_t>(p) * m + qi) * k + (e - p * k);
            key = merge_key(gdist[o], gids[o], l2);
        }
        a[e] = key;
    }
    __syncthreads();
    for (int n = p2; n > 1; n >>= 1) {
        const int outs = (n >> 1) * k;
        for (int e = threadIdx.x; e < outs; e += blockDim.x) {
            const int j = e / k;
            const int t = e - j * k;
            b[e] = merge_at(a + static_cast<size_t>(2 * j) * k, a + static_cast<size_t>(2 * j + 1) * k, k, t);
        }
        __syncthreads();
        uint64_t* tmp = a;
        a = b;
        b = tmp;
    }
    const float empty = l2 ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
    for (int t = threadIdx.x; t < k; t += blockDim.x) {
        const uint64_t key = a[t];
        const int64_t o = static_cast<int64_t>(qi) * k + t;
        if (key == 0ull) {
            out_ids[o] = -1;
            out_dist[o] = empty;
        } else {
            const uint32_t h = static_cast<uint32_t>(key >> 32);
            const float s = __uint_as_float((h & 0x80000000u) ? (h & 0x7fffffffu) : ~h);
            out_ids[o] = static_cast<int32_t>(~static_cast<uint32_t>(key));
            out_dist[o] = l2 ? -s : s;
        }
    }
}

constexpr size_t kMergeSmemMax = 200u << 10;

int merge_p2(int world) {
    int p2 = 1;
    while (p2 < world) p2 <<= 1;
    return p2;
}

size_t merge_smem(int world, int k) {
    const int p2 = merge_p2(world);
    return static_cast<size_t>(p2) * k * 8 + static_cast<size_t>(p2 / 2) * k * 8;
}

}  // namespace

void comm_release(mflat_cu_index* ix) {
    if (ix->comm) {
        nccl().CommDestroy(static_cast<ncclComm_t>(ix->comm));
        ix->comm = nullptr;
    }
    ix->world = 1;
    ix->rank = 0;
    ix->id_base = 0;
}

// Wait for `st` while watching the communicator: a peer that died or hung
// surfaces as an error instead of a hang (MFLAT_NCCL_TIMEOUT_S, default 300).
int wait_collective(mflat_cu_index* ix, cudaStream_t st) {
    const char* env = std::getenv("MFLAT_NCCL_TIMEOUT_S");
    const double limit = env ? std::atof(env) : 300.0;
    const auto t0 = std::chrono::steady_clock::now();
    auto comm = static_cast<ncclComm_t>(ix->comm);
    for (;;) {
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) return ST_OK;
        if (q != cudaErrorNotReady) return fail(ST_DEVICE, "collective", q);
        ncclResult_t ar = ncclSuccess;
        nccl().CommGetAsyncError(comm, &ar);
        if (ar != ncclSuccess && ar != ncclInProgress) {
            nccl().CommAbort(comm);
            ix->comm = nullptr;
            ix->world = 1;
            return nccl_fail("all-gather failed", ar);
        }
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > limit) {
            nccl().CommAbort(comm);
            ix->comm = nullptr;
            ix->world = 1;
            return fail(ST_DEVICE, "all-gather timed out; communicator aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int shard_merge(mflat_cu_index* ix, int m, int k_out, int32_t* ids, float* dist, cudaStream_t st) {
    if (!ix->comm || ix->world <= 1) return ST_OK;
    if (merge_smem(ix->world, k_out) > kMergeSmemMax)
        return fail(ST_BAD_ARG, "too many ranks for this k: the on-device merge holds 1.5 x ranks"
                                " (rounded up to a power of two) x k x 8 bytes in 200 KB");
    const size_t cnt = static_cast<size_t>(m) * k_out;
    CU_TRY(ix->gather_ids.ensure(cnt * ix->world * sizeof(int32_t)), "gather buffer");
    CU_TRY(ix->gather_dist.ensure(cnt * ix->world * sizeof(float)), "gather buffer");
    auto comm = static_cast<ncclComm_t>(ix->comm);
    ncclResult_t r;
    if ((r = nccl().GroupStart()) != ncclSuccess) return nccl_fail("group start", r);
    nccl().AllGather(ids, ix->gather_ids.p, cnt, ncclInt32, comm, st);
    nccl().AllGather(dist, ix->gather_dist.p, cnt, ncclFloat32, comm, st);
    if ((r = nccl().GroupEnd()) != ncclSuccess) return nccl_fail("all-gather", r);
    CU_TRY(launch_merge_ranks(ix->gather_ids.as<int32_t>(), ix->gather_dist.as<float>(), ix->world, m,
                              k_out, ix->metric == kL2 ? kL2 : kIP, ids, dist, st),
           "merge launch");
    return ST_OK;
}

cudaError_t launch_merge_ranks(const int32_t* gids, const float* gdist, int world, int m, int k,
                               int metric, int32_t* out_ids, float* out_dist, cudaStream_t st) {
    const size_t smem = merge_smem(world, k);
    if (world < 1 || k < 1 || smem > kMergeSmemMax) return cudaErrorInvalidValue;
    if (m == 0) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(merge_ranks_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const int p2 = merge_p2(world);
    const int work = p2 * k;
    const int threads = work >= 256 ? 256 : (work + 31) / 32 * 32;
    merge_ranks_kernel<<<m, threads, smem, st>>>(gids, gdist, world, p2, m, k, metric, out_ids, out_dist);
    return cudaGetLastError();
}

}  // namespace mflat_cu

using namespace mflat_cu;

extern "C" int mflat_cu_merge_ranks(const int32_t* d_gids, const float* d_gdist, int world, int m,
                                    int k, int metric, int32_t* d_out_ids, float* d_out_dist,
                                    void* stream) {
    if (!d_gids || !d_gdist || !d_out_ids || !d_out_dist || world < 1 || m < 0 || k < 1)
        return fail(ST_BAD_ARG, "bad argument");
    CU_TRY(launch_merge_ranks(d_gids, d_gdist, world, m, k, metric == kL2 ? kL2 : kIP, d_out_ids,
                              d_out_dist, static_cast<cudaStream_t>(stream)),
           "merge launch");
    return ST_OK;
}

extern "C" int mflat_cu_comm_unique_id(uint8_t* out_id) {
    if (!out_id) return fail(ST_BAD_ARG, "null argument");
    if (!nccl().ok) return fail(ST_DEVICE, "NCCL (libnccl.so.2) not available");
    ncclUniqueId id;
    const ncclResult_t r = nccl().GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
    static_assert(sizeof(id.internal) == 128, "unique id size");
    std::memcpy(out_id, id.internal, 128);
    return ST_OK;
}

extern "C" int mflat_cu_index_set_shard(mflat_cu_index_t* ix, int rank, int world,
                                        const uint8_t* comm_id, int64_t id_base) {
    if (!ix || world < 1 || rank < 0 || rank >= world || id_base < 0)
        return fail(ST_BAD_ARG, "bad argument");
    DeviceGuard g(ix->device);
    cudaStreamSynchronize(ix->stream);
    comm_release(ix);
    if (world == 1) return ST_OK;
    if (!comm_id) return fail(ST_BAD_ARG, "null communicator id");
    if (world > kMaxRanks) return fail(ST_BAD_ARG, "too many ranks");
    if (!nccl().ok) return fail(ST_DEVICE, "NCCL (libnccl.so.2) not available");
    ncclUniqueId id;
    std::memcpy(id.internal, comm_id, 128);
    ncclComm_t comm = nullptr;
    const ncclResult_t r = nccl().CommInitRank(&comm, world, id, rank);
    if (r != ncclSuccess) return nccl_fail("ncclCommInitRank", r);
    ix->comm = comm;
    ix->rank = rank;
    ix->world = world;
    ix->id_base = id_base;
    return ST_OK;
}

// Used by the search path (index.cu) after enqueueing a sharded search with
// host outputs.
namespace mflat_cu {

int comm_create(void** out, int rank, int world, const uint8_t* comm_id) {
    *out = nullptr;
    if (world < 2 || rank < 0 || rank >= world || !comm_id) return fail(ST_BAD_ARG, "bad communicator");
    if (!nccl().ok) return fail(ST_DEVICE, "NCCL (libnccl.so.2) not available");
    ncclUniqueId id;
    std::memcpy(id.internal, comm_id, 128);
    ncclComm_t comm = nullptr;
    const ncclResult_t r = nccl().CommInitRank(&comm, world, id, rank);
    if (r != ncclSuccess) return nccl_fail("ncclCommInitRank", r);
    *out = comm;
    return ST_OK;
}

void comm_destroy(void* comm) {
    if (comm) nccl().CommDestroy(static_cast<ncclComm_t>(comm));
}

int comm_allgather_bytes(void* comm, const void* send, void* recv, size_t bytes, cudaStream_t st) {
    const ncclResult_t r =
        nccl().AllGather(send, recv, bytes, ncclChar, static_cast<ncclComm_t>(comm), st);
    if (r != ncclSuccess) return nccl_fail("all-gather", r);
    return ST_OK;
}

// Synchronise `st` while watching the communicator (as wait_collective); on a
// peer failure or after MFLAT_NCCL_TIMEOUT_S the communicator is aborted and
// *comm cleared.
int comm_wait(void** comm, cudaStream_t st) {
    const char* env = std::getenv("MFLAT_NCCL_TIMEOUT_S");
    const double limit = env ? std::atof(env) : 300.0;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) return ST_OK;
        if (q != cudaErrorNotReady) return fail(ST_DEVICE, "collective", q);
        ncclResult_t ar = ncclSuccess;
        nccl().CommGetAsyncError(static_cast<ncclComm_t>(*comm), &ar);
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if ((ar != ncclSuccess && ar != ncclInProgress) || el > limit) {
            nccl().CommAbort(static_cast<ncclComm_t>(*comm));
            *comm = nullptr;
            return ar != ncclSuccess && ar != ncclInProgress
                       ? nccl_fail("collective failed", ar)
                       : fail(ST_DEVICE, "collective timed out; communicator aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int wait_stream_checked(mflat_cu_index* ix, cudaStream_t st) {
    if (ix->comm && ix->world > 1) return wait_collective(ix, st);
    CU_TRY(cudaStreamSynchronize(st), "search");
    return ST_OK;
}
}  // namespace mflat_cu
