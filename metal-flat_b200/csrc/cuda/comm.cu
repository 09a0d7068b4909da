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

namespace mflat_cu {
namespace {

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

// One thread per query: P-way merge of the gathered per-rank lists
// ([P][m][k], each nearest-first, ids global) into [m][k].
__global__ void merge_ranks_kernel(const int32_t* __restrict__ gids, const float* __restrict__ gdist,
                                   int world, int m, int k, int metric, int32_t* __restrict__ out_ids,
                                   float* __restrict__ out_dist) {
    const int qi = blockIdx.x * blockDim.x + threadIdx.x;
    if (qi >= m) return;
    int head[8];
    for (int p = 0; p < world; ++p) head[p] = 0;
    const float empty = metric == kL2 ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
    for (int j = 0; j < k; ++j) {
        int bp = -1;
        int32_t bid = -1;
        float bd = 0.0f;
        for (int p = 0; p < world; ++p) {
            if (head[p] >= k) continue;
            const int64_t o = (static_cast<int64_t>(p) * m + qi) * k + head[p];
            const int32_t id = gids[o];
            if (id < 0) continue;
            const float d = gdist[o];
            bool take = bp < 0;
            if (!take) {
                if (d != bd) take = metric == kL2 ? (d < bd) : (d > bd);
                else take = id < bid;
            }
            if (take) { bp = p; bid = id; bd = d; }
        }
        const int64_t oo = static_cast<int64_t>(qi) * k + j;
        if (bp < 0) {
            out_ids[oo] = -1;
            out_dist[oo] = empty;
        } else {
            out_ids[oo] = bid;
            out_dist[oo] = bd;
            ++head[bp];
        }
    }
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
    if (ix->world > 8) return fail(ST_BAD_ARG, "at most 8 ranks");
    const size_t cnt = static_cast<size_t>(m) * k_out;
    CU_TRY(ix->gather_ids.ensure(cnt * ix->world * sizeof(int32_t)), "gather buffer");
    CU_TRY(ix->gather_dist.ensure(cnt * ix->world * sizeof(float)), "gather buffer");
    auto comm = static_cast<ncclComm_t>(ix->comm);
    ncclResult_t r;
    if ((r = nccl().GroupStart()) != ncclSuccess) return nccl_fail("group start", r);
    nccl().AllGather(ids, ix->gather_ids.p, cnt, ncclInt32, comm, st);
    nccl().AllGather(dist, ix->gather_dist.p, cnt, ncclFloat32, comm, st);
    if ((r = nccl().GroupEnd()) != ncclSuccess) return nccl_fail("all-gather", r);
    merge_ranks_kernel<<<blocks_for(m, 128), 128, 0, st>>>(
        ix->gather_ids.as<int32_t>(), ix->gather_dist.as<float>(), ix->world, m, k_out,
        ix->metric == kL2 ? kL2 : kIP, ids, dist);
    CU_TRY(cudaGetLastError(), "merge launch");
    return ST_OK;
}

}  // namespace mflat_cu

using namespace mflat_cu;

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
    if (world > 8) return fail(ST_BAD_ARG, "at most 8 ranks");
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
