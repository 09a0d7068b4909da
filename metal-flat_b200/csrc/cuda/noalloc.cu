// noalloc.cu -- exact search that allocates no device memory.
//
// Some callers cannot call cudaMalloc: a serving process whose device memory is
// already reserved by a framework's caching allocator (a raw cudaMalloc then
// fails or fragments that pool), or a latency-critical loop in which the
// implicit device-wide synchronisation of cudaMalloc / cudaFree would stall
// every other stream.  mflat_cu_index_search_noalloc serves them: the caller
// passes device inputs and outputs, and all per-call scratch of the search
// (split queries, candidate lists, score floors, fallback lists) lives in the
// fixed array below, which every GPU that loads this library holds until the
// process exits.
//
// Limits (sizes beyond them are rejected with ST_BAD_ARG and a message):
// at most kNaMaxQueries queries per call, dim <= kNaMaxDim, k <= kNaMaxK, fp32
// storage.  The database itself is the index's (allocated by add()).
//
// The array is shared by every call on a device and keeps the last call's
// contents; the parts that must start at zero (score floors, fallback count)
// are cleared on the call's stream.  Calls that overlap on the GPU -- two
// streams, or two indexes on one device -- race on the array; serialise them.
// The first call on a device resolves the array's device address with
// cudaGetSymbolAddress (the host-side name is only a stand-in); make that first
// call before any stream capture.  This entry point always runs the
// tensor-core screen (the MFLAT_SCREEN=simt cross-check does not apply to it)
// and records no timing events (mflat_cu_index_last_timing keeps describing
// the index's last regular search).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <mutex>

#include "index_impl.cuh"
#include "kernels.cuh"
#include "mflat_cuda.h"

namespace mflat_cu {
namespace {

constexpr int kNaMaxQueries = 128;                   // one query tile
constexpr int kNaMaxDim = 128;
constexpr int kNaMaxK = 21;
constexpr int kNaKP = 32;
constexpr int kNaMaxChunks = 16;                     // x 2 lists per chunk
constexpr size_t kNaScratchBytes = size_t(4) << 20; // 4 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNaScratchBytes];

constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Byte offsets of the per-call buffers inside g_noalloc_scratch: the fp32
// queries and their bf16 split planes, norms, candidate lists, floors and the
// exact fallback's lists.
constexpr size_t kOffQX = 0;
constexpr size_t kOffQH = kOffQX + align256(size_t(kNaMaxQueries) * kNaMaxDim * 4);
constexpr size_t kOffQL = kOffQH + align256(size_t(kNaMaxQueries) * kNaMaxDim * 2);
constexpr size_t kOffQNorm = kOffQL + align256(size_t(kNaMaxQueries) * kNaMaxDim * 2);
constexpr size_t kOffPartS = kOffQNorm + align256(size_t(kNaMaxQueries) * 4);
constexpr size_t kOffPartI = kOffPartS + align256(size_t(kNaMaxChunks) * kScreenListsPerChunk * kNaMaxQueries * kNaKP * 4);
constexpr size_t kOffThr = kOffPartI + align256(size_t(kNaMaxChunks) * kScreenListsPerChunk * kNaMaxQueries * kNaKP * 4);
constexpr size_t kOffFlag = kOffThr + align256(size_t(kNaMaxQueries) * 4);
constexpr size_t kOffFbS = kOffFlag + align256(size_t(kNaMaxQueries) * 4);
constexpr size_t kOffFbI = kOffFbS + align256(size_t(kNaMaxQueries) * kFbChunks * kNaMaxK * 8);
constexpr size_t kOffEnd = kOffFbI + align256(size_t(kNaMaxQueries) * kFbChunks * kNaMaxK * 4);
static_assert(kOffEnd <= kNaScratchBytes, "no-alloc scratch layout exceeds the array");

constexpr int kMaxDevices = 64;
std::mutex g_addr_mu;
unsigned char* g_addr[kMaxDevices] = {};

// Device address of the array on `device` (which must be current).
int scratch_base(int device, unsigned char** out) {
    if (device < 0 || device >= kMaxDevices) return fail(ST_BAD_ARG, "device index out of range");
    std::lock_guard<std::mutex> lk(g_addr_mu);
    if (!g_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return fail(ST_DEVICE, "cudaGetSymbolAddress(no-alloc scratch)", e);
        g_addr[device] = static_cast<unsigned char*>(p);
    }
    *out = g_addr[device];
    return ST_OK;
}

}  // namespace
}  // namespace mflat_cu

using namespace mflat_cu;

extern "C" int mflat_cu_index_search_noalloc(mflat_cu_index_t* ix, const float* d_queries, int m,
                                             int k_out, int32_t* d_ids, float* d_dist,
                                             void* stream) {
    if (!ix || (m > 0 && (!d_queries || !d_ids || !d_dist))) return fail(ST_BAD_ARG, "null argument");
    char msg[160];
    if (m < 0 || m > kNaMaxQueries) {
        std::snprintf(msg, sizeof msg, "no-alloc search: m=%d outside [0, %d] queries per call", m,
                      kNaMaxQueries);
        return fail(ST_BAD_ARG, msg);
    }
    if (k_out < 1 || k_out > kNaMaxK) {
        std::snprintf(msg, sizeof msg, "no-alloc search: k=%d outside [1, %d]", k_out, kNaMaxK);
        return fail(ST_BAD_ARG, msg);
    }
    if (ix->dim > kNaMaxDim || ix->storage != 0) {
        std::snprintf(msg, sizeof msg, "no-alloc search: needs fp32 storage and dim <= %d (dim=%d)",
                      kNaMaxDim, ix->dim);
        return fail(ST_BAD_ARG, msg);
    }
    if (ix->world > 1) return fail(ST_BAD_ARG, "no-alloc search: sharded indexes are not supported");
    if (m == 0) return ST_OK;
    DeviceGuard g(ix->device);
    unsigned char* base = nullptr;
    int rc = scratch_base(ix->device, &base);
    if (rc != ST_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    rc = check_device_error(ix, st);   // the previous asynchronous call on this index
    if (rc != ST_OK) return rc;
    const int64_t mk = static_cast<int64_t>(m) * k_out;
    const float empty = ix->metric == kL2 ? INFINITY : -INFINITY;
    if (ix->n == 0) {
        CU_TRY(launch_fill_empty(d_ids, d_dist, mk, empty, st), "fill");
        return ST_OK;
    }

    const int m_pad = kBM;
    const int d_pad = ix->d_pad;
    const int n_tiles = static_cast<int>((ix->n + kBN - 1) / kBN);
    int n_chunks = 1, tpc = n_tiles;
    plan_screen_chunks(1, n_tiles, ix->num_sms, kNaMaxChunks, n_chunks, tpc);

    float* q_x = reinterpret_cast<float*>(base + kOffQX);
    uint16_t* q_h = reinterpret_cast<uint16_t*>(base + kOffQH);
    uint16_t* q_l = reinterpret_cast<uint16_t*>(base + kOffQL);
    float* qnorm = reinterpret_cast<float*>(base + kOffQNorm);
    float* part_s = reinterpret_cast<float*>(base + kOffPartS);
    int32_t* part_i = reinterpret_cast<int32_t*>(base + kOffPartI);
    uint32_t* thr = reinterpret_cast<uint32_t*>(base + kOffThr);
    int* flag_list = reinterpret_cast<int*>(base + kOffFlag);
    double* fb_s = reinterpret_cast<double*>(base + kOffFbS);
    int32_t* fb_i = reinterpret_cast<int32_t*>(base + kOffFbI);

    CU_TRY(launch_prep_queries(d_queries, m, m_pad, ix->dim, d_pad, ix->metric, q_x, q_h, q_l, qnorm, st),
           "query prep launch");
    CU_TRY(cudaMemsetAsync(thr, 0, static_cast<size_t>(m_pad) * sizeof(uint32_t), st), "floors");
    CU_TRY(cudaMemsetAsync(ix->flag_count, 0, sizeof(int), st), "fallback count");

    ScreenParams sp{};
    sp.m = m;
    sp.m_pad = m_pad;
    sp.d_pad = d_pad;
    sp.n = ix->n;
    sp.n_tiles = n_tiles;
    sp.n_qtiles = 1;
    sp.n_chunks = n_chunks;
    sp.tiles_per_chunk = tpc;
    sp.alpha = ix->metric == kL2 ? 2.0f : 1.0f;
    sp.colbias = ix->colbias;
    sp.part_score = part_s;
    sp.part_id = part_i;
    sp.err = ix->err;
    sp.thr = thr;
    sp.tile_stride = 1;
    sp.use_floor = 1;
    sp.wait_ns = ix->wait_ns;
    ScreenMaps maps;
    if (!encode_map_bf16(&maps.a, q_h, d_pad, m_pad, kBM) ||
        !encode_map_bf16(&maps.a2, q_l, d_pad, m_pad, kBM) ||
        !encode_map_bf16(&maps.b, ix->db_h, d_pad, ix->n, kBN) ||
        !encode_map_bf16(&maps.b2, ix->db_l, d_pad, ix->n, kBN))
        return fail(ST_DEVICE, "tensor map encoding failed");
    // the rows' bias parts live with the rows (allocated by add); this only
    // brings rows added since the last search up to date, on `st`
    rc = prepare_bias_parts(ix, st, &maps.bias);
    if (rc != ST_OK) return rc;
    const int grid = n_chunks < ix->num_sms ? n_chunks : ix->num_sms;
    CU_TRY(launch_screen(kNaKP, ScreenKind::kBF16x3, maps, sp, grid, false, st), "screen launch");

    SelectParams sel{};
    sel.m = m;
    sel.m_pad = m_pad;
    sel.dim = ix->dim;
    sel.d_pad = d_pad;
    sel.k_out = k_out;
    sel.n_chunks = n_chunks * kScreenListsPerChunk;
    sel.metric = ix->metric == kL2 ? kL2 : kIP;
    sel.n = ix->n;
    sel.part_score = part_s;
    sel.part_id = part_i;
    sel.q_x = q_x;
    sel.qnorm = qnorm;
    sel.db_x = ix->db_x;
    sel.xmax_bits = ix->xmax_bits;
    sel.gamma = screen_gamma(d_pad);
    sel.out_ids = d_ids;
    sel.out_dist = d_dist;
    sel.flag_count = ix->flag_count;
    sel.flag_list = flag_list;
    sel.err = ix->err;
    sel.fb_s = fb_s;
    sel.fb_i = fb_i;
    CU_TRY(launch_select_exact(kNaKP, sel, st), "select launch");
    CU_TRY(launch_fallback_exact(sel, ix->num_sms, st), "fallback launch");
    cudaMemcpyAsync(&ix->host_words[0], ix->err, sizeof(int), cudaMemcpyDeviceToHost, st);
    return ST_OK;
}
