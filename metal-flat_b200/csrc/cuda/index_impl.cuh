// index_impl.cuh -- internal state of a device index, shared by index.cu
// (create / add / search), kmeans.cu and comm.cu.  Not installed.
#pragma once

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <cstdint>
#include <string>

#include "kernels.cuh"
#include "mflat_cuda.h"

namespace mflat_cu {

constexpr int kTimingRing = 32;   // searches whose timing events may be in flight
constexpr int kHostWords = 8 + kTimingRing;

enum : int { ST_OK = 0, ST_BAD_ARG = 2, ST_ALLOC = 3, ST_INTERNAL = 5, ST_DEVICE = 6 };

int fail(int status, const char* what, cudaError_t e = cudaSuccess);

#define CU_TRY(expr, what)                                                                   \
    do {                                                                                     \
        cudaError_t e_ = (expr);                                                             \
        if (e_ != cudaSuccess)                                                               \
            return ::mflat_cu::fail(e_ == cudaErrorMemoryAllocation ? ::mflat_cu::ST_ALLOC    \
                                                                    : ::mflat_cu::ST_DEVICE, \
                                    what, e_);                                               \
    } while (0)

// Scratch buffer grown on demand and reused across calls.
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    cudaError_t ensure(size_t need);
    void release();
    template <class T>
    T* as() const { return static_cast<T*>(p); }
};

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev);
    ~DeviceGuard();
};

// NVTX range for the host side of one operation (add, search, all-gather,
// merge); costs nothing unless a profiler is attached.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

inline unsigned blocks_for(int64_t n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

// Result of the screen stage of one search (per (query, chunk) top-KP lists).
struct ScreenRun {
    int kp = 0, m = 0, m_pad = 0, n_chunks = 0;
    int n_lists = 0;                  // lists per query (chunks x lists per chunk)
    const float* q_x = nullptr;       // fp32 queries [m_pad][d_pad] (exact re-rank)
    const float* qnorm = nullptr;
    const float* part_s = nullptr;
    const int32_t* part_i = nullptr;
    int launches = 0;
};

}  // namespace mflat_cu

struct mflat_cu_index {
    int device = 0;
    int dim = 0, d_pad = 0, metric = 0, storage = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    int64_t n = 0, cap = 0;
    void* db16 = nullptr;         // fp16 / bf16 storage: [cap][d_pad] 16-bit
    float* db_x = nullptr;        // fp32 storage: the rows [cap][d_pad]
    uint16_t* db_h = nullptr;     // fp32 storage: bf16 screen planes [cap][d_pad]
    uint16_t* db_l = nullptr;
    float* colbias = nullptr;     // [cap], -inf past n
    float* dnorm = nullptr;       // [cap]
    unsigned* xmax_bits = nullptr;
    int* err = nullptr;           // device error word
    int* flag_count = nullptr;    // queries routed to the exact full scan
    int* host_words = nullptr;    // pinned: [0] err, [4..7] status words, [8 + slot] fallback
                                  // query count of timing slot `slot`
    mflat_cu::DevBuf stage_in, q_in, q_x, q_h, q_l, qnorm, part_s, part_i, flag_list, out_ids, out_dist;
    mflat_cu::DevBuf thr, thr_stat, fb_s, fb_i;
    mflat_cu::DevBuf buf_cnt, buf_s, buf_i, lk_words;   // large-k candidate buffers
    size_t lk_budget = 0;                               // their byte budget (first large search)
    mflat_cu::DevBuf q16, qsq;                          // 16-bit queries, ||q||^2
    // Screen bias parts: colbias / alpha as three bf16 parts per row
    // ([cap][8] bf16 = (h, m, l, 0 ...); rows past n: (-inf, 0, 0)), the
    // operand of the screens' bias MMA.  Allocated with the rows (grow); rows
    // [0, bias16_rows) are current, add / reset lower it.
    uint4* bias16 = nullptr;
    int64_t bias16_rows = 0;
    // Timing (mflat_cu_index_set_timing): each search records 4 events into
    // one slot of a ring and returns without waiting for them; a slot is read
    // (and its device times added to `sum`) only when it is reused, or by
    // last_timing / timing_sum, so timing does not serialise back-to-back
    // searches.  `ev` points at the slot of the search in progress; `last`
    // collects that search's launch counts.
    bool timing = false;
    cudaEvent_t* ev = nullptr;
    struct TimingSlot {
        cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
        mflat_cu_timing_t t{};
        bool pending = false;
    };
    mutable TimingSlot ring[mflat_cu::kTimingRing];
    int ring_next = 0, ring_last = -1;
    mutable mflat_cu_timing_t sum{};
    mutable int sum_n = 0;
    mflat_cu_timing_t last{};
    bool force_simt = false;
    // Tensor-core screens of batches with two or more query tiles run as CTA
    // pairs (cta_group::2); MFLAT_SCREEN_PAIR=0 at creation keeps every screen
    // on single CTAs.
    bool screen_pair = true;
    // Limit of the screens' bounded waits in ns (MFLAT_WAIT_LIMIT_MS; 0 = 2 s).
    uint64_t wait_ns = 0;
    // Test hook (MFLAT_TEST_STALL_SCREEN set at creation): the next fp32
    // screen launch stalls on purpose until its bounded wait runs out; one shot.
    int test_stall = 0;
    // row sharding (comm.cu)
    void* comm = nullptr;
    int rank = 0, world = 1;
    int64_t id_base = 0;
    mflat_cu::DevBuf gather_ids, gather_dist, merge_tmp_ids, merge_tmp_dist;
};

namespace mflat_cu {

// Upload (if needed), split the queries and run the tensor-core screen with
// top-KP lists on stream `st`.  `queries` is device memory when on_device.
int run_screen(mflat_cu_index* ix, const float* queries, int m, int kp, int on_device,
               cudaStream_t st, ScreenRun& out, int max_chunks = kMaxChunks);
int check_device_error(mflat_cu_index* ix, cudaStream_t st);
// Timing ring (no-ops unless timing is on): begin points ix->ev at a free
// slot; end (after the search's last event is recorded on the stream) marks
// the slot pending with the counts in ix->last.
void timing_begin(mflat_cu_index* ix);
void timing_end(mflat_cu_index* ix);
void comm_release(mflat_cu_index* ix);
// Plain communicator helpers (k-means training over sharded points).
int comm_create(void** out, int rank, int world, const uint8_t* comm_id);
void comm_destroy(void* comm);
int comm_allgather_bytes(void* comm, const void* send, void* recv, size_t bytes, cudaStream_t st);
int comm_wait(void** comm, cudaStream_t st);
int shard_merge(mflat_cu_index* ix, int m, int k_out, int32_t* ids, float* dist, cudaStream_t st);
// Merge of gathered per-rank lists [world][m][k] into [m][k] (comm.cu).
cudaError_t launch_merge_ranks(const int32_t* gids, const float* gdist, int world, int m, int k,
                               int metric, int32_t* out_ids, float* out_dist, cudaStream_t st);
// Synchronise `st`; with a communicator attached, watch it for peer failure.
int wait_stream_checked(mflat_cu_index* ix, cudaStream_t st);
const char* last_error_message();
cudaError_t launch_prep_queries(const float* src, int m, int m_pad, int dim, int d_pad, int metric,
                                float* q_x, uint16_t* q_h, uint16_t* q_l, float* qnorm,
                                cudaStream_t st);
bool encode_map_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                     uint32_t box_rows);
// Bias parts of rows [0, rows_pad(n)) current (a kernel launch on `st` when
// rows were added; no allocation), and their tensor map (boxes for a single-CTA
// or a CTA-pair screen).
int prepare_bias_parts(mflat_cu_index* ix, cudaStream_t st, CUtensorMap* map, bool pair = false);
// Whether a screen over n_qtiles query tiles runs as CTA pairs, and its grid.
bool screen_pair_for(const mflat_cu_index* ix, int n_qtiles);
int screen_grid(const mflat_cu_index* ix, int n_qtiles, int n_chunks, bool pair);
// Screen lists per chunk of the fp32-storage screen in use (tensor core: 2,
// MFLAT_SCREEN=simt cross-check: 1).
int fp32_lists_per_chunk(const mflat_cu_index* ix);
cudaError_t launch_fill_empty(int32_t* ids, float* dist, int64_t n, float v, cudaStream_t st);
void plan_screen_chunks(int n_qtiles, int n_tiles, int num_sms, int max_chunks, int& n_chunks,
                        int& tiles_per_chunk);

}  // namespace mflat_cu
