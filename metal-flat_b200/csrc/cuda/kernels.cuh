// kernels.cuh -- shared layouts, parameter blocks and device helpers of the
// flat-search kernels.
//
// Data layout in HBM (one index on one device), fp32 storage:
//   db_x         : float [cap][d_pad]     the stored rows (exact fp32; Cosine
//                  rows normalised), read by the exact fp64 re-rank;
//   db_h, db_l   : bf16  [cap][d_pad]     screen planes, x = h + l + r with
//                  h = bf16(x), l = bf16(x - h) (round to nearest) and
//                  |r| <= 2^-16 |x|; d_pad is dim rounded up to 64 (one
//                  128-byte TMA/UMMA k-block of 16-bit elements), the padding
//                  is zero.
//   colbias      : float [cap]        per-row additive term of the screen
//                  score: -||x||^2 (L2) or 0 (IP / Cosine); -inf past n, so a
//                  ragged last tile can never enter a top-k list.
//   xmax_bits    : uint  [1]          bits of max_i ||x_i|| (error bound).
//   q_x, q_h, q_l: the queries in the same three forms ([m_pad][d_pad], zero
//                  rows past m); qnorm: float [m] = ||q|| (error bound).
//   part_score/part_id : [n_chunks][m_pad][KP] per (query, db chunk) top-KP
//                  lists of the screen, sorted by (score desc, id asc).
// fp16 / bf16 storage keeps one 16-bit plane (db16, q16) instead.
//
// Screen score (larger = nearer, reference src/Distance.h:65-69):
//   L2 : s = 2 q.x - ||x||^2      (= ||q||^2 - ||q - x||^2, ||q||^2 dropped)
//   IP : s = q.x
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "plan.h"

namespace mflat_cu {

constexpr int kBK = 64;           // 16-bit elements per k-block (128 bytes)
constexpr int kMaxDPadResident = 256;   // A (queries) kept resident in smem up to this
constexpr int kSelectMaxThreads = 256;   // one select thread per list
constexpr int kFbChunks = 64;     // database chunks of the exact fallback scan

enum Metric : int { kL2 = 0, kIP = 1, kCosine = 2 };

// Relative error bound gamma of the fp32-storage screen dot product over d_pad
// elements: |dot' - q.x| <= gamma * ||q|| * ||x||.  The screen sums
// q_h x_h + q_l x_h + q_h x_l (3 x bf16, each product exact in fp32); what
// the split leaves out of q_i x_i (the dropped q_l x_l and the residues r of
// both operands) is about 3 * 2^-16 |q_i x_i|, bounded here by 4 * 2^-16, and
// the fp32 accumulation of 3 * d_pad products adds (3 * d_pad + 16) * 2^-24,
// taken with an 8x safety factor since the tensor core's summation order
// and rounding are not specified.  Sum |q_i x_i| <= ||q|| ||x|| (Cauchy-Schwarz).
inline float screen_gamma(int d_pad) {
    return static_cast<float>(4.0 * 1.52587890625e-05 +                 // 4 * 2^-16
                              (3.0 * d_pad + 16.0) * 4.76837158203125e-07);   // 8 * 2^-24
}

struct ScreenParams {
    int m;                 // queries
    int m_pad;             // multiple of kBM
    int d_pad;             // multiple of kBK (64)
    int64_t n;             // database rows
    int n_tiles;           // ceil(n / kBN)
    int n_qtiles;          // m_pad / kBM
    int n_chunks;          // database chunks (units = n_qtiles * n_chunks)
    int tiles_per_chunk;
    float alpha;           // 2 (L2) or 1 (IP / Cosine)
    const float* colbias;  // [>= n_tiles * kBN]
    float* part_score;     // [n_chunks][m_pad][KP]
    int32_t* part_id;
    int* err;              // device error word (0 = ok)
    // Per query row: key (score_key) of a floor under which no row can enter
    // that query's global top-KP; raised by every finished work unit.
    uint32_t* thr;
    int use_floor;         // 0: ignore and never raise thr (floor pre-pass)
    // Database tiles visited are t * tile_stride for t in [0, n_tiles): a
    // stride > 1 screens an evenly spread sample (the floor pre-pass).
    int tile_stride;
    // Buffer mode (large k): per-query candidate buffers [m_pad][cap].
    uint32_t* buf_cnt;
    float* buf_s;
    int32_t* buf_i;
    uint32_t cap;
    // SIMT path only: the fp32 queries and rows
    const float* q_x;
    const float* db_x;
    // Limit of every bounded mbarrier wait in ns (0: kWaitTimeoutNs).
    uint64_t wait_ns;
    // Test hook (MFLAT_TEST_STALL_SCREEN): the MMA warp first waits on a
    // barrier nothing arrives at, so the bounded wait runs out and the launch
    // ends through its error path (error word kErrTimeout, TMEM freed).
    int test_stall;
};

struct SelectParams {
    double* fb_s; int32_t* fb_i;          // exact fallback scratch [m][kFbChunks][k_out]
    int m, m_pad, dim, d_pad, k_out, n_chunks, metric;
    int64_t n;
    const float* part_score; const int32_t* part_id;
    const float* q_x; const float* qnorm;     // fp32 queries [m_pad][d_pad], ||q||
    const float* db_x;                        // fp32 rows [n][d_pad]
    const unsigned* xmax_bits;
    float gamma;           // relative dot-product error bound of the screen
    int64_t id_base;       // added to every returned id (row sharding)
    int32_t* out_ids; float* out_dist;    // [m][k_out]
    int* flag_count; int* flag_list;      // queries needing the exact full scan
    int* err;
};

// Large-k selection over the candidate buffers (select_large.cu).
struct LargeSelectParams {
    int m, m_pad, dim, d_pad, k_out, metric;
    const uint32_t* cnt; const float* buf_s; const int32_t* buf_i; uint32_t cap;
    const uint32_t* thr;                  // floor keys used by the screen
    int exact;                            // 1: fp64 re-rank of the proven window
    const float* q_x; const float* qnorm;
    const float* db_x;
    const unsigned* xmax_bits; float gamma;
    const float* qsq;                     // recall path: ||q||^2 for L2 distances
    int64_t id_base;
    int32_t* out_ids; float* out_dist;
    int* flag_count; int* flag_list;      // proof failures (exact path)
    int* overflow;                        // buffers that overflowed / too many ties
    int64_t n;                            // database rows (candidate ids are below)
    const int* err;                       // device error word of the screens
};

// ---------------------------------------------------------------------------
// Per-thread top-KP list in registers, sorted by score descending.  insert()
// is called only when v > s[KP-1]; strict '>' keeps an earlier (lower) id
// ahead of a later equal score, matching the reference's cpuSearch scan
// (src/FlatIndex.mm:272-281) when ids are visited in ascending order.
template <int KP>
struct TopList {
    float s[KP];
    int id[KP];
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int i = 0; i < KP; ++i) { s[i] = -__int_as_float(0x7f800000); id[i] = -1; }
    }
    __device__ __forceinline__ float worst() const { return s[KP - 1]; }
    __device__ __forceinline__ void insert(float v, int vid) {
#pragma unroll
        for (int j = KP - 1; j >= 0; --j) {
            const bool cj = v > s[j];
            const bool cjm1 = (j > 0) ? (v > s[j > 0 ? j - 1 : 0]) : false;
            const float ns = cj ? (cjm1 ? s[j > 0 ? j - 1 : 0] : v) : s[j];
            const int nid = cj ? (cjm1 ? id[j > 0 ? j - 1 : 0] : vid) : id[j];
            s[j] = ns;
            id[j] = nid;
        }
    }
};

// (score desc, id asc) order with id < 0 ranked last.
__device__ __forceinline__ bool cand_better(float sa, int ia, float sb, int ib) {
    if (ia < 0) return false;
    if (ib < 0) return true;
    if (sa != sb) return sa > sb;
    return ia < ib;
}

// ------------------------------------------------------------- launchers
// All launchers enqueue on `stream` and return the launch status.
// kp = 0 selects buffer mode (append every score above the floor).
// The tensor-core screen (screen.cu).  kF16 / kBF16: 16-bit storage, one
// plane (maps a, b); kBF16x3: fp32 storage, bf16 split planes (a / a2: the
// queries' h / l planes, b / b2: the rows').  `bias`: the rows' bias parts,
// [rows][8] bf16 = (h, m, l, 0, ...) of colbias / alpha, no swizzle (split_bias
// in index.cu).  The b, b2 and bias maps' boxes are screen_rows_per_cta(pair)
// rows high.  kp 0 = buffer mode; list mode (kp 4 .. 32) writes two lists per
// (query, chunk), list index = chunk * 2 + half.  pair: CTA pairs (grid even,
// grid / 2 pairs; each pair works on two query tiles per unit).
enum class ScreenKind : int { kF16 = 0, kBF16 = 1, kBF16x3 = 2 };
struct ScreenMaps {
    CUtensorMap a, a2, b, b2, bias;
};
constexpr int kScreenListsPerChunk = 2;
cudaError_t launch_screen(int kp, ScreenKind kind, const ScreenMaps& maps, const ScreenParams& p,
                          int grid, bool pair, cudaStream_t stream);
int screen_smem_bytes(int d_pad, bool x3, bool pair);
int screen_rows_per_cta(bool pair);
cudaError_t launch_screen_simt(int kp, const ScreenParams& p, cudaStream_t stream);
cudaError_t launch_select_exact(int kp, const SelectParams& p, cudaStream_t stream);
cudaError_t launch_fallback_exact(const SelectParams& p, int grid, cudaStream_t stream);
cudaError_t launch_select_large(const LargeSelectParams& p, cudaStream_t stream);
// Recall path, list mode: merge n_lists lists per query, write the top k_out
// with screen distances (L2: max(0, ||q||^2 - s); IP / Cosine: s).
cudaError_t launch_select_recall(int kp, const SelectParams& p, const float* qsq, cudaStream_t stream);
cudaError_t launch_prepass_floor(const float* part_s, const int32_t* part_i, int n_lists, int m,
                                 int m_pad, int kp1, int want, int r_guess, uint32_t* thr,
                                 uint32_t* thr_guess, cudaStream_t stream);
cudaError_t launch_buffer_floor(const uint32_t* cnt, const float* buf_s, uint32_t cap, int want,
                                int r_stat, int m, uint32_t* thr, uint32_t* thr_stat, int* short_count,
                                cudaStream_t stream);
cudaError_t launch_floor_check(const uint32_t* cnt, const uint32_t* used, const uint32_t* valid,
                               int want, int m, int* failures, cudaStream_t stream);
cudaError_t launch_kmeans_select(const SelectParams& p, int32_t* out, int grid_fallback,
                                 cudaStream_t stream);

}  // namespace mflat_cu
