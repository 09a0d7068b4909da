// plan.h -- host-side planning of the screens: how the database tiles are cut
// into chunks (a work unit is one query tile x one chunk) and, for large k, the
// floor-estimate plan.  Plain C++ without CUDA types, so the CPU test suite
// compiles and checks it on its own.
#pragma once

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>

namespace mflat_cu {

constexpr int kBM = 128;          // queries per tile (TMEM lanes)
constexpr int kBN = 256;          // database rows per tile (UMMA N)
constexpr int kMaxChunks = 256;   // candidate lists per query (select kernel fan-in)
constexpr int kFloorMaxEntries = 4096;   // list entries per query the floor select takes
constexpr int64_t kAllRowsBuffered = 32768;   // large k below this many rows: no pre-pass

// Screens run as single CTAs or as CTA pairs (two SMs, two query tiles per
// work unit).  Query units of a batch and the units that run at once.
inline int screen_qunits(int n_qtiles, bool pair) { return pair ? (n_qtiles + 1) / 2 : n_qtiles; }
inline int screen_slots(int num_sms, bool pair) { return pair ? std::max(1, num_sms / 2) : num_sms; }
// CTA pairs when allowed and the batch has at least two query tiles.
inline bool screen_pair_for(bool allowed, int n_qtiles) { return allowed && n_qtiles >= 2; }

// Database chunks per query tile.  The critical path of a launch is the
// tiles its busiest SM (or pair) streams: waves x tiles per chunk, where a wave
// is one work unit on every slot.  The plan takes the fewest chunks whose
// critical path is within 1 % of the shortest (fewer chunks: fewer candidate
// lists to merge and fewer per-unit query-tile loads).
inline void plan_chunks(int n_qtiles, int n_tiles, int num_sms, int max_chunks, int& n_chunks,
                        int& tiles_per_chunk, int min_chunks = 1) {
    const int smin = std::max(1, std::min(min_chunks, std::min(max_chunks, n_tiles)));
    // beyond a few chunks per slot more chunks only add lists and unit overheads
    const int smax = std::min({max_chunks, n_tiles, smin + 4 * std::max(num_sms, 1)});
    auto span = [&](int s) -> int64_t {
        const int tpc = (n_tiles + s - 1) / s;
        const int sc = (n_tiles + tpc - 1) / tpc;
        const int64_t units = static_cast<int64_t>(n_qtiles) * sc;
        const int64_t waves = (units + num_sms - 1) / num_sms;
        return waves * tpc;
    };
    int64_t best = span(smin);
    for (int s = smin + 1; s <= smax; ++s) best = std::min(best, span(s));
    int pick = smin;
    for (int s = smin; s <= smax; ++s) {
        if (span(s) * 100 <= best * 101) { pick = s; break; }
    }
    tiles_per_chunk = (n_tiles + pick - 1) / pick;
    n_chunks = (n_tiles + tiles_per_chunk - 1) / tiles_per_chunk;
}

// Chunking of a buffer-mode pass (no per-chunk lists, so no fan-in limit):
// chunks of at most ~8 MB of rows.  The CTAs working on the same chunk share
// its tiles through L2, but in buffer mode their progress drifts apart (the
// appends differ per query tile); with small chunks the rows still in use by
// the leading and the trailing CTAs stay within L2 instead of being fetched
// from HBM again by each query tile.
inline void plan_buffer_chunks(int n_qtiles, int n_tiles, int num_sms, size_t tile_bytes,
                               int& n_chunks, int& tiles_per_chunk) {
    const int max_tpc = static_cast<int>(
        std::max<size_t>(16, (size_t(8) << 20) / std::max<size_t>(tile_bytes, 1)));
    const int min_chunks = (n_tiles + max_tpc - 1) / max_tpc;
    plan_chunks(n_qtiles, n_tiles, num_sms, n_tiles, n_chunks, tiles_per_chunk, min_chunks);
}

struct LargePlan {
    bool prepass = false;          // floor estimate before the main pass
    bool two_stage = false;        // stage A (list, sparse) + stage B (buffer, denser)
    int lists = 0;                 // stage-A lists (chunks)
    int stride_a = 1, sample_a = 0;
    int stride_b = 1, sample_b = 0;
    int chunks_a = 0, tpc_a = 0;   // stage-A chunking (>= lists, spread over the SMs)
    int r_stat = 0;                // rank of the statistical floor in the stage-B sample (0: none)
    int r_guess = 0;               // rank of stage B's statistical floor in the stage-A union
    uint32_t cap = 0;
    int batch = 0;
};

// Large-k plan (k > 21 fp32, or the 16-bit buffer path) for n rows and a batch
// of m queries.  want: rank whose sampled score becomes the floor (2k exact
// path, k recall); kp1: list length of the stage-A pass; lists_per_chunk: lists
// one list-mode chunk produces (f16 kernel: 2); budget_bytes: what the
// candidate buffers of one query batch may take; pair: CTA-pair screens are
// allowed (stage A's chunks are then planned in pair units).
inline LargePlan plan_large(int64_t n, int k, int m, int kp1, int want, int lists_per_chunk,
                            int num_sms, size_t budget_bytes, bool pair = false) {
    LargePlan P;
    const int n_tiles = static_cast<int>((n + kBN - 1) / kBN);
    const int64_t n_round = (n + 255) / 256 * 256;
    if (n <= kAllRowsBuffered) {
        P.cap = static_cast<uint32_t>(n_round);
    } else {
        // union of lists * kp1 >= 2 * want sampled scores; floor = its want-th best
        const int lists_total = std::min(4096 / kp1, std::max(1, (2 * want + kp1 - 1) / kp1));
        P.lists = std::max(1, (lists_total + lists_per_chunk - 1) / lists_per_chunk);
        P.stride_b = 16;
        while (P.stride_b > 1 && (n_tiles + P.stride_b - 1) / P.stride_b < 2 * P.lists) P.stride_b /= 2;
        P.sample_b = (n_tiles + P.stride_b - 1) / P.stride_b;
        if (P.sample_b < P.lists) {                      // too small to sample: buffer all
            P.cap = static_cast<uint32_t>(n_round);
        } else {
            P.prepass = true;
            P.stride_a = P.stride_b;
            P.sample_a = P.sample_b;
            // a list-mode pass over 1/stride_a of the tiles (the sparsest of
            // 1/256, 1/128, 1/64 that still gives every list two tiles), then a
            // buffer-mode pass over 1/stride_b sharpens its floor
            for (int sa = 256; sa >= 64 && P.stride_b == 16; sa /= 2) {
                if ((n_tiles + sa - 1) / sa >= 2 * P.lists) {
                    P.two_stage = true;
                    P.stride_a = sa;
                    P.sample_a = (n_tiles + sa - 1) / sa;
                    break;
                }
            }
            if (P.two_stage) {
                // about want / stride_b of the sampled rows are in the global
                // top-want; six standard deviations above that (see
                // buffer_floor_kernel) the floor admits ~r_stat * stride_b rows
                const double mean = static_cast<double>(want) / P.stride_b;
                const int r = static_cast<int>(std::ceil(mean + 6.0 * std::sqrt(mean))) + 1;
                P.r_stat = r < want ? r : 0;
                // stage B only needs its sample's top `want`, i.e. rows down to about
                // the global (want * stride_b)-th; the stage-A sample holds about
                // want * stride_b / stride_a of those
                const double mean_a = static_cast<double>(want) * P.stride_b / P.stride_a;
                const int ra = static_cast<int>(std::ceil(mean_a + 6.0 * std::sqrt(mean_a))) + 1;
                P.r_guess = ra < want ? ra : 0;
            }
            // the floor is about the (want * stride_b)-th best row overall; the
            // stage-B buffer holds about want * stride_a / stride_b rows
            const int64_t expect = static_cast<int64_t>(want) * P.stride_b;
            int64_t cap = std::max<int64_t>(4 * expect, 4096);
            cap = std::min<int64_t>((cap + 255) / 256 * 256, n_round);
            P.cap = static_cast<uint32_t>(cap);
        }
    }
    const size_t per_q = static_cast<size_t>(P.cap) * 8 + 64;
    P.batch = static_cast<int>(std::max<size_t>(kBM, std::min<size_t>(m, budget_bytes / per_q)));
    P.batch = std::min(P.batch, m);
    if (P.prepass) {
        // Stage A needs >= `lists` chunks for its union; more chunks only enlarge
        // the union (a sharper floor) and keep every SM busy when few query
        // tiles share the pass.
        const int n_qt = (P.batch + kBM - 1) / kBM;
        const int max_a = std::max(P.lists, kFloorMaxEntries / (kp1 * lists_per_chunk));
        const bool pr = screen_pair_for(pair, n_qt);
        plan_chunks(screen_qunits(n_qt, pr), P.sample_a, screen_slots(num_sms, pr), max_a, P.chunks_a,
                    P.tpc_a);
        if (P.chunks_a < P.lists) {
            // whole tiles per list, as few as keep >= `lists` chunks; coarser
            // only where that many lists would not fit the floor select
            int tpc = std::max(1, P.sample_a / P.lists);
            while ((P.sample_a + tpc - 1) / tpc > max_a) ++tpc;
            P.tpc_a = tpc;
            P.chunks_a = (P.sample_a + tpc - 1) / tpc;
        }
    }
    return P;
}

}  // namespace mflat_cu
