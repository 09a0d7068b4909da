// select.cu -- candidate merge, exactness proof and exact re-rank.
//
// The screen (screen.cu) leaves, per query and database chunk, the top-KP
// rows by the fp32 screen score s' (3 x bf16 dot + norm term).  Every screen
// score is within E of the exact score s (a-priori bound, see error_bound()).
// If the KP-th best merged screen score is below (k-th best) - 2E, every row
// of the true top-k is among the KP candidates (standard argument: the k rows
// of the true top-k all have s' >= s_(k) - E, hence s'_(k) >= s_(k) - E, and
// s'_(k) <= s_(k) + E; a true top-k row therefore has s' >= s'_(k) - 2E).
// The candidates are then re-scored exactly in fp64 from the stored fp32 rows
// and ordered by (distance, id), which is the fp64 brute-force
// oracle's order (reference semantics: src/Distance.h:26-81, ties to the
// lowest id as in src/FlatIndex.mm:272-281).  Queries whose proof fails
// (many near-equal scores, e.g. duplicated rows) are re-done by an exact
// full scan on the device.  There is no CPU fallback.
#include <cfloat>

#include "kernels.cuh"
#include "ptx.cuh"

namespace mflat_cu {
namespace {

struct Cand {
    double s;
    int id;
    int owner;
};

__device__ __forceinline__ bool better(const Cand& a, const Cand& b) {
    if (a.id < 0) return false;
    if (b.id < 0) return true;
    if (a.s != b.s) return a.s > b.s;
    return a.id < b.id;
}

__device__ __forceinline__ Cand warp_best(Cand c) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        Cand o;
        o.s = __shfl_xor_sync(0xffffffffu, c.s, off);
        o.id = __shfl_xor_sync(0xffffffffu, c.id, off);
        o.owner = __shfl_xor_sync(0xffffffffu, c.owner, off);
        if (better(o, c)) c = o;
    }
    return c;
}

// Block-wide best candidate; `red` holds >= 32 entries of shared memory.
__device__ Cand block_best(Cand c, Cand* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
    c = warp_best(c);
    if (lane == 0) red[warp] = c;
    __syncthreads();
    if (warp == 0) {
        Cand w = lane < nwarps ? red[lane] : Cand{-DBL_MAX, -1, -1};
        w = warp_best(w);
        if (lane == 0) red[32] = w;
    }
    __syncthreads();
    const Cand r = red[32];
    __syncthreads();
    return r;
}

// Upper bound E on |screen score - exact score| for one query.
//   dot:  |dot' - q.x| <= gamma * ||q|| * ||x||  (split + tensor-core
//         accumulation error; sum |q_i x_i| <= ||q|| ||x|| by Cauchy-Schwarz)
//   L2 adds the rounding of the fp32 ||x||^2 term (u X^2) and of the bias
//   step's accumulation into score / 2 (u (||q|| X + X^2 / 2), doubled).
__device__ __forceinline__ double error_bound(int metric, double qn, double xmax, double gamma) {
    const double u = 1.0 / 8388608.0;    // 2^-23
    if (metric == kL2) return 2.0 * gamma * qn * xmax + u * xmax * xmax + 2.0 * u * qn * xmax + 1e-30;
    return gamma * qn * xmax + 1e-30;
}

// fp64 score of the stored fp32 query and row, index order (the fp64 oracle's
// evaluation): -sum (q - x)^2 for L2, sum q x otherwise.
// q and x are 16-byte aligned rows (d_pad floats apart).  The terms are summed
// in ascending coordinate order; the rows are read four coordinates per load,
// several loads in flight, so a lane's row costs a few memory latencies rather
// than one per coordinate.
__device__ __forceinline__ double exact_score(int metric, const float* q, const float* x, int dim) {
    const float4* q4 = reinterpret_cast<const float4*>(q);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int d4 = dim >> 2;
    double acc = 0.0;
    if (metric == kL2) {
#pragma unroll 4
        for (int c = 0; c < d4; ++c) {
            const float4 a = __ldg(q4 + c), b = __ldg(x4 + c);
            double e = static_cast<double>(a.x) - static_cast<double>(b.x);
            acc += e * e;
            e = static_cast<double>(a.y) - static_cast<double>(b.y);
            acc += e * e;
            e = static_cast<double>(a.z) - static_cast<double>(b.z);
            acc += e * e;
            e = static_cast<double>(a.w) - static_cast<double>(b.w);
            acc += e * e;
        }
        for (int c = 4 * d4; c < dim; ++c) {
            const double e = static_cast<double>(q[c]) - static_cast<double>(x[c]);
            acc += e * e;
        }
        return -acc;
    }
#pragma unroll 4
    for (int c = 0; c < d4; ++c) {
        const float4 a = __ldg(q4 + c), b = __ldg(x4 + c);
        acc += static_cast<double>(a.x) * static_cast<double>(b.x);
        acc += static_cast<double>(a.y) * static_cast<double>(b.y);
        acc += static_cast<double>(a.z) * static_cast<double>(b.z);
        acc += static_cast<double>(a.w) * static_cast<double>(b.w);
    }
    for (int c = 4 * d4; c < dim; ++c) acc += static_cast<double>(q[c]) * static_cast<double>(x[c]);
    return acc;
}

// ---------------------------------------------------------------------------
// Warp-level merge of the per-chunk candidate lists.  A candidate is packed
// into a 64-bit key whose unsigned order is the selection order: the high
// word is the order-preserving key of the screen score (score desc), the low
// word ~id (id asc among equal scores); 0 marks an empty slot.  A warp holds
// one sorted list of 32 keys, one per lane (lane 0 = best).  Merging in the
// next chunk's sorted list keeps the 32 largest of the union: max(a[i],
// b[31 - i]) is a bitonic sequence holding exactly those, and five
// half-cleaner stages sort it again.  Lists are read with one coalesced load
// per chunk; nothing in the merge depends on a load of an earlier round.
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ uint64_t cand_key(float s, int id) {
    if (id < 0) return 0ull;
    return (static_cast<uint64_t>(score_key(s)) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(id));
}
__device__ __forceinline__ float key_score(uint64_t k) {
    const uint32_t h = static_cast<uint32_t>(k >> 32);
    return __uint_as_float((h & 0x80000000u) ? (h & 0x7fffffffu) : ~h);
}
__device__ __forceinline__ int key_id(uint64_t k) {
    return k == 0ull ? -1 : static_cast<int>(~static_cast<uint32_t>(k));
}

__device__ __forceinline__ uint64_t merge_top32(uint64_t a, uint64_t b, int lane) {
    const uint64_t br = __shfl_sync(kFull, b, 31 - lane);
    uint64_t v = a > br ? a : br;
#pragma unroll
    for (int st = 16; st >= 1; st >>= 1) {
        const uint64_t o = __shfl_xor_sync(kFull, v, st);
        v = (lane & st) == 0 ? (v > o ? v : o) : (v < o ? v : o);
    }
    return v;
}

// Top 32 keys over the query's n_lists lists of KP entries (each sorted best
// first); lane i returns the i-th best.  Lanes >= KP of a list read nothing.
template <int KP>
__device__ __forceinline__ uint64_t warp_merge_lists(const float* __restrict__ part_s,
                                                     const int32_t* __restrict__ part_i, int n_lists,
                                                     int m_pad, int qi, int lane) {
    uint64_t top = 0ull;
    constexpr int kU = 4;
    for (int c0 = 0; c0 < n_lists; c0 += kU) {
        uint64_t kk[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            kk[u] = 0ull;
            const int c = c0 + u;
            if (c < n_lists && lane < KP) {
                const int64_t o = (static_cast<int64_t>(c) * m_pad + qi) * KP + lane;
                kk[u] = cand_key(__ldg(part_s + o), __ldg(part_i + o));
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u)
            if (c0 + u < n_lists) top = (c0 + u == 0) ? kk[u] : merge_top32(top, kk[u], lane);
    }
    return top;
}

// Bitonic sort of one (score, id) pair per lane into better-first order
// (score desc, id asc, id < 0 last): lane 0 ends with the best.
__device__ __forceinline__ void warp_sort_better_first(double& s, int& id, int lane) {
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int st = size >> 1; st >= 1; st >>= 1) {
            const double os = __shfl_xor_sync(kFull, s, st);
            const int oid = __shfl_xor_sync(kFull, id, st);
            const Cand me{s, id, 0}, other{os, oid, 0};
            // blocks of `size` alternate direction until the last merge
            const bool ascending = (lane & size) == 0;
            const bool lower = (lane & st) == 0;
            // the pair's lower lane keeps the better entry in an ascending
            // (better-first) block, the worse one in a descending block
            if (lower == ascending ? better(other, me) : better(me, other)) {
                s = os;
                id = oid;
            }
        }
    }
}

// Exact fp64 scores of the warp's candidates (lane j holds candidate j's row id,
// -1 for none), the warp cooperating on each row: lane l reads coordinates
// [4l, 4l + 4) of every 128-wide slab of the row, so a row is one coalesced
// 512-byte read per slab, with kB rows in flight (two: fewer registers, more
// resident warps -- measured faster than four or eight).  Each lane sums its
// coordinates in ascending order; the 32 lane sums are added by the same
// shuffle tree for every row, so identical rows score identically.  Lane j
// returns candidate j's score (-DBL_MAX for none).  q and the rows are
// zero-padded to d_pad (a multiple of 64), 16-byte aligned.
template <int KP>
__device__ __forceinline__ double warp_rescore(int metric, const float* __restrict__ q,
                                               const float* __restrict__ db_x, int d_pad, int id, int lane) {
    constexpr int kB = 2;
    double mine = -DBL_MAX;
#pragma unroll 1
    for (int j0 = 0; j0 < KP; j0 += kB) {
        int rid[kB];
        double part[kB];
#pragma unroll
        for (int jj = 0; jj < kB; ++jj) {
            rid[jj] = __shfl_sync(kFull, id, j0 + jj);
            part[jj] = 0.0;
        }
#pragma unroll 1
        for (int c0 = 0; c0 < d_pad; c0 += 128) {
            const int c = c0 + 4 * lane;
            const bool in = c < d_pad;
            const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 qv = in ? __ldg(reinterpret_cast<const float4*>(q + c)) : zero;
            float4 xv[kB];
#pragma unroll
            for (int jj = 0; jj < kB; ++jj)
                xv[jj] = (in && rid[jj] >= 0)
                             ? __ldg(reinterpret_cast<const float4*>(db_x + static_cast<int64_t>(rid[jj]) * d_pad + c))
                             : zero;
#pragma unroll
            for (int jj = 0; jj < kB; ++jj) {
                if (metric == kL2) {
                    double e = static_cast<double>(qv.x) - static_cast<double>(xv[jj].x);
                    part[jj] += e * e;
                    e = static_cast<double>(qv.y) - static_cast<double>(xv[jj].y);
                    part[jj] += e * e;
                    e = static_cast<double>(qv.z) - static_cast<double>(xv[jj].z);
                    part[jj] += e * e;
                    e = static_cast<double>(qv.w) - static_cast<double>(xv[jj].w);
                    part[jj] += e * e;
                } else {
                    part[jj] += static_cast<double>(qv.x) * static_cast<double>(xv[jj].x);
                    part[jj] += static_cast<double>(qv.y) * static_cast<double>(xv[jj].y);
                    part[jj] += static_cast<double>(qv.z) * static_cast<double>(xv[jj].z);
                    part[jj] += static_cast<double>(qv.w) * static_cast<double>(xv[jj].w);
                }
            }
        }
#pragma unroll
        for (int jj = 0; jj < kB; ++jj) {
            double v = part[jj];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(kFull, v, o);
            v = __shfl_sync(kFull, v, 0);
            if (lane == j0 + jj && rid[jj] >= 0) mine = metric == kL2 ? -v : v;
        }
    }
    return mine;
}

// One warp per query: merge the chunk lists into the top KP candidates, prove
// that the true top-k is among them, re-score them exactly in fp64 and write
// the k nearest in (distance, id) order.  Queries whose proof fails are
// listed for the exact full scan and written by it.
template <int KP>
__global__ void __launch_bounds__(128) select_exact_kernel(const SelectParams p) {
    const int lane = threadIdx.x & 31;
    const int qi = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (qi >= p.m) return;                      // uniform per warp
    if (*p.err != 0) return;                    // the screen failed: its lists are not valid
    uint64_t top = warp_merge_lists<KP>(p.part_score, p.part_id, p.n_chunks, p.m_pad, qi, lane);
    if (lane >= KP) top = 0ull;                 // only the merged top-KP are proven candidates
    const float s_screen = key_score(top);
    const int id = key_id(top);
    if (__any_sync(kFull, id >= p.n)) {         // never produced by a screen: report, read nothing
        if (lane == 0) atomicExch(p.err, kErrInternal);
        return;
    }
    const int n_valid = __popc(__ballot_sync(kFull, id >= 0));

    // proof that the true top-k is inside the candidates
    bool ok = true;
    if (n_valid >= KP && p.k_out <= KP) {
        const float sk = __shfl_sync(kFull, s_screen, p.k_out - 1);
        const float skp = __shfl_sync(kFull, s_screen, KP - 1);
        const double xmax = static_cast<double>(__uint_as_float(*p.xmax_bits));
        const double E = error_bound(p.metric, p.qnorm[qi], xmax, p.gamma);
        ok = static_cast<double>(skp) < static_cast<double>(sk) - 2.0 * E;
    }
    if (!ok) {
        if (lane == 0) {
            const int slot = atomicAdd(p.flag_count, 1);
            p.flag_list[slot] = qi;
        }
        return;
    }

    // exact fp64 re-score (lane = candidate), then (distance, id) order
    double ex = warp_rescore<KP>(p.metric, p.q_x + static_cast<int64_t>(qi) * p.d_pad, p.db_x, p.d_pad, id, lane);
    int rid = id;
    warp_sort_better_first(ex, rid, lane);
    if (lane < p.k_out) {
        const int64_t o = static_cast<int64_t>(qi) * p.k_out + lane;
        if (rid >= 0) {
            p.out_ids[o] = static_cast<int32_t>(rid + p.id_base);
            p.out_dist[o] = static_cast<float>(p.metric == kL2 ? -ex : ex);
        } else {
            p.out_ids[o] = -1;
            p.out_dist[o] = p.metric == kL2 ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
        }
    }
}

// Exact fp64 full scan for the queries the proof rejected, in two stages.
// Stage 1: every block takes (flagged query, database chunk) pairs, chunk-major
// so that concurrently running blocks read the same rows; each thread keeps a
// best-k list of its rows (visited in ascending order, strict '>'), the block
// merges its 256 lists by a k-round tournament and stores the chunk's best k.
// Stage 2: one block per flagged query merges the kFbChunks chunk lists.
constexpr int kFbThreads = 256;
constexpr int kFbMaxK = 32;

__global__ void __launch_bounds__(kFbThreads) fallback_scan_kernel(const SelectParams p) {
    __shared__ Cand red[33];
    const int nflag = *p.flag_count;
    const int k = p.k_out;
    const int64_t per = (p.n + kFbChunks - 1) / kFbChunks;
    for (int pair = blockIdx.x; pair < nflag * kFbChunks; pair += gridDim.x) {
        const int c = pair / nflag;
        const int f = pair % nflag;
        const int qi = p.flag_list[f];
        const float* qx = p.q_x + static_cast<int64_t>(qi) * p.d_pad;
        const int64_t r0 = c * per;
        const int64_t r1 = min(p.n, r0 + per);
        double bs[kFbMaxK];
        int bi[kFbMaxK];
        for (int i = 0; i < k; ++i) { bs[i] = -DBL_MAX; bi[i] = -1; }   // sorted desc
        for (int64_t j = r0 + threadIdx.x; j < r1; j += blockDim.x) {
            const double s = exact_score(p.metric, qx, p.db_x + j * p.d_pad, p.dim);
            if (bi[k - 1] < 0 || s > bs[k - 1]) {
                int pos = k - 1;
                while (pos > 0 && (bi[pos - 1] < 0 || s > bs[pos - 1])) {
                    bs[pos] = bs[pos - 1];
                    bi[pos] = bi[pos - 1];
                    --pos;
                }
                bs[pos] = s;
                bi[pos] = static_cast<int>(j);
            }
        }
        int head = 0;
        const int64_t ob = (static_cast<int64_t>(f) * kFbChunks + c) * k;
        for (int r = 0; r < k; ++r) {
            Cand cd{-DBL_MAX, -1, static_cast<int>(threadIdx.x)};
            if (head < k && bi[head] >= 0) { cd.s = bs[head]; cd.id = bi[head]; }
            const Cand w = block_best(cd, red);
            if (threadIdx.x == 0) {
                p.fb_s[ob + r] = w.s;
                p.fb_i[ob + r] = w.id;
            }
            if (w.id >= 0 && w.owner == static_cast<int>(threadIdx.x)) ++head;
        }
    }
}

__global__ void __launch_bounds__(128) fallback_merge_kernel(const SelectParams p) {
    __shared__ Cand red[33];
    const int nflag = *p.flag_count;
    const int k = p.k_out;
    const int t = threadIdx.x;
    for (int f = blockIdx.x; f < nflag; f += gridDim.x) {
        const int qi = p.flag_list[f];
        int head = 0;
        const int64_t ob = (static_cast<int64_t>(f) * kFbChunks + t) * k;
        for (int r = 0; r < k; ++r) {
            Cand cd{-DBL_MAX, -1, t};
            if (t < kFbChunks && head < k) { cd.s = p.fb_s[ob + head]; cd.id = p.fb_i[ob + head]; }
            const Cand w = block_best(cd, red);
            if (t == 0) {
                const int64_t o = static_cast<int64_t>(qi) * k + r;
                if (w.id >= 0) {
                    p.out_ids[o] = static_cast<int32_t>(w.id + p.id_base);
                    p.out_dist[o] = static_cast<float>(p.metric == kL2 ? -w.s : w.s);
                } else {
                    p.out_ids[o] = -1;
                    p.out_dist[o] = p.metric == kL2 ? __int_as_float(0x7f800000)
                                                    : -__int_as_float(0x7f800000);
                }
            }
            if (w.id >= 0 && w.owner == t) ++head;
        }
    }
}

// ---------------------------------------------------------------- k-means
// Assignment of point qi = argmin_c sqL2_f32(p, c) with the reference's fp32
// sequential sqL2 (src/Distance.h:33-37, used by src/CoarseQuantizer.mm:
// 122-130) and strict '<' (lowest centroid wins a tie).  The screen gives the
// top-KP centroids by screen score; every centroid that could be the fp32
// argmin lies within a window W of the best screen score (W covers the screen
// error E on both sides and the rounding of the fp32 sequential sum,
// gamma_s = (dim + 8) 2^-23 relative).  If the KP-th candidate is outside the
// window the candidates inside it are re-scored with exactly the reference's
// operations (__fsub_rn / __fmul_rn / __fadd_rn in index order) and the
// minimum is taken; otherwise the point goes to the full fp32 scan.
__device__ __forceinline__ float sql2_f32_seq(const float* p, const float* x, int dim) {
    float acc = 0.0f;
    for (int c = 0; c < dim; ++c) {
        const float e = __fsub_rn(p[c], x[c]);
        acc = __fadd_rn(acc, __fmul_rn(e, e));
    }
    return acc;
}

struct MinCand {
    float v;
    int id;
};

__device__ __forceinline__ MinCand warp_min(MinCand c) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        MinCand o;
        o.v = __shfl_xor_sync(0xffffffffu, c.v, off);
        o.id = __shfl_xor_sync(0xffffffffu, c.id, off);
        const bool take = o.id >= 0 && (c.id < 0 || o.v < c.v || (o.v == c.v && o.id < c.id));
        if (take) c = o;
    }
    return c;
}

template <int KP>
__global__ void __launch_bounds__(128) kmeans_select_kernel(const SelectParams p,
                                                            int32_t* out_assign) {
    // one thread per point: the sequential fp32 re-check below is one chain
    // of dim operations per candidate, so a warp serves 32 points at once
    const int qi = blockIdx.x * blockDim.x + threadIdx.x;
    if (qi >= p.m) return;
    if (*p.err != 0) return;                    // the screen failed: its lists are not valid
    // the point's top KP over its lists, in (score desc, id asc) order, by a
    // static compare-and-swap insertion (lists are read coalesced: thread qi's
    // KP entries of a list are adjacent to thread qi + 1's)
    float sel_s[KP];
    int sel_id[KP];
#pragma unroll
    for (int i = 0; i < KP; ++i) {
        sel_s[i] = 0.0f;
        sel_id[i] = -1;
    }
    for (int c = 0; c < p.n_chunks; ++c) {
        const int64_t base = (static_cast<int64_t>(c) * p.m_pad + qi) * KP;
#pragma unroll
        for (int j = 0; j < KP; ++j) {
            float s = p.part_score[base + j];
            int id = p.part_id[base + j];
            if (id < 0) continue;
#pragma unroll
            for (int i = 0; i < KP; ++i) {
                const bool take = sel_id[i] < 0 || s > sel_s[i] || (s == sel_s[i] && id < sel_id[i]);
                if (take) {
                    const float ts = sel_s[i];
                    const int ti = sel_id[i];
                    sel_s[i] = s;
                    sel_id[i] = id;
                    s = ts;
                    id = ti;
                    if (id < 0) break;
                }
            }
        }
    }
    int n_valid = 0;
    bool bad_id = false;
#pragma unroll
    for (int i = 0; i < KP; ++i) {
        n_valid += sel_id[i] >= 0 ? 1 : 0;
        bad_id |= sel_id[i] >= p.n;
    }
    if (bad_id) {                               // never produced by a screen: report, read nothing
        atomicExch(p.err, kErrInternal);
        return;
    }
    const double qn = p.qnorm[qi];
    const double xmax = static_cast<double>(__uint_as_float(*p.xmax_bits));
    const double E = error_bound(kL2, qn, xmax, p.gamma);
    const double gs = (p.dim + 8.0) / 8388608.0;
    const double db = fmax(0.0, qn * qn - static_cast<double>(sel_s[0]));
    const double W = 2.0 * E + 3.0 * gs * (db + E) + 1e-30;
    const bool ok = n_valid < KP || static_cast<double>(sel_s[KP - 1]) < static_cast<double>(sel_s[0]) - W;
    if (!ok) {
        const int slot = atomicAdd(p.flag_count, 1);
        p.flag_list[slot] = qi;
        return;
    }
    // exact fp32 distance, in the reference's operation order, of every
    // candidate within W of the best screen score; argmin, lowest id on ties
    const float* px = p.q_x + static_cast<int64_t>(qi) * p.d_pad;
    MinCand mc{0.0f, -1};
#pragma unroll
    for (int i = 0; i < KP; ++i) {
        if (sel_id[i] >= 0 && static_cast<double>(sel_s[i]) >= static_cast<double>(sel_s[0]) - W) {
            const int id = sel_id[i];
            const float v = sql2_f32_seq(px, p.db_x + static_cast<int64_t>(id) * p.d_pad, p.dim);
            if (mc.id < 0 || v < mc.v || (v == mc.v && id < mc.id)) {
                mc.v = v;
                mc.id = id;
            }
        }
    }
    out_assign[qi] = mc.id;
}

__global__ void __launch_bounds__(128) kmeans_fallback_kernel(const SelectParams p,
                                                              int32_t* out_assign) {
    const int lane = threadIdx.x & 31;
    const int wid = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * 4;
    const int nflag = *p.flag_count;
    for (int f = wid; f < nflag; f += nwarps) {
        const int qi = p.flag_list[f];
        const float* px = p.q_x + static_cast<int64_t>(qi) * p.d_pad;
        MinCand mc{0.0f, -1};
        for (int64_t c = lane; c < p.n; c += 32) {
            const float v = sql2_f32_seq(px, p.db_x + c * p.d_pad, p.dim);
            if (mc.id < 0 || v < mc.v) { mc.v = v; mc.id = static_cast<int>(c); }
        }
        mc = warp_min(mc);
        if (lane == 0) out_assign[qi] = mc.id;
    }
}

// Recall path (fp16 / bf16 storage): the screen's scores are the answer.  One
// warp per query merges the lists (k_out <= KP); lane r writes rank r.
template <int KP>
__global__ void __launch_bounds__(128) select_recall_kernel(const SelectParams p, const float* qsq) {
    const int lane = threadIdx.x & 31;
    const int qi = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (qi >= p.m) return;
    const uint64_t top = warp_merge_lists<KP>(p.part_score, p.part_id, p.n_chunks, p.m_pad, qi, lane);
    if (lane < p.k_out) {
        const int64_t o = static_cast<int64_t>(qi) * p.k_out + lane;
        const int id = key_id(top);
        if (id >= 0) {
            const float s = key_score(top);
            p.out_ids[o] = static_cast<int32_t>(id + p.id_base);
            p.out_dist[o] = p.metric == kL2
                                ? fmaxf(0.0f, static_cast<float>(static_cast<double>(qsq[qi]) - s))
                                : s;
        } else {
            p.out_ids[o] = -1;
            p.out_dist[o] = p.metric == kL2 ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
        }
    }
}

// Four queries (warps) per block.
inline unsigned select_blocks(int m) { return static_cast<unsigned>((m + 3) / 4); }

template <int KP>
cudaError_t launch_select_kp(const SelectParams& p, cudaStream_t stream) {
    select_exact_kernel<KP><<<select_blocks(p.m), 128, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_select_exact(int kp, const SelectParams& p, cudaStream_t stream) {
    if (p.n_chunks > kMaxChunks || p.n_chunks < 1) return cudaErrorInvalidValue;
    switch (kp) {
        case 4: return launch_select_kp<4>(p, stream);
        case 8: return launch_select_kp<8>(p, stream);
        case 16: return launch_select_kp<16>(p, stream);
        case 32: return launch_select_kp<32>(p, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_kmeans_select(const SelectParams& p, int32_t* out, int grid_fallback,
                                 cudaStream_t stream) {
    if (p.n_chunks > 32 || p.n_chunks < 1) return cudaErrorInvalidValue;
    kmeans_select_kernel<4><<<(p.m + 127) / 128, 128, 0, stream>>>(p, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    kmeans_fallback_kernel<<<grid_fallback, 128, 0, stream>>>(p, out);
    return cudaGetLastError();
}

cudaError_t launch_select_recall(int kp, const SelectParams& p, const float* qsq, cudaStream_t stream) {
    if (p.n_chunks > kMaxChunks || p.n_chunks < 1 || p.k_out > kp) return cudaErrorInvalidValue;
    switch (kp) {
        case 4: select_recall_kernel<4><<<select_blocks(p.m), 128, 0, stream>>>(p, qsq); break;
        case 8: select_recall_kernel<8><<<select_blocks(p.m), 128, 0, stream>>>(p, qsq); break;
        case 16: select_recall_kernel<16><<<select_blocks(p.m), 128, 0, stream>>>(p, qsq); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_fallback_exact(const SelectParams& p, int grid, cudaStream_t stream) {
    if (p.k_out > kFbMaxK || p.k_out < 1) return cudaErrorInvalidValue;
    fallback_scan_kernel<<<grid * 2, kFbThreads, 0, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    fallback_merge_kernel<<<grid, 128, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace mflat_cu
