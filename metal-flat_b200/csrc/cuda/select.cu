// select.cu -- candidate merge, exactness proof and exact re-rank.
//
// The screen (screen_tc.cu) leaves, per query and database chunk, the top-KP
// rows by the fp32 screen score s' (3xTF32 dot + norm term).  Every screen
// score is within E of the exact score s (a-priori bound, see error_bound()).
// If the KP-th best merged screen score is below (k-th best) - 2E, every row
// of the true top-k is among the KP candidates (standard argument: the k rows
// of the true top-k all have s' >= s_(k) - E, hence s'_(k) >= s_(k) - E, and
// s'_(k) <= s_(k) + E; a true top-k row therefore has s' >= s'_(k) - 2E).
// The candidates are then re-scored exactly in fp64 from the stored fp32 rows
// (hi + lo) and ordered by (distance, id), which is the fp64 brute-force
// oracle's order (reference semantics: src/Distance.h:26-81, ties to the
// lowest id as in src/FlatIndex.mm:272-281).  Queries whose proof fails
// (many near-equal scores, e.g. duplicated rows) are re-done by an exact
// full scan on the device.  There is no CPU fallback.
#include <cfloat>

#include "kernels.cuh"

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
//   L2 adds the rounding of the fp32 ||x||^2 term and of the score FMA.
__device__ __forceinline__ double error_bound(int metric, double qn, double xmax, double gamma) {
    const double u = 1.0 / 8388608.0;    // 2^-23
    if (metric == kL2) return 2.0 * gamma * qn * xmax + u * xmax * xmax + u * qn * xmax + 1e-30;
    return gamma * qn * xmax + 1e-30;
}

__device__ __forceinline__ double exact_score(int metric, const float* qh, const float* ql,
                                              const float* xh, const float* xl, int dim) {
    double acc = 0.0;
    if (metric == kL2) {
        for (int c = 0; c < dim; ++c) {
            const double e = static_cast<double>(qh[c] + ql[c]) - static_cast<double>(xh[c] + xl[c]);
            acc += e * e;
        }
        return -acc;
    }
    for (int c = 0; c < dim; ++c)
        acc += static_cast<double>(qh[c] + ql[c]) * static_cast<double>(xh[c] + xl[c]);
    return acc;
}

template <int KP>
__global__ void __launch_bounds__(kSelectMaxThreads) select_exact_kernel(const SelectParams p) {
    const int qi = blockIdx.x;
    if (qi >= p.m) return;
    __shared__ Cand red[33];
    __shared__ float sel_s[KP];
    __shared__ int sel_id[KP];
    __shared__ double ex_s[KP];
    __shared__ int s_ok;

    // 1. tournament merge of the per-chunk lists (each sorted best-first)
    const int t = threadIdx.x;
    int head = 0;
    const int64_t base = (static_cast<int64_t>(t) * p.m_pad + qi) * KP;
    for (int r = 0; r < KP; ++r) {
        Cand c{-DBL_MAX, -1, t};
        if (t < p.n_chunks && head < KP) {
            c.s = p.part_score[base + head];
            c.id = p.part_id[base + head];
        }
        const Cand w = block_best(c, red);
        if (t == 0) {
            sel_s[r] = static_cast<float>(w.s);
            sel_id[r] = w.id;
        }
        if (w.id >= 0 && w.owner == t) ++head;
    }
    __syncthreads();

    // 2. proof that the true top-k is inside the candidates
    int n_valid = 0;
    for (int i = 0; i < KP; ++i) n_valid += sel_id[i] >= 0 ? 1 : 0;
    if (t == 0) {
        int ok = 1;
        if (n_valid >= KP && p.k_out <= KP) {
            const double xmax = static_cast<double>(__uint_as_float(*p.xmax_bits));
            const double E = error_bound(p.metric, p.qnorm[qi], xmax, p.gamma);
            ok = static_cast<double>(sel_s[KP - 1]) < static_cast<double>(sel_s[p.k_out - 1]) - 2.0 * E;
        }
        if (!ok) {
            const int slot = atomicAdd(p.flag_count, 1);
            p.flag_list[slot] = qi;
        }
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;

    // 3. exact fp64 re-score of the candidates
    const float* qh = p.q_hi + static_cast<int64_t>(qi) * p.d_pad;
    const float* ql = p.q_lo + static_cast<int64_t>(qi) * p.d_pad;
    if (t < n_valid) {
        const int64_t id = sel_id[t];
        ex_s[t] = exact_score(p.metric, qh, ql, p.db_hi + id * p.d_pad, p.db_lo + id * p.d_pad, p.dim);
    }
    __syncthreads();

    // 4. order by (exact score desc, id asc) and emit nearest-first
    if (t < n_valid) {
        const Cand me{ex_s[t], sel_id[t], t};
        int rank = 0;
        for (int u = 0; u < n_valid; ++u) {
            const Cand o{ex_s[u], sel_id[u], u};
            if (better(o, me)) ++rank;
        }
        if (rank < p.k_out) {
            const int64_t o = static_cast<int64_t>(qi) * p.k_out + rank;
            p.out_ids[o] = static_cast<int32_t>(me.id + p.id_base);
            p.out_dist[o] = static_cast<float>(p.metric == kL2 ? -me.s : me.s);
        }
    }
    for (int pos = n_valid + t; pos < p.k_out; pos += blockDim.x) {
        const int64_t o = static_cast<int64_t>(qi) * p.k_out + pos;
        p.out_ids[o] = -1;
        p.out_dist[o] = p.metric == kL2 ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
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
        const float* qh = p.q_hi + static_cast<int64_t>(qi) * p.d_pad;
        const float* ql = p.q_lo + static_cast<int64_t>(qi) * p.d_pad;
        const int64_t r0 = c * per;
        const int64_t r1 = min(p.n, r0 + per);
        double bs[kFbMaxK];
        int bi[kFbMaxK];
        for (int i = 0; i < k; ++i) { bs[i] = -DBL_MAX; bi[i] = -1; }   // sorted desc
        for (int64_t j = r0 + threadIdx.x; j < r1; j += blockDim.x) {
            const double s = exact_score(p.metric, qh, ql, p.db_hi + j * p.d_pad,
                                         p.db_lo + j * p.d_pad, p.dim);
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
// top-KP centroids by 3xTF32 score; every centroid that could be the fp32
// argmin lies within a window W of the best screen score (W covers the screen
// error E on both sides and the rounding of the fp32 sequential sum,
// gamma_s = (dim + 8) 2^-23 relative).  If the KP-th candidate is outside the
// window the candidates inside it are re-scored with exactly the reference's
// operations (__fsub_rn / __fmul_rn / __fadd_rn in index order) and the
// minimum is taken; otherwise the point goes to the full fp32 scan.
__device__ __forceinline__ float sql2_f32_seq(const float* ph, const float* pl, const float* xh,
                                              const float* xl, int dim) {
    float acc = 0.0f;
    for (int c = 0; c < dim; ++c) {
        const float e = __fsub_rn(__fadd_rn(ph[c], pl[c]), __fadd_rn(xh[c], xl[c]));
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
    const int lane = threadIdx.x & 31;
    const int qi = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (qi >= p.m) return;
    float sel_s[KP];
    int sel_id[KP];
    int head = 0;
    const int64_t base = (static_cast<int64_t>(lane) * p.m_pad + qi) * KP;
    for (int r = 0; r < KP; ++r) {
        Cand c{-DBL_MAX, -1, lane};
        if (lane < p.n_chunks && head < KP) {
            c.s = p.part_score[base + head];
            c.id = p.part_id[base + head];
        }
        const Cand w = warp_best(c);
        sel_s[r] = static_cast<float>(w.s);
        sel_id[r] = w.id;
        if (w.id >= 0 && w.owner == lane) ++head;
    }
    int n_valid = 0;
#pragma unroll
    for (int i = 0; i < KP; ++i) n_valid += sel_id[i] >= 0 ? 1 : 0;
    const double qn = p.qnorm[qi];
    const double xmax = static_cast<double>(__uint_as_float(*p.xmax_bits));
    const double E = error_bound(kL2, qn, xmax, p.gamma);
    const double gs = (p.dim + 8.0) / 8388608.0;
    const double db = fmax(0.0, qn * qn - static_cast<double>(sel_s[0]));
    const double W = 2.0 * E + 3.0 * gs * (db + E) + 1e-30;
    const bool ok = n_valid < KP || static_cast<double>(sel_s[KP - 1]) < static_cast<double>(sel_s[0]) - W;
    if (!ok) {
        if (lane == 0) {
            const int slot = atomicAdd(p.flag_count, 1);
            p.flag_list[slot] = qi;
        }
        return;
    }
    const float* ph = p.q_hi + static_cast<int64_t>(qi) * p.d_pad;
    const float* pl = p.q_lo + static_cast<int64_t>(qi) * p.d_pad;
    MinCand mc{0.0f, -1};
#pragma unroll
    for (int i = 0; i < KP; ++i) {
        if (lane == i && sel_id[i] >= 0 &&
            static_cast<double>(sel_s[i]) >= static_cast<double>(sel_s[0]) - W) {
            const int64_t id = sel_id[i];
            mc.v = sql2_f32_seq(ph, pl, p.db_hi + id * p.d_pad, p.db_lo + id * p.d_pad, p.dim);
            mc.id = sel_id[i];
        }
    }
    mc = warp_min(mc);
    if (lane == 0) out_assign[qi] = mc.id;
}

__global__ void __launch_bounds__(128) kmeans_fallback_kernel(const SelectParams p,
                                                              int32_t* out_assign) {
    const int lane = threadIdx.x & 31;
    const int wid = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * 4;
    const int nflag = *p.flag_count;
    for (int f = wid; f < nflag; f += nwarps) {
        const int qi = p.flag_list[f];
        const float* ph = p.q_hi + static_cast<int64_t>(qi) * p.d_pad;
        const float* pl = p.q_lo + static_cast<int64_t>(qi) * p.d_pad;
        MinCand mc{0.0f, -1};
        for (int64_t c = lane; c < p.n; c += 32) {
            const float v = sql2_f32_seq(ph, pl, p.db_hi + c * p.d_pad, p.db_lo + c * p.d_pad, p.dim);
            if (mc.id < 0 || v < mc.v) { mc.v = v; mc.id = static_cast<int>(c); }
        }
        mc = warp_min(mc);
        if (lane == 0) out_assign[qi] = mc.id;
    }
}

// Recall path (fp16 / bf16 storage): the screen's scores are the answer.
template <int KP>
__global__ void __launch_bounds__(kSelectMaxThreads) select_recall_kernel(const SelectParams p, const float* qsq) {
    const int qi = blockIdx.x;
    if (qi >= p.m) return;
    __shared__ Cand red[33];
    const int t = threadIdx.x;
    int head = 0;
    const int64_t base = (static_cast<int64_t>(t) * p.m_pad + qi) * KP;
    const float empty = p.metric == kL2 ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
    for (int r = 0; r < p.k_out; ++r) {
        Cand c{-DBL_MAX, -1, t};
        if (t < p.n_chunks && head < KP) {
            c.s = p.part_score[base + head];
            c.id = p.part_id[base + head];
        }
        const Cand w = block_best(c, red);
        if (t == 0) {
            const int64_t o = static_cast<int64_t>(qi) * p.k_out + r;
            if (w.id >= 0) {
                p.out_ids[o] = static_cast<int32_t>(w.id + p.id_base);
                p.out_dist[o] = p.metric == kL2
                                    ? fmaxf(0.0f, static_cast<float>(static_cast<double>(qsq[qi]) - w.s))
                                    : static_cast<float>(w.s);
            } else {
                p.out_ids[o] = -1;
                p.out_dist[o] = empty;
            }
        }
        if (w.id >= 0 && w.owner == t) ++head;
    }
}

// One thread per candidate list in the tournament merge.
inline int select_threads(int n_lists) { return n_lists > 128 ? kSelectMaxThreads : 128; }

template <int KP>
cudaError_t launch_select_kp(const SelectParams& p, cudaStream_t stream) {
    select_exact_kernel<KP><<<p.m, select_threads(p.n_chunks), 0, stream>>>(p);
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
    kmeans_select_kernel<4><<<(p.m + 3) / 4, 128, 0, stream>>>(p, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    kmeans_fallback_kernel<<<grid_fallback, 128, 0, stream>>>(p, out);
    return cudaGetLastError();
}

cudaError_t launch_select_recall(int kp, const SelectParams& p, const float* qsq, cudaStream_t stream) {
    if (p.n_chunks > kMaxChunks || p.n_chunks < 1 || p.k_out > kp) return cudaErrorInvalidValue;
    switch (kp) {
        case 4: select_recall_kernel<4><<<p.m, select_threads(p.n_chunks), 0, stream>>>(p, qsq); break;
        case 8: select_recall_kernel<8><<<p.m, select_threads(p.n_chunks), 0, stream>>>(p, qsq); break;
        case 16: select_recall_kernel<16><<<p.m, select_threads(p.n_chunks), 0, stream>>>(p, qsq); break;
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
