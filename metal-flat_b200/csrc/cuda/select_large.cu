// select_large.cu -- selection for large k (up to 1024): floor from the
// sampling pre-pass, then per-query top-k from the candidate buffers that the
// buffer-mode screen filled.
//
// Floor.  The pre-pass screens an evenly spread sample of database tiles in
// list mode and leaves, per query, L lists of the KP1 best sampled rows.  The
// minimum over the lists of their KP1-th score is met by at least L*KP1 sampled
// rows, so it is <= the global (L*KP1)-th best score: with L*KP1 >= KP no row of
// the query's global top-KP scores below it (the screen then keeps s >= floor).
//
// Select.  Per query, a block radix-selects over the buffer (4 passes of 8 bits
// on order-preserving keys), gathers the winners (ties at the threshold broken
// by lowest id), sorts them by (score desc, id asc) and writes the results.
//   recall path (fp16 / bf16 storage): the top-k by screen score, distances
//     from the screen (L2: max(0, ||q||^2 - s), reference Distance.h:79-81).
//   exact path (fp32 storage): the k-th screen score s'_(k) gives the window
//     [s'_(k) - 2E, inf) that must hold the true top-k (see select.cu); it lies
//     inside the buffer when the floor is below it, and every buffered row in
//     it is re-scored in fp64 and sorted by (distance, id).
#include <cfloat>
#include <climits>

#include "kernels.cuh"
#include "ptx.cuh"

namespace mflat_cu {
namespace {

constexpr int kSelThreads = 512;
constexpr int kSelMax = 2048;       // winners sorted in shared memory

__device__ __forceinline__ float key_to_score(uint32_t key) {
    const uint32_t u = (key & 0x80000000u) ? (key & 0x7fffffffu) : ~key;
    return __uint_as_float(u);
}

// Key of the want-th largest key among s[0..n) (want in [1, n]) and how many
// entries equal to it belong to the top-want.
__device__ void radix_select(const float* __restrict__ s, int n, int want, uint32_t* hist,
                             uint32_t* sh_prefix, int* sh_remaining) {
    if (threadIdx.x == 0) { *sh_prefix = 0; *sh_remaining = want; }
    uint32_t mask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = *sh_prefix;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t key = score_key(s[i]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // Digit d of the want-th largest key: the highest d whose count of
            // keys in digits [d, 255] reaches `rem` (d = 0 when none of 255..1
            // does), and acc = the count in digits above d.  Warp 0 scans the
            // 256 bins, 8 per lane, from the top.
            const int lane = threadIdx.x;
            const uint32_t rem = static_cast<uint32_t>(*sh_remaining);
            uint32_t t = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) t += hist[8 * lane + j];
            uint32_t incl = t;   // sum over lanes >= lane
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t v = __shfl_down_sync(0xffffffffu, incl, off);
                if (lane + off < 32) incl += v;
            }
            uint32_t acc = incl - t;   // keys in digits above this lane's bins
            int found = -1;
            uint32_t found_acc = 0;
            if (acc < rem && rem <= acc + t) {
                for (int j = 7; j >= 0; --j) {
                    const int d = 8 * lane + j;
                    if (d == 0) break;
                    if (acc + hist[d] >= rem) {
                        found = d;
                        found_acc = acc;
                        break;
                    }
                    acc += hist[d];
                }
            }
            const unsigned who = __ballot_sync(0xffffffffu, found >= 0);
            const uint32_t total = __shfl_sync(0xffffffffu, incl, 0);
            int d = 0;
            uint32_t above = total - hist[0];
            if (who) {
                const int src = __ffs(who) - 1;
                d = __shfl_sync(0xffffffffu, found, src);
                above = __shfl_sync(0xffffffffu, found_acc, src);
            }
            if (lane == 0) {
                *sh_prefix = prefix | (static_cast<uint32_t>(d) << shift);
                *sh_remaining = static_cast<int>(rem - above);
            }
        }
        mask |= 255u << shift;
        __syncthreads();
    }
}

// Bitonic sort of cnt (<= kSelMax) entries: key descending, then id ascending.
__device__ void bitonic_sort(double* key, int* id, int cnt) {
    int P = 1;
    while (P < cnt) P <<= 1;
    for (int i = cnt + threadIdx.x; i < P; i += blockDim.x) { key[i] = -DBL_MAX; id[i] = INT_MAX; }
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const bool i_first = key[i] > key[j] || (key[i] == key[j] && id[i] < id[j]);
                    if (i_first != desc) {
                        const double tk = key[i]; key[i] = key[j]; key[j] = tk;
                        const int ti = id[i]; id[i] = id[j]; id[j] = ti;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// Bitonic sort of cnt (<= kSelMax) ints ascending.
__device__ void bitonic_sort_int(int* a, int cnt) {
    int P = 1;
    while (P < cnt) P <<= 1;
    for (int i = cnt + threadIdx.x; i < P; i += blockDim.x) a[i] = INT_MAX;
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool asc = (i & size) == 0;
                    if ((a[i] > a[j]) == asc) { const int t = a[i]; a[i] = a[j]; a[j] = t; }
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ double exact_score_l(int metric, const float* q, const float* x, int dim) {
    double acc = 0.0;
    if (metric == kL2) {
        for (int c = 0; c < dim; ++c) {
            const double e = static_cast<double>(q[c]) - static_cast<double>(x[c]);
            acc += e * e;
        }
        return -acc;
    }
    for (int c = 0; c < dim; ++c) acc += static_cast<double>(q[c]) * static_cast<double>(x[c]);
    return acc;
}

__device__ __forceinline__ double bound_e(int metric, double qn, double xmax, double gamma) {
    const double u = 1.0 / 8388608.0;
    if (metric == kL2) return 2.0 * gamma * qn * xmax + u * xmax * xmax + 2.0 * u * qn * xmax + 1e-30;
    return gamma * qn * xmax + 1e-30;
}

__global__ void __launch_bounds__(kSelThreads) select_large_kernel(const LargeSelectParams p) {
    const int qi = blockIdx.x;
    if (qi >= p.m) return;
    if (p.err && *p.err != 0) return;                     // a screen failed: buffers not valid
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sh_prefix;
    __shared__ int sh_remaining, sh_pos, sh_tpos, sh_status;
    __shared__ double key[kSelMax];
    __shared__ int ids[kSelMax];
    __shared__ int ties[kSelMax];

    const uint32_t n_raw = p.cnt[qi];
    const float* bs = p.buf_s + static_cast<int64_t>(qi) * p.cap;
    const int32_t* bi = p.buf_i + static_cast<int64_t>(qi) * p.cap;
    const float empty = p.metric == kL2 ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
    int64_t orow = static_cast<int64_t>(qi) * p.k_out;

    if (n_raw > p.cap) {                                  // buffer overflow: report, write nothing
        if (threadIdx.x == 0) atomicAdd(p.overflow, 1);
        return;
    }
    const int n = static_cast<int>(n_raw);
    const int k = p.k_out;
    const int want = min(k, n);
    if (threadIdx.x == 0) { sh_pos = 0; sh_tpos = 0; sh_status = 0; }
    int cnt = 0;     // entries gathered into key/ids

    if (want > 0) {
        radix_select(bs, n, want, hist, &sh_prefix, &sh_remaining);
        const uint32_t T = sh_prefix;
        if (!p.exact) {
            // winners: keys > T, plus the lowest-id entries equal to T
            const int need_eq = sh_remaining;
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const uint32_t kk = score_key(bs[i]);
                if (kk > T) {
                    const int slot = atomicAdd(&sh_pos, 1);
                    key[slot] = bs[i];
                    ids[slot] = bi[i];
                } else if (kk == T) {
                    const int slot = atomicAdd(&sh_tpos, 1);
                    if (slot < kSelMax) ties[slot] = bi[i];
                }
            }
            __syncthreads();
            const int ngt = sh_pos, nt = sh_tpos;
            if (nt > kSelMax) {
                if (threadIdx.x == 0) atomicAdd(p.overflow, 1);
                return;
            }
            bitonic_sort_int(ties, nt);                  // lowest ids first
            const float tsc = key_to_score(T);
            for (int i = threadIdx.x; i < need_eq; i += blockDim.x) {
                key[ngt + i] = tsc;
                ids[ngt + i] = ties[i];
            }
            __syncthreads();
            cnt = ngt + need_eq;
            bitonic_sort(key, ids, cnt);
            for (int pos = threadIdx.x; pos < k; pos += blockDim.x) {
                if (pos < cnt) {
                    const double s = key[pos];
                    float d;
                    if (p.metric == kL2) d = fmaxf(0.0f, static_cast<float>(static_cast<double>(p.qsq[qi]) - s));
                    else d = static_cast<float>(s);
                    p.out_ids[orow + pos] = static_cast<int32_t>(ids[pos] + p.id_base);
                    p.out_dist[orow + pos] = d;
                } else {
                    p.out_ids[orow + pos] = -1;
                    p.out_dist[orow + pos] = empty;
                }
            }
            return;
        }
        // ---- exact path: window [s'_(k) - 2E, inf) must lie above the floor
        const double sk = key_to_score(T);
        const double xmax = static_cast<double>(__uint_as_float(*p.xmax_bits));
        const double E = bound_e(p.metric, p.qnorm[qi], xmax, p.gamma);
        const double W = sk - 2.0 * E;
        const double floor_s = (p.thr[qi] == 0u) ? -DBL_MAX : static_cast<double>(key_to_score(p.thr[qi]));
        if (!(W >= floor_s)) {                    // window reaches below the floor
            if (threadIdx.x == 0) sh_status = 1;
        } else {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                if (static_cast<double>(bs[i]) >= W) {
                    const int slot = atomicAdd(&sh_pos, 1);
                    if (slot < kSelMax) ids[slot] = bi[i];
                }
            }
        }
        __syncthreads();
        if (threadIdx.x == 0 && sh_status == 0 && sh_pos > kSelMax) sh_status = 1;   // too many near-ties
        __syncthreads();
        if (sh_status) {
            if (threadIdx.x == 0) {
                const int slot = atomicAdd(p.flag_count, 1);
                p.flag_list[slot] = qi;
            }
            return;
        }
        cnt = sh_pos;
        const float* qx = p.q_x + static_cast<int64_t>(qi) * p.d_pad;
        for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
            const int64_t id = ids[i];
            if (id < 0 || id >= p.n) {                  // never produced by a screen
                atomicExch(const_cast<int*>(p.err), kErrInternal);
                key[i] = -DBL_MAX;
                continue;
            }
            key[i] = exact_score_l(p.metric, qx, p.db_x + id * p.d_pad, p.dim);
        }
        __syncthreads();
        bitonic_sort(key, ids, cnt);
        for (int pos = threadIdx.x; pos < k; pos += blockDim.x) {
            if (pos < cnt) {
                p.out_ids[orow + pos] = static_cast<int32_t>(ids[pos] + p.id_base);
                p.out_dist[orow + pos] = static_cast<float>(p.metric == kL2 ? -key[pos] : key[pos]);
            } else {
                p.out_ids[orow + pos] = -1;
                p.out_dist[orow + pos] = empty;
            }
        }
        return;
    }
    for (int pos = threadIdx.x; pos < k; pos += blockDim.x) {
        p.out_ids[orow + pos] = -1;
        p.out_dist[orow + pos] = empty;
    }
}

// Floor of one query from the pre-pass lists: the want-th largest score in the
// union of its L lists (each the KP1 best rows of one sample chunk).  At least
// `want` sampled rows score at or above it, so it is <= the global want-th
// best.  thr[q] = 0 (no floor) when the union holds fewer than `want` rows.
// thr_guess (when non-null) gets max(thr, r_guess-th best): a statistical
// floor for the next, denser sample pass (see buffer_floor_kernel).
constexpr int kFloorMax = kFloorMaxEntries;

__global__ void __launch_bounds__(256) prepass_floor_kernel(const float* __restrict__ part_s,
                                                            const int32_t* __restrict__ part_i,
                                                            int n_lists, int m, int m_pad, int kp1,
                                                            int want, int r_guess, uint32_t* thr,
                                                            uint32_t* thr_guess) {
    const int q = blockIdx.x;
    if (q >= m_pad) return;
    if (q >= m) {
        if (threadIdx.x == 0) {
            thr[q] = 0u;
            if (thr_guess) thr_guess[q] = 0u;
        }
        return;
    }
    __shared__ float vals[kFloorMax];
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sh_prefix;
    __shared__ int sh_remaining, sh_valid;
    if (threadIdx.x == 0) sh_valid = 0;
    __syncthreads();
    const int total = n_lists * kp1;
    int valid = 0;
    for (int e = threadIdx.x; e < total; e += blockDim.x) {
        const int l = e / kp1, j = e % kp1;
        const int64_t o = (static_cast<int64_t>(l) * m_pad + q) * kp1 + j;
        const bool ok = part_i[o] >= 0;
        vals[e] = ok ? part_s[o] : -__int_as_float(0x7f800000);
        valid += ok ? 1 : 0;
    }
    atomicAdd(&sh_valid, valid);
    __syncthreads();
    const int have = sh_valid;
    uint32_t valid_floor = 0u;
    if (have >= want) {
        radix_select(vals, total, want, hist, &sh_prefix, &sh_remaining);
        valid_floor = sh_prefix;
        __syncthreads();
    }
    uint32_t guess = valid_floor;
    if (thr_guess && r_guess > 0 && have >= r_guess) {
        radix_select(vals, total, r_guess, hist, &sh_prefix, &sh_remaining);
        guess = max(guess, sh_prefix);
    }
    if (threadIdx.x == 0) {
        thr[q] = valid_floor;
        if (thr_guess) thr_guess[q] = guess;
    }
}

// Sharper floor from a buffer-mode pass over a sample: the want-th best score
// among the rows the query's buffer kept (real rows, at or above the previous
// floor) is met by `want` rows, hence <= the global want-th best.  That holds
// for any subset, so an overflowed buffer (the first `cap` appends) still
// gives a valid floor.  Leaves thr unchanged when fewer than `want` were kept.
//
// thr_stat (when r_stat > 0) gets the r_stat-th best kept score, r_stat <
// want: a statistical floor.  With the sample a 1/s slice of the rows, the
// number of sampled rows among the global top-`want` is about want/s, and
// r_stat sits several standard deviations above that, so the floor is almost
// always below the global want-th best while admitting ~r_stat * s rows
// instead of ~want * s.  It is only a guess: floor_check_kernel verifies it
// after the full pass (at least `want` rows must reach it) and the caller
// redoes the pass with the valid floor when it fails.
__global__ void __launch_bounds__(512) buffer_floor_kernel(const uint32_t* __restrict__ cnt,
                                                           const float* __restrict__ buf_s, uint32_t cap,
                                                           int want, int r_stat, int m, uint32_t* thr,
                                                           uint32_t* thr_stat, int* short_count) {
    const int q = blockIdx.x;
    if (q >= m) return;
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sh_prefix;
    __shared__ int sh_remaining;
    const uint32_t n = min(cnt[q], cap);
    const float* s = buf_s + static_cast<int64_t>(q) * cap;
    uint32_t valid = thr[q];
    if (n >= static_cast<uint32_t>(want)) {
        radix_select(s, static_cast<int>(n), want, hist, &sh_prefix, &sh_remaining);
        valid = max(valid, sh_prefix);
        __syncthreads();
    } else if (short_count && threadIdx.x == 0) {
        atomicAdd(short_count, 1);    // the sample pass's floor kept too few rows
    }
    uint32_t stat = valid;
    if (r_stat > 0 && n >= static_cast<uint32_t>(r_stat)) {
        radix_select(s, static_cast<int>(n), r_stat, hist, &sh_prefix, &sh_remaining);
        stat = max(stat, sh_prefix);
    }
    if (threadIdx.x == 0) {
        thr[q] = valid;
        if (thr_stat) thr_stat[q] = stat;
    }
}

// A query whose full pass used a statistical floor above its valid one must
// have kept at least `want` rows; count the ones that did not.
__global__ void floor_check_kernel(const uint32_t* __restrict__ cnt, const uint32_t* __restrict__ used,
                                   const uint32_t* __restrict__ valid, int want, int m, int* failures) {
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= m) return;
    if (used[q] > valid[q] && cnt[q] < static_cast<uint32_t>(want)) atomicAdd(failures, 1);
}

}  // namespace

cudaError_t launch_buffer_floor(const uint32_t* cnt, const float* buf_s, uint32_t cap, int want,
                                int r_stat, int m, uint32_t* thr, uint32_t* thr_stat, int* short_count,
                                cudaStream_t stream) {
    buffer_floor_kernel<<<m, 512, 0, stream>>>(cnt, buf_s, cap, want, r_stat, m, thr, thr_stat,
                                                short_count);
    return cudaGetLastError();
}

cudaError_t launch_floor_check(const uint32_t* cnt, const uint32_t* used, const uint32_t* valid,
                               int want, int m, int* failures, cudaStream_t stream) {
    floor_check_kernel<<<(m + 255) / 256, 256, 0, stream>>>(cnt, used, valid, want, m, failures);
    return cudaGetLastError();
}

cudaError_t launch_select_large(const LargeSelectParams& p, cudaStream_t stream) {
    if (p.k_out < 1 || p.k_out > kSelMax) return cudaErrorInvalidValue;
    select_large_kernel<<<p.m, kSelThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_prepass_floor(const float* part_s, const int32_t* part_i, int n_lists, int m,
                                 int m_pad, int kp1, int want, int r_guess, uint32_t* thr,
                                 uint32_t* thr_guess, cudaStream_t stream) {
    if (n_lists * kp1 > kFloorMax || want < 1) return cudaErrorInvalidValue;
    prepass_floor_kernel<<<m_pad, 256, 0, stream>>>(part_s, part_i, n_lists, m, m_pad, kp1, want,
                                                    r_guess, thr, thr_guess);
    return cudaGetLastError();
}

}  // namespace mflat_cu
