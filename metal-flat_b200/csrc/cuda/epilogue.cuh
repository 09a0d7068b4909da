// epilogue.cuh -- per-32-column score processing shared by the screen
// kernels (thread = query row, 32 accumulator columns in registers).
#pragma once

#include <cstdint>

#include "kernels.cuh"
#include "ptx.cuh"

namespace mflat_cu {

// Two fp32 FMAs in one instruction (sm_100 packed f32x2), each lane rounded
// to nearest exactly like fmaf.
__device__ __forceinline__ void ffma2(float a, float x0, float x1, float c0, float c1, float& d0,
                                      float& d1) {
    asm("{\n\t.reg .b64 ra, rx, rc, rd;\n\t"
        "mov.b64 ra, {%2, %2};\n\t"
        "mov.b64 rx, {%3, %4};\n\t"
        "mov.b64 rc, {%5, %6};\n\t"
        "fma.rn.f32x2 rd, ra, rx, rc;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a), "f"(x0), "f"(x1), "f"(c0), "f"(c1));
}

// Three-input fp32 maximum (one instruction on sm_100).
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Maximum of 32 scores in 17 max instructions.
__device__ __forceinline__ float max_tree32(const float (&sc)[32]) {
    float t[11];
#pragma unroll
    for (int i = 0; i < 10; ++i) t[i] = max3f(sc[3 * i], sc[3 * i + 1], sc[3 * i + 2]);
    t[10] = fmaxf(sc[30], sc[31]);
    const float u0 = max3f(t[0], t[1], t[2]);
    const float u1 = max3f(t[3], t[4], t[5]);
    const float u2 = max3f(t[6], t[7], t[8]);
    const float u3 = fmaxf(t[9], t[10]);
    return fmaxf(max3f(u0, u1, u2), u3);
}

// s = alpha * acc + bias for 32 columns, as 16 packed FMAs.
__device__ __forceinline__ void chunk_scores(const uint32_t (&r)[32], const float4 (&cb)[8],
                                             float alpha, float (&sc)[32]) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        ffma2(alpha, __uint_as_float(r[4 * q + 0]), __uint_as_float(r[4 * q + 1]), cb[q].x, cb[q].y,
              sc[4 * q + 0], sc[4 * q + 1]);
        ffma2(alpha, __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]), cb[q].z, cb[q].w,
              sc[4 * q + 2], sc[4 * q + 3]);
    }
}

// Eight float4 of the per-row score bias for 32 columns, from global memory.
// Every lane of the warp reads the same addresses (an L1 broadcast).
__device__ __forceinline__ void load_bias(float4 (&cb)[8], const float* src) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
    for (int q = 0; q < 8; ++q) cb[q] = __ldg(s4 + q);
}

// The same from shared memory (a broadcast read; `src` must point into this
// CTA's shared memory -- the read-only global path cannot address it).
__device__ __forceinline__ void load_bias_shared(float4 (&cb)[8], const float* src) {
    const uint32_t a = smem_u32(src);
#pragma unroll
    for (int q = 0; q < 8; ++q)
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(cb[q].x), "=f"(cb[q].y), "=f"(cb[q].z), "=f"(cb[q].w)
                     : "r"(a + q * 16)
                     : "memory");
}

// Bit mask of the columns scoring above `gate` (slow paths only).  The eight
// 4-column groups are screened by their maxima (recomputed here rather than
// kept live from the hot path's tree) and only passing groups are compared
// column by column.
__device__ __forceinline__ uint32_t passing_mask(const float (&sc)[32], float gate) {
    uint32_t mask = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (fmaxf(max3f(sc[4 * i], sc[4 * i + 1], sc[4 * i + 2]), sc[4 * i + 3]) > gate) {
#pragma unroll
            for (int e = 0; e < 4; ++e) mask |= (sc[4 * i + e] > gate ? 1u : 0u) << (4 * i + e);
        }
    }
    return mask;
}

// sc[j] for a run-time j, as a 5-level select tree over registers (a dynamic
// index into a register array would place it in local memory).
__device__ __forceinline__ float select32(const float (&sc)[32], uint32_t j) {
    float a[16], b[8], c[4], d[2];
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] = (j & 1u) ? sc[2 * i + 1] : sc[2 * i];
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = (j & 2u) ? a[2 * i + 1] : a[2 * i];
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = (j & 4u) ? b[2 * i + 1] : b[2 * i];
#pragma unroll
    for (int i = 0; i < 2; ++i) d[i] = (j & 8u) ? c[2 * i + 1] : c[2 * i];
    return (j & 16u) ? d[1] : d[0];
}

// List mode, slow path: insert the columns beating the gate (the list's worst
// entry or the published floor) in ascending id order, re-testing each
// against the raised gate.  One copy of the insertion network.
template <int KP>
__device__ __forceinline__ void insert_passing(const float (&sc)[32], float floor_adj, TopList<KP>& L,
                                               int id0) {
    uint32_t mask = passing_mask(sc, fmaxf(L.worst(), floor_adj));
#pragma unroll 1
    while (mask) {
        const uint32_t j = __ffs(mask) - 1;
        mask &= mask - 1u;
        const float v = select32(sc, j);
        if (v > fmaxf(L.worst(), floor_adj)) L.insert(v, id0 + static_cast<int>(j));
    }
}

// Scores of one 32-column chunk: s = alpha * dot + bias.  Hot path: 16 packed
// FMAs, a 17-instruction max tree and one compare; the slow path runs only
// when some score beats the gate.
template <int KP>
__device__ __forceinline__ void scan_chunk(const uint32_t (&r)[32], const float4 (&cb)[8],
                                           float alpha, float floor_adj, TopList<KP>& L, int id0) {
    float sc[32];
    chunk_scores(r, cb, alpha, sc);
    if (max_tree32(sc) > fmaxf(L.worst(), floor_adj)) insert_passing<KP>(sc, floor_adj, L, id0);
}

// Buffer mode: every score above the query's floor is appended to that
// query's candidate buffer (slots past `cap` are counted but not stored, so the
// select stage can detect an overflow).  The passing columns of a chunk are
// found group-wise, one atomic reserves their slots, and the passing groups
// are visited again to write them, all from registers.
struct BufferRow {
    uint32_t* cnt;
    float* s;
    int32_t* id;
    uint32_t cap;
};

// `scale` converts the compared values to scores (1, or 2 for the L2 screen
// whose accumulator holds half the score); an exact power of two.
__device__ __forceinline__ void append_passing(const float (&sc)[32], float floor_adj, float scale,
                                               const BufferRow& br, int id0) {
    const uint32_t mask = passing_mask(sc, floor_adj);
    uint32_t slot = atomicAdd(br.cnt, static_cast<uint32_t>(__popc(mask)));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if ((mask >> (4 * i)) & 0xFu) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = 4 * i + e;
                if ((mask >> j) & 1u) {
                    if (slot < br.cap) {
                        br.s[slot] = scale * sc[j];
                        br.id[slot] = id0 + j;
                    }
                    ++slot;
                }
            }
        }
    }
}

// Per-thread stage of up to kStage appends, held in registers.  Staged entries
// are published -- one atomic reserves their slots, then the stores -- when the
// stage would overflow and at the end of each unit, so the atomic's round trip
// (which all warps of the tile wait for before the accumulator is released)
// leaves the per-chunk slow path.  A chunk with more than kStage passing columns
// is appended directly.
struct AppendStage {
    static constexpr uint32_t kStage = 2;
    float s0, s1;
    int i0, i1;
    uint32_t n;

    __device__ __forceinline__ void init() {
        n = 0;
        s0 = s1 = 0.0f;
        i0 = i1 = 0;
    }
    // static register slots chosen by a compare (no local memory)
    __device__ __forceinline__ void put(float v, int id) {
        if (n == 0) { s0 = v; i0 = id; }
        else { s1 = v; i1 = id; }
        ++n;
    }
    __device__ __forceinline__ void flush(const BufferRow& br) {
        if (n == 0) return;
        const uint32_t base = atomicAdd(br.cnt, n);
        if (base < br.cap) { br.s[base] = s0; br.id[base] = i0; }
        if (n > 1 && base + 1 < br.cap) { br.s[base + 1] = s1; br.id[base + 1] = i1; }
        n = 0;
    }
};

__device__ __forceinline__ void stage_passing(const float (&sc)[32], float floor_adj, float scale,
                                              const BufferRow& br, AppendStage& st, int id0) {
    const uint32_t mask = passing_mask(sc, floor_adj);
    const uint32_t np = __popc(mask);
    if (st.n + np > AppendStage::kStage) {
        st.flush(br);
        if (np > AppendStage::kStage) {
            append_passing(sc, floor_adj, scale, br, id0);
            return;
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if ((mask >> (4 * i)) & 0xFu) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int j = 4 * i + e;
                if ((mask >> j) & 1u) st.put(scale * sc[j], id0 + j);
            }
        }
    }
}

__device__ __forceinline__ void buffer_chunk(const uint32_t (&r)[32], const float4 (&cb)[8],
                                             float alpha, float floor_adj, const BufferRow& br,
                                             AppendStage& st, int id0) {
    float sc[32];
    chunk_scores(r, cb, alpha, sc);
    if (max_tree32(sc) > floor_adj) stage_passing(sc, floor_adj, 1.0f, br, st, id0);
}

// Accumulator compared as it is (no bias load, no FFMA): inner product on
// chunks wholly inside the database (bias 0, scale 1), or the L2 screen with
// the bias folded into the MMA (accumulator = score / 2: floor_adj halved,
// scale 2).
__device__ __forceinline__ void buffer_chunk_raw(const uint32_t (&r)[32], float floor_adj, float scale,
                                                 const BufferRow& br, AppendStage& st, int id0) {
    float sc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) sc[j] = __uint_as_float(r[j]);
    if (max_tree32(sc) > floor_adj) stage_passing(sc, floor_adj, scale, br, st, id0);
}

template <int KP>
__device__ __forceinline__ void scan_chunk_raw(const uint32_t (&r)[32], float floor_adj,
                                               TopList<KP>& L, int id0) {
    float sc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) sc[j] = __uint_as_float(r[j]);
    if (max_tree32(sc) > fmaxf(L.worst(), floor_adj)) insert_passing<KP>(sc, floor_adj, L, id0);
}

}  // namespace mflat_cu
