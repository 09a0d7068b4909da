// epilogue.cuh -- per-32-column score processing shared by the screen
// kernels (thread = query row, 32 accumulator columns in registers).
#pragma once

#include <cstdint>

#include "kernels.cuh"
#include "ptx.cuh"

namespace mflat_cu {

// Eight float4 of the per-row score bias for 32 columns.  Every lane of the
// warp reads the same addresses (an L1 broadcast).
__device__ __forceinline__ void load_bias(float4 (&cb)[8], const float* src) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
    for (int q = 0; q < 8; ++q) cb[q] = __ldg(s4 + q);
}

// Scores of one 32-column chunk: s = alpha * dot + bias.  Hot path: 32 FFMA
// and a 31-FMNMX max tree, one compare.  Only when some score beats the gate
// (the list's worst entry or the published floor) are the scores spilled to
// a small local array and inserted one by one, in ascending id order.
template <int KP>
__device__ __forceinline__ void scan_chunk(const uint32_t (&r)[32], const float4 (&cb)[8],
                                           float alpha, float floor_adj, TopList<KP>& L, int id0) {
    float sc[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        sc[4 * q + 0] = fmaf(alpha, __uint_as_float(r[4 * q + 0]), cb[q].x);
        sc[4 * q + 1] = fmaf(alpha, __uint_as_float(r[4 * q + 1]), cb[q].y);
        sc[4 * q + 2] = fmaf(alpha, __uint_as_float(r[4 * q + 2]), cb[q].z);
        sc[4 * q + 3] = fmaf(alpha, __uint_as_float(r[4 * q + 3]), cb[q].w);
    }
    float m16[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) m16[i] = fmaxf(sc[2 * i], sc[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 8; ++i) m16[i] = fmaxf(m16[2 * i], m16[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 4; ++i) m16[i] = fmaxf(m16[2 * i], m16[2 * i + 1]);
    const float mx = fmaxf(fmaxf(m16[0], m16[1]), fmaxf(m16[2], m16[3]));
    if (mx > fmaxf(L.worst(), floor_adj)) {
        float tmp[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) tmp[j] = sc[j];
#pragma unroll 1
        for (int j = 0; j < 32; ++j) {
            const float v = tmp[j];
            if (v > fmaxf(L.worst(), floor_adj)) L.insert(v, id0 + j);
        }
    }
}

// Buffer mode: every score above the query's floor is appended to that
// query's candidate buffer (slot from an atomic counter; slots past `cap` are
// counted but not stored, so the select stage can detect an overflow).
struct BufferRow {
    uint32_t* cnt;
    float* s;
    int32_t* id;
    uint32_t cap;
};

__device__ __forceinline__ void buffer_chunk(const uint32_t (&r)[32], const float4 (&cb)[8],
                                             float alpha, float floor_adj, const BufferRow& br,
                                             int id0) {
    float sc[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        sc[4 * q + 0] = fmaf(alpha, __uint_as_float(r[4 * q + 0]), cb[q].x);
        sc[4 * q + 1] = fmaf(alpha, __uint_as_float(r[4 * q + 1]), cb[q].y);
        sc[4 * q + 2] = fmaf(alpha, __uint_as_float(r[4 * q + 2]), cb[q].z);
        sc[4 * q + 3] = fmaf(alpha, __uint_as_float(r[4 * q + 3]), cb[q].w);
    }
    float m16[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) m16[i] = fmaxf(sc[2 * i], sc[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 8; ++i) m16[i] = fmaxf(m16[2 * i], m16[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 4; ++i) m16[i] = fmaxf(m16[2 * i], m16[2 * i + 1]);
    const float mx = fmaxf(fmaxf(m16[0], m16[1]), fmaxf(m16[2], m16[3]));
    if (mx > floor_adj) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (sc[j] > floor_adj) {
                const uint32_t slot = atomicAdd(br.cnt, 1u);
                if (slot < br.cap) {
                    br.s[slot] = sc[j];
                    br.id[slot] = id0 + j;
                }
            }
        }
    }
}

}  // namespace mflat_cu
