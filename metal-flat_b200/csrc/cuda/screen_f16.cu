// screen_f16.cu -- tcgen05 kind::f16 distance GEMM with fused selection, for
// fp16 / bf16 database storage (the recall path: no fp32 rows are kept, the
// screen's own scores are the result).
//
// Same structure as screen_tc.cu, with these differences:
//   * one operand plane (no hi/lo split): tcgen05.mma.kind::f16, M=128 N=256
//     K=16, fp32 accumulation in TMEM; a 128-byte k-block holds 64 halves;
//   * the query tile stays resident in shared memory when it fits
//     (d <= 384); otherwise it is streamed with the database tile, one
//     k-block of each per ring stage (d = 768 for config 2);
//   * the epilogue warpgroups split each tile's 256 columns (the MMA of a
//     d = 128 tile lasts only ~1k cycles): four in buffer mode, two in list
//     mode, where each keeps its own top-KP, written as two lists per
//     (query, chunk) for the select stage;
//   * each warp hands its accumulator back after its last TMEM load of the
//     tile, before scoring that chunk.
#include "epilogue.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace mflat_cu {
namespace {

// Epilogue warpgroups: 2 in list mode (per-thread lists need the registers),
// 4 in buffer mode (4 warps per SMSP hide the TMEM-load / FMA latency of a
// d = 128 tile, whose MMA lasts only ~1.5k cycles).  Producer and MMA warps
// follow the epilogue warps.
__host__ __device__ constexpr int epi_wg(bool buf) { return buf ? 4 : 2; }
__host__ __device__ constexpr int threads_h(bool buf) { return epi_wg(buf) * 128 + 64; }
constexpr int kBKH = 64;                          // halves per 128-byte k-block
constexpr int kATileBytesH = kBM * 128;           // 16 KB
constexpr int kBTileBytesH = kBN * 128;           // 32 KB
constexpr int kMaxStagesH = 6;
constexpr int kMaxResidentKb = 6;                 // d_pad <= 384 keeps A resident
constexpr int kBarBytesH = 256;                   // mbarriers, TMEM slot, abort flag
constexpr int kBiasBytesH = kBN * 4;              // one tile's score bias (fp32)
// Folded L2 bias (kFold): one more K = 16 MMA step per tile adds -||x||^2 / 2,
// held as three bf16 parts per row, to the accumulator (A = a tile of ones),
// so the accumulator is half the score and the epilogue compares it as it is.
constexpr int kFoldSlots = 4;                     // bias tiles in flight (loaded one tile ahead)
constexpr int kFoldSlotBytes = kBN * 16;          // 256 rows x 8 bf16: the 3 parts, then zeros
constexpr int kOnesBytes = kBM * 16;              // 128 rows x 8 bf16: 1, 1, 1, 0, ...
constexpr int kZeroBytes = kBN * 16;              // K columns 8..15 of both operands
constexpr int kFoldBytes = kFoldSlots * kFoldSlotBytes + kOnesBytes + kZeroBytes;
constexpr int kSmemMaxH = 232448;                 // opt-in shared memory per CTA
constexpr uint32_t kOneBf16x2 = 0x3F803F80u;      // two bf16 1.0

__host__ __device__ inline bool a_streamed(int kb) { return kb > kMaxResidentKb; }
__host__ __device__ inline int stage_bytes_h(int kb) {
    return a_streamed(kb) ? kATileBytesH + kBTileBytesH : kBTileBytesH;
}
__host__ __device__ inline int extra_bytes_h(bool fold) { return fold ? kFoldBytes : 2 * kBiasBytesH; }
__host__ __device__ inline int n_stages_h(int kb, bool fold) {
    const int a = a_streamed(kb) ? 0 : kb * kATileBytesH;
    const int budget = kSmemMaxH - kBarBytesH - extra_bytes_h(fold);
    const int s = (budget - a) / stage_bytes_h(kb);
    return s > kMaxStagesH ? kMaxStagesH : s;
}

struct SmemH {
    uint8_t* a;         // resident A [kb][16 KB] (resident mode)
    uint8_t* ring;      // [stages][stage bytes]: ([A 16 KB]) [B 32 KB]
    uint64_t *full, *empty, *a_full, *a_empty, *acc_full, *acc_empty, *drain;
    uint64_t* bias_full;   // [2] (bias copy of accumulator buffer b) or [kFoldSlots]
    uint32_t* tmem_slot;
    int* abort_flag;
    float* bias;        // [2][kBN]: score bias of the tile in accumulator buffer b
    uint8_t* fold;      // kFold: [kFoldSlots][4 KB] bias parts, ones [2 KB], zeros [4 KB]
};

__device__ inline SmemH carve_h(uint8_t* base, int kb, int stages) {
    SmemH S;
    S.a = base;
    S.ring = base + (a_streamed(kb) ? 0 : kb * kATileBytesH);
    uint64_t* bars = reinterpret_cast<uint64_t*>(S.ring + stages * stage_bytes_h(kb));
    S.full = bars;
    S.empty = bars + kMaxStagesH;
    S.a_full = bars + 2 * kMaxStagesH;
    S.a_empty = S.a_full + 1;
    S.acc_full = S.a_full + 2;
    S.acc_empty = S.a_full + 4;
    S.drain = S.a_full + 6;
    S.bias_full = S.a_full + 7;                          // up to kFoldSlots barriers
    S.tmem_slot = reinterpret_cast<uint32_t*>(S.bias_full + kFoldSlots);
    S.abort_flag = reinterpret_cast<int*>(S.tmem_slot + 1);
    S.bias = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + kBarBytesH);
    S.fold = reinterpret_cast<uint8_t*>(bars) + kBarBytesH;
    return S;
}

template <int KP, bool kBuf, bool kBF16, bool kFold>
__global__ void __launch_bounds__(threads_h(kBuf), 1)
screen_f16_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                  const __grid_constant__ CUtensorMap tm_bias, const ScreenParams p) {
    // SWIZZLE_128B tiles need 1024-byte aligned shared memory.  The declared
    // alignment is checked, not assumed: a misaligned base ends the launch
    // with a configuration error before any copy is issued.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = smem_raw;
    const int kb_count = p.d_pad / kBKH;
    if (kb_count < 1 || kb_count * kBKH != p.d_pad || (smem_u32(smem_raw) & 1023u) != 0u) {
        if (threadIdx.x == 0) atomicExch(p.err, kErrConfig);
        return;
    }
    const bool stream_a = a_streamed(kb_count);
    const int stages = n_stages_h(kb_count, kFold);
    const int sbytes = stage_bytes_h(kb_count);
    SmemH S = carve_h(base, kb_count, stages);
    constexpr uint32_t kIdesc = make_idesc(kBF16 ? 1u : 0u, kBM, kBN);
    constexpr uint32_t kIdescBias = make_idesc(1u, kBM, kBN);   // the bias step is bf16

    constexpr int kEpiWG = epi_wg(kBuf);
    constexpr int kProducerWarpH = kEpiWG * 4;
    constexpr int kMmaWarpH = kProducerWarpH + 1;
    constexpr int kCols = kBN / kEpiWG;          // accumulator columns per warpgroup
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxStagesH; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        mbar_init(S.a_full, 1);
        mbar_init(S.a_empty, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.acc_full[b], 1);
            mbar_init(&S.acc_empty[b], kEpiWG * 4);   // one arrival per epilogue warp
        }
        mbar_init(S.drain, 1);
        for (int s = 0; s < kFoldSlots; ++s) mbar_init(&S.bias_full[s], 1);
        *S.abort_flag = 0;
        fence_mbar_init();
    }
    if constexpr (kFold) {
        // the constant operand rows of the bias step: A = (1, 1, 1, 0, ...),
        // and zeros for K columns 8..15 of A and B; written once, then made
        // visible to the tensor core's (async-proxy) reads
        uint4* ones = reinterpret_cast<uint4*>(S.fold + kFoldSlots * kFoldSlotBytes);
        uint4* zeros = ones + kOnesBytes / 16;
        for (int i = threadIdx.x; i < kOnesBytes / 16 + kZeroBytes / 16; i += blockDim.x) {
            if (i < kOnesBytes / 16) ones[i] = make_uint4(kOneBf16x2, kOneBf16x2 & 0xFFFFu, 0u, 0u);
            else zeros[i - kOnesBytes / 16] = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_shared();
    }
    if (warp == kMmaWarpH) {
        tmem_alloc(S.tmem_slot, 512);
        tmem_relinquish();
    }
    if (warp == kProducerWarpH && lane == 0) {
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
        if constexpr (kFold) tma_prefetch_desc(&tm_bias);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *S.tmem_slot;
    volatile int* abort_flag = S.abort_flag;
    const int n_units = p.n_qtiles * p.n_chunks;

    if (warp == kProducerWarpH) {
        if (lane == 0) {
            int stage = 0;
            uint32_t sphase = 0, a_phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;
            bool a_issued = false;
            uint32_t a_issue_phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
                const int qt = u % p.n_qtiles;
                const int ch = u / p.n_qtiles;
                const int t0 = ch * p.tiles_per_chunk;
                const int t1 = min(t0 + p.tiles_per_chunk, p.n_tiles);
                if (!stream_a) {
                    if (!mbar_wait(S.a_empty, a_phase ^ 1u, abort_flag, p.wait_ns)) { ok = false; break; }
                    mbar_arrive_expect_tx(S.a_full, static_cast<uint32_t>(kb_count * kATileBytesH));
                    for (int kb = 0; kb < kb_count; ++kb)
                        tma_load_2d(&tm_a, S.a_full, S.a + kb * kATileBytesH, kb * kBKH, qt * kBM);
                    a_issued = true;
                    a_issue_phase = a_phase;
                    a_phase ^= 1u;
                }
                for (int t = t0; t < t1 && ok; ++t) {
                    for (int kb = 0; kb < kb_count; ++kb) {
                        if (!mbar_wait(&S.empty[stage], sphase ^ 1u, abort_flag, p.wait_ns)) { ok = false; break; }
                        uint8_t* st = S.ring + stage * sbytes;
                        mbar_arrive_expect_tx(&S.full[stage], static_cast<uint32_t>(sbytes));
                        if (stream_a) {
                            tma_load_2d(&tm_a, &S.full[stage], st, kb * kBKH, qt * kBM);
                            st += kATileBytesH;
                        }
                        tma_load_2d(&tm_b, &S.full[stage], st, kb * kBKH, t * p.tile_stride * kBN);
                        issued_mask |= 1u << stage;
                        issued_phase = (issued_phase & ~(1u << stage)) | (sphase << stage);
                        if (++stage == stages) { stage = 0; sphase ^= 1u; }
                    }
                }
            }
            if (*abort_flag) {
                for (int s = 0; s < stages; ++s)
                    if (issued_mask & (1u << s))
                        mbar_wait_drain(&S.full[s], (issued_phase >> s) & 1u, 200000000ull);
                if (a_issued) mbar_wait_drain(S.a_full, a_issue_phase, 200000000ull);
            }
        }
    } else if (warp == kMmaWarpH) {
        if (lane == 0) {
            int stage = 0;
            uint32_t sphase = 0, a_phase = 0, tcount = 0;
            uint32_t bias_pending = 0, bias_phase = 0;   // bias copies issued (drain on abort)
            bool ok = true, issued_any = false;
            // kFold: the bias parts of the CTA's tile number tc go to slot tc % 4,
            // loaded one tile ahead.  Slot (tc + 1) % 4 last served tile tc - 3,
            // whose bias step has completed once acc_empty of tile tc has been
            // observed (the epilogue had received tile tc - 2, committed after it).
            const uint32_t ones = smem_u32(S.fold + kFoldSlots * kFoldSlotBytes);
            const uint32_t zeros = ones + kOnesBytes;
            auto load_bias_parts = [&](uint32_t tc, int tile) {
                const uint32_t sl = tc % kFoldSlots;
                mbar_arrive_expect_tx(&S.bias_full[sl], kFoldSlotBytes);
                tma_load_2d(&tm_bias, &S.bias_full[sl], S.fold + sl * kFoldSlotBytes, 0,
                            tile * p.tile_stride * kBN);
                bias_pending |= 1u << sl;
                bias_phase = (bias_phase & ~(1u << sl)) | (((tc / kFoldSlots) & 1u) << sl);
            };
            if constexpr (kFold) {
                if (static_cast<int>(blockIdx.x) < n_units)
                    load_bias_parts(0, (blockIdx.x / p.n_qtiles) * p.tiles_per_chunk);
            }
            for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
                const int ch = u / p.n_qtiles;
                const int t0 = ch * p.tiles_per_chunk;
                const int t1 = min(t0 + p.tiles_per_chunk, p.n_tiles);
                if (!stream_a) {
                    if (!mbar_wait(S.a_full, a_phase, abort_flag, p.wait_ns)) { ok = false; break; }
                    a_phase ^= 1u;
                    tc_fence_after();
                }
                for (int t = t0; t < t1 && ok; ++t, ++tcount) {
                    const uint32_t b = tcount & 1u;
                    const uint32_t ph = (tcount >> 1) & 1u;
                    if (!mbar_wait(&S.acc_empty[b], ph ^ 1u, abort_flag, p.wait_ns)) { ok = false; break; }
                    tc_fence_after();
                    if constexpr (kFold) {
                        // the CTA's next tile: the rest of this unit, else the
                        // first tile of its next unit
                        int nt = -1;
                        if (t + 1 < t1) nt = t + 1;
                        else if (u + static_cast<int>(gridDim.x) < n_units)
                            nt = ((u + static_cast<int>(gridDim.x)) / p.n_qtiles) * p.tiles_per_chunk;
                        if (nt >= 0) load_bias_parts(tcount + 1, nt);
                    } else {
                        // the epilogue is done with buffer b's tile (two tiles
                        // back), so its bias slot takes this tile's bias; the copy
                        // lands while the MMAs run
                        mbar_arrive_expect_tx(&S.bias_full[b], kBiasBytesH);
                        bulk_load_g2s(S.bias + b * kBN,
                                      p.colbias + static_cast<int64_t>(t) * p.tile_stride * kBN,
                                      kBiasBytesH, &S.bias_full[b]);
                        bias_pending |= 1u << b;
                        bias_phase = (bias_phase & ~(1u << b)) | (ph << b);
                    }
                    const uint32_t d_tmem = tmem_base + b * kBN;
                    for (int kb = 0; kb < kb_count; ++kb) {
                        if (!mbar_wait(&S.full[stage], sphase, abort_flag, p.wait_ns)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t st = smem_u32(S.ring + stage * sbytes);
                        const uint64_t ad = smem_desc_k_sw128(
                            stream_a ? st : smem_u32(S.a + kb * kATileBytesH));
                        const uint64_t bd = smem_desc_k_sw128(stream_a ? st + kATileBytesH : st);
#pragma unroll
                        for (int ks = 0; ks < kBKH / 16; ++ks) {
                            const uint64_t o = static_cast<uint64_t>(ks * 2);   // 32 B >> 4
                            tc_mma_f16(d_tmem, ad + o, bd + o, kIdesc, (kb | ks) != 0 ? 1u : 0u);
                        }
                        issued_any = true;
                        tc_commit(&S.empty[stage]);
                        if (++stage == stages) { stage = 0; sphase ^= 1u; }
                    }
                    if constexpr (kFold) {
                        if (ok) {
                            const uint32_t sl = tcount % kFoldSlots;
                            if (!mbar_wait(&S.bias_full[sl], (tcount / kFoldSlots) & 1u, abort_flag, p.wait_ns)) {
                                ok = false;
                            } else {
                                bias_pending &= ~(1u << sl);
                                tc_fence_after();
                                const uint32_t bslot = smem_u32(S.fold + sl * kFoldSlotBytes);
                                tc_mma_f16(d_tmem, smem_desc_k_none(ones, zeros - ones, 128u),
                                           smem_desc_k_none(bslot, zeros - bslot, 128u), kIdescBias, 1u);
                            }
                        }
                    }
                    if (ok) tc_commit(&S.acc_full[b]);
                }
                if (ok && !stream_a) tc_commit(S.a_empty);
            }
            if (*abort_flag && issued_any) {
                tc_commit(S.drain);
                mbar_wait_drain(S.drain, 0u, 200000000ull);
            }
            if (*abort_flag) {
                for (int sl = 0; sl < kFoldSlots; ++sl)
                    if (bias_pending & (1u << sl))
                        mbar_wait_drain(&S.bias_full[sl], (bias_phase >> sl) & 1u, 200000000ull);
            }
        }
    } else {
        // ---------------- epilogue: warpgroup g = warp / 4 owns columns [g*kCols, (g+1)*kCols)
        const int g = warp >> 2;
        const int wq = warp & 3;
        const int row_in_tile = wq * 32 + lane;
        const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(wq * 32) << 16);
        // Accumulator b (and its bias slot) goes back to the MMA warp as soon as
        // the warp's last tcgen05.ld of the tile has completed and that chunk's
        // bias loads are issued, before the last chunk is scored: the refill of
        // b (tile t + 2) then overlaps that scoring.  The arrival releases the
        // preceding shared-memory reads, and the bias copy into the slot is
        // issued only after the MMA thread has observed it.
        auto release_acc = [&](uint32_t b) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.acc_empty[b]);
        };
        uint32_t tcount = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            const int qt = u % p.n_qtiles;
            const int ch = u / p.n_qtiles;
            const int t0 = ch * p.tiles_per_chunk;
            const int t1 = min(t0 + p.tiles_per_chunk, p.n_tiles);
            const int row = qt * kBM + row_in_tile;
            const bool live = row < p.m;
            TopList<KP> L;
            L.init();
            BufferRow br{};
            AppendStage st;
            st.init();
            if constexpr (kBuf) {
                const int rr = live ? row : 0;
                br = BufferRow{p.buf_cnt + rr, p.buf_s + static_cast<int64_t>(rr) * p.cap,
                               p.buf_i + static_cast<int64_t>(rr) * p.cap, p.cap};
            }
            // Score floor: fixed during a buffer pass (one load per unit); in list
            // mode raised by finished units (monotone), reloaded one tile ahead.
            uint32_t fkey_next = (live && p.use_floor) ? __ldcg(p.thr + row) : 0u;
            for (int t = t0; t < t1; ++t, ++tcount) {
                const uint32_t b = tcount & 1u;
                const uint32_t ph = (tcount >> 1) & 1u;
                const uint32_t fkey = fkey_next;
                if (!kBuf && live && p.use_floor && t + 1 < t1) fkey_next = __ldcg(p.thr + row);
                // one lane polls the barriers, the warp follows
                bool ready = true;
                if (lane == 0)
                    ready = mbar_wait(&S.acc_full[b], ph, abort_flag, p.wait_ns) &&
                            (kFold || mbar_wait(&S.bias_full[b], ph, abort_flag, p.wait_ns));
                if (!__shfl_sync(0xffffffffu, ready ? 1 : 0, 0)) { ok = false; break; }
                // with the bias folded into the MMA the accumulator is half the
                // score: it is compared against half the floor (exact)
                const float floor_adj =
                    (!live ? __int_as_float(0x7f800000)
                           : (p.use_floor ? floor_below(fkey) : -__int_as_float(0x7f800000))) *
                    (kFold ? 0.5f : 1.0f);
                const int id_tile = t * p.tile_stride * kBN + g * kCols;
                const float* cb_tile = S.bias + b * kBN + g * kCols;   // shared memory
                const uint32_t taddr = lane_addr + b * kBN + g * kCols;
                // inner product on columns wholly inside the database: bias 0
                const bool raw = p.alpha == 1.0f && static_cast<int64_t>(id_tile) + kCols <= p.n;
                if constexpr (kBuf) {
                    // buffer mode, 4 warps per SMSP: one chunk at a time, latency
                    // hidden by the other warps (keeps the thread within 96 registers)
                    static_assert(kEpiWG == 4, "buffer mode runs four epilogue warpgroups");
                    __syncwarp();
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < kCols / 32; ++c) {
                        uint32_t r[32];
                        float4 cb[8];
                        __syncwarp();
                        tmem_ld_32x32b_x32(taddr + c * 32, r);
                        if (!kFold && !raw) load_bias_shared(cb, cb_tile + c * 32);
                        tmem_wait_ld_regs(r);
                        if (c == kCols / 32 - 1) release_acc(b);
                        if (kFold) buffer_chunk_raw(r, floor_adj, 2.0f, br, st, id_tile + c * 32);
                        else if (raw) buffer_chunk_raw(r, floor_adj, 1.0f, br, st, id_tile + c * 32);
                        else buffer_chunk(r, cb, p.alpha, floor_adj, br, st, id_tile + c * 32);
                    }
                } else {
                    // list mode, 2 warps per SMSP: the next chunk's TMEM load is in
                    // flight while a chunk is scored
                    uint32_t ra[32], rb[32];
                    float4 cb[8];
                    __syncwarp();
                    tc_fence_after();
                    tmem_ld_32x32b_x32(taddr, ra);
#pragma unroll 1
                    for (int c = 0; c < kCols / 32; c += 2) {
                        if (!kFold && !raw) load_bias_shared(cb, cb_tile + c * 32);
                        tmem_wait_ld_regs(ra);
                        __syncwarp();
                        tmem_ld_32x32b_x32(taddr + (c + 1) * 32, rb);
                        if (kFold || raw) scan_chunk_raw<KP>(ra, floor_adj, L, id_tile + c * 32);
                        else scan_chunk<KP>(ra, cb, p.alpha, floor_adj, L, id_tile + c * 32);
                        if (!kFold && !raw) load_bias_shared(cb, cb_tile + (c + 1) * 32);
                        tmem_wait_ld_regs(rb);
                        if (c + 2 < kCols / 32) {
                            __syncwarp();
                            tmem_ld_32x32b_x32(taddr + (c + 2) * 32, ra);
                        } else {
                            release_acc(b);
                        }
                        if (kFold || raw) scan_chunk_raw<KP>(rb, floor_adj, L, id_tile + (c + 1) * 32);
                        else scan_chunk<KP>(rb, cb, p.alpha, floor_adj, L, id_tile + (c + 1) * 32);
                    }
                }
            }
            if constexpr (kBuf) st.flush(br);   // the unit's staged appends
            if (!ok) break;
            if (!kBuf && live) {
                const int64_t o = (static_cast<int64_t>(ch * kEpiWG + g) * p.m_pad + row) * KP;
                float4* ps = reinterpret_cast<float4*>(p.part_score + o);
                int4* pi = reinterpret_cast<int4*>(p.part_id + o);
                const float sc = kFold ? 2.0f : 1.0f;   // list entries back to score units
#pragma unroll
                for (int i = 0; i < KP / 4; ++i) {
                    ps[i] = make_float4(sc * L.s[4 * i], sc * L.s[4 * i + 1], sc * L.s[4 * i + 2],
                                        sc * L.s[4 * i + 3]);
                    pi[i] = make_int4(L.id[4 * i], L.id[4 * i + 1], L.id[4 * i + 2], L.id[4 * i + 3]);
                }
                if (p.use_floor && L.id[KP - 1] >= 0)
                    atomicMax(p.thr + row, score_key(sc * L.s[KP - 1]));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarpH) tmem_dealloc(tmem_base, 512);
    if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, *abort_flag);
}

template <int KP, bool kBuf, bool kBF16, bool kFold>
cudaError_t launch_h(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& bias,
                     const ScreenParams& p, int grid, cudaStream_t stream) {
    const int smem = screen_f16_smem_bytes(p.d_pad, kFold);
    cudaError_t e = cudaFuncSetAttribute(screen_f16_kernel<KP, kBuf, kBF16, kFold>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    screen_f16_kernel<KP, kBuf, kBF16, kFold><<<grid, threads_h(kBuf), smem, stream>>>(a, b, bias, p);
    return cudaGetLastError();
}

template <bool kBF16, bool kFold>
cudaError_t launch_h_kp(int kp, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& bias,
                        const ScreenParams& p, int grid, cudaStream_t stream) {
    switch (kp) {
        case 0: return launch_h<4, true, kBF16, kFold>(a, b, bias, p, grid, stream);
        case 4: return launch_h<4, false, kBF16, kFold>(a, b, bias, p, grid, stream);
        case 8: return launch_h<8, false, kBF16, kFold>(a, b, bias, p, grid, stream);
        case 16: return launch_h<16, false, kBF16, kFold>(a, b, bias, p, grid, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

int screen_f16_smem_bytes(int d_pad, bool fold) {
    const int kb = d_pad / kBKH;
    const int a = a_streamed(kb) ? 0 : kb * kATileBytesH;
    return a + n_stages_h(kb, fold) * stage_bytes_h(kb) + kBarBytesH + extra_bytes_h(fold);
}

cudaError_t launch_screen_f16(int kp, bool bf16, const CUtensorMap& a, const CUtensorMap& b,
                              const CUtensorMap* fold_bias, const ScreenParams& p, int grid,
                              cudaStream_t stream) {
    if (p.d_pad % kBKH != 0 || p.d_pad < kBKH) return cudaErrorInvalidValue;
    if (fold_bias)
        return bf16 ? launch_h_kp<true, true>(kp, a, b, *fold_bias, p, grid, stream)
                    : launch_h_kp<false, true>(kp, a, b, *fold_bias, p, grid, stream);
    return bf16 ? launch_h_kp<true, false>(kp, a, b, b, p, grid, stream)
                : launch_h_kp<false, false>(kp, a, b, b, p, grid, stream);
}

}  // namespace mflat_cu
