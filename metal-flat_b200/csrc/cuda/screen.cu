// screen.cu -- the tcgen05 distance GEMM with the top-k selection fused into
// its epilogue: the B200 replacement of the reference's per-tile pair
// GemmDistance::encode + topk_merge (src/GemmDistance.mm:15-60 and
// src/FlatIndex.mm:63-107, which round-tripped an m x tileW score matrix
// through device memory; here no score matrix is ever written).
//
// One kernel serves every storage precision:
//   * fp16 / bf16 storage: one operand plane, tcgen05.mma.kind::f16;
//   * fp32 storage (kX3): each operand is held as two bf16 planes, x ~ h + l
//     with h = bf16(x), l = bf16(x - h), and the kernel accumulates
//     A_h.B_h + A_l.B_h + A_h.B_l (3 x bf16).  Each product of bf16 values is
//     exact in fp32; what the split drops is ~3 * 2^-16 of |q_i x_i|, inside
//     the error bound the exact select works with (screen_gamma).
// M = 128 queries x N = 256 rows per tile, K = 16 per MMA, fp32 accumulators
// in TMEM (two 256-column buffers, so the epilogue of one tile overlaps the
// MMAs of the next).  The screen score bias (-||x||^2 for L2, 0 for inner
// product, -inf for rows past n) enters the accumulator through one more
// K = 16 MMA per tile against three bf16 parts of bias / alpha per row
// (split_bias in index.cu; the parts are exact and sum exactly in any order),
// so the accumulator holds score / alpha and the epilogue only compares.
//
// Work unit = (query tile, database chunk of whole tiles).  Persistent CTAs
// (one per SM) walk units chunk-major so that the CTAs running at the same
// time read the same database rows (L2 reuse).
//
// Warp roles: the epilogue warpgroups first (two in list mode, four in buffer
// mode; warpgroup g owns columns [g * kCols, (g + 1) * kCols) of each tile and,
// in list mode, its own top-KP per query row -- two lists per (query, chunk)),
// then the TMA producer warp, then the MMA warp (TMEM allocator, one issuing
// thread).  The query tile (all k-blocks, both planes for kX3) stays resident
// in shared memory for a unit when it fits in 64 KB; above, each ring stage
// carries the k-block's query plane with the database plane (kX3: a k-block's
// h and l stages are consumed as a pair).  Every mbarrier wait is bounded; a
// wait that runs out sets the CTA's abort flag, the warps drain what they
// issued, TMEM is freed and the error word records kErrTimeout.
#include "epilogue.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace mflat_cu {
namespace {

__host__ __device__ constexpr int epi_wg(bool buf) { return buf ? 4 : 2; }
__host__ __device__ constexpr int screen_threads(bool buf) { return epi_wg(buf) * 128 + 64; }
constexpr int kATile = kBM * 128;                 // 16 KB: 128 rows x 128 B (one plane, one k-block)
constexpr int kBTile = kBN * 128;                 // 32 KB: 256 rows x 128 B
constexpr int kMaxStages = 6;
constexpr int kAResidentMax = 64 * 1024;          // resident query tile budget
constexpr int kSmemMax = 232448;                  // opt-in shared memory per CTA
constexpr int kBarBytes = 256;                    // mbarriers, TMEM slot, abort flag
// Folded bias: slot s holds the bias parts of one tile, [256 rows][8 bf16]
// = (h, m, l, 0, ...); three slots, loaded one tile ahead (slot (t + 1) % 3
// last served tile t - 2, whose MMAs have completed once the MMA warp has
// seen tile t - 2's accumulator released).  The constant block holds 128
// rows of (1, 1, 1, 0, ...) -- the A operand's K columns 0..7 -- then 128
// zero rows -- its K columns 8..15.  B's K columns 8..15 read the whole
// constant block (finite values, multiplied by A's zeros).
constexpr int kFoldSlots = 3;
constexpr int kFoldSlotBytes = kBN * 16;          // 4 KB
constexpr int kConstBytes = 2 * kBM * 16;         // 4 KB: ones rows, then zero rows
constexpr int kFoldBytes = kFoldSlots * kFoldSlotBytes + kConstBytes;
constexpr uint32_t kOneBf16x2 = 0x3F803F80u;      // two bf16 1.0

__host__ __device__ inline int a_bytes(int kb, int planes) { return kb * planes * kATile; }
__host__ __device__ inline bool a_streamed(int kb, int planes) { return a_bytes(kb, planes) > kAResidentMax; }
__host__ __device__ inline int stage_bytes(bool streamed) { return streamed ? kATile + kBTile : kBTile; }
__host__ __device__ inline int n_stages(int kb, int planes) {
    const bool st = a_streamed(kb, planes);
    const int a = st ? 0 : a_bytes(kb, planes);
    int s = (kSmemMax - kBarBytes - kFoldBytes - a) / stage_bytes(st);
    if (s > kMaxStages) s = kMaxStages;
    if (st && planes == 2) s &= ~1;               // a k-block's h and l stages form a pair
    return s;
}
__host__ __device__ inline int smem_bytes(int kb, int planes) {
    const bool st = a_streamed(kb, planes);
    return (st ? 0 : a_bytes(kb, planes)) + n_stages(kb, planes) * stage_bytes(st) + kBarBytes + kFoldBytes;
}

struct Smem {
    uint8_t* a;          // resident A: [planes][kb][16 KB]
    uint8_t* ring;       // [stages][stage bytes]: ([A plane 16 KB]) [B plane 32 KB]
    uint64_t *full, *empty, *a_full, *a_empty, *acc_full, *acc_empty, *drain, *bias_full;
    uint32_t* tmem_slot;
    int* abort_flag;
    uint8_t* fold;       // [kFoldSlots][4 KB] bias parts, then the 4 KB constant block
};

__device__ inline Smem carve(uint8_t* base, int kb, int planes, int stages) {
    Smem S;
    const bool st = a_streamed(kb, planes);
    S.a = base;
    S.ring = base + (st ? 0 : a_bytes(kb, planes));
    uint64_t* bars = reinterpret_cast<uint64_t*>(S.ring + stages * stage_bytes(st));
    S.full = bars;
    S.empty = bars + kMaxStages;
    S.a_full = bars + 2 * kMaxStages;
    S.a_empty = S.a_full + 1;
    S.acc_full = S.a_full + 2;
    S.acc_empty = S.a_full + 4;
    S.drain = S.a_full + 6;
    S.bias_full = S.a_full + 7;
    S.tmem_slot = reinterpret_cast<uint32_t*>(S.bias_full + kFoldSlots);
    S.abort_flag = reinterpret_cast<int*>(S.tmem_slot + 1);
    S.fold = reinterpret_cast<uint8_t*>(bars) + kBarBytes;
    return S;
}

template <int KP, bool kBuf, bool kBF16, bool kX3>
__global__ void __launch_bounds__(screen_threads(kBuf), 1)
screen_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_a2,
              const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_b2,
              const __grid_constant__ CUtensorMap tm_bias, const ScreenParams p) {
    // SWIZZLE_128B tiles need 1024-byte aligned shared memory; the declared
    // alignment is checked, not assumed.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    constexpr int kPlanes = kX3 ? 2 : 1;
    const int kb_count = p.d_pad / kBK;
    if (kb_count < 1 || kb_count * kBK != p.d_pad || (smem_u32(smem_raw) & 1023u) != 0u) {
        if (threadIdx.x == 0) atomicExch(p.err, kErrConfig);
        return;
    }
    const bool stream_a = a_streamed(kb_count, kPlanes);
    const int sbytes = stage_bytes(stream_a);
    const int stages = n_stages(kb_count, kPlanes);
    Smem S = carve(smem_raw, kb_count, kPlanes, stages);
    constexpr uint32_t kIdesc = make_idesc(kBF16 ? 1u : 0u, kBM, kBN);
    constexpr uint32_t kIdescBias = make_idesc(1u, kBM, kBN);   // the bias step is bf16

    constexpr int kEpiWG = epi_wg(kBuf);
    constexpr int kProducerWarp = kEpiWG * 4;
    constexpr int kMmaWarp = kProducerWarp + 1;
    constexpr int kCols = kBN / kEpiWG;          // accumulator columns per warpgroup
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
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
    {
        // constant operand rows of the bias step, written once and made
        // visible to the tensor core's (async-proxy) reads
        uint4* cst = reinterpret_cast<uint4*>(S.fold + kFoldSlots * kFoldSlotBytes);
        for (int i = threadIdx.x; i < kConstBytes / 16; i += blockDim.x)
            cst[i] = i < kBM ? make_uint4(kOneBf16x2, kOneBf16x2 & 0xFFFFu, 0u, 0u)
                             : make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_shared();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(S.tmem_slot, 512);
        tmem_relinquish();
    }
    if (warp == kProducerWarp && lane == 0) {
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
        if constexpr (kX3) {
            tma_prefetch_desc(&tm_a2);
            tma_prefetch_desc(&tm_b2);
        }
        tma_prefetch_desc(&tm_bias);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *S.tmem_slot;
    volatile int* abort_flag = S.abort_flag;
    const int n_units = p.n_qtiles * p.n_chunks;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            int stage = 0;
            uint32_t sphase = 0, a_phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;   // per stage, for the drain
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
                    mbar_arrive_expect_tx(S.a_full, static_cast<uint32_t>(a_bytes(kb_count, kPlanes)));
                    for (int pl = 0; pl < kPlanes; ++pl)
                        for (int kb = 0; kb < kb_count; ++kb)
                            tma_load_2d(pl ? &tm_a2 : &tm_a, S.a_full, S.a + (pl * kb_count + kb) * kATile,
                                        kb * kBK, qt * kBM);
                    a_issued = true;
                    a_issue_phase = a_phase;
                    a_phase ^= 1u;
                }
                for (int t = t0; t < t1 && ok; ++t) {
                    for (int kb = 0; kb < kb_count && ok; ++kb) {
                        for (int pl = 0; pl < kPlanes; ++pl) {
                            if (!mbar_wait(&S.empty[stage], sphase ^ 1u, abort_flag, p.wait_ns)) { ok = false; break; }
                            uint8_t* dst = S.ring + stage * sbytes;
                            mbar_arrive_expect_tx(&S.full[stage], static_cast<uint32_t>(sbytes));
                            if (stream_a) {
                                tma_load_2d(pl ? &tm_a2 : &tm_a, &S.full[stage], dst, kb * kBK, qt * kBM);
                                dst += kATile;
                            }
                            tma_load_2d(pl ? &tm_b2 : &tm_b, &S.full[stage], dst, kb * kBK,
                                        t * p.tile_stride * kBN);
                            issued_mask |= 1u << stage;
                            issued_phase = (issued_phase & ~(1u << stage)) | (sphase << stage);
                            if (++stage == stages) { stage = 0; sphase ^= 1u; }
                        }
                    }
                }
            }
            if (*abort_flag) {
                // Drain: let every copy this thread issued land before exit.
                for (int s = 0; s < stages; ++s)
                    if (issued_mask & (1u << s))
                        mbar_wait_drain(&S.full[s], (issued_phase >> s) & 1u, 200000000ull);
                if (a_issued) mbar_wait_drain(S.a_full, a_issue_phase, 200000000ull);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            int stage = 0;
            uint32_t sphase = 0, a_phase = 0, tcount = 0;
            uint32_t bias_pending = 0, bias_phase = 0;   // bias copies issued (drain on abort)
            bool ok = true, issued_any = false;
            const uint32_t cst = smem_u32(S.fold + kFoldSlots * kFoldSlotBytes);
            // bias-step operand descriptors: K-major, no swizzle, 8-row x 16-byte
            // core matrices (SBO 128 B between row groups, LBO to the K columns 8..15)
            const uint64_t bias_a = smem_desc_k_none(cst, kConstBytes / 2, 128u);
            auto load_bias_parts = [&](uint32_t tc, int tile) {
                const uint32_t sl = tc % kFoldSlots;
                mbar_arrive_expect_tx(&S.bias_full[sl], kFoldSlotBytes);
                tma_load_2d(&tm_bias, &S.bias_full[sl], S.fold + sl * kFoldSlotBytes, 0,
                            tile * p.tile_stride * kBN);
                bias_pending |= 1u << sl;
                bias_phase = (bias_phase & ~(1u << sl)) | (((tc / kFoldSlots) & 1u) << sl);
            };
            // test hook: the drain barrier completes no phase before an abort,
            // so this bounded wait runs out and the CTA takes its error path
            if (p.test_stall) ok = mbar_wait(S.drain, 0u, abort_flag, p.wait_ns) && false;
            if (ok && static_cast<int>(blockIdx.x) < n_units)
                load_bias_parts(0, (blockIdx.x / p.n_qtiles) * p.tiles_per_chunk);
            for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
                const int ch = u / p.n_qtiles;
                const int t0 = ch * p.tiles_per_chunk;
                const int t1 = min(t0 + p.tiles_per_chunk, p.n_tiles);
                if (!stream_a) {
                    if (!mbar_wait(S.a_full, a_phase, abort_flag, p.wait_ns)) { ok = false; break; }
                    a_phase ^= 1u;
                    tc_fence_after();
                }
                const uint32_t a_addr = smem_u32(S.a);
                for (int t = t0; t < t1 && ok; ++t, ++tcount) {
                    const uint32_t b = tcount & 1u;
                    const uint32_t ph = (tcount >> 1) & 1u;
                    if (!mbar_wait(&S.acc_empty[b], ph ^ 1u, abort_flag, p.wait_ns)) { ok = false; break; }
                    tc_fence_after();
                    {
                        // the bias parts of the CTA's next tile: the rest of this
                        // unit, else the first tile of its next unit
                        int nt = -1;
                        if (t + 1 < t1) nt = t + 1;
                        else if (u + static_cast<int>(gridDim.x) < n_units)
                            nt = ((u + static_cast<int>(gridDim.x)) / p.n_qtiles) * p.tiles_per_chunk;
                        if (nt >= 0) load_bias_parts(tcount + 1, nt);
                    }
                    const uint32_t d_tmem = tmem_base + b * kBN;
                    if constexpr (!kX3) {
                        for (int kb = 0; kb < kb_count && ok; ++kb) {
                            if (!mbar_wait(&S.full[stage], sphase, abort_flag, p.wait_ns)) { ok = false; break; }
                            tc_fence_after();
                            const uint32_t st = smem_u32(S.ring + stage * sbytes);
                            const uint64_t ad = smem_desc_k_sw128(stream_a ? st : a_addr + kb * kATile);
                            const uint64_t bd = smem_desc_k_sw128(stream_a ? st + kATile : st);
#pragma unroll
                            for (int ks = 0; ks < kBK / 16; ++ks) {
                                const uint64_t o = static_cast<uint64_t>(ks * 2);   // 32 B >> 4
                                tc_mma_f16(d_tmem, ad + o, bd + o, kIdesc, (kb | ks) != 0 ? 1u : 0u);
                            }
                            issued_any = true;
                            tc_commit(&S.empty[stage]);
                            if (++stage == stages) { stage = 0; sphase ^= 1u; }
                        }
                    } else if (!stream_a) {
                        for (int kb = 0; kb < kb_count && ok; ++kb) {
                            const uint64_t a_h = smem_desc_k_sw128(a_addr + kb * kATile);
                            const uint64_t a_l = smem_desc_k_sw128(a_addr + (kb_count + kb) * kATile);
                            // stage holding B_h of this k-block
                            if (!mbar_wait(&S.full[stage], sphase, abort_flag, p.wait_ns)) { ok = false; break; }
                            tc_fence_after();
                            uint64_t bd = smem_desc_k_sw128(smem_u32(S.ring + stage * sbytes));
#pragma unroll
                            for (int ks = 0; ks < kBK / 16; ++ks) {
                                const uint64_t o = static_cast<uint64_t>(ks * 2);
                                tc_mma_f16(d_tmem, a_h + o, bd + o, kIdesc, (kb | ks) != 0 ? 1u : 0u);
                                tc_mma_f16(d_tmem, a_l + o, bd + o, kIdesc, 1u);
                            }
                            issued_any = true;
                            tc_commit(&S.empty[stage]);
                            if (++stage == stages) { stage = 0; sphase ^= 1u; }
                            // stage holding B_l of this k-block
                            if (!mbar_wait(&S.full[stage], sphase, abort_flag, p.wait_ns)) { ok = false; break; }
                            tc_fence_after();
                            bd = smem_desc_k_sw128(smem_u32(S.ring + stage * sbytes));
#pragma unroll
                            for (int ks = 0; ks < kBK / 16; ++ks) {
                                const uint64_t o = static_cast<uint64_t>(ks * 2);
                                tc_mma_f16(d_tmem, a_h + o, bd + o, kIdesc, 1u);
                            }
                            tc_commit(&S.empty[stage]);
                            if (++stage == stages) { stage = 0; sphase ^= 1u; }
                        }
                    } else {
                        for (int kb = 0; kb < kb_count && ok; ++kb) {
                            // the k-block's h stage [A_h | B_h] and l stage [A_l | B_l]
                            const int s_h = stage;
                            const uint32_t ph_h = sphase;
                            if (++stage == stages) { stage = 0; sphase ^= 1u; }
                            const int s_l = stage;
                            const uint32_t ph_l = sphase;
                            if (++stage == stages) { stage = 0; sphase ^= 1u; }
                            if (!mbar_wait(&S.full[s_h], ph_h, abort_flag, p.wait_ns) ||
                                !mbar_wait(&S.full[s_l], ph_l, abort_flag, p.wait_ns)) { ok = false; break; }
                            tc_fence_after();
                            const uint32_t base_h = smem_u32(S.ring + s_h * sbytes);
                            const uint32_t base_l = smem_u32(S.ring + s_l * sbytes);
                            const uint64_t a_h = smem_desc_k_sw128(base_h);
                            const uint64_t b_h = smem_desc_k_sw128(base_h + kATile);
                            const uint64_t a_l = smem_desc_k_sw128(base_l);
                            const uint64_t b_l = smem_desc_k_sw128(base_l + kATile);
#pragma unroll
                            for (int ks = 0; ks < kBK / 16; ++ks) {
                                const uint64_t o = static_cast<uint64_t>(ks * 2);
                                tc_mma_f16(d_tmem, a_h + o, b_h + o, kIdesc, (kb | ks) != 0 ? 1u : 0u);
                                tc_mma_f16(d_tmem, a_l + o, b_h + o, kIdesc, 1u);
                                tc_mma_f16(d_tmem, a_h + o, b_l + o, kIdesc, 1u);
                            }
                            issued_any = true;
                            tc_commit(&S.empty[s_h]);
                            tc_commit(&S.empty[s_l]);
                        }
                    }
                    if (ok) {
                        // bias step: acc += (1, 1, 1, 0 ...) . (h, m, l, 0 ...) per row
                        const uint32_t sl = tcount % kFoldSlots;
                        if (!mbar_wait(&S.bias_full[sl], (tcount / kFoldSlots) & 1u, abort_flag, p.wait_ns)) {
                            ok = false;
                        } else {
                            bias_pending &= ~(1u << sl);
                            tc_fence_after();
                            const uint32_t bslot = smem_u32(S.fold + sl * kFoldSlotBytes);
                            tc_mma_f16(d_tmem, bias_a, smem_desc_k_none(bslot, cst - bslot, 128u), kIdescBias, 1u);
                            tc_commit(&S.acc_full[b]);
                        }
                    }
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
        // ---------------- epilogue: warpgroup g owns columns [g*kCols, (g+1)*kCols)
        const int g = warp >> 2;
        const int wq = warp & 3;
        const int row_in_tile = wq * 32 + lane;
        const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(wq * 32) << 16);
        // the accumulator holds score / alpha (alpha = 2 for L2, 1 otherwise,
        // an exact power of two): compare against floor / alpha, store * alpha
        const float alpha = p.alpha;
        const float inv_alpha = 1.0f / alpha;
        // Accumulator b goes back to the MMA warp as soon as the warp's last
        // tcgen05.ld of the tile has completed, before that data is scored.
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
                // one lane polls the barrier, the warp follows
                bool ready = true;
                if (lane == 0) ready = mbar_wait(&S.acc_full[b], ph, abort_flag, p.wait_ns);
                if (!__shfl_sync(0xffffffffu, ready ? 1 : 0, 0)) { ok = false; break; }
                const float floor_adj =
                    !live ? __int_as_float(0x7f800000)
                          : (p.use_floor ? floor_below(fkey) * inv_alpha : -__int_as_float(0x7f800000));
                const int id_tile = t * p.tile_stride * kBN + g * kCols;
                const uint32_t taddr = lane_addr + b * kBN + g * kCols;
                uint32_t ra[32], rb[32];
                __syncwarp();
                tc_fence_after();
                if constexpr (kBuf) {
                    // buffer mode, 4 warps per SMSP, 64 columns per warp: both
                    // loads in flight together, one wait
                    static_assert(kCols == 64, "buffer mode: four warpgroups of 64 columns");
                    tmem_ld_32x32b_x32(taddr, ra);
                    tmem_ld_32x32b_x32(taddr + 32, rb);
                    tmem_wait_ld_regs(ra);
                    tmem_wait_ld_regs(rb);
                    release_acc(b);
                    buffer_chunk_raw(ra, floor_adj, alpha, br, st, id_tile);
                    buffer_chunk_raw(rb, floor_adj, alpha, br, st, id_tile + 32);
                } else {
                    // list mode, 2 warps per SMSP: the next chunk's TMEM load is
                    // in flight while a chunk is scored
                    tmem_ld_32x32b_x32(taddr, ra);
#pragma unroll 1
                    for (int c = 0; c < kCols / 32; c += 2) {
                        tmem_wait_ld_regs(ra);
                        __syncwarp();
                        tmem_ld_32x32b_x32(taddr + (c + 1) * 32, rb);
                        scan_chunk_raw<KP>(ra, floor_adj, L, id_tile + c * 32);
                        tmem_wait_ld_regs(rb);
                        if (c + 2 < kCols / 32) {
                            __syncwarp();
                            tmem_ld_32x32b_x32(taddr + (c + 2) * 32, ra);
                        } else {
                            release_acc(b);
                        }
                        scan_chunk_raw<KP>(rb, floor_adj, L, id_tile + (c + 1) * 32);
                    }
                }
            }
            if constexpr (kBuf) st.flush(br);   // the unit's staged appends
            if (!ok) break;
            if (!kBuf && live) {
                const int64_t o = (static_cast<int64_t>(ch * kEpiWG + g) * p.m_pad + row) * KP;
                float4* ps = reinterpret_cast<float4*>(p.part_score + o);
                int4* pi = reinterpret_cast<int4*>(p.part_id + o);
#pragma unroll
                for (int i = 0; i < KP / 4; ++i) {
                    ps[i] = make_float4(alpha * L.s[4 * i], alpha * L.s[4 * i + 1], alpha * L.s[4 * i + 2],
                                        alpha * L.s[4 * i + 3]);
                    pi[i] = make_int4(L.id[4 * i], L.id[4 * i + 1], L.id[4 * i + 2], L.id[4 * i + 3]);
                }
                // A full list's KP-th score is a lower bound of the query's
                // global KP-th best: no row below it can matter any more.
                if (p.use_floor && L.id[KP - 1] >= 0)
                    atomicMax(p.thr + row, score_key(alpha * L.s[KP - 1]));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc(tmem_base, 512);
    if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, *abort_flag);
}

template <int KP, bool kBuf, bool kBF16, bool kX3>
cudaError_t launch_one(const ScreenMaps& m, const ScreenParams& p, int grid, cudaStream_t stream) {
    const int smem = smem_bytes(p.d_pad / kBK, kX3 ? 2 : 1);
    cudaError_t e = cudaFuncSetAttribute(screen_kernel<KP, kBuf, kBF16, kX3>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    screen_kernel<KP, kBuf, kBF16, kX3><<<grid, screen_threads(kBuf), smem, stream>>>(
        m.a, kX3 ? m.a2 : m.a, m.b, kX3 ? m.b2 : m.b, m.bias, p);
    return cudaGetLastError();
}

template <bool kBF16, bool kX3>
cudaError_t launch_kind(int kp, const ScreenMaps& m, const ScreenParams& p, int grid, cudaStream_t stream) {
    switch (kp) {
        case 0: return launch_one<4, true, kBF16, kX3>(m, p, grid, stream);
        case 4: return launch_one<4, false, kBF16, kX3>(m, p, grid, stream);
        case 8: return launch_one<8, false, kBF16, kX3>(m, p, grid, stream);
        case 16: return launch_one<16, false, kBF16, kX3>(m, p, grid, stream);
        case 32: return launch_one<32, false, kBF16, kX3>(m, p, grid, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

int screen_smem_bytes(int d_pad, bool x3) { return smem_bytes(d_pad / kBK, x3 ? 2 : 1); }

cudaError_t launch_screen(int kp, ScreenKind kind, const ScreenMaps& maps, const ScreenParams& p,
                          int grid, cudaStream_t stream) {
    if (p.d_pad % kBK != 0 || p.d_pad < kBK || !(p.alpha == 1.0f || p.alpha == 2.0f))
        return cudaErrorInvalidValue;
    switch (kind) {
        case ScreenKind::kF16: return launch_kind<false, false>(kp, maps, p, grid, stream);
        case ScreenKind::kBF16: return launch_kind<true, false>(kp, maps, p, grid, stream);
        case ScreenKind::kBF16x3: return launch_kind<true, true>(kp, maps, p, grid, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace mflat_cu
