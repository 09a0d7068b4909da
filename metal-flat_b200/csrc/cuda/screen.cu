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
// Per CTA a tile is 128 queries x 256 rows, K = 16 per MMA, fp32 accumulators
// in TMEM (two 256-column buffers, so the epilogue of one tile overlaps the
// MMAs of the next).  The screen score bias (-||x||^2 for L2, 0 for inner
// product, -inf for rows past n) enters the accumulator through one more
// K = 16 MMA per tile against three bf16 parts of bias / alpha per row
// (split_bias in index.cu; the parts are exact and sum exactly in any order),
// so the accumulator holds score / alpha and the epilogue only compares.
// The bias parts travel in the tile's last ring stage.
//
// CTA pairs (kPair): the two CTAs of a cluster issue their MMAs as one
// tcgen05 cta_group::2 instruction (M = 256: CTA r holds query tile 2j + r
// and rows [r * 128, r * 128 + 128) of each 256-row database tile; each CTA's
// TMEM receives its 128 queries x all 256 columns).  Each SM then loads and
// holds half of every database tile, which halves the per-SM L2 -> shared
// memory traffic and doubles the tiles the ring holds in flight.  The
// leader CTA (rank 0) owns the full / a_full / acc_empty
// barriers and the one MMA-issuing thread; both CTAs' TMA loads complete on
// the leader's barriers (cta_group::2 loads, no multicast), MMA completion is
// committed to the barriers of both CTAs, and the peer's epilogue warps
// release accumulators on the leader's barrier.
//
// Work unit = (query tile (pair), database chunk of whole tiles).  Persistent
// CTAs (pairs) walk units chunk-major so that the CTAs running at the same
// time read the same database rows (L2 reuse).  Warp roles: the epilogue
// warpgroups first (two in list mode, each owning 128 of a tile's 256 columns
// and its own top-KP per query row -- two lists per (query, chunk); four in
// buffer mode, 64 columns each), then the TMA producer warp, then the MMA warp
// (TMEM allocator, one issuing thread).  The query tile stays resident in
// shared memory for a unit when it fits in 64 KB; above, each ring stage
// carries the k-block's query planes with its database planes.  Every mbarrier wait is
// bounded; a wait that runs out sets the CTA's abort flag, the warps drain
// what they issued, TMEM is freed and the error word records kErrTimeout.
//
// Ring stages: a stage holds kps k-blocks (two where that still leaves three
// stages, else one), each with all its planes ([query plane when streamed]
// [database plane]), and room for the tile's bias parts, which the tile's last
// stage carries.  A 16-bit d = 128 pair tile is then one stage: one full wait
// and one release per tile besides the accumulator hand-off.
#include "epilogue.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace mflat_cu {
namespace {

__host__ __device__ constexpr int epi_wg(bool buf) { return buf ? 4 : 2; }
__host__ __device__ constexpr int screen_threads(bool buf) { return epi_wg(buf) * 128 + 64; }
constexpr int kATile = kBM * 128;                 // 16 KB: 128 rows x 128 B (one plane, one k-block)
constexpr int kAResidentMax = 64 * 1024;          // resident query tile budget
constexpr int kSmemMax = 232448;                  // opt-in shared memory per CTA
constexpr int kBarBytes = 512;                    // mbarriers, TMEM slot, abort flag
constexpr int kMaxStagesAll = 12;                 // barrier slots of the ring
// Bias step operands: the bias parts of the CTA's rows of a tile, [rows][8]
// bf16 = (h, m, l, 0, ...), sit at the end of the tile's last stage.  The
// constant block holds 128 rows of (1, 1, 1, 0, ...) -- the A operand's K
// columns 0..7 -- then 128 zero rows -- its K columns 8..15.  B's K columns
// 8..15 read the constant block (finite values, multiplied by A's zeros).
constexpr int kConstBytes = 2 * kBM * 16;         // 4 KB: ones rows, then zero rows
constexpr uint32_t kOneBf16x2 = 0x3F803F80u;      // two bf16 1.0

// Per-CTA geometry of one mode.
struct Geo {
    int rows_b;          // database rows of a tile this CTA holds (256, or 128 in a pair)
    int b_tile;          // bytes of one B plane k-block
    int slot;            // bytes of the tile's bias parts
};
__host__ __device__ constexpr Geo geo(bool pair) {
    return pair ? Geo{kBN / 2, (kBN / 2) * 128, (kBN / 2) * 16} : Geo{kBN, kBN * 128, kBN * 16};
}

__host__ __device__ inline int a_bytes(int kb, int planes) { return kb * planes * kATile; }
__host__ __device__ inline bool a_streamed(int kb, int planes) { return a_bytes(kb, planes) > kAResidentMax; }
// one k-block, all planes: ([A plane]) [B plane] per plane
__host__ __device__ inline int kblock_bytes(bool streamed, int planes, bool pair) {
    return planes * ((streamed ? kATile : 0) + geo(pair).b_tile);
}
__host__ __device__ inline int stage_bytes(int kps, bool streamed, int planes, bool pair) {
    return kps * kblock_bytes(streamed, planes, pair) + geo(pair).slot;
}
__host__ __device__ inline int stages_for(int kps, int kb, int planes, bool pair) {
    const bool st = a_streamed(kb, planes);
    const int a = st ? 0 : a_bytes(kb, planes);
    const int s = (kSmemMax - kBarBytes - kConstBytes - a) / stage_bytes(kps, st, planes, pair);
    return s < kMaxStagesAll ? s : kMaxStagesAll;
}
// k-blocks per stage: two where that still leaves three stages, else one
__host__ __device__ inline int kblocks_per_stage(int kb, int planes, bool pair) {
    return (kb % 2 == 0 && stages_for(2, kb, planes, pair) >= 3) ? 2 : 1;
}
__host__ __device__ inline int smem_bytes(int kb, int planes, bool pair) {
    const bool st = a_streamed(kb, planes);
    const int kps = kblocks_per_stage(kb, planes, pair);
    return (st ? 0 : a_bytes(kb, planes)) + stages_for(kps, kb, planes, pair) * stage_bytes(kps, st, planes, pair) +
           kBarBytes + kConstBytes;
}

struct Smem {
    uint8_t* a;          // resident A: [planes][kb][16 KB]
    uint8_t* ring;       // [stages][stage bytes]
    uint64_t *full, *empty, *a_full, *a_empty, *acc_full, *acc_empty, *drain;
    uint32_t* tmem_slot;
    int* abort_flag;
    uint8_t* cst;        // the 4 KB constant block of the bias step
};

__device__ inline Smem carve(uint8_t* base, int kb, int planes, int stages, int sbytes) {
    Smem S;
    const bool st = a_streamed(kb, planes);
    S.a = base;
    S.ring = base + (st ? 0 : a_bytes(kb, planes));
    uint64_t* bars = reinterpret_cast<uint64_t*>(S.ring + stages * sbytes);
    S.full = bars;
    S.empty = bars + kMaxStagesAll;
    S.a_full = bars + 2 * kMaxStagesAll;
    S.a_empty = S.a_full + 1;
    S.acc_full = S.a_full + 2;
    S.acc_empty = S.a_full + 4;
    S.drain = S.a_full + 6;
    S.tmem_slot = reinterpret_cast<uint32_t*>(S.drain + 1);
    S.abort_flag = reinterpret_cast<int*>(S.tmem_slot + 1);
    S.cst = reinterpret_cast<uint8_t*>(bars) + kBarBytes;
    return S;
}

template <int KP, bool kBuf, bool kBF16, bool kX3, bool kPair>
__global__ void __launch_bounds__(screen_threads(kBuf), 1)
screen_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_a2,
              const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_b2,
              const __grid_constant__ CUtensorMap tm_bias, const ScreenParams p) {
    // SWIZZLE_128B tiles need 1024-byte aligned shared memory; the declared
    // alignment is checked, not assumed.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    constexpr int kPlanes = kX3 ? 2 : 1;
    constexpr Geo G = geo(kPair);
    constexpr uint16_t kBoth = 0x3;              // CTA mask of a pair
    const int kb_count = p.d_pad / kBK;
    // identical in both CTAs of a pair, so both leave together
    if (kb_count < 1 || kb_count * kBK != p.d_pad || (smem_u32(smem_raw) & 1023u) != 0u) {
        if (threadIdx.x == 0) atomicExch(p.err, kErrConfig);
        return;
    }
    const uint32_t crank = kPair ? cluster_rank() : 0u;
    const bool leader = crank == 0;
    const bool stream_a = a_streamed(kb_count, kPlanes);
    const int kps = kblocks_per_stage(kb_count, kPlanes, kPair);
    const int kbb = kblock_bytes(stream_a, kPlanes, kPair);
    const int sbytes = stage_bytes(kps, stream_a, kPlanes, kPair);
    const int stages = stages_for(kps, kb_count, kPlanes, kPair);
    Smem S = carve(smem_raw, kb_count, kPlanes, stages, sbytes);
    constexpr uint32_t kM = kPair ? 2 * kBM : kBM;
    constexpr uint32_t kIdesc = make_idesc(kBF16 ? 1u : 0u, kM, kBN);
    constexpr uint32_t kIdescBias = make_idesc(1u, kM, kBN);   // the bias step is bf16

    constexpr int kEpiWG = epi_wg(kBuf);
    constexpr int kProducerWarp = kEpiWG * 4;
    constexpr int kMmaWarp = kProducerWarp + 1;
    constexpr int kCols = kBN / kEpiWG;          // accumulator columns per warpgroup
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxStagesAll; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        mbar_init(S.a_full, 1);
        mbar_init(S.a_empty, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.acc_full[b], 1);
            // one arrival per epilogue warp (of both CTAs of a pair)
            mbar_init(&S.acc_empty[b], kEpiWG * 4 * (kPair ? 2 : 1));
        }
        mbar_init(S.drain, 1);
        *S.abort_flag = 0;
        fence_mbar_init();
    }
    {
        // constant operand rows of the bias step, written once and made
        // visible to the tensor core's (async-proxy) reads
        uint4* cst = reinterpret_cast<uint4*>(S.cst);
        for (int i = threadIdx.x; i < kConstBytes / 16; i += blockDim.x)
            cst[i] = i < kBM ? make_uint4(kOneBf16x2, kOneBf16x2 & 0xFFFFu, 0u, 0u)
                             : make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_shared();
    }
    if (warp == kMmaWarp) {
        if constexpr (kPair) {
            tmem_alloc_pair(S.tmem_slot, 512);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(S.tmem_slot, 512);
            tmem_relinquish();
        }
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
    if constexpr (kPair) cluster_sync();         // barriers of both CTAs initialised
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *S.tmem_slot;
    volatile int* abort_flag = S.abort_flag;
    // query units: tiles, or pairs of tiles (the peer's tile may lie past m_pad:
    // its TMA rows then read as zero and none of its rows is live)
    const int n_qunits = kPair ? (p.n_qtiles + 1) / 2 : p.n_qtiles;
    const int n_units = n_qunits * p.n_chunks;
    const int unit0 = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
    const int unit_step = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

    if (warp == kProducerWarp) {
        if (lane == 0) {
            int stage = 0;
            uint32_t sphase = 0, a_phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;   // per stage, for the drain
            bool a_issued = false, any_issued = false;
            uint32_t a_issue_phase = 0;
            bool ok = true;
            // barrier the loads complete on: the leader's (pair) or this CTA's
            auto bar_of = [&](uint64_t* bar) -> uint32_t {
                if constexpr (kPair) return cluster_addr(bar, 0);
                else return smem_u32(bar);
            };
            auto load = [&](const CUtensorMap* map, uint64_t* bar, void* dst, int x, int y) {
                if constexpr (kPair) tma_load_2d_pair(map, bar_of(bar), dst, x, y);
                else tma_load_2d(map, bar, dst, x, y);
            };
            constexpr uint32_t kShare = kPair ? 2u : 1u;   // the leader expects both CTAs' bytes
            for (int u = unit0; u < n_units && ok; u += unit_step) {
                const int qt = (u % n_qunits) * (kPair ? 2 : 1) + static_cast<int>(crank);
                const int ch = u / n_qunits;
                const int t0 = ch * p.tiles_per_chunk;
                const int t1 = min(t0 + p.tiles_per_chunk, p.n_tiles);
                if (!stream_a) {
                    if (!mbar_wait(S.a_empty, a_phase ^ 1u, abort_flag, p.wait_ns)) { ok = false; break; }
                    if (leader)
                        mbar_arrive_expect_tx(S.a_full, kShare * static_cast<uint32_t>(a_bytes(kb_count, kPlanes)));
                    for (int pl = 0; pl < kPlanes; ++pl)
                        for (int kb = 0; kb < kb_count; ++kb)
                            load(pl ? &tm_a2 : &tm_a, S.a_full, S.a + (pl * kb_count + kb) * kATile, kb * kBK,
                                 qt * kBM);
                    a_issued = any_issued = true;
                    a_issue_phase = a_phase;
                    a_phase ^= 1u;
                }
                for (int t = t0; t < t1 && ok; ++t) {
                    const int row0 = t * p.tile_stride * kBN + static_cast<int>(crank) * G.rows_b;
                    for (int kb0 = 0; kb0 < kb_count && ok; kb0 += kps) {
                        if (!mbar_wait(&S.empty[stage], sphase ^ 1u, abort_flag, p.wait_ns)) { ok = false; break; }
                        const bool last = kb0 + kps >= kb_count;
                        uint8_t* base = S.ring + stage * sbytes;
                        if (leader)
                            mbar_arrive_expect_tx(&S.full[stage],
                                                  kShare * static_cast<uint32_t>(kps * kbb + (last ? G.slot : 0)));
                        uint8_t* dst = base;
                        for (int j = 0; j < kps; ++j) {
                            const int kb = kb0 + j;
                            for (int pl = 0; pl < kPlanes; ++pl) {
                                if (stream_a) {
                                    load(pl ? &tm_a2 : &tm_a, &S.full[stage], dst, kb * kBK, qt * kBM);
                                    dst += kATile;
                                }
                                load(pl ? &tm_b2 : &tm_b, &S.full[stage], dst, kb * kBK, row0);
                                dst += G.b_tile;
                            }
                        }
                        // the tile's bias parts travel with its last stage
                        if (last) load(&tm_bias, &S.full[stage], base + kps * kbb, 0, row0);
                        issued_mask |= 1u << stage;
                        issued_phase = (issued_phase & ~(1u << stage)) | (sphase << stage);
                        any_issued = true;
                        if (++stage == stages) { stage = 0; sphase ^= 1u; }
                    }
                }
            }
            if (ok && !*abort_flag) {
                // Tail: wait until the MMAs have released every stage and query
                // tile this warp filled, so that no commit (multicast in a pair)
                // is still on its way to this CTA's barriers at exit.
                for (int i = 0; i < stages && ok; ++i) {
                    ok = mbar_wait(&S.empty[stage], sphase ^ 1u, abort_flag, p.wait_ns);
                    if (++stage == stages) { stage = 0; sphase ^= 1u; }
                }
                if (ok && !stream_a) ok = mbar_wait(S.a_empty, a_phase ^ 1u, abort_flag, p.wait_ns);
            }
            if (*abort_flag) {
                if (leader) {
                    // Drain: every copy issued into the full barriers (both CTAs'
                    // bytes, in a pair) lands before exit.
                    for (int s = 0; s < stages; ++s)
                        if (issued_mask & (1u << s))
                            mbar_wait_drain(&S.full[s], (issued_phase >> s) & 1u, 200000000ull);
                    if (a_issued) mbar_wait_drain(S.a_full, a_issue_phase, 200000000ull);
                } else if (any_issued) {
                    // the peer's copies complete on the leader's barriers: give them
                    // time to land in this CTA's shared memory before it exits
                    const uint64_t t0 = globaltimer_ns();
                    while (globaltimer_ns() - t0 < 200000ull) {
                    }
                }
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0 && leader) {
            int stage = 0;
            uint32_t sphase = 0, a_phase = 0, tcount = 0;
            bool ok = true, issued_any = false;
            const uint32_t cst = smem_u32(S.cst);
            // bias-step operand descriptors: K-major, no swizzle, 8-row x 16-byte
            // core matrices (SBO 128 B between row groups, LBO to the K columns 8..15)
            const uint64_t bias_a = smem_desc_k_none(cst, kConstBytes / 2, 128u);
            auto mma = [&](uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
                if constexpr (kPair) tc_mma_f16_pair(d, a, b, idesc, acc);
                else tc_mma_f16(d, a, b, idesc, acc);
            };
            // every tcgen05 op of a kernel uses one cta_group: pair commits
            // (multicast to both CTAs' barriers) in pair mode
            auto commit = [&](uint64_t* bar) {
                if constexpr (kPair) tc_commit_pair(bar, kBoth);
                else tc_commit(bar);
            };
            // test hook: the drain barrier completes no phase before an abort,
            // so this bounded wait runs out and the CTA takes its error path
            if (p.test_stall) ok = mbar_wait(S.drain, 0u, abort_flag, p.wait_ns) && false;
            const uint32_t a_addr = smem_u32(S.a);
            for (int u = unit0; u < n_units && ok; u += unit_step) {
                const int ch = u / n_qunits;
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
                    const uint32_t d_tmem = tmem_base + b * kBN;
                    for (int kb0 = 0; kb0 < kb_count && ok; kb0 += kps) {
                        if (!mbar_wait(&S.full[stage], sphase, abort_flag, p.wait_ns)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t base = smem_u32(S.ring + stage * sbytes);
                        for (int j = 0; j < kps; ++j) {
                            const int kb = kb0 + j;
                            const uint32_t blk = base + j * kbb;
                            // this k-block's operands: A from the stage (streamed) or the
                            // resident tile; B planes from the stage
                            uint32_t ah, bh, al = 0, bl = 0;
                            if (stream_a) {
                                ah = blk;
                                bh = blk + kATile;
                                if constexpr (kX3) {
                                    al = blk + kATile + G.b_tile;
                                    bl = al + kATile;
                                }
                            } else {
                                ah = a_addr + kb * kATile;
                                bh = blk;
                                if constexpr (kX3) {
                                    al = a_addr + (kb_count + kb) * kATile;
                                    bl = blk + G.b_tile;
                                }
                            }
                            const uint64_t a_h = smem_desc_k_sw128(ah), b_h = smem_desc_k_sw128(bh);
                            const uint64_t a_l = kX3 ? smem_desc_k_sw128(al) : 0ull;
                            const uint64_t b_l = kX3 ? smem_desc_k_sw128(bl) : 0ull;
#pragma unroll
                            for (int ks = 0; ks < kBK / 16; ++ks) {
                                const uint64_t o = static_cast<uint64_t>(ks * 2);   // 32 B >> 4
                                mma(d_tmem, a_h + o, b_h + o, kIdesc, (kb | ks) != 0 ? 1u : 0u);
                                if constexpr (kX3) {
                                    mma(d_tmem, a_l + o, b_h + o, kIdesc, 1u);
                                    mma(d_tmem, a_h + o, b_l + o, kIdesc, 1u);
                                }
                            }
                        }
                        issued_any = true;
                        if (kb0 + kps >= kb_count) {
                            // bias step: acc += (1, 1, 1, 0 ...) . (h, m, l, 0 ...) per row
                            const uint32_t bslot = base + kps * kbb;
                            mma(d_tmem, bias_a, smem_desc_k_none(bslot, cst - bslot, 128u), kIdescBias, 1u);
                        }
                        commit(&S.empty[stage]);
                        if (++stage == stages) { stage = 0; sphase ^= 1u; }
                    }
                    if (ok) commit(&S.acc_full[b]);
                }
                if (ok && !stream_a) commit(S.a_empty);
            }
            if (*abort_flag && issued_any) {
                commit(S.drain);
                mbar_wait_drain(S.drain, 0u, 200000000ull);
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
        // Accumulator b goes back to the MMA thread as soon as the warp's last
        // tcgen05.ld of the tile has completed, before that data is scored.
        auto release_acc = [&](uint32_t b) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (kPair) mbar_arrive_cluster(cluster_addr(&S.acc_empty[b], 0));
                else mbar_arrive(&S.acc_empty[b]);
            }
        };
        uint32_t tcount = 0;
        bool ok = true;
        for (int u = unit0; u < n_units && ok; u += unit_step) {
            const int qt = (u % n_qunits) * (kPair ? 2 : 1) + static_cast<int>(crank);
            const int ch = u / n_qunits;
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
                    // list mode, 2 warps per SMSP, 128 columns per warp: two
                    // chunks' TMEM loads in flight together and one wait per
                    // pair (a TMEM load's round trip is several hundred cycles,
                    // more than scoring a chunk takes)
#pragma unroll 1
                    for (int c = 0; c < kCols / 32; c += 2) {
                        if (c > 0) __syncwarp();
                        tmem_ld_32x32b_x32(taddr + c * 32, ra);
                        tmem_ld_32x32b_x32(taddr + (c + 1) * 32, rb);
                        tmem_wait_ld_regs(ra);
                        tmem_wait_ld_regs(rb);
                        if (c + 2 >= kCols / 32) release_acc(b);
                        scan_chunk_raw<KP>(ra, floor_adj, L, id_tile + c * 32);
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

    __syncwarp();
    tc_fence_before();
    if constexpr (kPair) cluster_sync();         // no CTA leaves while its peer may still use it
    else __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) {
        if constexpr (kPair) tmem_dealloc_pair(tmem_base, 512);
        else tmem_dealloc(tmem_base, 512);
    }
    if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, *abort_flag);
}

template <int KP, bool kBuf, bool kBF16, bool kX3, bool kPair>
cudaError_t launch_one(const ScreenMaps& m, const ScreenParams& p, int grid, cudaStream_t stream) {
    auto kernel = screen_kernel<KP, kBuf, kBF16, kX3, kPair>;
    const int smem = smem_bytes(p.d_pad / kBK, kX3 ? 2 : 1, kPair);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const CUtensorMap& a2 = kX3 ? m.a2 : m.a;
    const CUtensorMap& b2 = kX3 ? m.b2 : m.b;
    if constexpr (!kPair) {
        kernel<<<grid, screen_threads(kBuf), smem, stream>>>(m.a, a2, m.b, b2, m.bias, p);
        return cudaGetLastError();
    } else {
        cudaLaunchConfig_t cfg{};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
        cfg.blockDim = dim3(screen_threads(kBuf), 1, 1);
        cfg.dynamicSmemBytes = static_cast<size_t>(smem);
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kernel, m.a, a2, m.b, b2, m.bias, p);
    }
}

template <bool kBF16, bool kX3, bool kPair>
cudaError_t launch_kind(int kp, const ScreenMaps& m, const ScreenParams& p, int grid, cudaStream_t stream) {
    switch (kp) {
        case 0: return launch_one<4, true, kBF16, kX3, kPair>(m, p, grid, stream);
        case 4: return launch_one<4, false, kBF16, kX3, kPair>(m, p, grid, stream);
        case 8: return launch_one<8, false, kBF16, kX3, kPair>(m, p, grid, stream);
        case 16: return launch_one<16, false, kBF16, kX3, kPair>(m, p, grid, stream);
        case 32: return launch_one<32, false, kBF16, kX3, kPair>(m, p, grid, stream);
        default: return cudaErrorInvalidValue;
    }
}

template <bool kPair>
cudaError_t launch_mode(int kp, ScreenKind kind, const ScreenMaps& maps, const ScreenParams& p,
                        int grid, cudaStream_t stream) {
    switch (kind) {
        case ScreenKind::kF16: return launch_kind<false, false, kPair>(kp, maps, p, grid, stream);
        case ScreenKind::kBF16: return launch_kind<true, false, kPair>(kp, maps, p, grid, stream);
        case ScreenKind::kBF16x3: return launch_kind<true, true, kPair>(kp, maps, p, grid, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

int screen_smem_bytes(int d_pad, bool x3, bool pair) { return smem_bytes(d_pad / kBK, x3 ? 2 : 1, pair); }

int screen_rows_per_cta(bool pair) { return geo(pair).rows_b; }

cudaError_t launch_screen(int kp, ScreenKind kind, const ScreenMaps& maps, const ScreenParams& p,
                          int grid, bool pair, cudaStream_t stream) {
    if (p.d_pad % kBK != 0 || p.d_pad < kBK || !(p.alpha == 1.0f || p.alpha == 2.0f))
        return cudaErrorInvalidValue;
    if (pair) {
        if (grid < 2 || (grid & 1)) return cudaErrorInvalidValue;
        return launch_mode<true>(kp, kind, maps, p, grid, stream);
    }
    return launch_mode<false>(kp, kind, maps, p, grid, stream);
}

}  // namespace mflat_cu
