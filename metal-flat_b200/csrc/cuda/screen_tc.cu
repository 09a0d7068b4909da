// screen_tc.cu -- tcgen05 distance GEMM with the top-k selection fused into
// its epilogue (the B200 replacement of the reference's per-tile pair
// GemmDistance::encode + topk_merge, src/GemmDistance.mm:15-60 and
// src/FlatIndex.mm:63-107, which round-tripped an m x tileW score matrix
// through device memory; here no score matrix is ever written).
//
// fp32 storage: each operand is held as two bf16 planes, x ~ h + l with
// h = bf16(x) and l = bf16(x - h); the kernel accumulates
// A_h.B_h + A_l.B_h + A_h.B_l (3 x bf16, kind::f16 at twice the kind::tf32
// rate) in a TMEM fp32 accumulator.  Each product of bf16 values is exact in
// fp32; what the split drops is ~3 * 2^-16 of |q_i x_i|, inside the error
// bound the select kernel works with (screen_gamma).  The result is a
// *screen*: the top-KP candidates per (query, database chunk) by screen
// score, KP > k, which the select kernel re-ranks exactly in fp64 from the
// stored fp32 rows after proving (with that a-priori bound) that the true
// top-k is inside the candidate set.
//
// Work unit = (query tile of 128 rows, database chunk of whole 256-row tiles).
// Persistent CTAs (one per SM) walk units chunk-major so that the CTAs
// running at the same time read the same database rows (L2 reuse).
//
// Warp roles (192 threads):
//   warps 0-3  epilogue: thread t owns query row t of the tile = TMEM lane t;
//              reads 32 fp32 columns at a time with tcgen05.ld, forms the
//              score s = alpha*dot + colbias[row] and keeps a register top-KP.
//   warp 4     TMA producer: for d_pad <= 256 the query tile (A, h and l
//              planes, all k-blocks) stays resident in shared memory for the
//              unit and the database tile is streamed one (k-block, plane) of
//              32 KB per ring stage; for larger d_pad each stage carries that
//              k-block's query plane too (16 + 32 KB), and a k-block's h and
//              l stages are consumed together.
//   warp 5     TMEM allocator + MMA issuer (one thread), M=128 N=256 K=16,
//              double-buffered accumulators (2 x 256 TMEM columns).
#include "epilogue.cuh"
#include "kernels.cuh"
#include "ptx.cuh"

namespace mflat_cu {
namespace {

constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kATileBytes = kBM * kBK * 2;        // 16 KB: 128 rows x 128 B
constexpr int kStageBytes = kBN * kBK * 2;        // 32 KB: 256 rows x 128 B
constexpr int kMaxStages = 6;
constexpr int kSmemBudget = 7 * kStageBytes;      // A + ring <= 224 KB
constexpr uint32_t kIdescBF16 = make_idesc(1u, kBM, kBN);   // bf16 x bf16 -> fp32

// Query tile resident up to d_pad = 256 (4 k-blocks, 128 KB for both planes);
// above, streamed with the database tile.
__host__ __device__ inline bool a_streamed(int kb) { return kb * kBK > kMaxDPadResident; }
__host__ __device__ inline int stage_bytes_for(int kb) {
    return a_streamed(kb) ? kATileBytes + kStageBytes : kStageBytes;
}
__host__ __device__ inline int n_stages_for(int kb) {
    const int a = a_streamed(kb) ? 0 : kb * 2 * kATileBytes;
    int s = (kSmemBudget - a) / stage_bytes_for(kb);
    if (s > kMaxStages) s = kMaxStages;
    if (a_streamed(kb)) s &= ~1;   // a k-block's h and l stages are used as a pair
    return s;
}

struct SmemLayout {
    uint8_t* a;          // [2 planes][kb][16 KB]
    uint8_t* b;          // [stages][32 KB]
    uint64_t* full;      // [kMaxStages]
    uint64_t* empty;     // [kMaxStages]
    uint64_t* a_full;
    uint64_t* a_empty;
    uint64_t* acc_full;  // [2]
    uint64_t* acc_empty; // [2]
    uint64_t* drain;
    uint32_t* tmem_slot;
    int* abort_flag;
};

__device__ inline SmemLayout carve(uint8_t* base, int kb, int stages) {
    SmemLayout L;
    L.a = base;
    L.b = base + (a_streamed(kb) ? 0 : kb * 2 * kATileBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(L.b + stages * stage_bytes_for(kb));
    L.full = bars;
    L.empty = bars + kMaxStages;
    L.a_full = bars + 2 * kMaxStages;
    L.a_empty = L.a_full + 1;
    L.acc_full = L.a_full + 2;
    L.acc_empty = L.a_full + 4;
    L.drain = L.a_full + 6;
    L.tmem_slot = reinterpret_cast<uint32_t*>(L.a_full + 7);
    L.abort_flag = reinterpret_cast<int*>(L.tmem_slot + 1);
    return L;
}

template <int KP, bool kBuf>
__global__ void __launch_bounds__(kThreads, 1)
screen_bf16x3_kernel(const __grid_constant__ CUtensorMap tm_a_h,
                     const __grid_constant__ CUtensorMap tm_a_l,
                     const __grid_constant__ CUtensorMap tm_b_h,
                     const __grid_constant__ CUtensorMap tm_b_l, const ScreenParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int kb_count = p.d_pad / kBK;
    if (kb_count < 1 || kb_count * kBK != p.d_pad) {
        if (threadIdx.x == 0) atomicExch(p.err, kErrConfig);
        return;
    }
    const bool stream_a = a_streamed(kb_count);
    const int sbytes = stage_bytes_for(kb_count);
    const int stages = n_stages_for(kb_count);
    SmemLayout S = carve(base, kb_count, stages);

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
            mbar_init(&S.acc_empty[b], kEpiWarps);   // one arrival per epilogue warp
        }
        mbar_init(S.drain, 1);
        *S.abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(S.tmem_slot, 512);
        tmem_relinquish();
    }
    if (warp == kProducerWarp && lane == 0) {
        tma_prefetch_desc(&tm_a_h);
        tma_prefetch_desc(&tm_a_l);
        tma_prefetch_desc(&tm_b_h);
        tma_prefetch_desc(&tm_b_l);
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
                    mbar_arrive_expect_tx(S.a_full, static_cast<uint32_t>(kb_count * 2 * kATileBytes));
                    for (int kb = 0; kb < kb_count; ++kb) {
                        tma_load_2d(&tm_a_h, S.a_full, S.a + kb * kATileBytes, kb * kBK, qt * kBM);
                        tma_load_2d(&tm_a_l, S.a_full, S.a + (kb_count + kb) * kATileBytes, kb * kBK,
                                    qt * kBM);
                    }
                    a_issued = true;
                    a_issue_phase = a_phase;
                    a_phase ^= 1u;
                }
                for (int t = t0; t < t1 && ok; ++t) {
                    for (int kb = 0; kb < kb_count && ok; ++kb) {
                        for (int plane = 0; plane < 2; ++plane) {
                            if (!mbar_wait(&S.empty[stage], sphase ^ 1u, abort_flag, p.wait_ns)) { ok = false; break; }
                            uint8_t* dst = S.b + stage * sbytes;
                            mbar_arrive_expect_tx(&S.full[stage], static_cast<uint32_t>(sbytes));
                            if (stream_a) {
                                tma_load_2d(plane ? &tm_a_l : &tm_a_h, &S.full[stage], dst, kb * kBK,
                                            qt * kBM);
                                dst += kATileBytes;
                            }
                            tma_load_2d(plane ? &tm_b_l : &tm_b_h, &S.full[stage], dst, kb * kBK,
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
            uint32_t sphase = 0, a_phase = 0;
            uint32_t tcount = 0;
            bool ok = true;
            bool issued_any = false;
            // test hook: the drain barrier completes no phase before an abort,
            // so this bounded wait runs out and the CTA takes its error path
            if (p.test_stall) ok = mbar_wait(S.drain, 0u, abort_flag, p.wait_ns) && false;
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
                    const uint32_t d_tmem = tmem_base + b * kBN;
                    for (int kb = 0; kb < kb_count && ok && stream_a; ++kb) {
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
                        const uint32_t base_h = smem_u32(S.b + s_h * sbytes);
                        const uint32_t base_l = smem_u32(S.b + s_l * sbytes);
                        const uint64_t a_h = smem_desc_k_sw128(base_h);
                        const uint64_t b_h = smem_desc_k_sw128(base_h + kATileBytes);
                        const uint64_t a_l = smem_desc_k_sw128(base_l);
                        const uint64_t b_l = smem_desc_k_sw128(base_l + kATileBytes);
#pragma unroll
                        for (int ks = 0; ks < kBK / 16; ++ks) {
                            const uint64_t o = static_cast<uint64_t>(ks * 2);   // 32 B >> 4
                            tc_mma_f16(d_tmem, a_h + o, b_h + o, kIdescBF16,
                                        (kb | ks) != 0 ? 1u : 0u);
                            tc_mma_f16(d_tmem, a_l + o, b_h + o, kIdescBF16, 1u);
                            tc_mma_f16(d_tmem, a_h + o, b_l + o, kIdescBF16, 1u);
                        }
                        issued_any = true;
                        tc_commit(&S.empty[s_h]);
                        tc_commit(&S.empty[s_l]);
                    }
                    for (int kb = 0; kb < kb_count && ok && !stream_a; ++kb) {
                        const uint64_t a_h = smem_desc_k_sw128(a_addr + kb * kATileBytes);
                        const uint64_t a_l =
                            smem_desc_k_sw128(a_addr + (kb_count + kb) * kATileBytes);
                        // stage holding B_h of this k-block
                        if (!mbar_wait(&S.full[stage], sphase, abort_flag, p.wait_ns)) { ok = false; break; }
                        tc_fence_after();
                        uint64_t bd = smem_desc_k_sw128(smem_u32(S.b + stage * kStageBytes));
#pragma unroll
                        for (int ks = 0; ks < kBK / 16; ++ks) {
                            const uint64_t o = static_cast<uint64_t>(ks * 2);   // 32 B >> 4
                            tc_mma_f16(d_tmem, a_h + o, bd + o, kIdescBF16,
                                        (kb | ks) != 0 ? 1u : 0u);
                            tc_mma_f16(d_tmem, a_l + o, bd + o, kIdescBF16, 1u);
                        }
                        issued_any = true;
                        tc_commit(&S.empty[stage]);
                        if (++stage == stages) { stage = 0; sphase ^= 1u; }
                        // stage holding B_l of this k-block
                        if (!mbar_wait(&S.full[stage], sphase, abort_flag, p.wait_ns)) { ok = false; break; }
                        tc_fence_after();
                        bd = smem_desc_k_sw128(smem_u32(S.b + stage * kStageBytes));
#pragma unroll
                        for (int ks = 0; ks < kBK / 16; ++ks) {
                            const uint64_t o = static_cast<uint64_t>(ks * 2);
                            tc_mma_f16(d_tmem, a_h + o, bd + o, kIdescBF16, 1u);
                        }
                        tc_commit(&S.empty[stage]);
                        if (++stage == stages) { stage = 0; sphase ^= 1u; }
                    }
                    if (ok) tc_commit(&S.acc_full[b]);
                }
                if (ok && !stream_a) tc_commit(S.a_empty);
            }
            if (*abort_flag && issued_any) {
                tc_commit(S.drain);
                mbar_wait_drain(S.drain, 0u, 200000000ull);
            }
        }
    } else {
        // ---------------- epilogue: warps 0..3, thread = query row
        const int row_in_tile = warp * 32 + lane;
        const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
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
            // Score floor of the query.  A buffer pass reads a floor fixed before
            // the launch: one load per unit.  In list mode finished units of the
            // same query raise it (monotone), so any earlier value is a valid
            // bound: it is reloaded one tile ahead, keeping the load's latency off
            // the tile loop.
            uint32_t fkey_next = (live && p.use_floor) ? __ldcg(p.thr + row) : 0u;
            for (int t = t0; t < t1; ++t, ++tcount) {
                const uint32_t b = tcount & 1u;
                const uint32_t ph = (tcount >> 1) & 1u;
                const uint32_t fkey = fkey_next;
                if (!kBuf && live && p.use_floor && t + 1 < t1) fkey_next = __ldcg(p.thr + row);
                // the next tile's bias prefetch overlaps the accumulator wait
                if (lane < 8 && t + 1 < t1)
                    prefetch_l1(p.colbias + static_cast<int64_t>(t + 1) * p.tile_stride * kBN + lane * 32);
                // one lane polls the barrier, the warp follows
                bool ready = true;
                if (lane == 0) ready = mbar_wait(&S.acc_full[b], ph, abort_flag, p.wait_ns);
                if (!__shfl_sync(0xffffffffu, ready ? 1 : 0, 0)) { ok = false; break; }
                const float floor_adj =
                    !live ? __int_as_float(0x7f800000)
                          : (p.use_floor ? floor_below(fkey) : -__int_as_float(0x7f800000));
                const int id_tile = t * p.tile_stride * kBN;
                const float* cb_tile = p.colbias + id_tile;
                const uint32_t taddr = lane_addr + b * kBN;
                uint32_t ra[32], rb[32];
                float4 ca[8], cbv[8];
                __syncwarp();
                tc_fence_after();
                tmem_ld_32x32b_x32(taddr, ra);
                load_bias(ca, cb_tile);
#pragma unroll 1
                for (int c = 0; c < kBN / 32; c += 2) {
                    tmem_wait_ld_regs(ra);
                    __syncwarp();
                    tmem_ld_32x32b_x32(taddr + (c + 1) * 32, rb);
                    load_bias(cbv, cb_tile + (c + 1) * 32);
                    if constexpr (kBuf) buffer_chunk(ra, ca, p.alpha, floor_adj, br, st, id_tile + c * 32);
                    else scan_chunk<KP>(ra, ca, p.alpha, floor_adj, L, id_tile + c * 32);
                    tmem_wait_ld_regs(rb);
                    if (c + 2 < kBN / 32) {
                        __syncwarp();
                        tmem_ld_32x32b_x32(taddr + (c + 2) * 32, ra);
                        load_bias(ca, cb_tile + (c + 2) * 32);
                    }
                    if constexpr (kBuf)
                        buffer_chunk(rb, cbv, p.alpha, floor_adj, br, st, id_tile + (c + 1) * 32);
                    else scan_chunk<KP>(rb, cbv, p.alpha, floor_adj, L, id_tile + (c + 1) * 32);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.acc_empty[b]);
            }
            if constexpr (kBuf) st.flush(br);   // the unit's staged appends
            if (!ok) break;
            if (!kBuf && live) {
                const int64_t o = (static_cast<int64_t>(ch) * p.m_pad + row) * KP;
                float4* ps = reinterpret_cast<float4*>(p.part_score + o);
                int4* pi = reinterpret_cast<int4*>(p.part_id + o);
#pragma unroll
                for (int i = 0; i < KP / 4; ++i) {
                    ps[i] = make_float4(L.s[4 * i], L.s[4 * i + 1], L.s[4 * i + 2], L.s[4 * i + 3]);
                    pi[i] = make_int4(L.id[4 * i], L.id[4 * i + 1], L.id[4 * i + 2], L.id[4 * i + 3]);
                }
                // A full list's KP-th score is a lower bound of the query's
                // global KP-th best: no row below it can matter any more.
                if (p.use_floor && L.id[KP - 1] >= 0) atomicMax(p.thr + row, score_key(L.s[KP - 1]));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc(tmem_base, 512);
    if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, *abort_flag);
}

template <int KP, bool kBuf = false>
cudaError_t launch_kp(const CUtensorMap& a_h, const CUtensorMap& a_l, const CUtensorMap& b_h,
                      const CUtensorMap& b_l, const ScreenParams& p, int grid,
                      cudaStream_t stream) {
    const int smem = screen_bf16x3_smem_bytes(p.d_pad);
    cudaError_t e = cudaFuncSetAttribute(screen_bf16x3_kernel<KP, kBuf>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    screen_bf16x3_kernel<KP, kBuf><<<grid, kThreads, smem, stream>>>(a_h, a_l, b_h, b_l, p);
    return cudaGetLastError();
}

}  // namespace

int screen_bf16x3_smem_bytes(int d_pad) {
    const int kb = d_pad / kBK;
    const int a = a_streamed(kb) ? 0 : kb * 2 * kATileBytes;
    return 1024 + a + n_stages_for(kb) * stage_bytes_for(kb) + 256;
}

cudaError_t launch_screen_bf16x3(int kp, const CUtensorMap& a_h, const CUtensorMap& a_l,
                                 const CUtensorMap& b_h, const CUtensorMap& b_l,
                                 const ScreenParams& p, int grid, cudaStream_t stream) {
    if (p.d_pad % kBK != 0 || p.d_pad < kBK) return cudaErrorInvalidValue;
    switch (kp) {
        case 0: return launch_kp<4, true>(a_h, a_l, b_h, b_l, p, grid, stream);
        case 4: return launch_kp<4>(a_h, a_l, b_h, b_l, p, grid, stream);
        case 8: return launch_kp<8>(a_h, a_l, b_h, b_l, p, grid, stream);
        case 16: return launch_kp<16>(a_h, a_l, b_h, b_l, p, grid, stream);
        case 32: return launch_kp<32>(a_h, a_l, b_h, b_l, p, grid, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace mflat_cu
