// ptx.cuh -- hand-written sm_100a PTX wrappers used by the flat-search kernels:
// mbarriers (every wait is bounded), TMA tile loads (no multicast anywhere),
// and the tcgen05 tensor-core / tensor-memory instructions.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace mflat_cu {

// A wait that has not completed after this many nanoseconds marks the CTA as
// failed: the kernel records an error code, drains what it issued and exits.
// Legitimate waits in these kernels last microseconds.  The host can pass a
// different limit per launch (ScreenParams::wait_ns, MFLAT_WAIT_LIMIT_MS).
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

enum ErrCode : int {
    kErrNone = 0,
    kErrTimeout = 1,        // a bounded mbarrier wait ran out
    kErrConfig = 2,         // kernel launched with an unsupported shape
    kErrInternal = 3,       // a consistency check failed (e.g. a candidate id out of range)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false when the
// CTA-wide abort flag is (or becomes) set, or after limit_ns (0: the default
// kWaitTimeoutNs); in the timeout case this thread sets the abort flag itself.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint64_t limit_ns) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    const uint64_t limit = limit_ns ? limit_ns : kWaitTimeoutNs;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(addr, parity)) return true;
        if ((it & 63u) == 0u) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > limit) {
                *abort_flag = kErrTimeout;
                return false;
            }
        }
    }
}

// Short bounded wait used only while draining after an abort.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    const uint32_t addr = smem_u32(bar);
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(addr, parity)) {
        if (globaltimer_ns() - t0 > limit_ns) return;
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void prefetch_l1(const void* p) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load global -> this CTA's shared memory, completion counted in
// bytes on `bar`.  x (innermost) is in elements and must be 16-byte aligned.
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory, completing on `bar`
// (both addresses 16-byte aligned, bytes a multiple of 16; no multicast).
__device__ __forceinline__ void bulk_load_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .u64 g;\n\t"
        "cvta.to.global.u64 g, %1;\n\t"
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [g], %2, [%3];\n\t}" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------ CTA pairs (clusters of 2)
// Rank of this CTA in its cluster.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Shared::cluster address of this CTA's shared variable `p` as seen in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
    return a;
}
// All threads of both CTAs of the cluster (release / acquire).  Unbounded:
// reach it only after every bounded wait of the CTA has returned.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive once on an mbarrier given by its shared::cluster address (possibly
// in the peer CTA), with the default semantics (release, CTA scope): used to
// hand an accumulator back after this thread's TMEM loads have completed
// (tcgen05.wait::ld), which needs execution order only -- a cluster-scope
// release would also wait for this thread's outstanding global stores.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// Tile load into this CTA's shared memory completing on an mbarrier of either
// CTA of the pair (`cluster_bar`: shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t cluster_bar, void* dst,
                                                 int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y)
        : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// The same for a CTA pair: issued by the same warp in both CTAs, same slot.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (A and B both f16
// or both bf16, fp32 accumulation), issued by one thread.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// CTA pair (issued by the leader): M = 256 split over the two CTAs' shared
// memory (A rows and B rows each halved, same offsets in both CTAs), each
// CTA's TMEM receiving its 128 rows x N columns.
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the mbarrier at this offset in every CTA of `mask` when the
// pair's tcgen05 ops issued so far by this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(mask)
        : "memory");
}

// Arrive once on `bar` when every tcgen05 op issued so far by this thread has
// completed (also makes their shared-memory reads / TMEM writes visible).
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (base_lane + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Wait for outstanding tcgen05.ld and tie the destination registers to the
// wait: the asm of tcgen05.ld declares its outputs as if they were ready at
// once, so without this the compiler could schedule a use above the wait.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
          "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
          "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]),
          "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
          "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
          "+r"(r[31])
        :
        : "memory");
}

// Order-preserving map float -> uint32 (larger float -> larger key), so a
// per-query score floor can be raised with atomicMax.  Key 0 means "none".
__device__ __forceinline__ uint32_t score_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// Largest float strictly below the score encoded by `key` (-inf for none):
// admitting s > floor_below(key) admits exactly s >= decoded score.
__device__ __forceinline__ float floor_below(uint32_t key) {
    if (key == 0u) return -__int_as_float(0x7f800000);
    const uint32_t u = (key & 0x80000000u) ? (key & 0x7fffffffu) : ~key;
    return nextafterf(__uint_as_float(u), -__int_as_float(0x7f800000));
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row swizzle atoms 1024 bytes
// apart (SBO = 1024), leading-byte offset unused for swizzled K-major,
// descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B.  The tile base
// must be 1024-byte aligned; k-steps inside the 128-byte row advance the
// start address by 32 bytes.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);      // start address
    d |= static_cast<uint64_t>(1u) << 16;                           // LBO (unused)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;                   // SBO
    d |= static_cast<uint64_t>(1u) << 46;                           // version
    d |= static_cast<uint64_t>(2u) << 61;                           // SWIZZLE_128B
    return d;
}

// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core
// matrices, rows 16 bytes apart inside one; `lbo` = byte offset between core
// matrices adjacent in K, `sbo` = between core matrices adjacent in M / N.
__device__ __forceinline__ uint64_t smem_desc_k_none(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);      // start address
    d |= static_cast<uint64_t>((lbo & 0x3FFFFu) >> 4) << 16;       // LBO
    d |= static_cast<uint64_t>((sbo & 0x3FFFFu) >> 4) << 32;       // SBO
    d |= static_cast<uint64_t>(1u) << 46;                           // version
    return d;                                                       // layout 0: no swizzle
}

// Generic-proxy writes to shared memory made visible to the async proxy
// (tcgen05.mma operands written by plain stores).
__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Instruction descriptor: fp32 accumulator, A/B format code (tf32 = 2,
// f16 = 0, bf16 = 1), both operands K-major, N and M encoded as N>>3 / M>>4.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_format, uint32_t M, uint32_t N) {
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}



}  // namespace mflat_cu
