// zz_tc.cuh -- Blackwell (sm_100a) primitives: mbarriers with bounded waits, TMA
// tile loads, TMEM allocation, tcgen05 MMA / commit / load. Hand-written inline PTX.
//
// Every wait here has a time limit (2 s of %globaltimer). A wait that runs out sets the CTA's abort
// flag and the kernel's error word and returns false; the caller then stops issuing
// work, drains what it can with the same bounded waits, frees its TMEM and returns,
// so the context stays usable and the host sees the error.
#pragma once
#include <cuda.h>
#include "zz_common.cuh"

namespace zz {
namespace tc {

constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;  // a wait gives up after 2 s
constexpr uint32_t SUSPEND_NS = 20000;                        // suspend-time hint of one try

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{.reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0];}" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{.reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;}" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{.reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p;}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
#ifdef ZZ_TC_PROF
// diagnostic build only: cycles spent in each wait site, summed over block 0's warps
__device__ unsigned long long g_tc_prof[128];
#endif
#ifdef ZZ_TC_PROF
#define TC_PROF_T(v) const long long v = clock64()
#define TC_PROF_ADD(code, t0)                                                                        \
    do {                                                                                             \
        if (blockIdx.x == 0 && (threadIdx.x & 31) == 0)                                              \
            atomicAdd(&::zz::tc::g_tc_prof[code], (unsigned long long)(clock64() - (t0)));           \
    } while (0)
#else
#define TC_PROF_T(v)
#define TC_PROF_ADD(code, t0)
#endif
// as mbar_try, but the thread may be suspended (up to `ns`) until the phase completes,
// so a waiting role does not take issue slots from the warps doing the work
__device__ __forceinline__ bool mbar_try_suspend(uint64_t *bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{.reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p;}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// bounded wait for the phase with the given parity to complete
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort, int *err, int code) {
#ifdef ZZ_TC_PROF
    const long long t0 = clock64();
    struct Acc {
        long long t0;
        int code;
        __device__ ~Acc() {
            if (blockIdx.x == 0 && (threadIdx.x & 31) == 0)
                atomicAdd(&g_tc_prof[code], (unsigned long long)(clock64() - t0));
        }
    } acc_{t0, code};
#endif
    if (mbar_try(bar, parity)) return true;
    const unsigned long long w0 = global_ns();
    // try_wait with a short back-off: a waiting warp sleeps between tries instead of
    // taking issue slots from the warps doing the work (a suspend-time hint on the try
    // itself can sleep well past the phase change); the sleep grows from 32 to 256 ns.
    // The clock and the abort flag are read every 16 tries.
    uint32_t ns = 32;
    for (;;) {
#ifdef ZZ_TC_PROF
        if (blockIdx.x == 0 && (threadIdx.x & 31) == 0) atomicAdd(&g_tc_prof[64 + code], 1ull);
#endif
        for (int i = 0; i < 16; i++) {
#ifndef ZZ_TC_MAXSLEEP
#define ZZ_TC_MAXSLEEP 256
#endif
            if (ZZ_TC_MAXSLEEP) __nanosleep(ns);
            if (mbar_try(bar, parity)) return true;
            ns = ns < ZZ_TC_MAXSLEEP ? 2 * ns : ZZ_TC_MAXSLEEP;
        }
        if (*abort) return false;
        if (global_ns() - w0 > WAIT_LIMIT_NS) break;
    }
    *abort = 1;
    atomicCAS(err, 0, code);
    return false;
}

// non-blocking probe of the phase with the given parity (mbarrier.test_wait: no
// suspension window, so a completed phase costs one shared-memory round trip)
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{.reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p;}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait without back-off, for the roles on a pipeline's critical path (the MMA
// issuer, copy issuers, operand producers): a ready phase costs one probe, and a pending
// one is waited for in hardware (try_wait) instead of a sleep. The clock and the abort flag
// are read every 16 tries.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t *bar, uint32_t parity, volatile int *abort, int *err,
                                               int code) {
#ifdef ZZ_TC_PROF
    const long long t0 = clock64();
    struct Acc {
        long long t0;
        int code;
        __device__ ~Acc() {
            if (blockIdx.x == 0 && (threadIdx.x & 31) == 0)
                atomicAdd(&g_tc_prof[code], (unsigned long long)(clock64() - t0));
        }
    } acc_{t0, code};
#endif
    if (mbar_test(bar, parity)) return true;
    const unsigned long long w0 = global_ns();
    for (;;) {
        // try_wait parks the thread in hardware until the phase completes (or a short
        // time-out), so a waiting warp takes no issue slots from the warps doing the work
        for (int i = 0; i < 16; i++)
            if (mbar_try(bar, parity)) return true;
        if (*abort) return false;
        if (global_ns() - w0 > WAIT_LIMIT_NS) break;
    }
    *abort = 1;
    atomicCAS(err, 0, code);
    return false;
}

// wait, bounded by time only (not by the abort flag), for copies or MMAs this thread has
// issued: a CTA must not exit, nor free TMEM, while they may still write its memory
__device__ __forceinline__ bool mbar_drain(uint64_t *bar, uint32_t parity) {
    const unsigned long long w0 = global_ns();
    while (!mbar_try(bar, parity))
        if (global_ns() - w0 > WAIT_LIMIT_NS) return false;
    return true;
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 2-D TMA tile load global -> shared, completion counted on an mbarrier (no multicast)
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 3-D TMA tile load (no multicast)
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}
// contiguous bulk copy global -> shared (16-byte aligned, size a multiple of 16)
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// TMEM: allocation by one full warp; the base address is written to shared memory
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core matrices,
// `lbo` bytes between K-adjacent core matrices, `sbo` bytes between 8-row groups.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for sm_100
    return d;                // base offset 0, layout type 0 (no swizzle)
}
// K-major with 64-byte swizzle (the layout a SWIZZLE_64B TMA box of 64-byte rows
// writes): 8-row x 64-byte atoms `sbo` bytes apart; the leading offset is unused
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t addr, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;  // leading byte offset field = 1 (ignored for swizzled K-major)
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for sm_100
    d |= (uint64_t)4 << 61;  // layout type: 64-byte swizzle
    return d;
}
// K-major operand in 128-byte-swizzled atoms (8 rows x 128 bytes, 1024 bytes apart):
// the layout a SWIZZLE_128B TMA box of 128-byte rows writes. A 32-byte K slice (K = 32 int8 or K = 16 fp16) at byte
// offset 32j inside the atom is addressed by advancing the start address.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;                 // leading offset: unused for swizzled K-major
    d |= (uint64_t)(1024 >> 4) << 32;       // 8-row groups 1024 bytes apart
    d |= (uint64_t)1 << 46;                 // descriptor version for sm_100
    d |= (uint64_t)2 << 61;                 // layout type: 128-byte swizzle
    return d;
}
// Instruction descriptor, kind::f16: f16 A and B (K-major), f32 accumulator, M x N
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread
__device__ __forceinline__ void mma_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{.reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// the same MMA issued by a whole warp in uniform control flow: one elected lane issues
// it, and the operands (warp-uniform values) can stay in uniform registers
__device__ __forceinline__ void mma_f16_ss_warp(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{.reg .pred p, e; setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_f16_ts_warp(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{.reg .pred p, e; setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// commit issued by one elected lane of a warp in uniform control flow
__device__ __forceinline__ void mma_commit_warp(uint64_t *bar) {
    asm volatile(
        "{.reg .pred e; elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];}" ::"r"(smem_u32(bar))
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T: A is M lanes x K columns of packed fp16 pairs (the
// 32-bit column c of lane m holds A[m][2c] in its low half and A[m][2c + 1] in its high
// half), issued by one thread
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{.reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns from 16 registers per thread
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t *r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// the mbarrier fires when all previously issued tcgen05 ops of this thread complete
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns -> 16 registers per thread
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// 16 lanes x 4 x 256 bits: thread t gets, for i = 0..3, lane (t/4) columns 8i + 2(t%4) + {0,1}
// in r[4i], r[4i+1] and lane (t/4)+8 the same columns in r[4i+2], r[4i+3]
__device__ __forceinline__ void tmem_ld16x256_x4(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// named barrier among a subset of warps
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace tc
}  // namespace zz
