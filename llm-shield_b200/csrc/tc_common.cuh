// tc_common.cuh — tcgen05 / TMEM / mbarrier / bulk-copy helpers shared by the tensor-core
// kernels (the prefill GEMM in gemm_tc.cu and the prefill attention in attn_tc.cu).
#pragma once

#include "jv_internal.h"

namespace jv {
namespace {

// Bound of every wait, in SM clock cycles (%clock64): about 2 s at the 1.965 GHz maximum,
// longer at lower clocks. The cycle counter of the SM running the thread only moves forward;
// %globaltimer is not used for bounds, since a step of it (the driver may re-synchronise it
// with the host clock) would end a wait early, and a backward step would underflow the
// elapsed-time difference.
constexpr long long WAIT_CYCLES = 4000000000ll;

__device__ __forceinline__ uint32_t s_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
// try_wait with a suspend-time hint: the thread sleeps until the phase completes (woken at
// completion) or ~1 ms passes, instead of spinning.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
// Bounded wait: false after `bound` cycles without the phase completing.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long bound = WAIT_CYCLES) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(bar, parity))
        if (clock64() - t0 > bound) return false;
    return true;
}
// Bounded wait that polls with the non-blocking mbarrier.test_wait instead of sleeping in
// try_wait: for the single thread that issues the MMAs, whose wake-up latency after a phase
// completes would otherwise sit between the data landing and the next MMA.
__device__ __forceinline__ bool mbar_poll(uint32_t bar, uint32_t parity, long long bound = WAIT_CYCLES) {
    uint32_t ok;
    const long long t0 = clock64();
    for (;;) {
        asm volatile(
            "{\n.reg .pred p;\nmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > bound) return false;
    }
}
// A bounded wait gave up: the error word takes JV_ERR_DEVICE_TIMEOUT and the word after it
// the first site that gave up (kernel x 16 + role), which the host names in its message.
__device__ __forceinline__ void report_timeout(int* err, int site) {
    // takes the place of a numeric report, not of an out-of-range index (its cause, in a checked build)
    atomicCAS(err, 0, JV_ERR_DEVICE_TIMEOUT);
    atomicCAS(err, JV_ERR_NUMERIC, JV_ERR_DEVICE_TIMEOUT);
    atomicCAS(err + 1, 0, site);
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// Bulk prefetch of [src, src + bytes) into L2 (no shared memory, no completion to wait for).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(slot), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

// UMMA shared-memory matrix descriptor, K-major SWIZZLE_128B: start address >> 4 in bits
// 0-13, leading byte offset (unused by this layout) 16 B, stride byte offset 1024 B (one
// 8-row x 128-byte swizzle atom), descriptor version 1 (bits 46-47), layout 2 = SWIZZLE_128B
// (bits 61-63).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)(16u >> 4) << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A/B fp16 (bits 7-9, 10-12 = 0;
// 1 would be bf16), both K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_f16(int n, int m) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\ntcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}

// tcgen05.ld of 16 consecutive accumulator columns (32 lanes x 32 bit) without waiting; the
// registers are valid only after tmem_wait16 on the same array, which names them as in/out
// operands so no use of them can be scheduled above the wait.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait16(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

}  // namespace
}  // namespace jv
