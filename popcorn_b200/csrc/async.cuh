// async.cuh — mbarrier and 1-D bulk-copy (cp.async.bulk) primitives for
// sm_100a, with bounded waits.
//
// Only the non-multicast, CTA-local forms are used: every copy lands in the
// issuing CTA's own shared memory from this GPU's global memory.
#pragma once

#include <stdint.h>

namespace popcorn {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// dst (shared) <- src (global), `bytes` a multiple of 16, both 16-B aligned;
// completion is signalled as transaction bytes on `bar`.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// Warm L2 with [src, src+bytes) (bytes a multiple of 16, 16-B aligned).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}

// Bounded wait (about 20k suspended tries of at most 0.1 ms each). On give-up
// it sets bit 0 of *err and returns false; the caller leaves cleanly.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned int* err) {
    for (int i = 0; i < 20000; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicOr(err, 1u);
    return false;
}

__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded spin for latency-critical hand-offs: polls without suspending
// (about 2^26 polls, seconds) so a completed phase is seen at once. On
// give-up it sets bit 0 of *err and returns false.
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, unsigned int* err) {
    for (uint32_t i = 0; i < (1u << 26); ++i)
        if (mbar_test_wait(bar, parity)) return true;
    atomicOr(err, 1u);
    return false;
}

// Pulls this CTA's share (part `part` of `nparts`) of [ptr, ptr+bytes) into
// L2, in pieces of at most 64 KB. Ranges are trimmed to 16-byte boundaries.
__device__ __forceinline__ void prefetch_share_l2(const void* ptr, uint64_t bytes, int part, int nparts) {
    if (!ptr || bytes < 16) return;
    uint64_t base = (reinterpret_cast<uint64_t>(ptr) + 15) & ~uint64_t(15);
    uint64_t end = (reinterpret_cast<uint64_t>(ptr) + bytes) & ~uint64_t(15);
    if (end <= base) return;
    uint64_t total = end - base;
    uint64_t share = ((total / uint64_t(nparts)) + 15) & ~uint64_t(15);
    uint64_t lo = base + share * uint64_t(part);
    uint64_t hi = lo + share < end ? lo + share : end;
    for (uint64_t a = lo; a < hi; a += 65536) {
        uint64_t n = hi - a < 65536 ? hi - a : 65536;
        bulk_prefetch_l2(reinterpret_cast<const void*>(a), uint32_t(n));
    }
}

// Named barrier over `threads` threads (a multiple of 32) with id `id` (1..15).
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace popcorn
