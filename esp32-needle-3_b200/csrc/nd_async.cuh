// nd_async.cuh - mbarrier, TMA and tcgen05 fence helpers shared by the
// asynchronous kernels (tensor-core prefill, TMA-staged decode). Every wait is
// bounded: kTimeoutCycles of SM clock (~2 s), after which the caller's abort
// flag is raised and the wait reports failure instead of spinning on.
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace nda {
namespace {

constexpr long long kTimeoutCycles = 4000000000LL;   // ~2 s at 1.9 GHz

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-blocking test of the same (test_wait never suspends the thread, where
// try_wait may, up to a hardware time limit): for event loops that poll
// several barriers.
__device__ __forceinline__ bool mbar_ready(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase of parity `parity`. False when the CTA is
// aborting (another role timed out) or this wait timed out (then it raises
// the abort itself).
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, volatile int *abort_flag) {
    if (mbar_test(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_test(b, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > kTimeoutCycles) {
            *abort_flag = 1;
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ void mbar_drain(uint64_t *b, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_test(b, parity) && clock64() - t0 < kTimeoutCycles) {
    }
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            su32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(su32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

}  // namespace
}  // namespace nda
