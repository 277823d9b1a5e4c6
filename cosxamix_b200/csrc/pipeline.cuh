// Bulk-copy (TMA unit) and mbarrier primitives for sm_100a, with bounded
// waits: no wait in this library can spin forever. A wait that runs out sets
// an error flag the host reads, and the kernel drains its own copies in
// flight before it returns.
#pragma once

#include <stdint.h>

namespace cxm {

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// One bounded try: the thread is suspended until the phase completes or the
// hint (in ns) runs out, instead of spinning on the barrier word the bulk
// copies are completing.
constexpr uint32_t kSuspendHintNs = 20000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` of
// transaction count on `bar`. src and dst 16-byte aligned, bytes % 16 == 0.
// No multicast: the source is always this GPU's own memory.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Bounded wait on a phase of `bar`: at most `limit` tries of up to
// kSuspendHintNs each (2^16 x 20 us ~ 1.3 s), or until another role of the
// CTA raised `abort`.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, volatile int *abort,
                                                  uint32_t limit = (1u << 16)) {
    for (uint32_t i = 0; i < limit; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
    }
    return false;
}

// 16-byte asynchronous global -> shared copies (many in flight per thread)
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Programmatic dependent launch: the next kernel in the stream may start its
// prologue (weight streaming) before this one ends; griddep_wait() blocks
// until the previous kernel's writes are visible.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace cxm
