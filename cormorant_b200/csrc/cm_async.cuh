// cm_async.cuh -- shared-memory mbarriers and bulk async copies (TMA engine),
// with every wait bounded by %globaltimer.
#pragma once

#include "cm_common.cuh"

namespace cm {

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// The same test, letting the thread sleep in hardware until the phase completes or
// about `hint_ns` pass (instead of returning at once), so waiting warps do not spin
// through issue slots.
__device__ __forceinline__ bool mbar_try_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

struct WaitCtl {
    volatile int* abort;   // shared flag: some role gave up
    int* status;           // device status word
    uint64_t timeout_ns;
};

// Bounded wait: returns false (and raises the abort flag) on timeout or abort.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtl& w) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_sleep(bar, parity, 20000u)) return true;
        if ((it & 7u) == 0) {
            if (*w.abort) return false;
            if (gtimer() - t0 > w.timeout_ns) {
                atomicCAS(w.status, 0, CM_ETIMEOUT);
                *w.abort = 1;
                return false;
            }
        }
    }
}

// Contiguous global -> shared copy on the TMA engine, completing `bytes` on the
// mbarrier.  Both addresses 16-byte aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"((uint64_t)src), "r"(bytes), "r"(bar)
                 : "memory");
}

}  // namespace cm
