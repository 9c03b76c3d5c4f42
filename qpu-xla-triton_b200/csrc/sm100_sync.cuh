// mbarrier, bounded-wait and TMA helpers shared by the sm_100a kernels.
//
// Every wait a kernel performs on an mbarrier goes through wait_bounded: after
// kKernelWaitLimitNs of %globaltimer it records kKernelWaitTimeout in the
// context's error word, raises the CTA's abort flag (so the CTA's other waits
// give up too) and returns false. wait_drain is the bounded wait used on the
// abort path to let a CTA's own copies and MMAs land before it exits.
#pragma once

#include <cuda.h>

#include <cstdint>

#include "qpucuda_internal.h"

namespace qpucuda {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void *pointer) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(pointer));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t value;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(value));
    return value;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// false when the CTA was aborted or the wait exceeded limit_ns (the latter records the error
// and aborts the CTA).
__device__ __forceinline__ bool wait_bounded_ns(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                                unsigned int *error_word, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer();
    for (uint32_t spin = 1;; ++spin) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((spin & 63u) == 0) {
            if (*abort_flag != 0) return false;
            if (globaltimer() - start > limit_ns) {
                *abort_flag = 1;
                atomicExch(error_word, static_cast<unsigned int>(kKernelWaitTimeout));
                return false;
            }
        }
    }
}

// try_wait that may suspend the thread for up to suspend_ns (it resumes as soon as the phase
// completes): a waiting warp then takes no issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint32_t bar, uint32_t parity, uint32_t suspend_ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(suspend_ns)
        : "memory");
    return done != 0;
}

// wait_bounded_ns built on the suspending try_wait (each attempt sleeps up to 20 us at most).
__device__ __forceinline__ bool wait_bounded_suspend(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                                     unsigned int *error_word) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer();
    for (;;) {
        if (mbar_try_wait_suspend(bar, parity, 20000u)) return true;
        if (*abort_flag != 0) return false;
        if (globaltimer() - start > kKernelWaitLimitNs) {
            *abort_flag = 1;
            atomicExch(error_word, static_cast<unsigned int>(kKernelWaitTimeout));
            return false;
        }
    }
}

// The product kernels' waits: bounded by kKernelWaitLimitNs.
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                             unsigned int *error_word) {
    return wait_bounded_ns(bar, parity, abort_flag, error_word, kKernelWaitLimitNs);
}

// Bounded wait that ignores the abort flag (abort path only).
__device__ __forceinline__ void wait_drain(uint32_t bar, uint32_t parity) {
    const uint64_t start = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - start > kKernelWaitLimitNs) return;
    }
}

// 2D tiled TMA load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t destination, const CUtensorMap *map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(destination),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 1D bulk copy global -> this CTA's shared memory (16-byte aligned addresses, size a
// multiple of 16), completing on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t destination, const void *source, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(destination),
        "l"(reinterpret_cast<uint64_t>(source)), "r"(bytes), "r"(bar)
        : "memory");
}

}  // namespace sm100
}  // namespace qpucuda
