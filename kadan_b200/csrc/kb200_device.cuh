// sm_100a device helpers shared by the kadan_b200 kernels: mbarriers with
// bounded waits, bulk async global->shared copies, packed f32x2 FMA and the
// watchdog word every bounded wait reports to.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace kb200 {

enum : unsigned {
    watchdog_full_barrier = 1u,
    watchdog_empty_barrier = 2u,
    watchdog_drain = 4u,
    watchdog_fixup = 8u,  // a cut tile's other pieces never arrived
};

// Upper bound on polls of one mbarrier phase. mbarrier.try_wait suspends the
// thread for a hardware time slice per poll, so this is far beyond any copy
// that can complete, yet ends a lost wait in well under a second.
constexpr uint32_t wait_polls = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
        : "memory"
    );
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory"
    );
    return done != 0;
}

// Non-blocking check that phase `parity` completed (try_wait, in contrast,
// suspends the thread for a hardware time slice before it gives up).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory"
    );
    return done != 0;
}

// Bounded wait for `parity` to complete. False (after flagging `cause` in the
// watchdog word, see watchdog_word()) when the phase never completed within
// wait_polls polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned cause, unsigned* watchdog) {
    for (uint32_t i = 0; i < wait_polls; ++i)
        if (mbar_try_wait(bar, parity))
            return true;
    atomicOr(watchdog, cause);
    return false;
}

// Bulk (non-tensor) async copy of `bytes` (multiple of 16; both addresses
// 16-byte aligned) from global to this CTA's shared memory, completing as
// transaction bytes on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)
        ),
        "l"(src),
        "r"(bytes),
        "r"(smem_addr(bar))
        : "memory"
    );
}

// Named barrier among the first `threads` threads (the consumer warps).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// d = a * b + c on two independent fp32 lanes in one instruction (sm_100).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)),
          "l"(*reinterpret_cast<unsigned long long*>(&b)),
          "l"(*reinterpret_cast<unsigned long long*>(&c)));
    return *reinterpret_cast<float2*>(&d);
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

}  // namespace kb200
