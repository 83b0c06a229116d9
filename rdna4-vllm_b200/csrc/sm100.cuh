// sm100.cuh — device helpers shared by the sm_100a kernels: mbarriers with bounded waits,
// TMA tile / bulk copies (no cluster multicast anywhere), shared-memory addresses.
#pragma once

#include <cudaTypedefs.h>
#include <stdint.h>

namespace w4a8 {

constexpr uint64_t kWaitLimitNs = 1000000000ull;  // a bounded wait gives up after 1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// try_wait that may suspend the thread in hardware for up to hint_ns (it resumes as soon as
// the phase completes), so a waiting warp does not spin on the issue slots its neighbours need.
__device__ __forceinline__ bool mbar_try_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return done != 0;
}

// Bounded wait: a plain try_wait first, then suspending try_waits (up to 20 us each), giving up
// after kWaitLimitNs; once any wait in the CTA has given up, later waits return at once.
__device__ __forceinline__ void mbar_wait(uint64_t* bar, uint32_t parity, volatile int* bad) {
    if (mbar_try(bar, parity)) return;
    if (*bad) return;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_sleep(bar, parity, 20000u)) return;
        if (*bad) return;
        if (global_ns() - t0 > kWaitLimitNs) {
            *bad = 1;
            return;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}


// 2D u8 tensor map over rows x row_bytes (row stride row_bytes), box box_bytes x box_rows
// (host side; defined in gemm_tc.cu).
bool make_tma_map_u8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes,
                     uint32_t box_bytes, uint32_t box_rows, CUtensorMapSwizzle sw);

}  // namespace w4a8
