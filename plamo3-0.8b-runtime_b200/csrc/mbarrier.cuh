// Shared-memory mbarriers and TMA tensor copies used by the tiled GEMMs (gemm.cu, gemm_tc.cu).
#pragma once
#include <cuda.h>
#include <cstdint>

namespace plamo {

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_test(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok)
                 : "r"(smem_addr(b)), "r"(parity)
                 : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait (2 s): a copy or an MMA that never completes ends the kernel's use of the barrier
// instead of hanging.
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity) {
    if (bar_test(b, parity)) return true;
    const uint64_t t0 = now_ns();
    for (uint32_t i = 1;; i++) {
        if (bar_test(b, parity)) return true;
        if ((i & 63u) == 0 && now_ns() - t0 > 2000000000ull) return false;
    }
}
__device__ __forceinline__ void tma2(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_addr(b))
        : "memory");
}
__device__ __forceinline__ void tma3(void* dst, const CUtensorMap* map, int c1, int c2, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(0), "r"(c1), "r"(c2), "r"(smem_addr(b))
        : "memory");
}

}  // namespace plamo
