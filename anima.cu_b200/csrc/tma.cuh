// tma.cuh -- Tensor Memory Accelerator staging for sm_100a: bulk tensor loads into shared
// memory that complete on an mbarrier, with bounded waits.
//
// Only loads from this GPU's own memory, never with .multicast::cluster: the kernels that use
// this header can run in multi-GPU jobs. Every wait polls a bounded number of times; a wait
// that runs out returns false and the kernel records it (the caller's counter) instead of
// spinning forever.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace anima {

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t arrivals) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(arrivals) : "memory");
}

// Makes the initialised barriers visible to the async proxy (the TMA unit).
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// One arrival that also announces `bytes` of transactions the barrier must see complete.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase with the given parity to complete; false after kMbarPolls polls. A poll
// may suspend the thread for a while, so the limit is far beyond any real transfer's latency
// (microseconds) but still ends.
constexpr uint32_t kMbarPolls = 1u << 22;
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < kMbarPolls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// 3-D tiled bulk tensor load of one box at (x, y, z) into shared memory, completing on `bar`.
// x (the innermost coordinate) times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// Host side (abi.cu): a bf16 3-D tensor map with dims {d0, d1, d2} (d0 innermost, contiguous),
// byte strides s1 (between d1 rows) and s2, box {b0, b1, 1}, no swizzle, zero fill out of
// bounds. False if the driver entry point is missing or the encoding is refused.
bool encode_bf16_map_3d(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                        uint64_t s2, uint32_t b0, uint32_t b1);

}  // namespace anima
