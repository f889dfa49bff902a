// tc.cuh — tcgen05 (5th-generation tensor core) building blocks shared by the
// tensor-core kernels (qgemm.cu, sgemm_tc.cu): the UMMA shared-memory and
// instruction descriptors, the 128-byte swizzle, fences and 1-D bulk copies.
#pragma once
#include "common.cuh"

namespace cats {

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// K-major, 128-byte swizzle, 8-row groups 1024 bytes apart (the canonical
// UMMA K-major SW128 layout: SBO = 1024 B, LBO unused = 1, version 1).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr)
{
    return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: D f32 (bits 4-5 = 1), A and B of format `fmt`
// (bits 7-9 and 10-12: 0 f16, 1 bf16, 2 tf32), both K-major, N >> 3 at bit
// 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t umma_idesc(int fmt, int M, int N)
{
    return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// byte offset of 16-byte chunk c of row r in a 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw128(int r, int c)
{
    return (uint32_t)r * 128 + (uint32_t)((c ^ (r & 7)) * 16);
}

// 1-D bulk copy global -> shared completing on an mbarrier (no L2 hint).
__device__ __forceinline__ void bulk_g2s_keep(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Bounded wait for an mbarrier phase that also gives up when the CTA is
// unwinding (abort flag); records `code` in err when it times out.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_s, int *err, int code)
{
    for (uint32_t i = 0; i < CATS_SPIN_LIMIT; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_s) return false;
        if (i > 64) __nanosleep(32);
    }
    if (!*abort_s && err) atomicOr(err, code);
    *abort_s = 1;
    return false;
}

} // namespace cats
