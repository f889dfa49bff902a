// common.cuh — shared device helpers for libcatsgpu (sm_100a only).
//
// Bulk-copy (TMA 1-D) staging with mbarriers, programmatic dependent launch,
// the sticky error word, and the weight-type table.  No multicast form of any
// bulk copy is used anywhere in this library.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libcatsgpu is written for sm_100a (Blackwell B200) only"
#endif

namespace cats {

// ggml type numbers (llm/catseye_llm.h:2557-2580)
enum WType : int { W_F32 = 0, W_Q4_0 = 2, W_Q8_0 = 8, W_Q3_K = 11, W_Q6_K = 14 };

// error codes recorded in the sticky status (include/catsgpu.h lists them)
enum Err : int {
    E_OK = 0, E_CUDA = 1, E_ARG = 2, E_NOMEM = 3, E_TIMEOUT = 4, E_UNSUPPORTED = 5,
    E_NOT_INIT = 6, E_NCCL = 7
};

// device-side error word: kernels OR bits into it when a bounded wait gives up
#define CATS_DEVERR_MBAR_FULL 0x1
#define CATS_DEVERR_MBAR_EMPTY 0x2
#define CATS_DEVERR_PEER_WAIT 0x4
#define CATS_DEVERR_ATTN_WAIT 0x8
#define CATS_DEVERR_POS_RANGE 0x10   // a step ran with pos >= seq_len; its cache writes were skipped
#define CATS_DEVERR_TOKEN_RANGE 0x20 // the greedy argmax gave no valid token

// bounded-wait budget: ~2^24 polls with backoff is far beyond any legitimate
// wait in these kernels (a few microseconds) and well under a second.
#define CATS_SPIN_LIMIT (1u << 22)

__host__ __device__ inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
__host__ __device__ inline int cdiv(int a, int b) { return (a + b - 1) / b; }

// A kernel's dynamic shared-memory limit is an attribute of the kernel on one
// device: raising it on device 0 leaves it at the default on device 1.  Each
// call site keeps one bit per device ordinal (ordinals >= 64 set the
// attribute on every call); concurrent first calls both set it, which is
// harmless because the value is the same.
template <class F>
inline cudaError_t once_per_device(unsigned long long &mask, F &&set_attr)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = dev >= 0 && dev < 64 ? 1ull << dev : 0ull;
    if (bit && (__atomic_load_n(&mask, __ATOMIC_ACQUIRE) & bit)) return cudaSuccess;
    e = set_attr();
    if (e == cudaSuccess && bit) __atomic_fetch_or(&mask, bit, __ATOMIC_RELEASE);
    return e;
}

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Invalidate an mbarrier before its shared memory is used for anything else
// (the next kernel on this SM reuses the bytes for other data).
__device__ __forceinline__ void mbar_inval(uint64_t *bar)
{
    asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase; returns false (and records `code` in the
// error word) if the phase did not complete within CATS_SPIN_LIMIT polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err, int code)
{
    for (uint32_t i = 0; i < CATS_SPIN_LIMIT; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (i > 64) __nanosleep(32);
    }
    if (err) atomicOr(err, code);
    return false;
}

// L2 policy for streamed-once weights: evict first so activations, the KV cache
// and the next kernel's prefetch keep their L2 lines.
__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> shared (TMA engine), completion counted on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16.  Never multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Programmatic dependent launch: wait for the upstream grid's memory, and let
// the downstream grid start its (weight-prefetching) prologue.
__device__ __forceinline__ void pdl_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// dp4a with unsigned bytes in a and signed bytes in b
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c)
{
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(int a, int b, int c)
{
    return __dp4a(a, b, c);
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h)
{
    return __half2float(__ushort_as_half(h));
}

// Greedy-argmax key: larger key wins; among equal values the lower index wins
// (sample_argmax keeps the first maximum, llm/catseye_llm.h:1944-1956).
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx)
{
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (uint32_t)(0x7fffffff - idx);
}

} // namespace cats
