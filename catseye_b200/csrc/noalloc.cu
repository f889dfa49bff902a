// noalloc.cu — the device sgemm for callers that cannot allocate device memory.
//
// cats_sgemm_dev may split K across CTAs for skinny problems; the partial
// sums then need a workspace, which it grows with cudaMalloc.  Some callers
// cannot let a library do that: a process whose device memory is already
// owned by another allocator (a framework's caching allocator that reserved
// the pool), or a latency-critical loop where cudaMalloc's implicit
// device-wide synchronisation is not acceptable.  cats_sgemm_dev_noalloc does
// the same arithmetic with its split-K workspace in a fixed array compiled
// into the library, and allocates nothing.
#include "../../include/catsgpu.h"
#include "sgemm.cuh"
#include <cstdio>

namespace cats {
int capi_fail(int code, const char *what);   // sticky status (capi.cu)
}

using namespace cats;

namespace {

// Split-K workspace shared by every call on a device.  Every GPU that loads
// the library holds these CATS_SGEMM_NOALLOC_SCRATCH_FLOATS floats (8 MiB)
// until the process exits.  In host code the symbol is only a host-side
// stand-in: the device address comes from cudaGetSymbolAddress below.
__device__ __align__(256) float g_splitk_scratch[CATS_SGEMM_NOALLOC_SCRATCH_FLOATS];
// Status word of the tensor-core kernel's bounded waits for these calls (the
// library's own error word is allocated by cats_gpu_init, which this entry
// point does not call).  Zero at load; cats_gpu_device_error reads it.
__device__ int g_noalloc_status;

constexpr int MAX_DEVICES = 64;
float *g_scratch_addr[MAX_DEVICES] = {};   // device address of g_splitk_scratch, per device ordinal
int *g_status_addr[MAX_DEVICES] = {};      // device address of g_noalloc_status, per device ordinal
int g_scratch_sms[MAX_DEVICES] = {};

// Once per device, with that device current: resolve the arrays' device
// addresses and the SM count.  None of these calls allocates.
int scratch_setup(int dev)
{
    if (g_scratch_addr[dev]) return CATS_OK;
    float *p = nullptr;
    int *st = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void **>(&p), g_splitk_scratch);
    if (e != cudaSuccess || !p) return capi_fail(CATS_ERR_CUDA, "cats_sgemm_dev_noalloc: cudaGetSymbolAddress");
    e = cudaGetSymbolAddress(reinterpret_cast<void **>(&st), g_noalloc_status);
    if (e != cudaSuccess || !st) return capi_fail(CATS_ERR_CUDA, "cats_sgemm_dev_noalloc: cudaGetSymbolAddress");
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess || sms <= 0) return capi_fail(CATS_ERR_CUDA, "cats_sgemm_dev_noalloc: SM count");
    g_scratch_sms[dev] = sms;
    g_status_addr[dev] = st;
    g_scratch_addr[dev] = p;
    return CATS_OK;
}

int current_device()
{
    int dev = -1;
    return cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < MAX_DEVICES ? dev : -1;
}

} // namespace

namespace cats {
// CATS_DEVERR_* bits the no-allocation sgemm's kernels left on the current
// device (0 when it never ran there); clear = reset them to 0.  Reads and
// writes the word with plain copies, which allocate nothing.
int noalloc_device_error(bool clear)
{
    const int dev = current_device();
    if (dev < 0 || !g_status_addr[dev]) return 0;
    int h = 0;
    if (cudaMemcpy(&h, g_status_addr[dev], 4, cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
    if (clear && h) cudaMemset(g_status_addr[dev], 0, 4);
    return h;
}
} // namespace cats

extern "C" int cats_sgemm_dev_noalloc(char ta, char tb, int m, int n, int k, float alpha, const float *a, int lda,
                                      const float *b, int ldb, float beta, float *c, int ldc, void *stream)
{
    const char *what = "cats_sgemm_dev_noalloc";
    const bool at = ta == 'T' || ta == 't', bt = tb == 'T' || tb == 't';
    if ((!at && ta != 'N' && ta != 'n') || (!bt && tb != 'N' && tb != 'n') || m < 0 || n < 0 || k < 0)
        return capi_fail(CATS_ERR_ARG, what);
    if (m == 0 || n == 0) return CATS_OK;
    if (!c || (k > 0 && (!a || !b)) || ldc < n || (k > 0 && (lda < (at ? m : k) || ldb < (bt ? k : n))))
        return capi_fail(CATS_ERR_ARG, what);
    const int dev = current_device();
    if (dev < 0) return capi_fail(CATS_ERR_CUDA, "cats_sgemm_dev_noalloc: no current device");
    if (int rc = scratch_setup(dev)) return rc;
    // the plan fits its K splits to the array (fewer splits, down to none)
    const SgemmPlan p = sgemm_plan(m, n, k, g_scratch_sms[dev], CATS_SGEMM_NOALLOC_SCRATCH_FLOATS);
    if (p.work_floats > (size_t)CATS_SGEMM_NOALLOC_SCRATCH_FLOATS) {   // defensive: the plan honours the cap
        char msg[160];
        snprintf(msg, sizeof msg,
                 "cats_sgemm_dev_noalloc: %dx%dx%d needs %zu split-K workspace floats, the fixed array holds %d",
                 m, n, k, p.work_floats, (int)CATS_SGEMM_NOALLOC_SCRATCH_FLOATS);
        return capi_fail(CATS_ERR_ARG, msg);
    }
    // Each split writes every element of its partial slab before the reduce
    // reads it, so nothing left in the array by an earlier call is ever used.
    const cudaError_t e = launch_sgemm(p, at, bt, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc,
                                       g_scratch_addr[dev], g_status_addr[dev], static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? CATS_OK : capi_fail(CATS_ERR_CUDA, what);
}
