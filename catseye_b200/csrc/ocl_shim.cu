// ocl_shim.cu — the library side of include/cats_ocl_cuda.h: the device
// buffer and the three kernels of catseye's OpenCL sgemm backend
// (sgemm_ocl2.h), by name, over this library.
//
// sgemm_ocl (sgemm_ocl2.h:208-261) packs A, B and C into one buffer, runs
// "transpose" for a T operand (input [Q][P] at float offset s2 -> output
// [P][Q] at s3, :94-126), then "gemm_rnn" on row-major operands at float
// offsets s3, s4, s5 with alpha = param.s0, beta = param.s1 (C read only when
// beta != 0, :14-90).  A transpose is not copied here: its output offset is
// remembered, and the GEMM that reads that offset takes the untransposed
// source in its 'T' form (cats_sgemm_dev), which is the same product.
#include "../../include/catsgpu.h"
#include "common.cuh"
#include "conv.cuh"
#include <cstdlib>
#include <cstring>

namespace cats {
int capi_fail(int code, const char *what);
cudaStream_t capi_stream();
}
using namespace cats;

namespace {

struct PendingT {
    void *buf;
    int dst, src, P, Q;   // float offsets; source [Q][P] whose [P][Q] transpose "is" at dst
};
PendingT g_pending[4];
int g_npending = 0;

const PendingT *pending(void *buf, int off)
{
    for (int i = 0; i < g_npending; i++)
        if (g_pending[i].buf == buf && g_pending[i].dst == off) return &g_pending[i];
    return nullptr;
}

} // namespace

extern "C" {

unsigned long cats_ocl_setup(int device)
{
    if (cats_gpu_init(device) != CATS_OK) return 0;
    const char *e = getenv("CATS_OCL_BUFFER_BYTES");
    const unsigned long long v = e ? strtoull(e, nullptr, 10) : 0ull;
    return (unsigned long)(v ? v : 1ull << 30);
}

void *cats_ocl_alloc(size_t bytes)
{
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        capi_fail(CATS_ERR_NOMEM, "cats_ocl_alloc");
        return nullptr;
    }
    return p;
}

void cats_ocl_free(void *p)
{
    if (p) cudaFree(p);
    g_npending = 0;
}

// Copies go on the library's stream, the one the GEMMs run on, and are waited
// for: a plain cudaMemcpy from pageable memory may return before its data has
// landed, and it is not ordered with that (non-blocking) stream.
int cats_ocl_write(void *buf, size_t off, size_t size, const void *host)
{
    if (!buf || !host) return capi_fail(CATS_ERR_ARG, "cats_ocl_write");
    cudaStream_t st = capi_stream();
    const bool ok = cudaMemcpyAsync(static_cast<uint8_t *>(buf) + off, host, size, cudaMemcpyHostToDevice, st) ==
                        cudaSuccess &&
                    cudaStreamSynchronize(st) == cudaSuccess;
    return ok ? CATS_OK : capi_fail(CATS_ERR_CUDA, "cats_ocl_write");
}

int cats_ocl_read(void *buf, size_t off, size_t size, void *host)
{
    if (!buf || !host) return capi_fail(CATS_ERR_ARG, "cats_ocl_read");
    cudaStream_t st = capi_stream();
    const bool ok = cudaMemcpyAsync(host, static_cast<const uint8_t *>(buf) + off, size, cudaMemcpyDeviceToHost, st) ==
                        cudaSuccess &&
                    cudaStreamSynchronize(st) == cudaSuccess;
    return ok ? CATS_OK : capi_fail(CATS_ERR_CUDA, "cats_ocl_read");
}

int cats_ocl_run(const char *kernel, void *buf, const int *info, const float *param)
{
    if (!kernel || !buf || !info) return capi_fail(CATS_ERR_ARG, "cats_ocl_run");
    float *gm = static_cast<float *>(buf);
    if (!strcmp(kernel, "transpose")) {
        if (g_npending == 4) g_npending = 0;
        g_pending[g_npending++] = PendingT{buf, info[3], info[2], info[0], info[1]};
        return CATS_OK;
    }
    if (!strcmp(kernel, "gemm_rnn")) {
        if (!param) return capi_fail(CATS_ERR_ARG, "cats_ocl_run");
        const int M = info[0], N = info[1], K = info[2];
        const PendingT *ta = pending(buf, info[3]), *tb = pending(buf, info[4]);
        // A^T written [M][K] from [K][M]: the 'T' form of the source (P = M, Q = K)
        const float *A = gm + (ta ? ta->src : info[3]);
        const float *B = gm + (tb ? tb->src : info[4]);
        int rc = cats_sgemm_dev(ta ? 'T' : 'N', tb ? 'T' : 'N', M, N, K, param[0], A, ta ? M : K, B, tb ? K : N,
                                param[1], gm + info[5], N, nullptr);
        g_npending = 0;
        if (rc) return rc;
        return cudaStreamSynchronize(capi_stream()) == cudaSuccess ? CATS_OK : capi_fail(CATS_ERR_CUDA, "cats_ocl_run");
    }
    if (!strcmp(kernel, "im2col")) {   // sgemm_ocl2.h:128-168 (square kernel, pad and stride)
        int rc = cats_im2col_dev(gm + info[0], info[1], info[2], info[3], info[4], info[4], info[5], info[5], info[6],
                                 info[6], gm + info[7], nullptr);
        if (rc) return rc;
        return cudaStreamSynchronize(capi_stream()) == cudaSuccess ? CATS_OK : capi_fail(CATS_ERR_CUDA, "cats_ocl_run");
    }
    return capi_fail(CATS_ERR_UNSUPPORTED, "cats_ocl_run: kernel name");
}

} // extern "C"
