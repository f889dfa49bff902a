/*
 * cats_ocl_cuda.h — the OpenCL host API that catseye's OpenCL sgemm backend
 * (sgemm_ocl2.h, over ocl.h) calls, implemented over libcatsgpu.
 *
 * catseye.h selects its GEMM backend by macro (catseye.h:61-75) and includes
 * sgemm_ocl2.h by quoted path, so the header itself cannot be swapped.  This
 * header is force-included instead; an unchanged catseye program builds on
 * the B200 with
 *
 *     cc -DCATS_OPENCL -include cats_ocl_cuda.h -I<this dir> prog.c \
 *        -L<lib dir> -lcatsgpu -Wl,-rpath,<lib dir>
 *
 * It defines OCL_H_INCLUDED first, so sgemm_ocl2.h's #include "ocl.h"
 * (ocl.h:7-8) expands to nothing, and supplies the names sgemm_ocl2.h uses:
 * args_t, ocl_t, cl_mem, OCL_BUFFER, CL_MEM_READ_WRITE, OCLSTRINGIFY,
 * ceil_int, oclSetup, oclKernel, oclKernelArgs, oclWrite, oclRead, oclRun,
 * oclReleaseKernel, oclFinish (ocl.h:90-400).  The device buffer is a CUDA
 * allocation; the kernels are the library's, looked up by the name the
 * backend gives them ("gemm_rnn", "transpose", "im2col", sgemm_ocl2.h:14-169)
 * and fed the backend's own argument block (the int8 _info and float4
 * _param), so sgemm_ocl (sgemm_ocl2.h:208-261) runs unchanged: its transposes
 * are folded into the GEMM's operand forms, and the GEMM is cats_sgemm_dev on
 * the buffer.  Every call is synchronous, like the blocking OpenCL calls it
 * replaces.
 */
#ifndef CATS_OCL_CUDA_H
#define CATS_OCL_CUDA_H

#define OCL_H_INCLUDED 1   /* the reference's ocl.h: already provided */

#include <assert.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "catsgpu.h"

typedef void *cl_mem;
typedef void *cl_kernel;
typedef int cl_int;
typedef unsigned long cl_ulong;

#define CL_MEM_READ_WRITE 1
#define OCL_OUTPUT 1
#define OCL_INPUT 2
#define OCL_INPUT_ONCE 4
#define OCL_BUFFER 8
#define OCL_SVM 16
#define MAX_PLATFORMS 10
#define MAX_DEVICES 10
#define _OCL_(...) #__VA_ARGS__
#define OCLSTRINGIFY(...) #__VA_ARGS__   /* the kernel source text: kept, not compiled */

typedef struct {
    int type;
    size_t size;
    void *s;     /* host memory of a by-value argument */
    int flag;
    cl_mem p;    /* device buffer */
} args_t;

typedef struct {
    args_t *a;
    char *f;     /* kernel name */
    cl_kernel k;
    int dim;
    size_t local_size[3];
    size_t global_size[3];
} ocl_t;

static inline int ceil_int_div(int i, int div) { return (i + div - 1) / div; }
static inline int ceil_int(int i, int div) { return ceil_int_div(i, div) * div; }

/* the device, and the size of the one buffer the backend packs its operands into */
static unsigned long oclSetup(int platform, int device)
{
    (void)platform;
    const char *d = getenv("DEVICE");
    return cats_ocl_setup(d ? atoi(d) : device);
}

/* the kernels are the library's; nothing to build */
static void oclKernel(ocl_t *kernel, int n, char *opt, char *kernel_code)
{
    (void)kernel; (void)n; (void)opt; (void)kernel_code;
}

static void oclKernelArgs(ocl_t *kernel, int n)
{
    for (int i = 0; i < n; i++, kernel++)
        for (args_t *a = kernel->a; a->size; a++)
            if (a->type > 0 && a->flag == OCL_BUFFER && !a->p) {
                a->p = cats_ocl_alloc(a->size);
                assert(a->p);
            }
}

static inline void oclWrite(cl_mem mem, size_t offset, size_t size, void *p) { cats_ocl_write(mem, offset, size, p); }
static inline void oclRead(cl_mem mem, size_t offset, size_t size, void *p) { cats_ocl_read(mem, offset, size, p); }

/* a[0]: the buffer; a[1]: _info (int8); a[2]: _param (float4) */
static inline void oclRun(ocl_t *kernel)
{
    const args_t *a = kernel->a;
    cats_ocl_run(kernel->f, a[0].p, (const int *)a[1].s, (const float *)a[2].s);
}

static void oclReleaseKernel(ocl_t *kernel, int n)
{
    for (int i = 0; i < n; i++, kernel++)
        for (args_t *a = kernel->a; a->size; a++)
            if (a->type > 0 && a->p) {
                cats_ocl_free(a->p);
                a->p = 0;
            }
}

static void oclWait(void) {}
static void oclFinish(void) {}

#endif
