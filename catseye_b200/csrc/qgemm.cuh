// qgemm.cuh — batched quantized-weight product on the tensor cores (tcgen05).
#pragma once
#include "matvec.cuh"
#include <cuda_fp16.h>

namespace cats {

// Weights qgemm handles: Q4_0 / Q8_0 in the tile layout, n a multiple of 64.
bool qgemm_supported(const WeightLayout &L);

// Y[T][d] = X16[T][n] * W[d][n]^T with fp16 operands and fp32 accumulation.
cudaError_t launch_qgemm(const WeightLayout &L, const uint8_t *w, const __half *x16, float *y, int T, int *err,
                         cudaStream_t st);

// y = fp16(x), round to nearest
cudaError_t launch_f32_to_f16(const float *x, __half *y, long long n, cudaStream_t st);

size_t qgemm_smem_bytes(int bn);

} // namespace cats
