// qgemm.cuh — batched quantized-weight product on the tensor cores (tcgen05).
#pragma once
#include "matvec.cuh"
#include <cuda_fp16.h>

namespace cats {

// Weights qgemm handles: Q4_0 / Q8_0 in the tile layout, n a multiple of 64.
bool qgemm_supported(const WeightLayout &L);

// Bytes of the fp16 activation scratch launch_qgemm needs for T tokens.
size_t qgemm_x16_bytes(int n, int T);

// Y[T][d] = X[T][n] * W[d][n]^T with fp16 operands and fp32 accumulation.
// x (fp32, 16-byte aligned) is converted into x16 (qgemm_x16_bytes) first.
cudaError_t launch_qgemm(const WeightLayout &L, const uint8_t *w, const float *x, __half *x16, float *y, int T,
                         int *err, cudaStream_t st);

size_t qgemm_smem_bytes(int bn);

} // namespace cats
