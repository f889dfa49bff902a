// kquant.cuh — Q3_K / Q6_K weights against Q8_K activations (kquant.cu).
#pragma once
#include "common.cuh"

namespace cats {

// quantize_q8_K of x[n] (n % 256 == 0) into n/256 blocks of 260 bytes
// {int8 q[256]; float d}, bit-exact with the reference.
cudaError_t launch_quantize_q8_K(uint8_t *y, const float *x, int n, cudaStream_t st);

// out[d] = W x for a Q3_K / Q6_K weight in the reference's row layout and a
// Q8_K activation (n/256 blocks).
cudaError_t launch_matvec_kquant(int type, float *out, const uint8_t *xq, const uint8_t *w, int n, int d,
                                 cudaStream_t st);

// `rows` rows of a Q3_K / Q6_K weight into fp32 (bit-exact).
cudaError_t launch_dequantize_kquant(int type, float *y, const uint8_t *w, int n, int rows, cudaStream_t st);

} // namespace cats
