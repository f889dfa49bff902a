// conv.cuh — the CNN forward callers of the GEMM, on the device.
#pragma once
#include "common.cuh"

namespace cats {

// Output size of a convolution axis (catseye.h:508-532 im2col's height_col).
__host__ __device__ inline int conv_out(int in, int k, int pad, int stride) { return (in + 2 * pad - k) / stride + 1; }

// im2col of one image: col[(c*kh + i)*kw + j][oh][ow] (catseye.h:508-532).
cudaError_t launch_im2col(const float *im, int channels, int height, int width, int kh, int kw, int ph, int pw,
                          int sh, int sw, float *col, cudaStream_t st);

// Batched convolution forward, one implicit GEMM over the whole batch
// (CatsEye_convolutional_forward, catseye.h:557-588, which runs im2col +
// gemm_rnn per sample): z[b][ch][oh*ow] = sum_k w[ch][k] * im2col(x[b])[k][oh*ow],
// k = (ic*ks + i)*ks + j, no bias.
// Shapes the tensor cores take (conv_tc_usable) run as 3xTF32 on tcgen05
// (launch_conv_tc, sgemm_tc.cu); the rest on the CUDA cores.  `err` (may be
// null) receives CATS_DEVERR_* bits when a tensor-core wait times out.
// `wperm` (may be null): room for ch * ich * ks^2 floats, where the weights
// are permuted into the channel-blocked order the tensor-core path gathers
// fastest in (input channels a multiple of 32).
cudaError_t launch_conv2d_forward(const float *x, const float *w, float *z, int batch, int ich, int h, int wd, int ch,
                                  int ks, int pad, int stride, int *err, float *wperm, cudaStream_t st);

bool conv_tc_usable(const float *w, int batch, int ich, int h, int wd, int ch, int ks, int pad, int stride);
cudaError_t launch_conv_tc(const float *x, const float *w, float *z, int batch, int ich, int h, int wd, int ch, int ks,
                           int pad, int stride, int *err, float *wperm, cudaStream_t st);

// z[b][o] = w[in*out + o] (the bias the linear forward adds, catseye.h:416-444).
cudaError_t launch_bias_rows(const float *bias, float *z, int batch, int out, cudaStream_t st);

} // namespace cats
