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

// ---- training (the GEMMs themselves run through launch_sgemm)
// col2im (catseye.h:533-556) of `batch` images whose columns are [k][b*P + p]
// with rows col_ld floats apart (one image: batch 1, col_ld = P); a gather in
// the reference's summation order, so bit-exact.
cudaError_t launch_col2im(const float *col, long long col_ld, int batch, int channels, int height, int width, int kh,
                          int kw, int ph, int pw, int sh, int sw, float *im, cudaStream_t st);
// im2col (catseye.h:508-532) of x[b][c][h][w] for every sample, into col[k][b*P + p]
cudaError_t launch_im2col_cols(const float *x, int batch, int channels, int height, int width, int kh, int kw, int ph,
                               int pw, int sh, int sw, float *col, cudaStream_t st);
// dst[c][b][p] = src[b][c][p]
cudaError_t launch_batch_to_channel_major(const float *src, int batch, int ch, int P, float *dst, cudaStream_t st);
// bias[o] -= eta * dout[b][o], b in order (CatsEye_linear_update's bias step, catseye.h:494-496)
cudaError_t launch_bias_update(float *bias, const float *dout, int batch, int out, float eta, cudaStream_t st);

} // namespace cats
