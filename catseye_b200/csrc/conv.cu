// conv.cu — the CNN forward callers of the GEMM on CUDA cores.
//
// The reference's convolution forward (CatsEye_convolutional_forward,
// catseye.h:557-588) runs, per sample, im2col (catseye.h:508-532) into a
// [ich*k*k][oh*ow] workspace and gemm_rnn(ch, oh*ow, ich*k*k) into z.  Here
// the whole batch is one implicit GEMM: M = ch, N = batch*oh*ow, K = ich*k*k,
// with the B operand gathered from the images while a tile is loaded, so the
// im2col matrix never exists in memory.  Tiling follows sgemm.cu (8-deep
// k-slabs, double-buffered shared memory, 256 threads, 8 columns per thread);
// the M tile is 64 rows when ch <= 64, so 64-channel layers waste no work.
// The output goes to z[b][ch][oh*ow], the reference's per-sample CHW order.
#include "conv.cuh"
#include <algorithm>

namespace cats {

constexpr int CV_BN = 128, CV_BK = 8, CV_NT = 256;

__global__ void k_im2col(const float *__restrict__ im, int channels, int height, int width, int kh, int kw, int ph,
                         int pw, int sh, int sw, int hc, int wc, float *__restrict__ col)
{
    const long long total = (long long)channels * kh * kw * hc * wc;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const int x = (int)(idx % wc);
        const long long r = idx / wc;
        const int y = (int)(r % hc);
        const int c = (int)(r / hc);
        const int wo = c % kw, ho = (c / kw) % kh, ci = c / kh / kw;
        const int yp = y * sh - ph + ho, xp = x * sw - pw + wo;
        col[idx] = (yp >= 0 && yp < height && xp >= 0 && xp < width) ? im[((size_t)ci * height + yp) * width + xp] : 0.f;
    }
}

cudaError_t launch_im2col(const float *im, int channels, int height, int width, int kh, int kw, int ph, int pw,
                          int sh, int sw, float *col, cudaStream_t st)
{
    const int hc = conv_out(height, kh, ph, sh), wc = conv_out(width, kw, pw, sw);
    const long long total = (long long)channels * kh * kw * hc * wc;
    if (total <= 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    k_im2col<<<grid, 256, 0, st>>>(im, channels, height, width, kh, kw, ph, pw, sh, sw, hc, wc, col);
    return cudaGetLastError();
}

struct ConvArgs {
    const float *x, *w;
    float *z;
    int ich, h, wd, ch, ks, pad, stride, oh, ow, K;
    long long N;   // batch * oh * ow
};

// BM output channels x 128 output pixels per CTA.
template <int BM>
__global__ void __launch_bounds__(CV_NT, 2) k_conv_fwd(const __grid_constant__ ConvArgs a)
{
    constexpr int TM = BM / 16;          // rows per thread (8 or 4)
    constexpr int EA = BM * CV_BK / CV_NT;   // A elements a thread loads per slab (4 or 2)
    __shared__ __align__(16) float As[2][CV_BK][BM];
    __shared__ __align__(16) float Bs[2][CV_BK][CV_BN];
    const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
    const int m0 = blockIdx.y * BM;
    const long long n0 = (long long)blockIdx.x * CV_BN;
    const int ohw = a.oh * a.ow, kk2 = a.ks * a.ks;

    // this thread's four B columns: sample base pointer and the input corner
    const float *xb[4];
    int iy0[4], ix0[4];
    bool nv[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const long long n = n0 + (t & 31) * 4 + j;
        nv[j] = n < a.N;
        const long long nn = nv[j] ? n : 0;
        const int b = (int)(nn / ohw), p = (int)(nn % ohw);
        xb[j] = a.x + (size_t)b * a.ich * a.h * a.wd;
        iy0[j] = (p / a.ow) * a.stride - a.pad;
        ix0[j] = (p % a.ow) * a.stride - a.pad;
    }
    const int am = t / (CV_BK / EA), ak = (t % (CV_BK / EA)) * EA;   // A: row, first k of the thread
    const int bk = t >> 5;                                           // B: k row of the thread

    float ra[EA], rb[4];
    auto load = [&](int k0) {
#pragma unroll
        for (int i = 0; i < EA; i++) {
            const int m = m0 + am, k = k0 + ak + i;
            ra[i] = (m < a.ch && k < a.K) ? a.w[(size_t)m * a.K + k] : 0.f;
        }
        const int k = k0 + bk;
        const int ci = k / kk2, r = k - ci * kk2, ky = r / a.ks, kx = r - ky * a.ks;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int iy = iy0[j] + ky, ix = ix0[j] + kx;
            rb[j] = (nv[j] && k < a.K && iy >= 0 && iy < a.h && ix >= 0 && ix < a.wd)
                        ? xb[j][((size_t)ci * a.h + iy) * a.wd + ix]
                        : 0.f;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int i = 0; i < EA; i++) As[buf][ak + i][am] = ra[i];
        *reinterpret_cast<float4 *>(&Bs[buf][bk][(t & 31) * 4]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
    };

    float acc[TM][8];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

    int buf = 0;
    load(0);
    store(0);
    __syncthreads();
    for (int k0 = 0; k0 < a.K; k0 += CV_BK) {
        const bool more = k0 + CV_BK < a.K;
        if (more) load(k0 + CV_BK);
#pragma unroll
        for (int kk = 0; kk < CV_BK; kk++) {
            float av[TM], bv[8];
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4]);
            av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
            if (TM == 8) {
                const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][64 + ty * 4]);
                av[TM - 4] = a1.x; av[TM - 3] = a1.y; av[TM - 2] = a1.z; av[TM - 1] = a1.w;
            }
            const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][64 + tx * 4]);
            bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
            bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (more) {
            store(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }

    // z[b][m][p] for column n = b*oh*ow + p
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const long long n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
        if (n >= a.N) continue;
        const int b = (int)(n / ohw), p = (int)(n % ohw);
        float *zb = a.z + (size_t)b * a.ch * ohw + p;
#pragma unroll
        for (int i = 0; i < TM; i++) {
            const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
            if (m < a.ch) zb[(size_t)m * ohw] = acc[i][j];
        }
    }
}

cudaError_t launch_conv2d_forward(const float *x, const float *w, float *z, int batch, int ich, int h, int wd, int ch,
                                  int ks, int pad, int stride, int *err, float *wperm, cudaStream_t st)
{
    if (conv_tc_usable(w, batch, ich, h, wd, ch, ks, pad, stride))
        return launch_conv_tc(x, w, z, batch, ich, h, wd, ch, ks, pad, stride, err, wperm, st);
    ConvArgs a;
    a.x = x;
    a.w = w;
    a.z = z;
    a.ich = ich;
    a.h = h;
    a.wd = wd;
    a.ch = ch;
    a.ks = ks;
    a.pad = pad;
    a.stride = stride;
    a.oh = conv_out(h, ks, pad, stride);
    a.ow = conv_out(wd, ks, pad, stride);
    a.K = ich * ks * ks;
    a.N = (long long)batch * a.oh * a.ow;
    if (a.N <= 0 || ch <= 0) return cudaSuccess;
    const long long tn = (a.N + CV_BN - 1) / CV_BN;
    if (tn > 0x7fffffffLL) return cudaErrorInvalidValue;
    if (ch <= 64) {
        k_conv_fwd<64><<<dim3((unsigned)tn, 1), CV_NT, 0, st>>>(a);
    } else {
        k_conv_fwd<128><<<dim3((unsigned)tn, cdiv(ch, 128)), CV_NT, 0, st>>>(a);
    }
    return cudaGetLastError();
}

__global__ void k_bias_rows(const float *__restrict__ bias, float *__restrict__ z, int batch, int out)
{
    const long long total = (long long)batch * out;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x)
        z[i] = bias[i % out];
}

cudaError_t launch_bias_rows(const float *bias, float *z, int batch, int out, cudaStream_t st)
{
    const long long total = (long long)batch * out;
    if (total <= 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((total + 255) / 256, 148LL * 8);
    k_bias_rows<<<grid, 256, 0, st>>>(bias, z, batch, out);
    return cudaGetLastError();
}

// ------------------------------------------------------------- training
// col2im as a gather: each image element sums the column entries that cover
// it, in the order the reference's scatter adds them (column row k =
// (c*kh + i)*kw + j ascending, catseye.h:533-556), starting from zero as its
// memset does, so the sums are the reference's bit for bit.  No atomics: the
// result does not depend on scheduling.  Columns of sample b start at b*P
// of each column row (row length col_ld): the batched layout [k][b][P].
__global__ void k_col2im(const float *__restrict__ col, long long col_ld, int batch, int channels, int height,
                         int width, int kh, int kw, int ph, int pw, int sh, int sw, int hc, int wc,
                         float *__restrict__ im)
{
    const long long total = (long long)batch * channels * height * width;
    const int P = hc * wc;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const int x = (int)(idx % width);
        long long r = idx / width;
        const int y = (int)(r % height);
        r /= height;
        const int c = (int)(r % channels);
        const int b = (int)(r / channels);
        const float *cb = col + (long long)b * P;
        float sum = 0.f;
        for (int i = 0; i < kh; i++) {
            const int ty = y + ph - i;
            if (ty < 0 || ty % sh) continue;
            const int oy = ty / sh;
            if (oy >= hc) continue;
            for (int j = 0; j < kw; j++) {
                const int tx = x + pw - j;
                if (tx < 0 || tx % sw) continue;
                const int ox = tx / sw;
                if (ox >= wc) continue;
                sum += cb[(long long)((c * kh + i) * kw + j) * col_ld + oy * wc + ox];
            }
        }
        im[idx] = sum;
    }
}

cudaError_t launch_col2im(const float *col, long long col_ld, int batch, int channels, int height, int width, int kh,
                          int kw, int ph, int pw, int sh, int sw, float *im, cudaStream_t st)
{
    const int hc = conv_out(height, kh, ph, sh), wc = conv_out(width, kw, pw, sw);
    const long long total = (long long)batch * channels * height * width;
    if (total <= 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    k_col2im<<<grid, 256, 0, st>>>(col, col_ld, batch, channels, height, width, kh, kw, ph, pw, sh, sw, hc, wc, im);
    return cudaGetLastError();
}

// im2col of a batch into the columns [k][b*P + p] (catseye.h:508-532 per sample)
__global__ void k_im2col_cols(const float *__restrict__ x, int batch, int channels, int height, int width, int kh,
                              int kw, int ph, int pw, int sh, int sw, int hc, int wc, float *__restrict__ col)
{
    const int P = hc * wc;
    const long long N = (long long)batch * P;
    const long long total = (long long)channels * kh * kw * N;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const long long n = idx % N;
        const int k = (int)(idx / N);
        const int b = (int)(n / P), p = (int)(n % P);
        const int ox = p % wc, oy = p / wc;
        const int j = k % kw, i = (k / kw) % kh, c = k / kh / kw;
        const int yp = oy * sh - ph + i, xp = ox * sw - pw + j;
        col[idx] = (yp >= 0 && yp < height && xp >= 0 && xp < width)
                       ? x[(((size_t)b * channels + c) * height + yp) * width + xp]
                       : 0.f;
    }
}

cudaError_t launch_im2col_cols(const float *x, int batch, int channels, int height, int width, int kh, int kw, int ph,
                               int pw, int sh, int sw, float *col, cudaStream_t st)
{
    const int hc = conv_out(height, kh, ph, sh), wc = conv_out(width, kw, pw, sw);
    const long long total = (long long)channels * kh * kw * batch * hc * wc;
    if (total <= 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    k_im2col_cols<<<grid, 256, 0, st>>>(x, batch, channels, height, width, kh, kw, ph, pw, sh, sw, hc, wc, col);
    return cudaGetLastError();
}

// dst[c][b][p] = src[b][c][p]: the per-sample CHW gradients as one [ch][batch*P] operand
__global__ void k_batch_to_channel_major(const float *__restrict__ src, int batch, int ch, int P,
                                         float *__restrict__ dst)
{
    const long long total = (long long)batch * ch * P;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const int p = (int)(idx % P);
        const long long r = idx / P;
        const int b = (int)(r % batch), c = (int)(r / batch);
        dst[idx] = src[((size_t)b * ch + c) * P + p];
    }
}

cudaError_t launch_batch_to_channel_major(const float *src, int batch, int ch, int P, float *dst, cudaStream_t st)
{
    const long long total = (long long)batch * ch * P;
    if (total <= 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    k_batch_to_channel_major<<<grid, 256, 0, st>>>(src, batch, ch, P, dst);
    return cudaGetLastError();
}

// bias[o] -= eta * dout[b][o] for b = 0, 1, ... in order (catseye.h:494-496)
__global__ void k_bias_update(float *__restrict__ bias, const float *__restrict__ dout, int batch, int out, float eta)
{
    for (int o = blockIdx.x * blockDim.x + threadIdx.x; o < out; o += gridDim.x * blockDim.x) {
        float v = bias[o];
        for (int b = 0; b < batch; b++) v -= eta * dout[(size_t)b * out + o];
        bias[o] = v;
    }
}

cudaError_t launch_bias_update(float *bias, const float *dout, int batch, int out, float eta, cudaStream_t st)
{
    if (out <= 0 || batch <= 0) return cudaSuccess;
    const int grid = std::min(cdiv(out, 256), 148 * 4);
    k_bias_update<<<grid, 256, 0, st>>>(bias, dout, batch, out, eta);
    return cudaGetLastError();
}

} // namespace cats
