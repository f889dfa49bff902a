// kquant.cu — the K-quant path of the llm runtime: Q3_K and Q6_K weights
// (256-element super-blocks) against Q8_K activations.
//
// Reference: quantize_q8_K (llm/catseye_llm.h:262-296), the dequantizers
// (:349-426) and the dots dot_q3_K_q8_K / dot_q6_K_q8_K (:1057-1261,
// 1332-1511) bound through gguf_matmul[] (:2583-2607).  Real Q4_0 GGUF files
// often carry a Q6_K output.weight, so a runtime that loads them needs these.
// Weights stay in the reference's GGUF row layout on the device (no repack):
//   Q3_K (110 B): hmask[32], qs[64] (2-bit codes), scales[12] (16 six-bit
//                 scales), d (fp16); value = d * (scale - 32) * (low2 - (hbit ? 0 : 4))
//   Q6_K (210 B): ql[128] (low nibbles), qh[64] (2 high bits), scales[16]
//                 (int8), d (fp16); value = d * scale * (6-bit code - 32)
//   Q8_K (260 B): int8 q[256], float d
// Matvec: one warp per row, super-block by super-block.  Lane L unpacks the
// eight codes 8L..8L+7 (group L/2 of 16 shares one scale), dots them with
// the activation bytes by dp4a; the block's integer sum is reduced exactly
// and scaled by the float product d_w * d_x, as the reference does.
#include "kquant.cuh"
#include <algorithm>

namespace cats {

constexpr int KQ_WARPS = 8;

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// ---------------------------------------------------------- quantize_q8_K
// One warp per 256-element block, 8 elements per lane.  The signed maximum
// is the element of largest magnitude, the first one on ties; iscale =
// -128/max in double rounded to float; q = round-half-even(iscale * x),
// at most 127; d = 1/iscale (:262-296).
__global__ void k_quantize_q8_K(uint8_t *__restrict__ y, const float *__restrict__ x, int nblocks)
{
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= nblocks) return;   // whole warps leave together
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)b * 256 + 8 * lane);
    const float4 v0 = src[0], v1 = src[1];
    const float e[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float amax = 0.f, mx = 0.f;
    int at = 1 << 30;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const float ax = fabsf(e[k]);
        if (ax > amax) { amax = ax; mx = e[k]; at = 8 * lane + k; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const float om = __shfl_xor_sync(0xffffffffu, mx, o);
        const int ot = __shfl_xor_sync(0xffffffffu, at, o);
        if (oa > amax || (oa == amax && ot < at)) { amax = oa; mx = om; at = ot; }
    }
    uint8_t *dst = y + (size_t)b * 260;
    uint32_t *dw = reinterpret_cast<uint32_t *>(dst);   // blocks are 260 bytes: 4-byte aligned only
    if (amax == 0.f) {
        dw[2 * lane] = 0u;
        dw[2 * lane + 1] = 0u;
        if (lane == 0) *reinterpret_cast<float *>(dst + 256) = 0.f;
        return;
    }
    const float iscale = (float)(-128.0 / (double)mx);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int q = min(127, __float2int_rn(__fmul_rn(iscale, e[k])));
        w[k >> 2] |= (uint32_t)(q & 0xff) << (8 * (k & 3));
    }
    dw[2 * lane] = w[0];
    dw[2 * lane + 1] = w[1];
    if (lane == 0) *reinterpret_cast<float *>(dst + 256) = __fdiv_rn(1.f, iscale);
}

cudaError_t launch_quantize_q8_K(uint8_t *y, const float *x, int n, cudaStream_t st)
{
    if (n <= 0 || n % 256) return cudaErrorInvalidValue;
    const int nb = n / 256;
    k_quantize_q8_K<<<cdiv(nb, 8), 256, 0, st>>>(y, x, nb);
    return cudaGetLastError();
}

// ------------------------------------------------------------ code unpack
// The 16 six-bit Q3_K scales from their 12 packed bytes (:360-368), minus 32.
__device__ __forceinline__ int q3k_scale(const uint8_t *sc12, int g)
{
    // scale g: low 4 bits from byte g (g < 8) low nibble or byte g - 8 high
    // nibble; high 2 bits from byte 8 + (g & 3), bits 2 * (g >> 2)
    const int lo = g < 8 ? (sc12[g] & 0xF) : (sc12[g - 8] >> 4);
    const int hi = (sc12[8 + (g & 3)] >> (2 * (g >> 2))) & 3;
    return (lo | (hi << 4)) - 32;
}

// Lane L's eight codes (elements 8L..8L+7) of a super-block as int8 in two
// words, and the scale of their 16-element group.
template <int WT>
__device__ __forceinline__ void unpack8(const uint8_t *blk, int lane, uint32_t (&q)[2], int &scale)
{
    const int l0 = 8 * (lane & 3);   // position within the 32-element run
    if (WT == W_Q3_K) {
        const int half = lane >> 4, s = (lane >> 2) & 3;
        const uint8_t *hm = blk, *qs = blk + 32 + 32 * half;
        const uint32_t mbit = 1u << (4 * half + s);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int low2 = (qs[l0 + k] >> (2 * s)) & 3;
            const int v = low2 - ((hm[l0 + k] & mbit) ? 0 : 4);
            q[k >> 2] = (k & 3) ? q[k >> 2] | ((uint32_t)(v & 0xff) << (8 * (k & 3))) : (uint32_t)(v & 0xff);
        }
        scale = q3k_scale(blk + 96, lane >> 1);
    } else {
        const int h = lane >> 4, part = (lane >> 2) & 3;
        const uint8_t *ql = blk + 64 * h + 32 * (part & 1), *qh = blk + 128 + 32 * h;
        const int lsh = 4 * (part >> 1), hsh = 2 * part;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int v = (((ql[l0 + k] >> lsh) & 0xF) | (((qh[l0 + k] >> hsh) & 3) << 4)) - 32;
            q[k >> 2] = (k & 3) ? q[k >> 2] | ((uint32_t)(v & 0xff) << (8 * (k & 3))) : (uint32_t)(v & 0xff);
        }
        scale = (int)(int8_t)blk[192 + (lane >> 1)];
    }
}

template <int WT>
__device__ __forceinline__ float kq_d(const uint8_t *blk)
{
    return half_bits_to_float(ld_u16(blk + (WT == W_Q3_K ? 108 : 208)));
}

// --------------------------------------------------------------- matvec
template <int WT>
__global__ void __launch_bounds__(32 * KQ_WARPS) k_matvec_kquant(float *__restrict__ out, const uint8_t *__restrict__ xq,
                                                                 const uint8_t *__restrict__ w, int n, int d)
{
    constexpr int BS = WT == W_Q3_K ? 110 : 210;
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * KQ_WARPS + (threadIdx.x >> 5);
    if (row >= d) return;   // whole warps leave together
    const int nb = n / 256;
    const uint8_t *wr = w + (size_t)row * nb * BS;
    float acc = 0.f;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = wr + (size_t)b * BS;
        const uint8_t *y = xq + (size_t)b * 260;
        uint32_t q[2];
        int sc;
        unpack8<WT>(blk, lane, q, sc);
        const uint32_t *yw = reinterpret_cast<const uint32_t *>(y + 8 * lane);   // 4-byte aligned blocks
        int part = __dp4a((int)q[0], (int)yw[0], 0);
        part = __dp4a((int)q[1], (int)yw[1], part);
        int isum = sc * part;
#pragma unroll
        for (int o = 16; o; o >>= 1) isum += __shfl_xor_sync(0xffffffffu, isum, o);
        const float delta = __fmul_rn(kq_d<WT>(blk), *reinterpret_cast<const float *>(y + 256));
        acc = fmaf(delta, (float)isum, acc);   // every lane holds the same sum
    }
    if (lane == 0) out[row] = acc;
}

cudaError_t launch_matvec_kquant(int type, float *out, const uint8_t *xq, const uint8_t *w, int n, int d,
                                 cudaStream_t st)
{
    if (n <= 0 || n % 256 || d <= 0) return cudaErrorInvalidValue;
    const int grid = cdiv(d, KQ_WARPS);
    if (type == W_Q3_K) k_matvec_kquant<W_Q3_K><<<grid, 32 * KQ_WARPS, 0, st>>>(out, xq, w, n, d);
    else if (type == W_Q6_K) k_matvec_kquant<W_Q6_K><<<grid, 32 * KQ_WARPS, 0, st>>>(out, xq, w, n, d);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

// ----------------------------------------------------------- dequantize
// One warp per super-block: value = (d * scale) * code, exact in fp32
// (:349-426).
template <int WT>
__global__ void k_dequantize_kquant(float *__restrict__ y, const uint8_t *__restrict__ w, long long nblocks)
{
    constexpr int BS = WT == W_Q3_K ? 110 : 210;
    const int lane = threadIdx.x & 31;
    for (long long b = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; b < nblocks;
         b += ((long long)gridDim.x * blockDim.x) >> 5) {
        const uint8_t *blk = w + b * BS;
        uint32_t q[2];
        int sc;
        unpack8<WT>(blk, lane, q, sc);
        const float ds = kq_d<WT>(blk) * (float)sc;
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = ds * (float)(int8_t)(q[k >> 2] >> (8 * (k & 3)));
        float4 *o = reinterpret_cast<float4 *>(y + b * 256 + 8 * lane);
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
}

cudaError_t launch_dequantize_kquant(int type, float *y, const uint8_t *w, int n, int rows, cudaStream_t st)
{
    if (n <= 0 || n % 256 || rows <= 0) return cudaErrorInvalidValue;
    const long long nb = (long long)rows * (n / 256);
    const int grid = (int)std::min<long long>((nb + 7) / 8, 148LL * 16);
    if (type == W_Q3_K) k_dequantize_kquant<W_Q3_K><<<grid, 256, 0, st>>>(y, w, nb);
    else if (type == W_Q6_K) k_dequantize_kquant<W_Q6_K><<<grid, 256, 0, st>>>(y, w, nb);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

} // namespace cats
