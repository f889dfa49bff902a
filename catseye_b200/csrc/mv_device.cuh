// mv_device.cuh — device building blocks shared by the standalone matvec
// (matvec.cu) and the persistent decode kernel (decode.cu): the Q8 activation
// quantizer, activation staging into shared memory, the per-chunk dot
// products, and RoPE.
//
// Shared-memory activation layout ("xs"):
//   quantized weights: lo[units][16] int8 (elements 0-15 of each 32-block),
//                      hi[units][16] int8 (elements 16-31),
//                      dxs[units] = (float d, int sum of the 32 codes)
//   F32 weights:       float[n]
#pragma once
#include "matvec.cuh"

namespace cats {

// Eight consecutive lanes hold one 32-element block, four elements each
// (lane g of the group holds elements 4g..4g+3).  Implements the AVX
// quantize_q8 (llm/catseye_llm.h:155-225): d = amax/127 and id = 127/amax,
// both correctly rounded floats (the reference divides in double and stores
// float); q = round-half-even(x*id), saturated to int8.  scalar_mode follows
// the plain build (:227-251): id = 1/d, q = roundf(x*id).
__device__ __forceinline__ uint32_t q8_group_quant(float4 v, unsigned gmask, bool scalar_mode, float &d_out,
                                                   int &sum_out)
{
    float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    a = fmaxf(a, __shfl_xor_sync(gmask, a, 1));
    a = fmaxf(a, __shfl_xor_sync(gmask, a, 2));
    a = fmaxf(a, __shfl_xor_sync(gmask, a, 4));
    const float d = __fdiv_rn(a, 127.f);
    int q[4];
    const float e[4] = {v.x, v.y, v.z, v.w};
    if (!scalar_mode) {
        const float id = a != 0.f ? __fdiv_rn(127.f, a) : 0.f;
#pragma unroll
        for (int k = 0; k < 4; k++) q[k] = max(-128, min(127, __float2int_rn(__fmul_rn(e[k], id))));
    } else {
        const float id = d != 0.f ? (float)(1.0 / (double)d) : 0.f;
#pragma unroll
        for (int k = 0; k < 4; k++) q[k] = (int)(signed char)(int)roundf(__fmul_rn(e[k], id));
    }
    int s = q[0] + q[1] + q[2] + q[3];
    s += __shfl_xor_sync(gmask, s, 1);
    s += __shfl_xor_sync(gmask, s, 2);
    s += __shfl_xor_sync(gmask, s, 4);
    d_out = d;
    sum_out = s;
    return (uint32_t)(q[0] & 0xff) | ((uint32_t)(q[1] & 0xff) << 8) | ((uint32_t)(q[2] & 0xff) << 16) |
           ((uint32_t)(q[3] & 0xff) << 24);
}

// float4 source of the activation: plain loads between kernels, L2-coherent
// (ld.global.cg) loads for vectors other CTAs of the same kernel wrote.
struct Float4Src {
    const float4 *p;
    bool coherent;
    __device__ __forceinline__ float4 operator()(int i) const { return coherent ? __ldcg(p + i) : p[i]; }
    // elements i0, i0 + stride, ... (V of them; zero past n4), every load issued before any is used
    template <int V>
    __device__ __forceinline__ void fill(float4 (&v)[V], int i0, int stride, int n4) const
    {
#pragma unroll
        for (int k = 0; k < V; k++) {
            const int i = i0 + k * stride;
            v[k] = i < n4 ? (*this)(i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
};

// Stage the activation x[n] into xs: optional rmsnorm with norm_w
// (llm/catseye_llm.h:684-698: ss = mean(x^2) + 1e-5; o = w * (x / sqrt(ss))),
// then quantize_q8 for quantized weights or a plain copy for F32 weights.
// writeback (if set) receives the pre-norm vector.  Called by the `nthr`
// consumer threads (tid 0..nthr-1, a multiple of 32) of the CTA; synchronizes
// them on named barrier 1 before returning.
// Each thread issues all of its loads of a pass (V float4 each) before using
// any, so a pass costs one L2 round trip.  With rmsnorm the vector must fit
// one pass (n <= 4 * V * nthr; the hosts check it).
constexpr int STAGE_V = 8;

// NORM = false compiles the form without rmsnorm (norm_w must be null).
template <int WT, int V = STAGE_V, bool NORM = true, class Src>
__device__ __forceinline__ void stage_act(const Src &src, int n, const float *norm_w, float *writeback,
                                          uint8_t *xs, float *red, int tid, int nthr)
{
    if (!NORM) norm_w = nullptr;
    const int lane = tid & 31, warp = tid >> 5;
    const unsigned gmask = 0xffu << (lane & 24);
    const int units = WT == W_F32 ? n / 4 : n / 32;
    uint8_t *xlo = xs, *xhi = xs + (size_t)units * 16;
    float2 *dxs = reinterpret_cast<float2 *>(xs + (size_t)units * 32);
    const int n4 = n / 4;
    const float4 *nw4 = reinterpret_cast<const float4 *>(norm_w);
    float4 *wb4 = reinterpret_cast<float4 *>(writeback);
    for (int base = 0; base < n4; base += V * nthr) {
        float4 v[V], g[V];
#pragma unroll
        for (int k = 0; k < V; k++) {
            const int i = base + tid + k * nthr;
            g[k] = (norm_w && i < n4) ? nw4[i] : make_float4(1.f, 1.f, 1.f, 1.f);
        }
        src.template fill<V>(v, base + tid, nthr, n4);
        float scale = 1.f;
        if (norm_w) {
            float ss = 0.f;
#pragma unroll
            for (int k = 0; k < V; k++) ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            named_bar_sync(1, nthr);
            float tot = 0.f;
            for (int w = 0; w < nthr / 32; w++) tot += red[w];
            tot = __fdiv_rn(tot, (float)n);
            tot = __fadd_rn(tot, 1e-5f);
            scale = __fdiv_rn(1.f, __fsqrt_rn(tot));
        }
#pragma unroll
        for (int k = 0; k < V; k++) {
            const int i = base + tid + k * nthr;
            if (i >= n4) continue;   // whole 8-lane groups leave together (n4 % 8 == 0, nthr % 8 == 0)
            float4 x = v[k];
            if (wb4) wb4[i] = x;
            if (norm_w) {
                x.x = __fmul_rn(g[k].x, __fmul_rn(scale, x.x));
                x.y = __fmul_rn(g[k].y, __fmul_rn(scale, x.y));
                x.z = __fmul_rn(g[k].z, __fmul_rn(scale, x.z));
                x.w = __fmul_rn(g[k].w, __fmul_rn(scale, x.w));
            }
            if (WT == W_F32) {
                reinterpret_cast<float4 *>(xs)[i] = x;
            } else {
                float d;
                int s;
                const uint32_t packed = q8_group_quant(x, gmask, false, d, s);
                const int b = i >> 3, q = i & 7;
                uint8_t *dst = (q < 4 ? xlo : xhi) + (size_t)b * 16 + (q & 3) * 4;
                *reinterpret_cast<uint32_t *>(dst) = packed;
                if (q == 0) dxs[b] = make_float2(d, __int_as_float(s));
            }
        }
    }
    named_bar_sync(1, nthr);
}

// Stage n/32 reference Q8 blocks {int8 q[32]; float d} (what quantize_q8 wrote).
__device__ __forceinline__ void stage_q8_raw(const uint8_t *xq, int n, uint8_t *xs, int tid, int nthr)
{
    const int lane = tid & 31;
    const unsigned gmask = 0xffu << (lane & 24);
    const int units = n / 32;
    uint8_t *xlo = xs, *xhi = xs + (size_t)units * 16;
    float2 *dxs = reinterpret_cast<float2 *>(xs + (size_t)units * 32);
    const int nw = n / 4;   // 8 words per block
    for (int i = tid; i < nw; i += nthr) {
        const int b = i >> 3, g = i & 7;
        const uint32_t wv = *reinterpret_cast<const uint32_t *>(xq + (size_t)b * 36 + g * 4);
        int s = __dp4a((int)wv, 0x01010101, 0);
        s += __shfl_xor_sync(gmask, s, 1);
        s += __shfl_xor_sync(gmask, s, 2);
        s += __shfl_xor_sync(gmask, s, 4);
        uint8_t *dst = (g < 4 ? xlo : xhi) + (size_t)b * 16 + (g & 3) * 4;
        *reinterpret_cast<uint32_t *>(dst) = wv;
        if (g == 0) dxs[b] = make_float2(*reinterpret_cast<const float *>(xq + (size_t)b * 36 + 32), __int_as_float(s));
    }
    named_bar_sync(1, nthr);
}

// Dot one staged chunk into acc: the RPW rows of this warp, segment s
// holding `us` units (<= MV_SEG_UNITS = 64).  Lane j handles units j and
// j + 32 of the segment, so every wait for a chunk feeds 2 * RPW blocks per
// lane.  Q4_0: the low nibbles are dotted as bytes; the high nibbles are
// dotted in place (w & 0xF0F0F0F0, each code times 16) and the sum shifted
// down by 4, which is exact.
// XF (fp32 activations staged as floats, quantized weights): each weight is
// dequantized in registers, (code - offset) * d exactly, and multiplied
// with x in fp32, as matmul_q4_0 (llm/catseye_llm.h:880-914) does.
template <int WT, int RPW, bool XF = false>
__device__ __forceinline__ void consume_chunk(const uint8_t *ch, int us, int s, int warp, int lane, int units,
                                              const uint8_t *xs, float (&acc)[RPW])
{
    constexpr int R = MV_CONSUMER_WARPS * RPW;
    constexpr uint32_t UB = WT == W_F32 ? 16 : (WT == W_Q4_0 ? 16 : 32);
    const uint8_t *wrow = ch + ((size_t)warp * RPW * us + lane) * (WT == W_Q8_0 ? 16 : UB);
    const uint32_t rstride = us * UB;                     // bytes between this warp's rows
    const uint32_t sstride = (uint32_t)round_up((size_t)us * 2, 16);
    const uint8_t *srow = ch + (size_t)R * us * UB + warp * RPW * sstride + lane * 2;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int j = lane + 32 * h;
        if (j >= us) break;
        const int u = s * MV_SEG_UNITS + j;
        if (WT == W_F32) {
            const float4 xv = reinterpret_cast<const float4 *>(xs)[u];
#pragma unroll
            for (int r = 0; r < RPW; r++) {
                const float4 wv = *reinterpret_cast<const float4 *>(wrow + r * rstride + h * 512);
                acc[r] = fmaf(wv.x, xv.x, acc[r]);
                acc[r] = fmaf(wv.y, xv.y, acc[r]);
                acc[r] = fmaf(wv.z, xv.z, acc[r]);
                acc[r] = fmaf(wv.w, xv.w, acc[r]);
            }
            continue;
        }
        if (XF) {
            const float4 *xv = reinterpret_cast<const float4 *>(xs) + (size_t)u * 8;   // the unit's 32 floats
            float xf[32];
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const float4 v = xv[k];
                xf[4 * k] = v.x;
                xf[4 * k + 1] = v.y;
                xf[4 * k + 2] = v.z;
                xf[4 * k + 3] = v.w;
            }
#pragma unroll
            for (int r = 0; r < RPW; r++) {
                const float dw = half_bits_to_float(*reinterpret_cast<const uint16_t *>(srow + r * sstride + h * 64));
                uint32_t cw[8];
                if (WT == W_Q4_0) {
                    const uint4 wq = *reinterpret_cast<const uint4 *>(wrow + r * rstride + h * 512);
                    cw[0] = wq.x; cw[1] = wq.y; cw[2] = wq.z; cw[3] = wq.w;
                } else {
                    const uint8_t *wp = ch + ((size_t)(warp * RPW + r) * 2 * us + j) * 16;
                    const uint4 wl = *reinterpret_cast<const uint4 *>(wp);
                    const uint4 wh = *reinterpret_cast<const uint4 *>(wp + (size_t)us * 16);
                    cw[0] = wl.x; cw[1] = wl.y; cw[2] = wl.z; cw[3] = wl.w;
                    cw[4] = wh.x; cw[5] = wh.y; cw[6] = wh.z; cw[7] = wh.w;
                }
                float a = acc[r];
#pragma unroll
                for (int k = 0; k < 16; k++) {
                    const uint32_t byte = (cw[k >> 2] >> (8 * (k & 3))) & 0xffu;
                    float w0, w1;   // elements k and k + 16
                    if (WT == W_Q4_0) {
                        w0 = (float)((int)(byte & 0xf) - 8) * dw;
                        w1 = (float)((int)(byte >> 4) - 8) * dw;
                    } else {
                        w0 = (float)(int8_t)byte * dw;
                        w1 = (float)(int8_t)((cw[4 + (k >> 2)] >> (8 * (k & 3))) & 0xffu) * dw;
                    }
                    a = fmaf(w0, xf[k], a);
                    a = fmaf(w1, xf[k + 16], a);
                }
                acc[r] = a;
            }
            continue;
        }
        const int4 xl = *reinterpret_cast<const int4 *>(xs + (size_t)u * 16);
        const int4 xh = *reinterpret_cast<const int4 *>(xs + (size_t)units * 16 + (size_t)u * 16);
        const float2 dxs = reinterpret_cast<const float2 *>(xs + (size_t)units * 32)[u];
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            const uint16_t sc = *reinterpret_cast<const uint16_t *>(srow + r * sstride + h * 64);
            int isum;
            if (WT == W_Q4_0) {
                const uint4 wq = *reinterpret_cast<const uint4 *>(wrow + r * rstride + h * 512);
                const uint32_t lo = 0x0f0f0f0fu, hi = 0xf0f0f0f0u;
                int a = dp4a_us(wq.x & lo, xl.x, 0);
                int b = dp4a_us(wq.x & hi, xh.x, 0);
                a = dp4a_us(wq.y & lo, xl.y, a);
                b = dp4a_us(wq.y & hi, xh.y, b);
                a = dp4a_us(wq.z & lo, xl.z, a);
                b = dp4a_us(wq.z & hi, xh.z, b);
                a = dp4a_us(wq.w & lo, xl.w, a);
                b = dp4a_us(wq.w & hi, xh.w, b);
                // (nibble - 8) * q summed = lo dot + hi dot / 16 - 8 * sum(q)
                isum = a + (b >> 4) - 8 * __float_as_int(dxs.y);
            } else {
                const uint8_t *wp = ch + ((size_t)(warp * RPW + r) * 2 * us + j) * 16;
                const int4 wl = *reinterpret_cast<const int4 *>(wp);
                const int4 wh = *reinterpret_cast<const int4 *>(wp + (size_t)us * 16);
                int a = __dp4a(wl.x, xl.x, 0);
                int b = __dp4a(wh.x, xh.x, 0);
                a = __dp4a(wl.y, xl.y, a);
                b = __dp4a(wh.y, xh.y, b);
                a = __dp4a(wl.z, xl.z, a);
                b = __dp4a(wh.z, xh.z, b);
                a = __dp4a(wl.w, xl.w, a);
                b = __dp4a(wh.w, xh.w, b);
                isum = a + b;
            }
            const float delta = __fmul_rn(half_bits_to_float(sc), dxs.x);   // d_w * d_x in float
            acc[r] = fmaf(delta, (float)isum, acc[r]);
        }
    }
}

// rope_llama (llm/catseye_llm.h:1597-1620) on one (even, odd) pair at index i
__device__ __forceinline__ void rope_pair(float &a, float &b, int i, int head_size, int pos)
{
    const int hd = i % head_size;
    const float p = powf(10000.f, (float)hd / (float)head_size);
    const float freq = (float)(1.0 / (double)p);
    const float val = (float)pos * freq;
    float s, c;
    sincosf(val, &s, &c);
    const float a0 = a, b0 = b;
    a = a0 * c - b0 * s;
    b = a0 * s + b0 * c;
}

} // namespace cats
