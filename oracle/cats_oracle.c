/*
 * cats_oracle.c — CPU restatement of catseye's matrix-multiply hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see cats_oracle.h).  Written from the reference's
 * algorithms; each function cites the reference lines it restates.  Matvec and
 * GEMM dot products accumulate in double so the oracle is at least as accurate
 * as the reference's float loops; quantizers and dequantizers are bit-exact
 * restatements (pinned against the compiled reference by tests/).
 */
#include "cats_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

size_t oracle_row_bytes(int type, int n)
{
    switch (type) {
    case OR_F32:  return (size_t)n * 4;
    case OR_Q4_0: return (size_t)(n / 32) * 18;
    case OR_Q8_0: return (size_t)(n / 32) * 34;
    case OR_Q3_K: return (size_t)(n / 256) * 110;
    case OR_Q6_K: return (size_t)(n / 256) * 210;
    }
    return 0;
}

/* IEEE half -> float; exact (llm/catseye_llm.h:75-125 computes the same value). */
float oracle_fp16_to_fp32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff;
    if (e == 0x1f) return bits_f(sign | 0x7f800000u | (m << 13));
    if (e == 0) {
        if (m == 0) return bits_f(sign);
        float v = (float)m * 0x1.0p-24f;          /* subnormal: m * 2^-24, exact */
        return sign ? -v : v;
    }
    return bits_f(sign | ((e + 112) << 23) | (m << 13));
}

/* float -> half, round to nearest even (F16C _cvtss_sh(x, 0), catseye_llm.h:79-80). */
uint16_t oracle_fp32_to_fp16(float f)
{
    uint32_t x = f_bits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return sign | (ax > 0x7f800000u ? 0x7e00 : 0x7c00);
    if (ax >= 0x477ff000u) return sign | 0x7c00;            /* rounds to >= 65520: inf */
    if (ax < 0x38800000u) {                                  /* result subnormal or zero */
        float a = bits_f(ax);
        /* a * 2^24 rounded to an integer (RNE) is the subnormal mantissa */
        float s = a * 0x1.0p24f;
        float r = nearbyintf(s);
        return sign | (uint16_t)r;
    }
    uint32_t mant = ax & 0x7fffff, exp = (ax >> 23) - 112;
    uint32_t h = (exp << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return sign | (uint16_t)h;
}

/* AVX quantize_q8 (llm/catseye_llm.h:155-225).  The reference computes
 * d = amax/127. and id = 127./amax in double and stores them as float, which is
 * the correctly rounded float quotient; v*id is a float multiply; the round is
 * _MM_ROUND_NEAREST (half to even); packs saturate to int8. */
void oracle_quantize_q8_avx(int8_t *q, const float *x, int n)
{
    for (int b = 0; b < n / 32; b++) {
        const float *xb = x + b * 32;
        float amax = 0.f;
        for (int i = 0; i < 32; i++) { float a = fabsf(xb[i]); if (a > amax) amax = a; }
        float d = (float)((double)amax / 127.0);
        float id = amax != 0.f ? (float)(127.0 / (double)amax) : 0.f;
        int8_t tmp[32];
        for (int i = 0; i < 32; i++) {
            float v = nearbyintf(xb[i] * id);
            int iv = (int)v;
            if (iv > 127) iv = 127;
            if (iv < -128) iv = -128;
            tmp[i] = (int8_t)iv;
        }
        int8_t *p = q + b * 36;
        memcpy(p, tmp, 32);
        memcpy(p + 32, &d, 4);
    }
}

/* Scalar quantize_q8 (llm/catseye_llm.h:227-251): id = 1.0/d in double, roundf. */
void oracle_quantize_q8_scalar(int8_t *q, const float *x, int n)
{
    for (int b = 0; b < n / 32; b++) {
        const float *xb = x + b * 32;
        float amax = 0.f;
        for (int i = 0; i < 32; i++) { float a = fabsf(xb[i]); amax = amax > a ? amax : a; }
        float d = (float)((double)amax / 127.0);
        float id = d != 0.f ? (float)(1.0 / (double)d) : 0.f;
        int8_t tmp[32];
        for (int i = 0; i < 32; i++) tmp[i] = (int8_t)(int)roundf(xb[i] * id);
        int8_t *p = q + b * 36;
        memcpy(p, tmp, 32);
        memcpy(p + 32, &d, 4);
    }
}

/* quantize_q8_K (llm/catseye_llm.h:262-296): signed max, iscale = -128/max,
 * nearest_int (round half to even through the 1.5*2^23 trick), clamp at 127. */
void oracle_quantize_q8_K(int8_t *y, const float *x, int n)
{
    for (int b = 0; b < n / 256; b++, x += 256, y += 260) {
        float amax = 0.f, max = 0.f;
        for (int j = 0; j < 256; j++) {
            float ax = fabsf(x[j]);
            if (ax > amax) { amax = ax; max = x[j]; }
        }
        if (amax == 0.f) { memset(y, 0, 260); continue; }
        float iscale = (float)(-128.0 / (double)max);
        for (int j = 0; j < 256; j++) {
            float v = nearbyintf(iscale * x[j]);
            int iv = (int)v;
            y[j] = (int8_t)(iv < 127 ? iv : 127);
        }
        float d = 1.f / iscale;
        memcpy(y + 256, &d, 4);
    }
}

/* Synthetic-model quantizers (no reference counterpart, see header). */
void oracle_quantize_row_q4_0(uint8_t *y, const float *x, int n)
{
    for (int b = 0; b < n / 32; b++, x += 32, y += 18) {
        float amax = 0.f, max = 0.f;
        for (int j = 0; j < 32; j++) {
            float a = fabsf(x[j]);
            if (a > amax) { amax = a; max = x[j]; }
        }
        float d = max / -8.f;
        float id = d != 0.f ? 1.f / d : 0.f;
        uint16_t hd = oracle_fp32_to_fp16(d);
        memcpy(y, &hd, 2);
        for (int j = 0; j < 16; j++) {
            int q0 = (int)(x[j] * id + 8.5f), q1 = (int)(x[j + 16] * id + 8.5f);
            if (q0 > 15) q0 = 15;
            if (q1 > 15) q1 = 15;
            y[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

void oracle_quantize_row_q8_0(uint8_t *y, const float *x, int n)
{
    for (int b = 0; b < n / 32; b++, x += 32, y += 34) {
        float amax = 0.f;
        for (int j = 0; j < 32; j++) { float a = fabsf(x[j]); if (a > amax) amax = a; }
        float d = amax / 127.f;
        float id = d != 0.f ? 1.f / d : 0.f;
        uint16_t hd = oracle_fp32_to_fp16(d);
        memcpy(y, &hd, 2);
        for (int j = 0; j < 32; j++) y[2 + j] = (uint8_t)(int8_t)(int)roundf(x[j] * id);
    }
}

static inline float ld_half(const uint8_t *p) { uint16_t h; memcpy(&h, p, 2); return oracle_fp16_to_fp32(h); }

/* dequantize_q4_0 (llm/catseye_llm.h:427-474): y[j] = (lo_nibble - 8)*d for j<16,
 * y[j+16] = (hi_nibble - 8)*d. */
static void deq_q4_0(float *y, const uint8_t *x, int n)
{
    for (int b = 0; b < n / 32; b++, x += 18, y += 32) {
        float d = ld_half(x);
        for (int j = 0; j < 16; j++) {
            y[j] = (float)((x[2 + j] & 0x0f) - 8) * d;
            y[j + 16] = (float)((x[2 + j] >> 4) - 8) * d;
        }
    }
}

/* Q8_0 weights: value = q*d (GGUF block {fp16 d; int8 qs[32]}). */
static void deq_q8_0(float *y, const uint8_t *x, int n)
{
    for (int b = 0; b < n / 32; b++, x += 34, y += 32) {
        float d = ld_half(x);
        for (int j = 0; j < 32; j++) y[j] = (float)(int8_t)x[2 + j] * d;
    }
}

/* Unpack the 16 six-bit Q3_K scales (llm/catseye_llm.h:360-368). */
static void q3k_scales(const uint8_t *sc12, int8_t out[16])
{
    uint32_t a[4];
    memcpy(a, sc12, 12);
    uint32_t tmp = a[2];
    const uint32_t k1 = 0x03030303, k2 = 0x0f0f0f0f;
    a[2] = ((a[0] >> 4) & k2) | (((tmp >> 4) & k1) << 4);
    a[3] = ((a[1] >> 4) & k2) | (((tmp >> 6) & k1) << 4);
    a[0] = (a[0] & k2) | (((tmp >> 0) & k1) << 4);
    a[1] = (a[1] & k2) | (((tmp >> 2) & k1) << 4);
    memcpy(out, a, 16);
}

/* Q3_K element values as small ints in element order, with per-16 scales
 * (llm/catseye_llm.h:349-393 dequant; 1200-1259 dot). */
static void q3k_unpack(const uint8_t *p, int8_t q[256], int8_t sc[16])
{
    const uint8_t *hm = p, *q3 = p + 32;
    int idx = 0;
    uint8_t m = 1;
    for (int half = 0; half < 2; half++, q3 += 32) {
        for (int s = 0; s < 4; s++, m <<= 1)
            for (int l = 0; l < 32; l++)
                q[idx++] = (int8_t)(((q3[l] >> (2 * s)) & 3) - ((hm[l] & m) ? 0 : 4));
    }
    int8_t raw[16];
    q3k_scales(p + 96, raw);
    for (int j = 0; j < 16; j++) sc[j] = (int8_t)(raw[j] - 32);
}

/* Q6_K element values (llm/catseye_llm.h:394-426 dequant; 1467-1511 dot). */
static void q6k_unpack(const uint8_t *p, int8_t q[256], int8_t sc[16])
{
    const uint8_t *ql = p, *qh = p + 128;
    for (int h = 0; h < 2; h++, ql += 64, qh += 32) {
        int8_t *a = q + 128 * h;
        for (int l = 0; l < 32; l++) {
            a[l + 0]  = (int8_t)(((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32);
            a[l + 32] = (int8_t)(((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32);
            a[l + 64] = (int8_t)(((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32);
            a[l + 96] = (int8_t)(((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32);
        }
    }
    memcpy(sc, p + 192, 16);
}

void oracle_dequantize_row(int type, float *y, const void *xv, int n)
{
    const uint8_t *x = (const uint8_t *)xv;
    switch (type) {
    case OR_F32: memcpy(y, x, (size_t)n * 4); return;
    case OR_Q4_0: deq_q4_0(y, x, n); return;
    case OR_Q8_0: deq_q8_0(y, x, n); return;
    case OR_Q3_K:
        for (int b = 0; b < n / 256; b++, x += 110, y += 256) {
            int8_t q[256], sc[16];
            q3k_unpack(x, q, sc);
            float d = ld_half(x + 108);
            for (int j = 0; j < 256; j++) y[j] = d * (float)sc[j / 16] * (float)q[j];
        }
        return;
    case OR_Q6_K:
        for (int b = 0; b < n / 256; b++, x += 210, y += 256) {
            int8_t q[256], sc[16];
            q6k_unpack(x, q, sc);
            float d = ld_half(x + 208);
            for (int j = 0; j < 256; j++) y[j] = d * (float)sc[j / 16] * (float)q[j];
        }
        return;
    }
}

/* matmul_f32 (llm/catseye_llm.h:1519-1529 with dot_avx :1449-1465). */
void oracle_matmul_f32(float *xout, const float *x, const float *w, int n, int d)
{
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < d; i++) {
        const float *r = w + (size_t)i * n;
        double s = 0;
        for (int j = 0; j < n; j++) s += (double)r[j] * x[j];
        xout[i] = (float)s;
    }
}

/* dot_q4_0_q8 (llm/catseye_llm.h:844-879 AVX, 916-972 scalar): per block the
 * integer sum of (nibble-8)*q8, times the float product d_w*d_x. */
void oracle_matmul_q4_0_q8(float *xout, const int8_t *xq, const uint8_t *w, int n, int d)
{
    const int nb = n / 32;
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < d; i++) {
        const uint8_t *r = w + (size_t)i * nb * 18;
        double s = 0;
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = r + b * 18;
            const int8_t *y = xq + b * 36;
            int isum = 0;
            for (int j = 0; j < 16; j++) {
                isum += ((blk[2 + j] & 0x0f) - 8) * y[j];
                isum += ((blk[2 + j] >> 4) - 8) * y[j + 16];
            }
            float dx;
            memcpy(&dx, y + 32, 4);
            float delta = ld_half(blk) * dx;
            s += (double)delta * isum;
        }
        xout[i] = (float)s;
    }
}

/* Q8_0 weights x Q8 activations (no reference counterpart; same block scheme). */
void oracle_matmul_q8_0_q8(float *xout, const int8_t *xq, const uint8_t *w, int n, int d)
{
    const int nb = n / 32;
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < d; i++) {
        const uint8_t *r = w + (size_t)i * nb * 34;
        double s = 0;
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = r + b * 34;
            const int8_t *y = xq + b * 36;
            int isum = 0;
            for (int j = 0; j < 32; j++) isum += (int8_t)blk[2 + j] * y[j];
            float dx;
            memcpy(&dx, y + 32, 4);
            float delta = ld_half(blk) * dx;
            s += (double)delta * isum;
        }
        xout[i] = (float)s;
    }
}

/* matmul_q4_0 = dot_avx_q4_0 (llm/catseye_llm.h:880-914): dequantized weights
 * (float) times fp32 x. */
void oracle_matmul_q4_0_f32(float *xout, const float *x, const uint8_t *w, int n, int d)
{
    const int nb = n / 32;
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < d; i++) {
        const uint8_t *r = w + (size_t)i * nb * 18;
        float wr[32];
        double s = 0;
        for (int b = 0; b < nb; b++) {
            deq_q4_0(wr, r + b * 18, 32);
            for (int j = 0; j < 32; j++) s += (double)wr[j] * x[b * 32 + j];
        }
        xout[i] = (float)s;
    }
}

/* Q8_0 weights times fp32 activations: value = q*d (GGUF Q8_0 block), the
 * f32-activation form of matmul_q4_0 (llm/catseye_llm.h:880-914) for Q8_0. */
void oracle_matmul_q8_0_f32(float *xout, const float *x, const uint8_t *w, int n, int d)
{
    const int nb = n / 32;
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < d; i++) {
        const uint8_t *r = w + (size_t)i * nb * 34;
        float wr[32];
        double s = 0;
        for (int b = 0; b < nb; b++) {
            deq_q8_0(wr, r + b * 34, 32);
            for (int j = 0; j < 32; j++) s += (double)wr[j] * x[b * 32 + j];
        }
        xout[i] = (float)s;
    }
}

/* dot_q3_K_q8_K / dot_q6_K_q8_K (llm/catseye_llm.h:1200-1259, 1467-1511):
 * per super-block, sum over 16-element groups of scale*int dot, times d_w*d_x. */
static void matmul_kquant(int type, float *xout, const int8_t *xq, const uint8_t *w, int n, int d)
{
    const int nb = n / 256;
    const int bs = type == OR_Q3_K ? 110 : 210;
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < d; i++) {
        const uint8_t *r = w + (size_t)i * nb * bs;
        double s = 0;
        for (int b = 0; b < nb; b++) {
            int8_t q[256], sc[16];
            const uint8_t *p = r + b * bs;
            float dw;
            if (type == OR_Q3_K) { q3k_unpack(p, q, sc); dw = ld_half(p + 108); }
            else                 { q6k_unpack(p, q, sc); dw = ld_half(p + 208); }
            const int8_t *y = xq + b * 260;
            int isum = 0;
            for (int g = 0; g < 16; g++) {
                int gs = 0;
                for (int l = 0; l < 16; l++) gs += q[g * 16 + l] * y[g * 16 + l];
                isum += sc[g] * gs;
            }
            float dx;
            memcpy(&dx, y + 256, 4);
            float delta = dw * dx;
            s += (double)delta * isum;
        }
        xout[i] = (float)s;
    }
}

void oracle_matmul_q3_K_q8_K(float *xout, const int8_t *xq, const uint8_t *w, int n, int d)
{ matmul_kquant(OR_Q3_K, xout, xq, w, n, d); }
void oracle_matmul_q6_K_q8_K(float *xout, const int8_t *xq, const uint8_t *w, int n, int d)
{ matmul_kquant(OR_Q6_K, xout, xq, w, n, d); }

/* Dispatch like gguf_matmul[] / gguf_quantize[] (llm/catseye_llm.h:2583-2607). */
static void matmul_q8mode(int type, int q8_mode, float *xout, const float *x, const void *w, int n, int d)
{
    if (type == OR_F32) { oracle_matmul_f32(xout, x, (const float *)w, n, d); return; }
    if (type == OR_Q3_K || type == OR_Q6_K) {
        int8_t *q = (int8_t *)malloc((size_t)(n / 256) * 260);
        oracle_quantize_q8_K(q, x, n);
        matmul_kquant(type, xout, q, (const uint8_t *)w, n, d);
        free(q);
        return;
    }
    if (q8_mode == 2) {   /* fp32 activations: matmul_q4_0 (:880-914) and its Q8_0 counterpart */
        if (type == OR_Q4_0) oracle_matmul_q4_0_f32(xout, x, (const uint8_t *)w, n, d);
        else                 oracle_matmul_q8_0_f32(xout, x, (const uint8_t *)w, n, d);
        return;
    }
    int8_t *q = (int8_t *)malloc((size_t)(n / 32) * 36);
    if (q8_mode) oracle_quantize_q8_scalar(q, x, n); else oracle_quantize_q8_avx(q, x, n);
    if (type == OR_Q4_0) oracle_matmul_q4_0_q8(xout, q, (const uint8_t *)w, n, d);
    else                 oracle_matmul_q8_0_q8(xout, q, (const uint8_t *)w, n, d);
    free(q);
}

void oracle_matmul(int type, float *xout, const float *x, const void *w, int n, int d)
{ matmul_q8mode(type, 0, xout, x, w, n, d); }

/* gemm_rnn / gemm_rnt / gemm_rtn (catseye.h:78-129). */
void oracle_sgemm(char ta, char tb, int M, int N, int K, float alpha,
                  const float *A, const float *B, float beta, float *C)
{
    const int at = (ta == 'T' || ta == 't'), bt = (tb == 'T' || tb == 't');
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        double *acc = (double *)calloc((size_t)N, sizeof(double));
        for (int k = 0; k < K; k++) {
            double a = at ? A[(size_t)k * M + m] : A[(size_t)m * K + k];
            if (a == 0.0) continue;
            if (bt) for (int n = 0; n < N; n++) acc[n] += a * B[(size_t)n * K + k];
            else    for (int n = 0; n < N; n++) acc[n] += a * B[(size_t)k * N + n];
        }
        float *c = C + (size_t)m * N;
        for (int n = 0; n < N; n++) {
            double base = beta == 0.f ? 0.0 : (double)beta * c[n];
            c[n] = (float)(base + (double)alpha * acc[n]);
        }
        free(acc);
    }
}

/* im2col (catseye.h:508-532). */
void oracle_im2col(const float *im, int channels, int height, int width, int kh, int kw,
                   int ph, int pw, int sh, int sw, float *col)
{
    int hc = (height + 2 * ph - kh) / sh + 1, wc = (width + 2 * pw - kw) / sw + 1;
    int cc = channels * kh * kw;
    for (int c = 0; c < cc; c++) {
        int wo = c % kw, ho = (c / kw) % kh, ci = c / kh / kw;
        for (int h = 0; h < hc; h++)
            for (int w = 0; w < wc; w++) {
                int hp = h * sh - ph + ho, wp = w * sw - pw + wo;
                col[((size_t)c * hc + h) * wc + w] =
                    (hp >= 0 && hp < height && wp >= 0 && wp < width) ? im[((size_t)ci * height + hp) * width + wp] : 0.f;
            }
    }
}

void oracle_conv2d_forward(const float *x, const float *w, float *z, int batch, int ich,
                           int h, int wd, int ch, int k, int pad, int stride)
{
    int oh = (h + 2 * pad - k) / stride + 1, ow = (wd + 2 * pad - k) / stride + 1;
    size_t K = (size_t)ich * k * k, Nn = (size_t)oh * ow;
    float *col = (float *)malloc(K * Nn * sizeof(float));
    for (int i = 0; i < batch; i++) {
        oracle_im2col(x + (size_t)i * ich * h * wd, ich, h, wd, k, k, pad, pad, stride, stride, col);
        oracle_sgemm('N', 'N', ch, (int)Nn, (int)K, 1.f, w, col, 0.f, z + (size_t)i * ch * Nn);
    }
    free(col);
}

void oracle_linear_forward(const float *x, const float *w, float *z, int batch, int in, int out)
{
    oracle_sgemm('N', 'T', batch, out, in, 1.f, x, w, 0.f, z);
    for (int b = 0; b < batch; b++)
        for (int i = 0; i < out; i++) z[(size_t)b * out + i] += w[(size_t)in * out + i];
}

/* col2im (catseye.h:533-556): scatter-add of every column entry into the
 * image, in column-row order, from a zeroed image. */
void oracle_col2im(const float *col, int channels, int height, int width, int kh, int kw,
                   int ph, int pw, int sh, int sw, float *im)
{
    int hc = (height + 2 * ph - kh) / sh + 1, wc = (width + 2 * pw - kw) / sw + 1;
    int cc = channels * kh * kw;
    memset(im, 0, sizeof(float) * (size_t)channels * height * width);
    for (int c = 0; c < cc; c++) {
        int wo = c % kw, ho = (c / kw) % kh, ci = c / kh / kw;
        for (int h = 0; h < hc; h++)
            for (int w = 0; w < wc; w++) {
                int hp = h * sh - ph + ho, wp = w * sw - pw + wo;
                if (hp >= 0 && hp < height && wp >= 0 && wp < width)
                    im[((size_t)ci * height + hp) * width + wp] += col[((size_t)c * hc + h) * wc + w];
            }
    }
}

/* CatsEye_convolutional_backward (catseye.h:589-620), per sample:
 * col = W^T dOut (gemm_rtn), dIn = col2im(col); ksize 1 writes W^T dOut. */
void oracle_conv2d_backward(const float *dout, const float *w, float *din, int batch, int ich,
                            int h, int wd, int ch, int k, int pad, int stride)
{
    int oh = (h + 2 * pad - k) / stride + 1, ow = (wd + 2 * pad - k) / stride + 1;
    size_t K = (size_t)ich * k * k, Nn = (size_t)oh * ow;
    float *col = (float *)malloc(K * Nn * sizeof(float));
    for (int i = 0; i < batch; i++) {
        float *di = din + (size_t)i * ich * h * wd;
        float *ws = k != 1 ? col : di;
        oracle_sgemm('T', 'N', (int)K, (int)Nn, ch, 1.f, w, dout + (size_t)i * ch * Nn, 0.f, ws);
        if (k != 1) oracle_col2im(col, ich, h, wd, k, k, pad, pad, stride, stride, di);
    }
    free(col);
}

/* CatsEye_convolutional_update (catseye.h:622-640), per sample:
 * dw += (1/batch) dOut im2col(x)^T (gemm_rnt, beta 1). */
void oracle_conv2d_update(const float *dout, const float *x, float *dw, int batch, int ich,
                          int h, int wd, int ch, int k, int pad, int stride)
{
    int oh = (h + 2 * pad - k) / stride + 1, ow = (wd + 2 * pad - k) / stride + 1;
    size_t K = (size_t)ich * k * k, Nn = (size_t)oh * ow;
    float *col = (float *)malloc(K * Nn * sizeof(float));
    const float alpha = (float)(1.0 / batch);
    for (int i = 0; i < batch; i++) {
        oracle_im2col(x + (size_t)i * ich * h * wd, ich, h, wd, k, k, pad, pad, stride, stride, col);
        oracle_sgemm('N', 'T', ch, (int)K, (int)Nn, alpha, dout + (size_t)i * ch * Nn, col, 1.f, dw);
    }
    free(col);
}

/* CatsEye_linear_backward (catseye.h:445-477): dIn = dOut W (gemm_rnn). */
void oracle_linear_backward(const float *dout, const float *w, float *din, int batch, int in, int out)
{
    oracle_sgemm('N', 'N', batch, in, out, 1.f, dout, w, 0.f, din);
}

/* CatsEye_linear_update (catseye.h:478-505): dw += dOut^T x (gemm_rtn, beta 1),
 * then the biases after the weights step by -eta dOut, sample after sample. */
void oracle_linear_update(const float *dout, const float *x, float *w, float *dw, int batch, int in, int out,
                          float eta)
{
    oracle_sgemm('T', 'N', out, in, batch, 1.f, dout, x, 1.f, dw);
    for (int b = 0; b < batch; b++)
        for (int i = 0; i < out; i++) w[(size_t)in * out + i] -= eta * dout[(size_t)b * out + i];
}

/* ---- llama decode step (llm/catseye_llm.h:684-721, 1574-1772) ---------------- */

static void rmsnorm(float *o, const float *x, const float *w, int n)
{
    float ss = 0.f;
    for (int j = 0; j < n; j++) ss += x[j] * x[j];
    ss /= n;
    ss += 1e-5f;
    ss = 1.f / sqrtf(ss);
    for (int j = 0; j < n; j++) o[j] = w[j] * (ss * x[j]);
}

static void softmax(float *x, int n)
{
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    float inv = 1.f / sum;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

static void rope_llama(float *q, float *k, int dim, int kv_dim, int hs, int pos)
{
    for (int i = 0; i < dim; i += 2) {
        int hd = i % hs;
        float freq = (float)(1.0 / (double)powf(10000.f, hd / (float)hs));
        float val = pos * freq;
        float c = cosf(val), s = sinf(val);
        float q0 = q[i], q1 = q[i + 1];
        q[i] = q0 * c - q1 * s;
        q[i + 1] = q0 * s + q1 * c;
        if (i < kv_dim) {
            float k0 = k[i], k1 = k[i + 1];
            k[i] = k0 * c - k1 * s;
            k[i + 1] = k0 * s + k1 * c;
        }
    }
}

int oracle_llm_alloc(oracle_llm *m)
{
    int kv_dim = m->dim * m->n_kv_heads / m->n_heads;
    m->x = calloc(m->dim, 4); m->xb = calloc(m->dim, 4); m->xb2 = calloc(m->dim, 4);
    m->hb = calloc(m->hidden, 4); m->hb2 = calloc(m->hidden, 4); m->q = calloc(m->dim, 4);
    m->att = calloc((size_t)m->n_heads * m->seq_len, 4);
    m->logits = calloc(m->vocab, 4);
    m->key_cache = calloc((size_t)m->n_layers * m->seq_len * kv_dim, 4);
    m->value_cache = calloc((size_t)m->n_layers * m->seq_len * kv_dim, 4);
    return m->x && m->xb && m->xb2 && m->hb && m->hb2 && m->q && m->att && m->logits &&
           m->key_cache && m->value_cache ? 0 : -1;
}

void oracle_llm_free(oracle_llm *m)
{
    free(m->x); free(m->xb); free(m->xb2); free(m->hb); free(m->hb2); free(m->q);
    free(m->att); free(m->logits); free(m->key_cache); free(m->value_cache);
    m->x = NULL;
}

static const void *layer_mat(const void *base, int type, int n, int d, int l)
{
    return (const uint8_t *)base + oracle_row_bytes(type, n) * (size_t)d * l;
}

float *oracle_llm_step(oracle_llm *m, int token, int pos)
{
    const int dim = m->dim, hidden = m->hidden, hs = dim / m->n_heads;
    const int kv_dim = dim * m->n_kv_heads / m->n_heads, kv_mul = m->n_heads / m->n_kv_heads;
    const int t = m->wtype;
    float *x = m->x;
    memcpy(x, m->emb + (size_t)token * dim, (size_t)dim * 4);
    for (int l = 0; l < m->n_layers; l++) {
        rmsnorm(m->xb, x, m->rms_att + (size_t)l * dim, dim);
        size_t loff = (size_t)l * m->seq_len * kv_dim;
        float *k = m->key_cache + loff + (size_t)pos * kv_dim;
        float *v = m->value_cache + loff + (size_t)pos * kv_dim;
        matmul_q8mode(t, m->q8_mode, m->q, m->xb, layer_mat(m->wq, t, dim, dim, l), dim, dim);
        matmul_q8mode(t, m->q8_mode, k, m->xb, layer_mat(m->wk, t, dim, kv_dim, l), dim, kv_dim);
        matmul_q8mode(t, m->q8_mode, v, m->xb, layer_mat(m->wv, t, dim, kv_dim, l), dim, kv_dim);
        rope_llama(m->q, k, dim, kv_dim, hs, pos);
        #pragma omp parallel for schedule(static)
        for (int h = 0; h < m->n_heads; h++) {
            const float *q = m->q + h * hs;
            float *att = m->att + (size_t)h * m->seq_len;
            for (int tt = 0; tt <= pos; tt++) {
                const float *kk = m->key_cache + loff + (size_t)tt * kv_dim + (h / kv_mul) * hs;
                float s = 0.f;
                for (int i = 0; i < hs; i++) s += q[i] * kk[i];
                att[tt] = s / sqrtf((float)hs);
            }
            softmax(att, pos + 1);
            float *xb = m->xb + h * hs;
            memset(xb, 0, (size_t)hs * 4);
            for (int tt = 0; tt <= pos; tt++) {
                const float *vv = m->value_cache + loff + (size_t)tt * kv_dim + (h / kv_mul) * hs;
                float a = att[tt];
                for (int i = 0; i < hs; i++) xb[i] += a * vv[i];
            }
        }
        matmul_q8mode(t, m->q8_mode, m->xb2, m->xb, layer_mat(m->wo, t, dim, dim, l), dim, dim);
        for (int i = 0; i < dim; i++) x[i] += m->xb2[i];
        rmsnorm(m->xb, x, m->rms_ffn + (size_t)l * dim, dim);
        matmul_q8mode(t, m->q8_mode, m->hb, m->xb, layer_mat(m->w1, t, dim, hidden, l), dim, hidden);
        matmul_q8mode(t, m->q8_mode, m->hb2, m->xb, layer_mat(m->w3, t, dim, hidden, l), dim, hidden);
        for (int i = 0; i < hidden; i++) {
            float val = m->hb[i];
            val *= 1.f / (1.f + expf(-val));
            m->hb[i] = val * m->hb2[i];
        }
        matmul_q8mode(t, m->q8_mode, m->xb, m->hb, layer_mat(m->w2, t, hidden, dim, l), hidden, dim);
        for (int i = 0; i < dim; i++) x[i] += m->xb[i];
    }
    rmsnorm(x, x, m->rms_final, dim);
    matmul_q8mode(t, m->q8_mode, m->logits, x, m->wcls, dim, m->vocab);
    return m->logits;
}

int oracle_argmax(const float *v, int n)
{
    int mi = 0;
    float mv = v[0];
    for (int i = 1; i < n; i++) if (v[i] > mv) { mv = v[i]; mi = i; }
    return mi;
}
