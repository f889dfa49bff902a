/*
 * cats_oracle.h — CPU restatement of catseye's matrix-multiply hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * it.  The product library (libcatsgpu.so) never links or calls it.
 *
 * Every function restates the algorithm of the reference function cited beside
 * it (paths are relative to the catseye project root).  Parity of this
 * restatement is pinned against the reference itself: oracle/ref_llm.c and
 * oracle/ref_cnn.c compile the reference's own headers into oracle/_ref/, and
 * tests/golden/make_golden.py records their outputs as committed fixtures.
 */
#ifndef CATS_ORACLE_H
#define CATS_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type numbers, as enumerated in llm/catseye_llm.h:2557-2580 */
enum { OR_F32 = 0, OR_Q4_0 = 2, OR_Q8_0 = 8, OR_Q3_K = 11, OR_Q6_K = 14 };

/* bytes of one row of n elements for a weight type (llm/catseye_llm.h:2808-2827) */
size_t oracle_row_bytes(int type, int n);

/* fp16 <-> fp32 (llm/catseye_llm.h:75-152); fp32->fp16 rounds to nearest even */
float    oracle_fp16_to_fp32(uint16_t h);
uint16_t oracle_fp32_to_fp16(float f);

/* Q8 activation quantizer: n/32 blocks of {int8 q[32]; float d} = 36 bytes.
 * _avx    restates the AVX build  (llm/catseye_llm.h:155-225): id = 127/amax, round half to even
 * _scalar restates the plain build (llm/catseye_llm.h:227-251): id = 1/(amax/127), roundf      */
void oracle_quantize_q8_avx(int8_t *q, const float *x, int n);
void oracle_quantize_q8_scalar(int8_t *q, const float *x, int n);

/* Q8_K activation quantizer for the K-quant matvecs (llm/catseye_llm.h:262-296):
 * n/256 blocks of {int8 q[256]; float d} = 260 bytes */
void oracle_quantize_q8_K(int8_t *q, const float *x, int n);

/* Weight quantizers used only to build synthetic GGUF-style models; the reference
 * has none (it only loads quantized files).  Q4_0: d = signed absmax / -8,
 * q = min(15, trunc(x/d + 8.5)).  Q8_0: d = absmax/127, q = roundf(x/d).        */
void oracle_quantize_row_q4_0(uint8_t *y, const float *x, int n);
void oracle_quantize_row_q8_0(uint8_t *y, const float *x, int n);

/* Dequantizers: one row of n elements (llm/catseye_llm.h:427-474, 349-426) */
void oracle_dequantize_row(int type, float *y, const void *x, int n);

/* matmul(xout, x, w, n, d): xout[i] = sum_j W[i][j] * x[j], W row-major [d][n]
 * (llm/catseye_llm.h:1519-1533).  x is what the tensor's quantize produced:
 * fp32 for F32 and Q4_0xF32, Q8 blocks for Q4_0/Q8_0, Q8_K blocks for K-quants. */
void oracle_matmul_f32(float *xout, const float *x, const float *w, int n, int d);
void oracle_matmul_q4_0_q8(float *xout, const int8_t *xq, const uint8_t *w, int n, int d);
void oracle_matmul_q8_0_q8(float *xout, const int8_t *xq, const uint8_t *w, int n, int d);
void oracle_matmul_q4_0_f32(float *xout, const float *x, const uint8_t *w, int n, int d);
void oracle_matmul_q8_0_f32(float *xout, const float *x, const uint8_t *w, int n, int d);
void oracle_matmul_q3_K_q8_K(float *xout, const int8_t *xq, const uint8_t *w, int n, int d);
void oracle_matmul_q6_K_q8_K(float *xout, const int8_t *xq, const uint8_t *w, int n, int d);
/* generic: quantizes x with the type's activation quantizer first (copy, not in place) */
void oracle_matmul(int type, float *xout, const float *x, const void *w, int n, int d);

/* Row-major sgemm as catseye.h's gemm_rnn / gemm_rnt / gemm_rtn (catseye.h:78-129):
 * C[MxN] = alpha*op(A)*op(B) + beta*C; ta/tb in {'N','T'}; lda = K|M, ldb = N|K,
 * ldc = N.  beta==0 does not read C.  Accumulates in double.                     */
void oracle_sgemm(char ta, char tb, int M, int N, int K, float alpha,
                  const float *A, const float *B, float beta, float *C);

/* darknet im2col for one image (catseye.h:508-532) */
void oracle_im2col(const float *im, int channels, int height, int width, int kh, int kw,
                   int ph, int pw, int sh, int sw, float *col);

/* catseye.h CatsEye_convolutional_forward (catseye.h:557-574): for every sample,
 * im2col + gemm_rnn(ch, oh*ow, kh*kw*ich, W, col) into z + i*ch*oh*ow (CHW). */
void oracle_conv2d_forward(const float *x, const float *w, float *z, int batch, int ich,
                           int h, int wd, int ch, int k, int pad, int stride);
/* CatsEye_linear_forward (catseye.h:416-444): z = x * W^T + bias, bias at w[in*out] */
void oracle_linear_forward(const float *x, const float *w, float *z, int batch, int in, int out);
void oracle_col2im(const float *col, int channels, int height, int width, int kh, int kw,
                   int ph, int pw, int sh, int sw, float *im);
void oracle_conv2d_backward(const float *dout, const float *w, float *din, int batch, int ich,
                            int h, int wd, int ch, int k, int pad, int stride);
void oracle_conv2d_update(const float *dout, const float *x, float *dw, int batch, int ich,
                          int h, int wd, int ch, int k, int pad, int stride);
void oracle_linear_backward(const float *dout, const float *w, float *din, int batch, int in, int out);
void oracle_linear_update(const float *dout, const float *x, float *w, float *dw, int batch, int in, int out,
                          float eta);

/* Llama decode step, restating cats_llama2_transformer (llm/catseye_llm.h:1625-1772).
 * Layer matrices of one kind are stored back to back: wq = L matrices [dim][dim] ... */
typedef struct {
    int dim, hidden, n_layers, n_heads, n_kv_heads, vocab, seq_len;
    int wtype;          /* type of wq..w3 and of the classifier */
    int q8_mode;        /* 0: AVX quantizer rounding, 1: scalar build rounding,
                           2: fp32 activations (matmul_q4_0, :880-914; no quantize_q8) */
    const float *emb;   /* [vocab][dim] fp32 */
    const float *rms_att, *rms_ffn, *rms_final;
    const void *wq, *wk, *wv, *wo, *w1, *w2, *w3, *wcls;
    /* state, allocated by oracle_llm_alloc */
    float *x, *xb, *xb2, *hb, *hb2, *q, *att, *logits, *key_cache, *value_cache;
} oracle_llm;

int    oracle_llm_alloc(oracle_llm *m);
void   oracle_llm_free(oracle_llm *m);
float *oracle_llm_step(oracle_llm *m, int token, int pos);
int    oracle_argmax(const float *v, int n);   /* sample_argmax, llm/catseye_llm.h:1944-1956 */

#ifdef __cplusplus
}
#endif
#endif
