/*
 * ref_llm.c — exports the reference's own LLM hot-path functions from a shared
 * library so the oracle restatement can be pinned against them.
 *
 * TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile from the reference
 * header where it lies (REF_DIR/llm/catseye_llm.h, never copied into this
 * repository) into oracle/_ref/.  The functions below only forward to the
 * reference's static functions; they add no arithmetic of their own.
 */
#include "catseye_llm.h"

int ref_is_avx(void)
{
#ifdef __AVX__
    return 1;
#else
    return 0;
#endif
}

float ref_fp16_to_fp32(uint16_t h) { return cats_fp16_to_fp32(h); }
uint16_t ref_fp32_to_fp16(float f) { return cats_fp32_to_fp16(f); }

/* quantize_q8 works in place in the reference; copy first so the caller's x survives */
void ref_quantize_q8(int8_t *q, const float *x, int n)
{
    float *tmp = malloc(sizeof(float) * n);
    memcpy(tmp, x, sizeof(float) * n);
    quantize_q8((int8_t *)tmp, tmp, n);
    memcpy(q, tmp, (size_t)(n / 32) * 36);
    free(tmp);
}

void ref_quantize_q8_K(int8_t *q, const float *x, int n) { quantize_q8_K(q, (real *)x, n); }

void ref_dequantize(int type, float *y, const void *w, int row, int n)
{
    gguf_dequantize[type](y, w, row, n);
}

void ref_matmul(int type, float *xout, void *x, void *w, int n, int d)
{
    gguf_matmul[type](xout, x, w, n, d);
}

#ifdef __AVX__
void ref_matmul_q4_0_f32(float *xout, void *x, void *w, int n, int d) { matmul_q4_0(xout, x, w, n, d); }
#endif

int ref_sample_argmax(float *v, int n) { return sample_argmax(v, n); }

/* A cats_llm_model whose tensors point at caller-owned blobs (layer matrices of
 * one kind stored back to back), bound like cats_checkpoint_load / the GGUF
 * loader bind them (llm/catseye_llm.h:2839-2840, 2985-2990). */
typedef struct { cats_llm_model m; } ref_model;

static size_t rowbytes(int type, int n)
{
    switch (type) {
    case GGML_TYPE_F32: return (size_t)n * 4;
    case GGML_TYPE_Q4_0: return (size_t)(n / 32) * 18;
    case GGML_TYPE_Q3_K: return (size_t)(n / 256) * 110;
    case GGML_TYPE_Q6_K: return (size_t)(n / 256) * 210;
    }
    return 0;
}

static void bind(cats_tensor *t, int type, void *data)
{
    t->type = type;
    t->data = data;
    t->quantize = gguf_quantize[type];
    t->matmul = gguf_matmul[type];
}

void *ref_llm_create(int dim, int hidden, int n_layers, int n_heads, int n_kv_heads, int vocab,
                     int seq_len, int wtype, const float *emb, const float *rms_att,
                     const float *rms_ffn, const float *rms_final, const void *wq, const void *wk,
                     const void *wv, const void *wo, const void *w1, const void *w2, const void *w3,
                     const void *wcls)
{
    if (wtype != GGML_TYPE_F32 && wtype != GGML_TYPE_Q4_0 && wtype != GGML_TYPE_Q3_K &&
        wtype != GGML_TYPE_Q6_K)
        return NULL;
    ref_model *r = calloc(1, sizeof(ref_model));
    cats_llm_model *m = &r->m;
    m->n_embd = dim; m->n_hidden = hidden; m->n_layer = n_layers; m->n_head = n_heads;
    m->n_kv_head = n_kv_heads; m->n_vocab = vocab; m->seq_len = seq_len;
    int kv_dim = dim * n_kv_heads / n_heads;
    m->token_embedding_table = &m->tensor[0];
    m->rms_final_weight = &m->tensor[1];
    m->wcls = &m->tensor[2];
    bind(m->token_embedding_table, GGML_TYPE_F32, (void *)emb);
    bind(m->rms_final_weight, GGML_TYPE_F32, (void *)rms_final);
    bind(m->wcls, wtype, (void *)wcls);
    for (int l = 0; l < n_layers; l++) {
        m->rms_att_weight[l] = &m->tensor[3 + l * 9];
        m->wq[l] = &m->tensor[4 + l * 9];
        m->wk[l] = &m->tensor[5 + l * 9];
        m->wv[l] = &m->tensor[6 + l * 9];
        m->wo[l] = &m->tensor[7 + l * 9];
        m->rms_ffn_weight[l] = &m->tensor[8 + l * 9];
        m->w1[l] = &m->tensor[9 + l * 9];
        m->w2[l] = &m->tensor[10 + l * 9];
        m->w3[l] = &m->tensor[11 + l * 9];
        bind(m->rms_att_weight[l], GGML_TYPE_F32, (void *)(rms_att + (size_t)l * dim));
        bind(m->rms_ffn_weight[l], GGML_TYPE_F32, (void *)(rms_ffn + (size_t)l * dim));
        bind(m->wq[l], wtype, (char *)wq + rowbytes(wtype, dim) * dim * l);
        bind(m->wk[l], wtype, (char *)wk + rowbytes(wtype, dim) * kv_dim * l);
        bind(m->wv[l], wtype, (char *)wv + rowbytes(wtype, dim) * kv_dim * l);
        bind(m->wo[l], wtype, (char *)wo + rowbytes(wtype, dim) * dim * l);
        bind(m->w1[l], wtype, (char *)w1 + rowbytes(wtype, dim) * hidden * l);
        bind(m->w2[l], wtype, (char *)w2 + rowbytes(wtype, hidden) * dim * l);
        bind(m->w3[l], wtype, (char *)w3 + rowbytes(wtype, dim) * hidden * l);
    }
    dequantize = _dequantize_memcpy;
    cats_llm_malloc(m);
    return r;
}

/* The reference's own loaders on a model file: fmt 1 cats_gguf_load
 * (llm/catseye_llm.h:2678-2895), 2 cats_ggml_load (:2326-2550), 3
 * cats_checkpoint_load (:2900-2993); then cats_llm_malloc.  hp receives
 * n_embd, n_hidden, n_layer, n_head, n_kv_head, n_vocab, seq_len. */
void *ref_llm_load(const char *path, int fmt, int *hp)
{
    ref_model *r = calloc(1, sizeof(ref_model));
    cats_llm_model *m = &r->m;
    int rc = 0;
    /* the runtime's global dequantizer starts as the plain copy (catseye_llm.h:521);
     * the GGUF and ggml loaders reassign it, the .bin loader relies on the
     * default: restore it, as a fresh process would have it */
    dequantize = _dequantize_memcpy;
    if (fmt == 1) rc = cats_gguf_load((char *)path, m);
    else if (fmt == 2) rc = cats_ggml_load((char *)path, m);
    else rc = cats_checkpoint_load((char *)path, m) > 0 ? 0 : 1;
    if (rc != 0) { free(r); return NULL; }
    if (fmt != 1) m->n_kv_head = m->n_kv_head ? m->n_kv_head : m->n_head;
    hp[0] = m->n_embd; hp[1] = m->n_hidden; hp[2] = m->n_layer; hp[3] = m->n_head;
    hp[4] = m->n_kv_head; hp[5] = m->n_vocab; hp[6] = m->seq_len;
    cats_llm_malloc(m);
    return r;
}

float *ref_llm_step(void *h, int token, int pos)
{
    ref_model *r = h;
    return cats_llama2_transformer(token, pos, &r->m);
}

#ifdef __AVX__
/* Rebind the Q4_0 tensors to the reference's fp32-activation matmul:
 * matmul_q4_0 (llm/catseye_llm.h:880-914) with quantize_null (:2593-2595),
 * the binding a runtime selects to skip quantize_q8.  Returns the number of
 * tensors rebound. */
int ref_llm_use_f32_activations(void *h)
{
    ref_model *r = h;
    int k = 0;
    for (int i = 0; i < (int)(sizeof(r->m.tensor) / sizeof(r->m.tensor[0])); i++) {
        cats_tensor *t = &r->m.tensor[i];
        if (t->data && t->type == GGML_TYPE_Q4_0) {
            t->matmul = matmul_q4_0;
            t->quantize = gguf_quantize[GGML_TYPE_F32];
            k++;
        }
    }
    return k;
}
#endif

/* Back to the runtime's default Q4_0 binding (gguf_matmul / gguf_quantize,
 * llm/catseye_llm.h:2583-2607): used after a prompt went through the
 * fp32-activation binding, so the decode steps that follow run the default
 * quantize_q8 + matmul_q4_0_q8 path over the cache the prompt left. */
int ref_llm_use_q8_activations(void *h)
{
    ref_model *r = h;
    int k = 0;
    for (int i = 0; i < (int)(sizeof(r->m.tensor) / sizeof(r->m.tensor[0])); i++) {
        cats_tensor *t = &r->m.tensor[i];
        if (t->data && t->type == GGML_TYPE_Q4_0) {
            bind(t, GGML_TYPE_Q4_0, t->data);
            k++;
        }
    }
    return k;
}

#ifdef CATS_DROPIN
/* The drop-in in place: the runtime's dispatch tables (llm/catseye_llm.h:
 * 2583-2607) rebound to libcatsgpu's matmuls and quantizers, as a program
 * binding the library would do before loading a model.  Tensors bound after
 * this (ref_llm_create, the loaders) call the GPU; the reference's own
 * cats_llama2_transformer drives them. */
#include "catsgpu.h"
void ref_llm_dropin_tables(void)
{
    cats_gpu_init(-1);
    gguf_matmul[GGML_TYPE_F32] = cats_gpu_matmul_f32;
    gguf_matmul[GGML_TYPE_Q4_0] = cats_gpu_matmul_q4_0_q8;
    gguf_quantize[GGML_TYPE_Q4_0] = cats_gpu_quantize_q8;
    gguf_dequantize[GGML_TYPE_Q4_0] = cats_gpu_dequantize_q4_0;
    gguf_matmul[GGML_TYPE_Q3_K] = cats_gpu_matmul_q3_K_q8_K;
    gguf_matmul[GGML_TYPE_Q6_K] = cats_gpu_matmul_q6_K_q8_K;
    gguf_quantize[GGML_TYPE_Q3_K] = cats_gpu_quantize_q8_K;
    gguf_quantize[GGML_TYPE_Q6_K] = cats_gpu_quantize_q8_K;
}
#endif

void ref_llm_destroy(void *h)
{
    ref_model *r = h;
    cats_llm_model *m = &r->m;
    free(m->x); free(m->xb); free(m->xb2); free(m->hb); free(m->hb2); free(m->q);
    free(m->att); free(m->logits); free(m->key_cache); free(m->value_cache);
    free(r);
}
