// llm.cu — device-resident decode step for the llama2.c-architecture runtime.
//
// Restates cats_llama2_transformer (llm/catseye_llm.h:1625-1772) as a chain
// of five kernels per layer, launched with programmatic dependent launch and
// captured once into a CUDA graph:
//   qkv   : rmsnorm + quantize_q8 (in the prologue) -> [wq;wk;wv] matvec -> RoPE,
//           k and v written straight into the KV cache at pos          (:1657-1674)
//   attn  : split-time attention over the fp32 KV cache, GQA via kv_mul (:1677-1723)
//   wo    : quantize -> matvec -> residual add into x                   (:1726-1733)
//   w13   : rmsnorm + quantize -> interleaved [w1;w3] matvec -> SwiGLU (:1735-1752)
//   w2    : quantize -> matvec -> residual add into x                   (:1754-1761)
// then the classifier (final rmsnorm + matvec + greedy argmax, :1765-1770)
// and a one-thread kernel that feeds the argmax back as the next token.
#include "llm.cuh"
#include "mv_device.cuh"
#include <algorithm>
#include <cstring>

namespace cats {

// ------------------------------------------------------- synthetic weights
__device__ __forceinline__ unsigned long long mix64(unsigned long long z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// two N(0,1) samples (Box-Muller) for pair index p of tensor `tid`
__device__ __forceinline__ float2 normal2(unsigned long long seed, int tid, unsigned long long p)
{
    const unsigned long long h = mix64(seed * 0xD1B54A32D192ED03ull ^ ((unsigned long long)tid << 44) ^ p);
    const float u1 = (float)((h >> 40) + 1) * 0x1.0p-24f;            // (0, 1]
    const float u2 = (float)((h >> 16) & 0xffffff) * 0x1.0p-24f;     // [0, 1)
    const float r = sqrtf(-2.f * logf(u1));
    float s, c;
    sincospif(2.f * u2, &s, &c);
    return make_float2(r * c, r * s);
}

// one thread per 32-element group of row-major [d][n]
__global__ void k_synth(uint8_t *__restrict__ dst, int type, int n, long long ngroups, unsigned long long seed,
                        int tid, float std, float constant)
{
    for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < ngroups;
         g += (long long)gridDim.x * blockDim.x) {
        float v[32];
        const unsigned long long p0 = (unsigned long long)g * 16;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            float2 z = std != 0.f ? normal2(seed, tid, p0 + k) : make_float2(0.f, 0.f);
            v[2 * k] = constant + std * z.x;
            v[2 * k + 1] = constant + std * z.y;
        }
        if (type == W_F32) {
            float *o = reinterpret_cast<float *>(dst) + g * 32;
#pragma unroll
            for (int k = 0; k < 32; k++) o[k] = v[k];
            continue;
        }
        float amax = 0.f, mx = 0.f;
#pragma unroll
        for (int k = 0; k < 32; k++) {
            const float a = fabsf(v[k]);
            if (a > amax) { amax = a; mx = v[k]; }
        }
        if (type == W_Q4_0) {
            // d = signed absmax / -8, q = min(15, trunc(x/d + 8.5)) (the oracle's synthetic rule)
            const float d = mx / -8.f;
            const float id = d != 0.f ? 1.f / d : 0.f;
            uint8_t *o = dst + g * 18;
            const uint16_t hd = __half_as_ushort(__float2half_rn(d));
            o[0] = hd & 0xff;
            o[1] = hd >> 8;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int q0 = min(15, (int)(v[j] * id + 8.5f));
                const int q1 = min(15, (int)(v[j + 16] * id + 8.5f));
                o[2 + j] = (uint8_t)(q0 | (q1 << 4));
            }
        } else {
            const float d = amax / 127.f;
            const float id = d != 0.f ? 1.f / d : 0.f;
            uint8_t *o = dst + g * 34;
            const uint16_t hd = __half_as_ushort(__float2half_rn(d));
            o[0] = hd & 0xff;
            o[1] = hd >> 8;
#pragma unroll
            for (int j = 0; j < 32; j++) o[2 + j] = (uint8_t)(int8_t)(int)roundf(v[j] * id);
        }
    }
}

cudaError_t synth_tensor(uint8_t *dst, int type, int n, int d, unsigned long long seed, int tensor_id,
                         float std, float constant, cudaStream_t st)
{
    if (n % 32) return cudaErrorInvalidValue;
    long long ng = (long long)d * (n / 32);
    int grid = (int)std::min<long long>((ng + 127) / 128, 148LL * 16);
    if (grid < 1) grid = 1;
    k_synth<<<grid, 128, 0, st>>>(dst, type, n, ng, seed, tensor_id, std, constant);
    return cudaGetLastError();
}

// ------------------------------------------------------------- attention
struct AttnArgs {
    const float *q;        // [heads_loc * hs]
    const float *kc, *vc;  // this layer's cache: [seq_len][kv_dim]
    float *xb;             // [heads_loc * hs]
    float *part;           // [heads][splits][hs + 2]
    int *counters;         // [heads]
    const StepParams *params;
    int hs, kv_dim, kv_mul, n_splits, max_chunk, seq_len;
    int *err;
};

// Split-time ("flash-decode") attention.  CTA (h, c) scores timesteps of chunk
// c against query head h (score = q.k / sqrtf(head_size), :1693-1704), takes a
// local softmax, and writes (max, sum, weighted V); the last CTA of a head to
// arrive merges the splits into xb (:1706-1722).
__global__ void __launch_bounds__(128) k_attention(const __grid_constant__ AttnArgs a)
{
    extern __shared__ float sm[];
    pdl_wait();
    pdl_launch_dependents();
    const int h = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hs = a.hs;
    const int pos = a.params->pos;
    if (pos < 0 || pos >= a.seq_len) {   // refused by the qkv kernel too; xb is left as it was
        if (threadIdx.x == 0 && a.err) atomicOr(a.err, CATS_DEVERR_POS_RANGE);
        return;
    }
    const int T = pos + 1;
    const int chunk = (T + a.n_splits - 1) / a.n_splits;
    const int t0 = min(T, c * chunk), t1 = min(T, t0 + chunk);
    const int len = t1 - t0;
    float *qs = sm, *sc = sm + hs, *red = sc + a.max_chunk;
    const int kvo = (h / a.kv_mul) * hs;
    for (int i = tid; i < hs; i += blockDim.x) qs[i] = a.q[h * hs + i];
    __syncthreads();
    const float rs = sqrtf((float)hs);
    for (int t = t0 + warp; t < t1; t += blockDim.x / 32) {
        const float *k = a.kc + (size_t)t * a.kv_dim + kvo;
        float s = 0.f;
        for (int i = lane; i < hs; i += 32) s = fmaf(qs[i], k[i], s);
        s = warp_sum(s);
        if (lane == 0) sc[t - t0] = __fdiv_rn(s, rs);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int t = tid; t < len; t += blockDim.x) m = fmaxf(m, sc[t]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float l = 0.f;
    for (int t = tid; t < len; t += blockDim.x) {
        const float p = expf(sc[t] - m);
        sc[t] = p;
        l += p;
    }
    l = warp_sum(l);
    if (lane == 0) red[warp] = l;
    __syncthreads();
    l = red[0] + red[1] + red[2] + red[3];
    float *pp = a.part + ((size_t)h * a.n_splits + c) * (hs + 2);
    for (int i = tid; i < hs; i += blockDim.x) {
        float acc = 0.f;
        for (int t = 0; t < len; t++) acc = fmaf(sc[t], a.vc[(size_t)(t0 + t) * a.kv_dim + kvo + i], acc);
        pp[2 + i] = acc;
    }
    if (tid == 0) { pp[0] = len > 0 ? m : -INFINITY; pp[1] = l; }
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (tid == 0) last = (atomicAdd(&a.counters[h], 1) == a.n_splits - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    const float *ph = a.part + (size_t)h * a.n_splits * (hs + 2);
    float M = -INFINITY;
    for (int s = 0; s < a.n_splits; s++) M = fmaxf(M, ((volatile const float *)ph)[s * (hs + 2)]);
    float L = 0.f;
    for (int s = 0; s < a.n_splits; s++) {
        const float ms = ((volatile const float *)ph)[s * (hs + 2)];
        if (ms != -INFINITY) L += expf(ms - M) * ((volatile const float *)ph)[s * (hs + 2) + 1];
    }
    const float inv = 1.f / L;
    for (int i = tid; i < hs; i += blockDim.x) {
        float v = 0.f;
        for (int s = 0; s < a.n_splits; s++) {
            const float ms = ((volatile const float *)ph)[s * (hs + 2)];
            if (ms != -INFINITY) v += expf(ms - M) * ((volatile const float *)ph)[s * (hs + 2) + 2 + i];
        }
        a.xb[h * hs + i] = v * inv;
    }
    if (tid == 0) a.counters[h] = 0;
}

// greedy argmax -> next token; pos advances (sample_argmax, llm/catseye_llm.h:2042)
__global__ void k_advance(StepParams *p, unsigned long long *argmax, int vocab, int *err)
{
    pdl_wait();
    const unsigned long long k = *argmax;
    int idx = 0x7fffffff - (int)(uint32_t)(k & 0xffffffffu);
    if (k == 0ull || idx < 0 || idx >= vocab) {
        idx = 0;
        if (err) atomicOr(err, CATS_DEVERR_TOKEN_RANGE);
    }
    p->next = idx;
    p->token = idx;
    p->pos += 1;
    p->steps += 1;
    *argmax = 0ull;
}

// x += delta (tensor parallel: the allreduced output of wo or w2, :1731-1733, :1759-1761)
__global__ void k_residual_add(float *__restrict__ x, const float *__restrict__ delta, int n)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) x[i] += delta[i];
}

static cudaError_t launch_residual_add(float *x, const float *delta, int n, cudaStream_t st)
{
    k_residual_add<<<std::min(cdiv(n, 256), 148), 256, 0, st>>>(x, delta, n);
    return cudaGetLastError();
}

// ------------------------------------------------------------ model setup
static int pick_stages(const WeightLayout &L)
{
    const size_t stride = round_up(L.full_chunk, 128);
    int s = (int)(MV_STAGE_BUDGET / stride);
    return std::max(2, std::min(8, s));
}

static MatvecArgs base_args(const DevWeight &W, int *err)
{
    MatvecArgs a;
    a.w = W.ptr;
    a.n = W.L.n;
    a.d = W.L.d;
    a.R = W.L.R;
    a.units = W.L.units;
    a.nseg = W.L.nseg;
    a.n_tiles = W.L.n_tiles;
    a.unit_bytes = W.L.unit_bytes;
    a.full_chunk = W.L.full_chunk;
    a.last_chunk = W.L.last_chunk;
    a.tile_bytes = W.L.tile_bytes;
    a.stages = pick_stages(W.L);
    a.err = err;
    return a;
}

int llm_alloc(LlmModel *m, const LlmConfig &c)
{
    m->c = c;
    const int tp = c.tp_size > 0 ? c.tp_size : 1;
    m->c.tp_size = tp;
    if (c.dim % c.n_heads || c.n_heads % c.n_kv_heads || c.n_heads % tp || c.n_kv_heads % tp ||
        c.hidden % tp || c.vocab % tp || c.dim % 32 || (c.hidden / tp) % 32 || (c.dim / tp) % 32)
        return E_ARG;
    // the matvec's rmsnorm prologue holds the whole vector in one staging pass
    if (c.dim > 4 * STAGE_V * 32 * MV_CONSUMER_WARPS) return E_ARG;
    m->head_size = c.dim / c.n_heads;
    m->heads_loc = c.n_heads / tp;
    m->kv_heads_loc = c.n_kv_heads / tp;
    m->q_dim = m->heads_loc * m->head_size;
    m->kv_dim = m->kv_heads_loc * m->head_size;
    m->hidden_loc = c.hidden / tp;
    m->vocab_loc = c.vocab / tp;
    m->vocab_off = c.tp_rank * m->vocab_loc;
    m->n_splits = 8;
    m->qkv.resize(c.n_layers);
    m->wo.resize(c.n_layers);
    m->w13.resize(c.n_layers);
    m->w2.resize(c.n_layers);
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) return E_CUDA;
    size_t kv = (size_t)c.n_layers * c.seq_len * m->kv_dim;
    bool ok = true;
    ok &= cudaMalloc(&m->x, (size_t)c.dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->x2, (size_t)c.dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->delta, (size_t)c.dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->q, (size_t)m->q_dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->xb, (size_t)m->q_dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->hb, (size_t)m->hidden_loc * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->logits, (size_t)c.vocab * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->kcache, kv * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->vcache, kv * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->part, (size_t)m->heads_loc * m->n_splits * (m->head_size + 2) * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->counters, (size_t)m->heads_loc * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->argmax, 8) == cudaSuccess;
    ok &= cudaMalloc(&m->params, sizeof(StepParams)) == cudaSuccess;
    ok &= cudaMalloc(&m->err, 4) == cudaSuccess;
    ok &= cudaMallocHost(&m->params_host, sizeof(StepParams)) == cudaSuccess;
    ok &= cudaMallocHost(&m->logits_host, (size_t)c.vocab * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->emb, (size_t)c.vocab * c.dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->rms_att, (size_t)c.n_layers * c.dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->rms_ffn, (size_t)c.n_layers * c.dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->rms_final, (size_t)c.dim * 4) == cudaSuccess;
    if (!ok) return E_NOMEM;
    cudaMemsetAsync(m->kcache, 0, kv * 4, m->stream);
    cudaMemsetAsync(m->vcache, 0, kv * 4, m->stream);
    cudaMemsetAsync(m->counters, 0, (size_t)m->heads_loc * 4, m->stream);
    cudaMemsetAsync(m->argmax, 0, 8, m->stream);
    cudaMemsetAsync(m->params, 0, sizeof(StepParams), m->stream);
    cudaMemsetAsync(m->err, 0, 4, m->stream);
    cudaMemsetAsync(m->logits, 0, (size_t)c.vocab * 4, m->stream);
    return cudaStreamSynchronize(m->stream) == cudaSuccess ? E_OK : E_CUDA;
}

static void free_w(DevWeight &w)
{
    if (w.ptr) cudaFree(w.ptr);
    w.ptr = nullptr;
}

void llm_free(LlmModel *m)
{
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    m->exec = nullptr;
    m->graph = nullptr;
    llm_batch_free(m);
    tp_release(m);   // after the graphs that hold its NCCL calls
    for (auto &w : m->qkv) free_w(w);
    for (auto &w : m->wo) free_w(w);
    for (auto &w : m->w13) free_w(w);
    for (auto &w : m->w2) free_w(w);
    free_w(m->cls);
    float **fp[] = {&m->x, &m->x2, &m->delta, &m->q, &m->xb, &m->hb, &m->logits, &m->kcache, &m->vcache,
                    &m->part, &m->emb, &m->rms_att, &m->rms_ffn, &m->rms_final};
    for (auto p : fp) if (*p) { cudaFree(*p); *p = nullptr; }
    if (m->wdesc) cudaFree(m->wdesc);
    if (m->dec_part) cudaFree(m->dec_part);
    if (m->dec_bar) cudaFree(m->dec_bar);
    m->wdesc = nullptr;
    m->dec_part = nullptr;
    m->dec_bar = nullptr;
    if (m->counters) cudaFree(m->counters);
    if (m->argmax) cudaFree(m->argmax);
    if (m->params) cudaFree(m->params);
    if (m->err) cudaFree(m->err);
    if (m->params_host) cudaFreeHost(m->params_host);
    if (m->logits_host) cudaFreeHost(m->logits_host);
    if (m->stream) cudaStreamDestroy(m->stream);
    m->counters = nullptr; m->argmax = nullptr; m->params = nullptr; m->err = nullptr;
    m->params_host = nullptr; m->logits_host = nullptr; m->stream = nullptr;
}

// A tensor source: a full [d][n] matrix in the reference's GGUF layout, either
// host memory (copied) or device memory.
struct Src {
    const uint8_t *p;
    bool host;
};

// Copy rows [r0, r0+nr) and byte columns [c0, c0+cw) of a source matrix with row
// pitch `sp` into dst with row pitch `dp`.
static cudaError_t copy_slice(uint8_t *dst, size_t dp, Src s, size_t sp, size_t r0, size_t nr, size_t c0, size_t cw,
                              cudaStream_t st)
{
    return cudaMemcpy2DAsync(dst, dp, s.p + r0 * sp + c0, sp, cw, nr,
                             s.host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, st);
}

static int finish_weight(DevWeight &W, int type, int n, int d, int rpw, const uint8_t *staging, cudaStream_t st)
{
    W.L = make_layout(type, n, d, rpw);
    if (cudaMalloc(&W.ptr, W.L.total_bytes) != cudaSuccess) return E_NOMEM;
    return launch_repack(staging, W.ptr, W.L, st) == cudaSuccess ? E_OK : E_CUDA;
}

// Build the fused, sharded device weights of one layer from full sources.
static int build_layer(LlmModel *m, int l, Src wq, Src wk, Src wv, Src wo, Src w1, Src w2, Src w3, uint8_t *stg)
{
    const LlmConfig &c = m->c;
    const int t = c.wtype, r = c.tp_rank;
    const int kvd_full = c.dim * c.n_kv_heads / c.n_heads;
    const size_t rb_dim = gguf_row_bytes(t, c.dim), rb_hid = gguf_row_bytes(t, c.hidden);
    cudaStream_t st = m->stream;
    cudaError_t e = cudaSuccess;
    // qkv: this rank's head rows of wq, wk, wv stacked
    e = copy_slice(stg, rb_dim, wq, rb_dim, (size_t)r * m->q_dim, m->q_dim, 0, rb_dim, st);
    if (e == cudaSuccess)
        e = copy_slice(stg + (size_t)m->q_dim * rb_dim, rb_dim, wk, rb_dim, (size_t)r * m->kv_dim, m->kv_dim, 0, rb_dim, st);
    if (e == cudaSuccess)
        e = copy_slice(stg + (size_t)(m->q_dim + m->kv_dim) * rb_dim, rb_dim, wv, rb_dim, (size_t)r * m->kv_dim,
                       m->kv_dim, 0, rb_dim, st);
    if (e != cudaSuccess) return E_CUDA;
    int rc = finish_weight(m->qkv[l], t, c.dim, m->q_dim + 2 * m->kv_dim, 2, stg, st);
    if (rc) return rc;
    if (cudaStreamSynchronize(st) != cudaSuccess) return E_CUDA;
    // wo: all dim rows, this rank's input columns
    const size_t cw_o = gguf_row_bytes(t, m->q_dim);
    if (copy_slice(stg, cw_o, wo, rb_dim, 0, c.dim, (size_t)r * cw_o, cw_o, st) != cudaSuccess) return E_CUDA;
    if ((rc = finish_weight(m->wo[l], t, m->q_dim, c.dim, 2, stg, st))) return rc;
    if (cudaStreamSynchronize(st) != cudaSuccess) return E_CUDA;
    // w13: this rank's hidden rows of w1 and w3, interleaved (row 2i = w1_i, 2i+1 = w3_i)
    if (copy_slice(stg, 2 * rb_dim, w1, rb_dim, (size_t)r * m->hidden_loc, m->hidden_loc, 0, rb_dim, st) != cudaSuccess)
        return E_CUDA;
    if (copy_slice(stg + rb_dim, 2 * rb_dim, w3, rb_dim, (size_t)r * m->hidden_loc, m->hidden_loc, 0, rb_dim, st) !=
        cudaSuccess)
        return E_CUDA;
    if ((rc = finish_weight(m->w13[l], t, c.dim, 2 * m->hidden_loc, 2, stg, st))) return rc;
    if (cudaStreamSynchronize(st) != cudaSuccess) return E_CUDA;
    // w2: all dim rows, this rank's hidden columns
    const size_t cw_2 = gguf_row_bytes(t, m->hidden_loc);
    if (copy_slice(stg, cw_2, w2, rb_hid, 0, c.dim, (size_t)r * cw_2, cw_2, st) != cudaSuccess) return E_CUDA;
    if ((rc = finish_weight(m->w2[l], t, m->hidden_loc, c.dim, 2, stg, st))) return rc;
    (void)kvd_full;
    return cudaStreamSynchronize(st) == cudaSuccess ? E_OK : E_CUDA;
}

static int build_cls(LlmModel *m, Src wcls, uint8_t *stg)
{
    const LlmConfig &c = m->c;
    const size_t rb = gguf_row_bytes(c.wtype, c.dim);
    if (copy_slice(stg, rb, wcls, rb, (size_t)m->vocab_off, m->vocab_loc, 0, rb, m->stream) != cudaSuccess) return E_CUDA;
    int rc = finish_weight(m->cls, c.wtype, c.dim, m->vocab_loc, 2, stg, m->stream);
    if (rc) return rc;
    return cudaStreamSynchronize(m->stream) == cudaSuccess ? E_OK : E_CUDA;
}

static size_t staging_bytes(const LlmConfig &c)
{
    const size_t rb_dim = gguf_row_bytes(c.wtype, c.dim), rb_hid = gguf_row_bytes(c.wtype, c.hidden);
    size_t s = std::max((size_t)c.dim * 3 * rb_dim, (size_t)c.hidden * 2 * rb_dim);
    s = std::max(s, (size_t)c.dim * rb_hid);
    s = std::max(s, (size_t)c.vocab * rb_dim);
    return s;
}

int llm_set_weights(LlmModel *m, const float *emb, const float *rms_att, const float *rms_ffn, const float *rms_final,
                    const void *wq, const void *wk, const void *wv, const void *wo, const void *w1, const void *w2,
                    const void *w3, const void *wcls)
{
    const LlmConfig &c = m->c;
    cudaStream_t st = m->stream;
    const int kvd_full = c.dim * c.n_kv_heads / c.n_heads;
    if (cudaMemcpyAsync(m->emb, emb, (size_t)c.vocab * c.dim * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(m->rms_att, rms_att, (size_t)c.n_layers * c.dim * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(m->rms_ffn, rms_ffn, (size_t)c.n_layers * c.dim * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(m->rms_final, rms_final, (size_t)c.dim * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return E_CUDA;
    uint8_t *stg = nullptr;
    if (cudaMalloc(&stg, staging_bytes(c)) != cudaSuccess) return E_NOMEM;
    const int t = c.wtype;
    const size_t rb_dim = gguf_row_bytes(t, c.dim), rb_hid = gguf_row_bytes(t, c.hidden);
    int rc = E_OK;
    for (int l = 0; l < c.n_layers && rc == E_OK; l++) {
        auto at = [&](const void *base, size_t mat_bytes) {
            return Src{static_cast<const uint8_t *>(base) + mat_bytes * l, true};
        };
        rc = build_layer(m, l, at(wq, rb_dim * c.dim), at(wk, rb_dim * kvd_full), at(wv, rb_dim * kvd_full),
                         at(wo, rb_dim * c.dim), at(w1, rb_dim * c.hidden), at(w2, rb_hid * c.dim),
                         at(w3, rb_dim * c.hidden), stg);
    }
    if (rc == E_OK) rc = build_cls(m, Src{static_cast<const uint8_t *>(wcls), true}, stg);
    cudaFree(stg);
    m->weights_ready = rc == E_OK;
    return rc;
}

int llm_set_weights_layers(LlmModel *m, const float *emb, const float *rms_att, const float *rms_ffn,
                           const float *rms_final, const void *const *layer_w, const void *wcls)
{
    const LlmConfig &c = m->c;
    cudaStream_t st = m->stream;
    if (cudaMemcpyAsync(m->emb, emb, (size_t)c.vocab * c.dim * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(m->rms_att, rms_att, (size_t)c.n_layers * c.dim * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(m->rms_ffn, rms_ffn, (size_t)c.n_layers * c.dim * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(m->rms_final, rms_final, (size_t)c.dim * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return E_CUDA;
    uint8_t *stg = nullptr;
    if (cudaMalloc(&stg, staging_bytes(c)) != cudaSuccess) return E_NOMEM;
    int rc = E_OK;
    for (int l = 0; l < c.n_layers && rc == E_OK; l++) {
        const void *const *w = layer_w + 7 * (size_t)l;
        auto h = [](const void *p) { return Src{static_cast<const uint8_t *>(p), true}; };
        rc = build_layer(m, l, h(w[0]), h(w[1]), h(w[2]), h(w[3]), h(w[4]), h(w[5]), h(w[6]), stg);
    }
    if (rc == E_OK) rc = build_cls(m, Src{static_cast<const uint8_t *>(wcls), true}, stg);
    cudaFree(stg);
    m->weights_ready = rc == E_OK;
    return rc;
}

// tensor ids of the synthetic generator (fixed so every TP rank regenerates the same tensors)
enum { T_EMB = 0, T_RMS_ATT = 1, T_RMS_FFN = 2, T_RMS_FINAL = 3, T_WCLS = 4, T_LAYER0 = 16 };
static int layer_tid(int l, int k) { return T_LAYER0 + l * 8 + k; }   // k: 0 wq 1 wk 2 wv 3 wo 4 w1 5 w2 6 w3

int llm_init_random(LlmModel *m, unsigned long long seed, float std)
{
    const LlmConfig &c = m->c;
    cudaStream_t st = m->stream;
    const int t = c.wtype;
    const int kvd_full = c.dim * c.n_kv_heads / c.n_heads;
    if (synth_tensor(reinterpret_cast<uint8_t *>(m->emb), W_F32, c.dim, c.vocab, seed, T_EMB, std, 0.f, st) ||
        synth_tensor(reinterpret_cast<uint8_t *>(m->rms_att), W_F32, c.dim, c.n_layers, seed, T_RMS_ATT, 0.f, 1.f, st) ||
        synth_tensor(reinterpret_cast<uint8_t *>(m->rms_ffn), W_F32, c.dim, c.n_layers, seed, T_RMS_FFN, 0.f, 1.f, st) ||
        synth_tensor(reinterpret_cast<uint8_t *>(m->rms_final), W_F32, c.dim, 1, seed, T_RMS_FINAL, 0.f, 1.f, st))
        return E_CUDA;
    const size_t rb_dim = gguf_row_bytes(t, c.dim), rb_hid = gguf_row_bytes(t, c.hidden);
    // full (unsharded) sources of one layer, generated on the device
    size_t sz[7] = {rb_dim * c.dim, rb_dim * kvd_full, rb_dim * kvd_full, rb_dim * c.dim,
                    rb_dim * c.hidden, rb_hid * c.dim, rb_dim * c.hidden};
    int nn[7] = {c.dim, c.dim, c.dim, c.dim, c.dim, c.hidden, c.dim};
    int dd[7] = {c.dim, kvd_full, kvd_full, c.dim, c.hidden, c.dim, c.hidden};
    uint8_t *src[7] = {};
    uint8_t *stg = nullptr;
    int rc = E_OK;
    for (int k = 0; k < 7 && rc == E_OK; k++) if (cudaMalloc(&src[k], sz[k]) != cudaSuccess) rc = E_NOMEM;
    if (rc == E_OK && cudaMalloc(&stg, staging_bytes(c)) != cudaSuccess) rc = E_NOMEM;
    for (int l = 0; l < c.n_layers && rc == E_OK; l++) {
        for (int k = 0; k < 7; k++)
            if (synth_tensor(src[k], t, nn[k], dd[k], seed, layer_tid(l, k), std, 0.f, st) != cudaSuccess) rc = E_CUDA;
        if (rc == E_OK)
            rc = build_layer(m, l, Src{src[0], false}, Src{src[1], false}, Src{src[2], false}, Src{src[3], false},
                             Src{src[4], false}, Src{src[5], false}, Src{src[6], false}, stg);
    }
    for (int k = 0; k < 7; k++) if (src[k]) cudaFree(src[k]);
    if (rc == E_OK) {
        uint8_t *cls = nullptr;
        if (cudaMalloc(&cls, rb_dim * c.vocab) != cudaSuccess) rc = E_NOMEM;
        else {
            if (t == W_F32)   // llama2.c checkpoints share the classifier with the embedding (:2924)
                rc = cudaMemcpyAsync(cls, m->emb, rb_dim * c.vocab, cudaMemcpyDeviceToDevice, st) ? E_CUDA : E_OK;
            else
                rc = synth_tensor(cls, t, c.dim, c.vocab, seed, T_WCLS, std, 0.f, st) ? E_CUDA : E_OK;
            if (rc == E_OK) rc = build_cls(m, Src{cls, false}, stg);
            cudaFree(cls);
        }
    }
    if (stg) cudaFree(stg);
    m->weights_ready = rc == E_OK;
    return rc;
}

// ------------------------------------------------------------------- step
static cudaError_t launch_attention(LlmModel *m, int l, cudaStream_t st)
{
    AttnArgs a;
    const size_t loff = (size_t)l * m->c.seq_len * m->kv_dim;
    a.q = m->q;
    a.kc = m->kcache + loff;
    a.vc = m->vcache + loff;
    a.xb = m->xb;
    a.part = m->part;
    a.counters = m->counters;
    a.params = m->params;
    a.hs = m->head_size;
    a.kv_dim = m->kv_dim;
    a.kv_mul = m->c.n_heads / m->c.n_kv_heads;
    a.n_splits = m->n_splits;
    a.max_chunk = (m->c.seq_len + m->n_splits - 1) / m->n_splits;
    a.seq_len = m->c.seq_len;
    a.err = m->err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m->heads_loc, m->n_splits);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = (size_t)(a.hs + a.max_chunk + 8) * 4;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_attention, a);
}

static cudaError_t launch_advance(LlmModel *m, cudaStream_t st)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_advance, m->params, m->argmax, m->c.vocab, m->err);
}

cudaError_t llm_enqueue_step(LlmModel *m, bool advance)
{
    const LlmConfig &c = m->c;
    cudaStream_t st = m->stream;
    const bool quant = c.wtype != W_F32;
    const int xmode = quant ? XM_Q8_FROM_F32 : XM_F32;
    const bool tp = c.tp_size > 1;
    cudaError_t e;
    for (int l = 0; l < c.n_layers; l++) {
        MatvecArgs a = base_args(m->qkv[l], m->err);
        a.xmode = xmode;
        if (l == 0) {
            a.x = m->emb;                   // dequantize(x, emb, token, dim): fp32 row copy (:1652)
            a.x_row = &m->params->token;
            a.x_writeback = m->x;
        } else {
            a.x = m->x;
        }
        a.norm_w = m->rms_att + (size_t)l * c.dim;
        a.epi = EPI_QKV_ROPE;
        a.out = m->q;
        a.k_out = m->kcache + (size_t)l * c.seq_len * m->kv_dim;
        a.v_out = m->vcache + (size_t)l * c.seq_len * m->kv_dim;
        a.pos = &m->params->pos;
        a.q_dim = m->q_dim;
        a.kv_dim = m->kv_dim;
        a.head_size = m->head_size;
        a.kv_rows = c.seq_len;
        if ((e = launch_matvec(a, 2, c.wtype, st, true))) return e;

        if ((e = launch_attention(m, l, st))) return e;

        // wo (and w2 below): with tensor parallelism each rank holds a column
        // slice, so its output is a partial sum: sum-allreduce, then add
        a = base_args(m->wo[l], m->err);
        a.xmode = xmode;
        a.x = m->xb;
        if (!tp) { a.epi = EPI_ADD; a.out = m->x; }
        else { a.epi = EPI_STORE; a.out = m->delta; }
        if ((e = launch_matvec(a, 2, c.wtype, st, true))) return e;
        if (tp) {
            m->allreduce(m->comm_ctx, m->delta, c.dim, st);
            if ((e = launch_residual_add(m->x, m->delta, c.dim, st))) return e;
        }

        a = base_args(m->w13[l], m->err);
        a.xmode = xmode;
        a.x = m->x;
        a.norm_w = m->rms_ffn + (size_t)l * c.dim;
        a.epi = EPI_SWIGLU;
        a.out = m->hb;
        if ((e = launch_matvec(a, 2, c.wtype, st, true))) return e;

        a = base_args(m->w2[l], m->err);
        a.xmode = xmode;
        a.x = m->hb;
        if (!tp) { a.epi = EPI_ADD; a.out = m->x; }
        else { a.epi = EPI_STORE; a.out = m->delta; }
        if ((e = launch_matvec(a, 2, c.wtype, st, true))) return e;
        if (tp) {
            m->allreduce(m->comm_ctx, m->delta, c.dim, st);
            if ((e = launch_residual_add(m->x, m->delta, c.dim, st))) return e;
        }
    }
    MatvecArgs a = base_args(m->cls, m->err);
    a.xmode = xmode;
    a.x = m->x;
    a.norm_w = m->rms_final;
    a.epi = EPI_STORE_ARGMAX;
    a.out = m->logits + m->vocab_off;
    a.argmax = m->argmax;
    a.argmax_base = m->vocab_off;
    if ((e = launch_matvec(a, 2, c.wtype, st, true))) return e;
    if (tp) {
        // the greedy token over every rank's vocabulary rows, and the full logits
        m->argmax_reduce(m->comm_ctx, m->argmax, st);
        m->allgather(m->comm_ctx, m->logits, (size_t)m->vocab_loc, c.tp_rank, st);
    }
    if (advance && (e = launch_advance(m, st))) return e;
    return cudaSuccess;
}

cudaError_t llm_time_matvec(LlmModel *m, int kind, int reps, float *ms_per_launch, double *bytes_per_launch)
{
    const LlmConfig &c = m->c;
    const bool quant = c.wtype != W_F32;
    std::vector<const DevWeight *> ws;
    for (int l = 0; l < c.n_layers; l++) {
        if (kind == 0) ws.push_back(&m->qkv[l]);
        else if (kind == 1) ws.push_back(&m->wo[l]);
        else if (kind == 2) ws.push_back(&m->w13[l]);
        else if (kind == 3) ws.push_back(&m->w2[l]);
    }
    if (kind == 4) ws.push_back(&m->cls);
    if (ws.empty() || reps <= 0) return cudaErrorInvalidValue;
    float *scratch = nullptr;
    size_t maxd = 0;
    for (auto w : ws) maxd = std::max(maxd, (size_t)w->L.d);
    cudaError_t e = cudaMalloc(&scratch, maxd * 4);
    if (e) return e;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    auto run = [&](int passes) -> cudaError_t {
        for (int r = 0; r < passes; r++)
            for (auto w : ws) {
                MatvecArgs a = base_args(*w, m->err);
                a.xmode = quant ? XM_Q8_FROM_F32 : XM_F32;
                a.x = (kind == 3) ? m->hb : (kind == 1 ? m->xb : m->x);
                a.norm_w = (kind == 0 || kind == 2) ? m->rms_att : (kind == 4 ? m->rms_final : nullptr);
                a.epi = EPI_STORE;
                a.out = scratch;
                cudaError_t le = launch_matvec(a, w->L.rpw, c.wtype, m->stream, true);
                if (le) return le;
            }
        return cudaSuccess;
    };
    e = run(1);   // warm-up
    if (!e) e = cudaEventRecord(e0, m->stream);
    if (!e) e = run(reps);
    if (!e) e = cudaEventRecord(e1, m->stream);
    if (!e) e = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (!e) cudaEventElapsedTime(&ms, e0, e1);
    const DevWeight *w = ws[0];
    const double xbytes = quant ? (double)w->L.n * 4 : (double)w->L.n * 4;
    *ms_per_launch = ms / (float)(reps * ws.size());
    *bytes_per_launch = (double)gguf_row_bytes(w->L.type, w->L.n) * w->L.d + xbytes + (double)w->L.d * 4;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(scratch);
    return e;
}

cudaError_t llm_build_graph(LlmModel *m)
{
    if (m->exec) return cudaSuccess;
    cudaError_t e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
    if (e) return e;
    cudaError_t e2 = llm_enqueue_step(m, true);
    e = cudaStreamEndCapture(m->stream, &m->graph);
    if (e2) return e2;
    if (e) return e;
    return cudaGraphInstantiate(&m->exec, m->graph, 0);
}

} // namespace cats
