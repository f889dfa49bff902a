// batch.cu — batched transformer step on the tensor cores: T tokens through
// the model at once, each with its own position and KV-cache sequence.
//
// It restates cats_llama2_transformer (llm/catseye_llm.h:1625-1772) for T
// tokens together, which serves two callers:
//  * prefill: the prompt of one sequence at positions p0 .. p0+T-1, which the
//    reference feeds one transformer call at a time;
//  * batched decode: one token of each of several sequences per step.
// Every weight product is one launch of the tcgen05 product (qgemm.cu) over
// all T tokens, so the weights stream from HBM once per step, not once per
// token.  The activations enter those products as fp16, so the step is the
// reference's fp32-activation binding (matmul_q4_0 with quantize_null,
// :880-914, :2593-2595) up to fp16 rounding of the operands.
//
// Per layer (the x16 operand is qgemm's swizzled fp16 layout, x16_chunk):
//   k_rmsnorm_x16     rmsnorm(x) -> x16                               (:1655, 684-698)
//   qgemm [wq;wk;wv]  -> y
//   k_rope_kv         RoPE on q and k; k and v into the cache          (:1657-1674, 1597-1620)
//   k_attn_batch      causal attention of every token over its
//                     sequence's cache, GQA via kv_mul                 (:1677-1723)
//   launch_x16        attention output -> x16
//   qgemm wo          accumulated into the residual stream x           (:1726-1733)
//   k_rmsnorm_x16, qgemm [w1;w3] (rows interleaved), k_swiglu_x16      (:1735-1752)
//   qgemm w2          accumulated into x                               (:1754-1761)
// then the final rmsnorm, the classifier product and a greedy argmax per
// token (:1765-1770, sample_argmax :1944-1956).  With tensor parallelism the
// wo and w2 products go to a delta buffer that is sum-allreduced and added,
// and the classifier slices are allgathered, as in the decode graph.
#include "llm.cuh"
#include "mv_device.cuh"
#include "qgemm.cuh"
#include <algorithm>
#include <cstring>
#include <vector>

namespace cats {

constexpr int AT_THREADS = 256;
constexpr int AT_KC = 32;          // cache positions per chunk
constexpr int DEC_MAX_HS_ATT = 128; // head size k_attn_tok holds as one float4 per lane
constexpr int AT_NQ = 64;          // query rows per CTA: tokens x the query heads of one kv head
constexpr int AT_MAXHS = 128;

// ------------------------------------------------------------- small kernels
// A product's element i: y[i], or, for a K split the product left to its
// reader (SplitOut), the sum of the partials in split order, the arithmetic
// of the split-sum kernel.
struct PartSrc {
    const float *y;
    const float *ws;
    int splits;
    long long count;   // elements of one partial slab ([T][d])

    __device__ __forceinline__ float ld1(size_t i) const
    {
        if (splits <= 1) return y[i];
        float p = 0.f;
        for (int z = 0; z < splits; z++) p += ws[(size_t)z * count + i];
        return p;
    }
    __device__ __forceinline__ float2 ld2(size_t i) const
    {
        if (splits <= 1) return *reinterpret_cast<const float2 *>(y + i);
        float2 p = make_float2(0.f, 0.f);
        for (int z = 0; z < splits; z++) {
            const float2 v = *reinterpret_cast<const float2 *>(ws + (size_t)z * count + i);
            p.x += v.x;
            p.y += v.y;
        }
        return p;
    }
    __device__ __forceinline__ float4 ld4(size_t i) const
    {
        if (splits <= 1) return *reinterpret_cast<const float4 *>(y + i);
        float4 p = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int z = 0; z < splits; z++) {
            const float4 v = *reinterpret_cast<const float4 *>(ws + (size_t)z * count + i);
            p.x += v.x;
            p.y += v.y;
            p.z += v.z;
            p.w += v.w;
        }
        return p;
    }
};

static PartSrc part_src(const float *y, const SplitOut &so, long long count)
{
    return PartSrc{y, so.ws, so.splits, count};
}

// x[t] = emb[token_t] (dequantize(x, emb, token, dim) of an fp32 table, :1652)
__global__ void k_embed(const BatchTok *__restrict__ bt, const float *__restrict__ emb, float *__restrict__ x, int dim,
                        int vocab, int *err)
{
    const int t = blockIdx.x;
    const int tok = bt[t].token;
    const bool ok = tok >= 0 && tok < vocab;
    if (!ok && threadIdx.x == 0 && err) atomicOr(err, CATS_DEVERR_TOKEN_RANGE);
    const float4 *src = reinterpret_cast<const float4 *>(emb + (size_t)(ok ? tok : 0) * dim);
    float4 *dst = reinterpret_cast<float4 *>(x + (size_t)t * dim);
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) dst[i] = ok ? __ldg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
}

// rmsnorm (llm/catseye_llm.h:684-698: ss = mean(x^2) + 1e-5, o = w * (x / sqrt(ss)))
// of token t's row, written as fp16 into the x16 operand.  One CTA per token.
// `add` (a residual product whose K split was left to this kernel): x += the
// product first, and the sum is written back (the residual stream).
__global__ void __launch_bounds__(256) k_rmsnorm_x16(float *__restrict__ x, const float *__restrict__ w,
                                                     __half *__restrict__ x16, int n, int Tpad, PartSrc add)
{
    __shared__ float red[8];
    const int t = blockIdx.x, tid = threadIdx.x;
    float4 *xr = reinterpret_cast<float4 *>(x + (size_t)t * n);
    float ss = 0.f;
    for (int i = tid; i < n / 4; i += blockDim.x) {
        float4 v = xr[i];
        if (add.splits > 1) {
            const float4 p = add.ld4((size_t)t * n + 4 * i);
            v = make_float4(v.x + p.x, v.y + p.y, v.z + p.z, v.w + p.w);
            xr[i] = v;
        }
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; k++) tot += red[k];
    tot = tot / (float)n + 1e-5f;
    const float sc = 1.f / sqrtf(tot);
    const float4 *wr = reinterpret_cast<const float4 *>(w);
    for (int ci = tid; ci < n / 8; ci += blockDim.x) {
        const int kb = ci >> 3, c = ci & 7, o4 = (kb * 64 + x16_src_off(c)) / 4;
        const float4 a0 = xr[o4], a1 = xr[o4 + 4];
        const float4 w0 = __ldg(wr + o4), w1 = __ldg(wr + o4 + 4);
        const float4 r0 = make_float4(w0.x * (sc * a0.x), w0.y * (sc * a0.y), w0.z * (sc * a0.z), w0.w * (sc * a0.w));
        const float4 r1 = make_float4(w1.x * (sc * a1.x), w1.y * (sc * a1.y), w1.z * (sc * a1.z), w1.w * (sc * a1.w));
        *reinterpret_cast<uint4 *>(x16 + x16_chunk(kb, c, t, Tpad)) = x16_pack(r0, r1);
    }
}

// RoPE (rope_llama, :1597-1620) on the q and k rows of the qkv product, q to
// q[t], k and v into the cache at (sequence, layer, pos).  One thread per pair.
__global__ void k_rope_kv(PartSrc y, int T, const BatchTok *__restrict__ bt, float *__restrict__ q,
                          float *__restrict__ kc, float *__restrict__ vc, size_t seq_stride, size_t layer_off,
                          int q_dim, int kv_dim, int hs, int seq_len, int n_seqs, int *err)
{
    const int qkv = q_dim + 2 * kv_dim, np = qkv / 2;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)T * np;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / np), r0 = 2 * (int)(i % np);
        const BatchTok b = bt[t];
        float2 v = y.ld2((size_t)t * qkv + r0);
        if (r0 < q_dim) {
            rope_pair(v.x, v.y, r0, hs, b.pos);
            *reinterpret_cast<float2 *>(q + (size_t)t * q_dim + r0) = v;
            continue;
        }
        if (b.pos < 0 || b.pos >= seq_len || b.seq < 0 || b.seq >= n_seqs) {
            if (r0 == q_dim && err) atomicOr(err, CATS_DEVERR_POS_RANGE);   // no cache write
            continue;
        }
        const bool is_k = r0 < q_dim + kv_dim;
        const int idx = r0 - q_dim - (is_k ? 0 : kv_dim);
        if (is_k) rope_pair(v.x, v.y, idx, hs, b.pos);
        float *c = (is_k ? kc : vc) + (size_t)b.seq * seq_stride + layer_off + (size_t)b.pos * kv_dim + idx;
        *reinterpret_cast<float2 *>(c) = v;
    }
}

// SwiGLU of the interleaved [w1;w3] product (row 2i = w1_i x, 2i+1 = w3_i x):
// h_i = silu(w1_i x) * (w3_i x) (:1744-1752), written as fp16 into x16.
__global__ void k_swiglu_x16(PartSrc y, int T, int hidden, __half *__restrict__ x16, int Tpad)
{
    const int cpr = hidden / 8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)T * cpr;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / cpr), ci = (int)(i % cpr), kb = ci >> 3, c = ci & 7;
        const int e0 = kb * 64 + x16_src_off(c);
        const size_t row = (size_t)t * 2 * hidden;
        float h[8];
#pragma unroll
        for (int run = 0; run < 2; run++) {
            const size_t src = row + 2 * (e0 + 16 * run);
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const float4 v = y.ld4(src + 4 * j);
                h[4 * run + 2 * j] = v.x * (1.f / (1.f + expf(-v.x))) * v.y;
                h[4 * run + 2 * j + 1] = v.z * (1.f / (1.f + expf(-v.z))) * v.w;
            }
        }
        *reinterpret_cast<uint4 *>(x16 + x16_chunk(kb, c, t, Tpad)) =
            x16_pack(make_float4(h[0], h[1], h[2], h[3]), make_float4(h[4], h[5], h[6], h[7]));
    }
}

__global__ void k_add(float *__restrict__ x, const float *__restrict__ d, long long n)
{
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        x[i] += d[i];
}

// Logits of token t from the classifier slices lg[tp][T][vocab_loc] into
// logits[t][vocab], and the greedy argmax (first maximum) into next[t].
__global__ void __launch_bounds__(256) k_logits_argmax(PartSrc lg, int T, int vocab_loc, int tp,
                                                       float *__restrict__ logits, int *__restrict__ next, int *err)
{
    __shared__ unsigned long long red[8];
    const int t = blockIdx.x, tid = threadIdx.x;
    const int vocab = vocab_loc * tp;
    unsigned long long best = 0ull;
    for (int j = tid; j < vocab; j += blockDim.x) {
        const int r = j / vocab_loc, jj = j - r * vocab_loc;
        const float v = lg.ld1(((size_t)r * T + t) * vocab_loc + jj);
        logits[(size_t)t * vocab + j] = v;
        const unsigned long long k = argmax_key(v, j);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if ((tid & 31) == 0) red[tid >> 5] = best;
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < 8; w++) best = red[w] > best ? red[w] : best;
        best = red[0] > best ? red[0] : best;
        int idx = 0x7fffffff - (int)(uint32_t)(best & 0xffffffffu);
        if (best == 0ull || idx < 0 || idx >= vocab) {
            idx = 0;
            if (err) atomicOr(err, CATS_DEVERR_TOKEN_RANGE);
        }
        next[t] = idx;
    }
}

// The generate loop's advance: every token's argmax becomes its next input
// at the next position; the ids are logged per step.
__global__ void k_batch_advance(BatchTok *bt, const int *next, int T, int *log, int log_cap, int *step)
{
    const int s = *step;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const int nx = next[t];
        bt[t].token = nx;
        bt[t].pos += 1;
        if (log && s < log_cap) log[(size_t)s * T + t] = nx;
    }
    __syncthreads();
    if (threadIdx.x == 0) *step = s + 1;
}

// --------------------------------------------------------------- attention
struct AttnBatchArgs {
    const float *q;          // [T][q_dim], RoPE applied
    const float *kc, *vc;    // cache base: [seq][layer][seq_len][kv_dim]
    size_t seq_stride, layer_off;
    const BatchTok *tok;
    const int2 *blocks;      // query blocks: (first token, count), tokens of one sequence
    float *xb;               // [T][q_dim]
    int q_dim, kv_dim, hs, kv_mul, seq_len, n_seqs;
};

__host__ __device__ inline size_t attn_smem_floats(int hs)
{
    // sQ [hs][NQ+1], sK [hs][KC+4], sV [KC][hs+4], sS [NQ][KC+1], sM/sL/sA [NQ], limits [NQ]
    return (size_t)hs * (AT_NQ + 1) + (size_t)hs * (AT_KC + 4) + (size_t)AT_KC * (hs + 4) + AT_NQ * (AT_KC + 1) +
           4 * AT_NQ;
}

// Causal attention for one query block (up to AT_NQ rows: the block's tokens
// times the kv_mul query heads that share kv head g) over the block's
// sequence, in chunks of AT_KC cache positions staged in shared memory:
// scores q.k / sqrt(head_size) (:1693-1704), an online softmax (max
// subtracted, expf), then the softmax-weighted sum of the value rows
// (:1706-1722).  Row r of the block is token t0 + r / kv_mul, query head
// g * kv_mul + r % kv_mul, and sees cache positions 0..pos_t.
__global__ void __launch_bounds__(AT_THREADS) k_attn_batch(const __grid_constant__ AttnBatchArgs a)
{
    extern __shared__ float sm[];
    const int hs = a.hs, hs4 = hs / 4;
    constexpr int SQ = AT_NQ + 1, SK = AT_KC + 4;
    const int SV = hs + 4;
    float *sQ = sm;                                   // [hs][SQ]   d-major
    float *sK = sQ + (size_t)hs * SQ;                 // [hs][SK]   d-major
    float *sV = sK + (size_t)hs * SK;                 // [KC][SV]
    float *sS = sV + (size_t)AT_KC * SV;              // [NQ][KC+1] scores, then probabilities
    float *sM = sS + AT_NQ * (AT_KC + 1);
    float *sL = sM + AT_NQ;
    float *sA = sL + AT_NQ;
    int *sLim = reinterpret_cast<int *>(sA + AT_NQ);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int2 blk = a.blocks[blockIdx.x];
    const int g = blockIdx.y;
    const int nq = blk.y * a.kv_mul;
    const int seq = a.tok[blk.x].seq;
    const bool seq_ok = seq >= 0 && seq < a.n_seqs;

    // query rows, d-major; limits; running statistics
    for (int e = tid; e < AT_NQ * hs4; e += AT_THREADS) {
        const int r = e % AT_NQ, d4 = e / AT_NQ;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < nq) {
            const int t = blk.x + r / a.kv_mul, h = g * a.kv_mul + r % a.kv_mul;
            v = *reinterpret_cast<const float4 *>(a.q + (size_t)t * a.q_dim + h * hs + 4 * d4);
        }
        sQ[(4 * d4 + 0) * SQ + r] = v.x;
        sQ[(4 * d4 + 1) * SQ + r] = v.y;
        sQ[(4 * d4 + 2) * SQ + r] = v.z;
        sQ[(4 * d4 + 3) * SQ + r] = v.w;
    }
    int maxpos = -1;
    for (int r = 0; r < nq; r += a.kv_mul) maxpos = max(maxpos, a.tok[blk.x + r / a.kv_mul].pos);
    maxpos = min(maxpos, a.seq_len - 1);
    if (!seq_ok) maxpos = -1;
    for (int r = tid; r < AT_NQ; r += AT_THREADS) {
        int lim = -1;
        if (r < nq && seq_ok) {
            const int p = a.tok[blk.x + r / a.kv_mul].pos;
            lim = (p >= 0 && p < a.seq_len) ? p : -1;
        }
        sLim[r] = lim;
        sM[r] = -INFINITY;
        sL[r] = 0.f;
        sA[r] = 0.f;
    }
    const float *kbase = a.kc + (size_t)(seq_ok ? seq : 0) * a.seq_stride + a.layer_off + (size_t)g * hs;
    const float *vbase = a.vc + (size_t)(seq_ok ? seq : 0) * a.seq_stride + a.layer_off + (size_t)g * hs;
    const float rs = sqrtf((float)hs);
    const bool small = nq <= 8;

    // PV ownership: rows rg + 16 i (i < 4), float4 columns c and c + 16
    const int rg = tid >> 4, cq = tid & 15;
    float4 o[4][2];
#pragma unroll
    for (int i = 0; i < 4; i++) o[i][0] = o[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);

    for (int p0 = 0; p0 <= maxpos; p0 += AT_KC) {
        const int nvalid = min(AT_KC, maxpos + 1 - p0);
        __syncthreads();   // the previous chunk's readers of sK/sV/sS are done
        // K rows, transposed (lane = position, warp = 8-dim group)
        for (int i8 = warp; i8 < hs / 8; i8 += AT_THREADS / 32) {
            float4 k0 = make_float4(0.f, 0.f, 0.f, 0.f), k1 = k0;
            if (lane < nvalid) {
                const float4 *src = reinterpret_cast<const float4 *>(kbase + (size_t)(p0 + lane) * a.kv_dim + 8 * i8);
                k0 = __ldg(src);
                k1 = __ldg(src + 1);
            }
            float *dst = sK + (size_t)(8 * i8) * SK + lane;
            dst[0 * SK] = k0.x; dst[1 * SK] = k0.y; dst[2 * SK] = k0.z; dst[3 * SK] = k0.w;
            dst[4 * SK] = k1.x; dst[5 * SK] = k1.y; dst[6 * SK] = k1.z; dst[7 * SK] = k1.w;
        }
        // V rows
        for (int e = tid; e < AT_KC * hs4; e += AT_THREADS) {
            const int j = e / hs4, c4 = e - j * hs4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (j < nvalid) v = __ldg(reinterpret_cast<const float4 *>(vbase + (size_t)(p0 + j) * a.kv_dim) + c4);
            *reinterpret_cast<float4 *>(sV + (size_t)j * SV + 4 * c4) = v;
        }
        __syncthreads();
        // scores
        if (!small) {
            // thread: positions 4*warp .. +3, rows lane and lane + 32
            float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            for (int d = 0; d < hs; d++) {
                const float4 kv = *reinterpret_cast<const float4 *>(sK + (size_t)d * SK + 4 * warp);
                const float q0 = sQ[d * SQ + lane], q1 = sQ[d * SQ + lane + 32];
                acc[0][0] = fmaf(q0, kv.x, acc[0][0]); acc[0][1] = fmaf(q0, kv.y, acc[0][1]);
                acc[0][2] = fmaf(q0, kv.z, acc[0][2]); acc[0][3] = fmaf(q0, kv.w, acc[0][3]);
                acc[1][0] = fmaf(q1, kv.x, acc[1][0]); acc[1][1] = fmaf(q1, kv.y, acc[1][1]);
                acc[1][2] = fmaf(q1, kv.z, acc[1][2]); acc[1][3] = fmaf(q1, kv.w, acc[1][3]);
            }
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int r = lane + 32 * i;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int p = p0 + 4 * warp + e;
                    sS[r * (AT_KC + 1) + 4 * warp + e] = p <= sLim[r] ? __fdiv_rn(acc[i][e], rs) : -INFINITY;
                }
            }
        } else {
            // few rows: 8 lanes per (row, position) pair split the head dimension
            const int l8 = tid & 7, pair = tid >> 3;            // 32 pairs per pass
            for (int pp = pair; pp < nq * AT_KC; pp += AT_THREADS / 8) {
                const int r = pp / AT_KC, j = pp - r * AT_KC;
                float s = 0.f;
                for (int d = l8; d < hs; d += 8) s = fmaf(sQ[d * SQ + r], sK[(size_t)d * SK + j], s);
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                s += __shfl_xor_sync(0xffffffffu, s, 4);
                if (l8 == 0) sS[r * (AT_KC + 1) + j] = p0 + j <= sLim[r] ? __fdiv_rn(s, rs) : -INFINITY;
            }
        }
        __syncthreads();
        // online softmax, one warp per row
        for (int r = warp; r < nq; r += AT_THREADS / 32) {
            const float s = sS[r * (AT_KC + 1) + lane];
            const float mx = warp_max(s);
            const float m_old = sM[r];
            const float m_new = fmaxf(m_old, mx);
            const float p = s == -INFINITY ? 0.f : expf(s - m_new);
            const float sum = warp_sum(p);
            sS[r * (AT_KC + 1) + lane] = p;
            if (lane == 0) {
                const float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
                sA[r] = alpha;
                sL[r] = sL[r] * alpha + sum;
                sM[r] = m_new;
            }
        }
        __syncthreads();
        // o = o * alpha + p . v
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = rg + 16 * i;
            if (r < nq) {
                const float al = sA[r];
                o[i][0].x *= al; o[i][0].y *= al; o[i][0].z *= al; o[i][0].w *= al;
                o[i][1].x *= al; o[i][1].y *= al; o[i][1].z *= al; o[i][1].w *= al;
            }
        }
        for (int j = 0; j < nvalid; j++) {
            const float4 v0 = cq < hs4 ? *reinterpret_cast<const float4 *>(sV + (size_t)j * SV + 4 * cq)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 v1 = cq + 16 < hs4 ? *reinterpret_cast<const float4 *>(sV + (size_t)j * SV + 4 * (cq + 16))
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int r = rg + 16 * i;
                if (r < nq) {
                    const float p = sS[r * (AT_KC + 1) + j];
                    o[i][0].x = fmaf(p, v0.x, o[i][0].x); o[i][0].y = fmaf(p, v0.y, o[i][0].y);
                    o[i][0].z = fmaf(p, v0.z, o[i][0].z); o[i][0].w = fmaf(p, v0.w, o[i][0].w);
                    o[i][1].x = fmaf(p, v1.x, o[i][1].x); o[i][1].y = fmaf(p, v1.y, o[i][1].y);
                    o[i][1].z = fmaf(p, v1.z, o[i][1].z); o[i][1].w = fmaf(p, v1.w, o[i][1].w);
                }
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = rg + 16 * i;
        if (r >= nq) continue;
        const int t = blk.x + r / a.kv_mul, h = g * a.kv_mul + r % a.kv_mul;
        const float l = sL[r];
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float *dst = a.xb + (size_t)t * a.q_dim + h * hs;
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int c = cq + 16 * k;
            if (c < hs4)
                *reinterpret_cast<float4 *>(dst + 4 * c) =
                    make_float4(o[i][k].x * inv, o[i][k].y * inv, o[i][k].z * inv, o[i][k].w * inv);
        }
    }
}

// ------------------------------------------------- attention on the tensor cores
// The same causal attention for query blocks of head size 128 (prefill),
// flash-attention style on the tensor cores (mma.sync m16n8k16, fp16
// operands, fp32 accumulation): warp w takes block rows 16w..16w+15; per
// chunk of MA_KC cache positions (staged as fp32 in shared memory by
// cp.async, double-buffered) S = Q K^T / sqrt(128) with the causal mask, an
// online softmax on the accumulators, then O += P V with P taken straight
// from the S accumulators.  The rounding of q, k, p and v to fp16 adds
// ~1e-4 relative to the attention output.
constexpr int MA_HS = 128;
constexpr int MA_KC = 32;
constexpr int MA_THREADS = 128;
constexpr int MA_SK = MA_HS + 8;   // K row stride (floats): 64-bit fragment loads conflict-free
constexpr int MA_SV = MA_HS + 4;   // V row stride (floats): 32-bit fragment loads conflict-free

__host__ __device__ constexpr size_t ma_smem_bytes() { return (size_t)2 * MA_KC * (MA_SK + MA_SV) * 4; }

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi)
{
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__global__ void __launch_bounds__(MA_THREADS) k_attn_mma(const __grid_constant__ AttnBatchArgs a)
{
    extern __shared__ __align__(16) float msm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, cq = lane & 3;   // mma fragment coordinates
    const int2 blk = a.blocks[blockIdx.x];
    const int kvh = blockIdx.y;
    const int nq = blk.y * a.kv_mul;
    const int seq = a.tok[blk.x].seq;
    const bool seq_ok = seq >= 0 && seq < a.n_seqs;
    int maxpos = -1;
    for (int r = 0; r < nq; r += a.kv_mul) maxpos = max(maxpos, a.tok[blk.x + r / a.kv_mul].pos);
    maxpos = seq_ok ? min(maxpos, a.seq_len - 1) : -1;
    const float *kbase = a.kc + (size_t)(seq_ok ? seq : 0) * a.seq_stride + a.layer_off + (size_t)kvh * MA_HS;
    const float *vbase = a.vc + (size_t)(seq_ok ? seq : 0) * a.seq_stride + a.layer_off + (size_t)kvh * MA_HS;

    // this thread's two block rows, g and g + 8 of the warp's 16
    int lim[2], tokr[2], headr[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int r = 16 * warp + g + 8 * i;
        lim[i] = -1;
        tokr[i] = -1;
        headr[i] = 0;
        if (r < nq && seq_ok) {
            tokr[i] = blk.x + r / a.kv_mul;
            headr[i] = kvh * a.kv_mul + r % a.kv_mul;
            const int p = a.tok[tokr[i]].pos;
            lim[i] = (p >= 0 && p < a.seq_len) ? p : -1;
        }
    }
    // Q fragments (A operand) for the 8 k-tiles of the head dimension
    uint32_t qf[8][4];
#pragma unroll
    for (int kt = 0; kt < 8; kt++) {
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {        // columns 2c.. and 2c+8..
#pragma unroll
            for (int i = 0; i < 2; i++) {       // rows g, g + 8
                float2 v = make_float2(0.f, 0.f);
                if (tokr[i] >= 0)
                    v = *reinterpret_cast<const float2 *>(a.q + (size_t)tokr[i] * a.q_dim + headr[i] * MA_HS +
                                                         16 * kt + 8 * hh + 2 * cq);
                qf[kt][2 * hh + i] = pack_f16x2(v.x, v.y);
            }
        }
    }
    const float scale = 1.f / sqrtf((float)MA_HS);
    float o[16][4];
#pragma unroll
    for (int nt = 0; nt < 16; nt++) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

    const int nchunks = maxpos >= 0 ? maxpos / MA_KC + 1 : 0;
    auto stage = [&](int ch, int buf) {
        float *ks = msm + (size_t)buf * MA_KC * (MA_SK + MA_SV);
        float *vs = ks + MA_KC * MA_SK;
        const int p0 = ch * MA_KC;
        // 2 x KC rows of 128 floats = KC * 64 16-byte pieces; rows past maxpos
        // are zeros (their probabilities are 0, and 0 * stale data could be NaN)
        for (int e = tid; e < MA_KC * 64; e += MA_THREADS) {
            const int j = e >> 6, piece = e & 63, isv = piece >> 5, c4 = piece & 31;
            float *dst = isv ? vs + j * MA_SV + 4 * c4 : ks + j * MA_SK + 4 * c4;
            if (p0 + j > maxpos) {
                *reinterpret_cast<float4 *>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
                continue;
            }
            cp_async16(dst, (isv ? vbase : kbase) + (size_t)(p0 + j) * a.kv_dim + 4 * c4);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (nchunks > 0) stage(0, 0);
    for (int ch = 0; ch < nchunks; ch++) {
        const int buf = ch & 1, p0 = ch * MA_KC;
        if (ch + 1 < nchunks) {
            stage(ch + 1, buf ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const float *ks = msm + (size_t)buf * MA_KC * (MA_SK + MA_SV);
        const float *vs = ks + MA_KC * MA_SK;
        // S = Q K^T over the chunk's 4 n-tiles of 8 positions
        float sacc[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; nt++) {
            sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
            const float *kr = ks + (8 * nt + g) * MA_SK + 2 * cq;
#pragma unroll
            for (int kt = 0; kt < 8; kt++) {
                const float2 b0 = *reinterpret_cast<const float2 *>(kr + 16 * kt);
                const float2 b1 = *reinterpret_cast<const float2 *>(kr + 16 * kt + 8);
                mma_16816(sacc[nt], qf[kt][0], qf[kt][1], qf[kt][2], qf[kt][3], pack_f16x2(b0.x, b0.y),
                          pack_f16x2(b1.x, b1.y));
            }
        }
        // mask, scale, online softmax (rows g and g + 8: accumulator halves 0-1 and 2-3)
        float alpha[2];
#pragma unroll
        for (int i = 0; i < 2; i++) {
            float mx = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 4; nt++)
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int p = p0 + 8 * nt + 2 * cq + e;
                    float v = sacc[nt][2 * i + e] * scale;
                    v = p <= lim[i] ? v : -INFINITY;
                    sacc[nt][2 * i + e] = v;
                    mx = fmaxf(mx, v);
                }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mn = fmaxf(mrow[i], mx);
            alpha[i] = mrow[i] == -INFINITY ? 0.f : expf(mrow[i] - mn);
            float sum = 0.f;
#pragma unroll
            for (int nt = 0; nt < 4; nt++)
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const float v = sacc[nt][2 * i + e];
                    const float pv = v == -INFINITY ? 0.f : expf(v - mn);
                    sacc[nt][2 * i + e] = pv;
                    sum += pv;
                }
            lrow[i] = lrow[i] * alpha[i] + sum;   // this thread's columns; the quad is summed at the end
            mrow[i] = mn;
        }
#pragma unroll
        for (int nt = 0; nt < 16; nt++) {
            o[nt][0] *= alpha[0];
            o[nt][1] *= alpha[0];
            o[nt][2] *= alpha[1];
            o[nt][3] *= alpha[1];
        }
        // O += P V: P's A fragments are the S accumulators of n-tiles 2kt, 2kt+1
#pragma unroll
        for (int kt = 0; kt < 2; kt++) {
            const uint32_t a0 = pack_f16x2(sacc[2 * kt][0], sacc[2 * kt][1]);
            const uint32_t a1 = pack_f16x2(sacc[2 * kt][2], sacc[2 * kt][3]);
            const uint32_t a2 = pack_f16x2(sacc[2 * kt + 1][0], sacc[2 * kt + 1][1]);
            const uint32_t a3 = pack_f16x2(sacc[2 * kt + 1][2], sacc[2 * kt + 1][3]);
            const float *vr = vs + (16 * kt + 2 * cq) * MA_SV + g;
#pragma unroll
            for (int nt = 0; nt < 16; nt++) {
                const float *v = vr + 8 * nt;
                mma_16816(o[nt], a0, a1, a2, a3, pack_f16x2(v[0], v[MA_SV]),
                          pack_f16x2(v[8 * MA_SV], v[9 * MA_SV]));
            }
        }
        __syncthreads();   // this buffer is restaged two chunks on
    }
    // normalise and store rows g, g + 8
#pragma unroll
    for (int i = 0; i < 2; i++) {
        float l = lrow[i];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        if (tokr[i] < 0) continue;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float *dst = a.xb + (size_t)tokr[i] * a.q_dim + headr[i] * MA_HS + 2 * cq;
#pragma unroll
        for (int nt = 0; nt < 16; nt++)
            *reinterpret_cast<float2 *>(dst + 8 * nt) = make_float2(o[nt][2 * i] * inv, o[nt][2 * i + 1] * inv);
    }
}

// ------------------------------------------------------------------- host
static int grid_for(long long items, int block)
{
    return (int)std::max<long long>(1, std::min<long long>((items + block - 1) / block, 148LL * 16));
}

// Tokens per attention query block: AT_NQ rows hold tokens x kv_mul heads.
static int block_tokens(const LlmModel *m)
{
    return std::max(1, AT_NQ / (m->c.n_heads / m->c.n_kv_heads));
}

bool batch_supported(const LlmModel *m)
{
    const LlmConfig &c = m->c;
    if (c.wtype != W_Q4_0 && c.wtype != W_Q8_0) return false;
    if (m->head_size > AT_MAXHS || m->head_size % 8) return false;
    if (c.n_heads / c.n_kv_heads > AT_NQ) return false;
    if (c.dim % 64 || m->q_dim % 64 || m->hidden_loc % 64) return false;
    for (int l = 0; l < c.n_layers; l++)
        if (!qgemm_supported(m->qkv[l].L) || !qgemm_supported(m->wo[l].L) || !qgemm_supported(m->w13[l].L) ||
            !qgemm_supported(m->w2[l].L))
            return false;
    return qgemm_supported(m->cls.L);
}

static void free_batch(LlmModel *m)
{
    if (m->bt_exec) cudaGraphExecDestroy(m->bt_exec);
    if (m->bt_graph) cudaGraphDestroy(m->bt_graph);
    m->bt_exec = nullptr;
    m->bt_graph = nullptr;
    m->bt_graph_T = 0;
    void *dp[] = {m->bt_tok, m->bt_blocks, m->bt_x, m->bt_delta, m->bt_y, m->bt_q, m->bt_xb, m->bt_lg, m->bt_logits,
                  m->bt_x16, m->bt_ws, m->bt_next, m->bt_step, m->bt_log};
    for (void *p : dp) if (p) cudaFree(p);
    if (m->bt_tok_host) cudaFreeHost(m->bt_tok_host);
    if (m->bt_blocks_host) cudaFreeHost(m->bt_blocks_host);
    m->bt_tok = nullptr; m->bt_blocks = nullptr; m->bt_x = nullptr; m->bt_delta = nullptr; m->bt_y = nullptr;
    m->bt_q = nullptr; m->bt_xb = nullptr; m->bt_lg = nullptr; m->bt_logits = nullptr; m->bt_x16 = nullptr;
    m->bt_ws = nullptr; m->bt_ws_bytes = 0;
    m->bt_next = nullptr; m->bt_step = nullptr; m->bt_log = nullptr; m->bt_log_cap = 0;
    m->bt_tok_host = nullptr; m->bt_blocks_host = nullptr;
    m->bt_cap = 0;
}

void llm_batch_free(LlmModel *m) { free_batch(m); }

int llm_batch_reserve(LlmModel *m, int cap, int n_seqs)
{
    const LlmConfig &c = m->c;
    if (cap <= 0 || n_seqs <= 0) return E_ARG;
    if (!m->weights_ready) return E_ARG;
    if (!batch_supported(m)) return E_UNSUPPORTED;
    if (cudaStreamSynchronize(m->stream) != cudaSuccess) return E_CUDA;
    if (n_seqs > m->n_seqs) {
        // more KV sequences: a new cache, sequence 0 kept where the decode engines read it
        const size_t per = (size_t)c.n_layers * c.seq_len * m->kv_dim;
        float *kc = nullptr, *vc = nullptr;
        if (cudaMalloc(&kc, per * n_seqs * 4) != cudaSuccess) return E_NOMEM;
        if (cudaMalloc(&vc, per * n_seqs * 4) != cudaSuccess) { cudaFree(kc); return E_NOMEM; }
        cudaMemcpyAsync(kc, m->kcache, per * m->n_seqs * 4, cudaMemcpyDeviceToDevice, m->stream);
        cudaMemcpyAsync(vc, m->vcache, per * m->n_seqs * 4, cudaMemcpyDeviceToDevice, m->stream);
        cudaMemsetAsync(kc + per * m->n_seqs, 0, per * (n_seqs - m->n_seqs) * 4, m->stream);
        cudaMemsetAsync(vc + per * m->n_seqs, 0, per * (n_seqs - m->n_seqs) * 4, m->stream);
        if (cudaStreamSynchronize(m->stream) != cudaSuccess) { cudaFree(kc); cudaFree(vc); return E_CUDA; }
        cudaFree(m->kcache);
        cudaFree(m->vcache);
        m->kcache = kc;
        m->vcache = vc;
        m->n_seqs = n_seqs;
        // the decode graph captured the old cache pointers
        if (m->exec) { cudaGraphExecDestroy(m->exec); m->exec = nullptr; }
        if (m->graph) { cudaGraphDestroy(m->graph); m->graph = nullptr; }
        if (m->bt_exec) { cudaGraphExecDestroy(m->bt_exec); m->bt_exec = nullptr; }
        if (m->bt_graph) { cudaGraphDestroy(m->bt_graph); m->bt_graph = nullptr; }
        m->bt_graph_T = 0;
    }
    if (cap <= m->bt_cap) return E_OK;
    free_batch(m);
    const int tp = c.tp_size;
    const size_t ymax = std::max((size_t)m->q_dim + 2 * m->kv_dim, (size_t)2 * m->hidden_loc);
    const size_t nmax = std::max(std::max((size_t)c.dim, (size_t)m->q_dim), (size_t)m->hidden_loc);
    bool ok = true;
    ok &= cudaMalloc(&m->bt_tok, (size_t)cap * sizeof(BatchTok)) == cudaSuccess;
    ok &= cudaMalloc(&m->bt_blocks, (size_t)cap * sizeof(int2)) == cudaSuccess;
    ok &= cudaMalloc(&m->bt_x, (size_t)cap * c.dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->bt_delta, (size_t)cap * c.dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->bt_y, (size_t)cap * ymax * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->bt_q, (size_t)cap * m->q_dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->bt_xb, (size_t)cap * m->q_dim * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->bt_lg, (size_t)tp * cap * m->vocab_loc * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->bt_logits, (size_t)cap * c.vocab * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->bt_x16, qgemm_x16_bytes((int)nmax, cap)) == cudaSuccess;
    // K-split partials: the most any product takes at any token count up to
    // cap (every layer has layer 0's shapes)
    size_t wsb = 0;
    for (int T = 1; T <= cap; T++)
        for (const DevWeight *w : {&m->qkv[0], &m->wo[0], &m->w13[0], &m->w2[0], &m->cls})
            wsb = std::max(wsb, qgemm_workspace_bytes(w->L, T));
    if (wsb) ok &= cudaMalloc(&m->bt_ws, wsb) == cudaSuccess;
    m->bt_ws_bytes = ok ? wsb : 0;
    ok &= cudaMalloc(&m->bt_next, (size_t)cap * 4) == cudaSuccess;
    ok &= cudaMalloc(&m->bt_step, 4) == cudaSuccess;
    ok &= cudaMallocHost(&m->bt_tok_host, (size_t)cap * sizeof(BatchTok)) == cudaSuccess;
    ok &= cudaMallocHost(&m->bt_blocks_host, (size_t)cap * sizeof(int2)) == cudaSuccess;
    if (!ok) {
        free_batch(m);
        return E_NOMEM;
    }
    cudaMemsetAsync(m->bt_x16, 0, qgemm_x16_bytes((int)nmax, cap), m->stream);
    cudaMemsetAsync(m->bt_step, 0, 4, m->stream);
    m->bt_cap = cap;
    return cudaStreamSynchronize(m->stream) == cudaSuccess ? E_OK : E_CUDA;
}

// Group tokens into attention query blocks: runs of consecutive tokens of one
// sequence, at most block_tokens(m) each.  Returns the number of blocks.
static int make_blocks(const LlmModel *m, const BatchTok *tok, int T, int2 *blocks)
{
    const int qb = block_tokens(m);
    int nb = 0;
    for (int t = 0; t < T;) {
        int n = 1;
        while (t + n < T && n < qb && tok[t + n].seq == tok[t].seq) n++;
        blocks[nb++] = make_int2(t, n);
        t += n;
    }
    return nb;
}

// Attention of single-token blocks (batched decode): one CTA per (block,
// query head) and eight warps over the cache positions, four in flight per
// warp, each lane holding four dimensions of q, k and v; every warp keeps its
// own online softmax and the warps merge in shared memory (:1693-1722, the
// same score, max-subtracted expf and weighted sum as k_attn_batch).
constexpr int AK_WARPS = 8;

__global__ void __launch_bounds__(AK_WARPS * 32) k_attn_tok(const __grid_constant__ AttnBatchArgs a)
{
    __shared__ float scr[AK_WARPS][DEC_MAX_HS_ATT + 4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int h = blockIdx.y, hs = a.hs;
    const int tok = a.blocks[blockIdx.x].x;
    const BatchTok bt = a.tok[tok];
    const int T = bt.pos + 1;
    const bool mine = lane * 4 < hs;
    const float rs = sqrtf((float)hs);
    const size_t base = (size_t)bt.seq * a.seq_stride + a.layer_off + (size_t)(h / a.kv_mul) * hs + lane * 4;
    const float *kc = a.kc + base, *vc = a.vc + base;
    constexpr int U = 4;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 qv = mine ? *(reinterpret_cast<const float4 *>(a.q + (size_t)tok * a.q_dim + h * hs) + lane) : z4;
    float4 acc = z4;
    float m = -INFINITY, lsum = 0.f;
    for (int tb = warp * U; tb < T; tb += AK_WARPS * U) {
        float4 kr[U], vr[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int t = min(tb + u, T - 1);   // clamped rows are loaded but not used
            kr[u] = mine ? *reinterpret_cast<const float4 *>(kc + (size_t)t * a.kv_dim) : z4;
            vr[u] = mine ? *reinterpret_cast<const float4 *>(vc + (size_t)t * a.kv_dim) : z4;
        }
        float dot[U];
#pragma unroll
        for (int u = 0; u < U; u++) dot[u] = qv.x * kr[u].x + qv.y * kr[u].y + qv.z * kr[u].z + qv.w * kr[u].w;
#pragma unroll
        for (int u = 0; u < U; u++) dot[u] = warp_sum(dot[u]);
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (tb + u >= T) break;
            const float sc = __fdiv_rn(dot[u], rs);
            const float mn = fmaxf(m, sc);
            const float corr = expf(m - mn);
            const float p = expf(sc - mn);
            lsum = lsum * corr + p;
            acc.x = acc.x * corr + p * vr[u].x;
            acc.y = acc.y * corr + p * vr[u].y;
            acc.z = acc.z * corr + p * vr[u].z;
            acc.w = acc.w * corr + p * vr[u].w;
            m = mn;
        }
    }
    if (lane == 0) { scr[warp][0] = m; scr[warp][1] = lsum; }
    if (mine) reinterpret_cast<float4 *>(&scr[warp][4])[lane] = acc;
    __syncthreads();
    if (tid < hs) {
        float M = -INFINITY;
        for (int w = 0; w < AK_WARPS; w++) M = fmaxf(M, scr[w][0]);
        float L = 0.f, v = 0.f;
        for (int w = 0; w < AK_WARPS; w++) {
            const float mw = scr[w][0];
            if (mw == -INFINITY) continue;
            const float e = expf(mw - M);
            L += e * scr[w][1];
            v += e * scr[w][4 + tid];
        }
        a.xb[(size_t)tok * a.q_dim + h * hs + tid] = v / L;
    }
}

static cudaError_t launch_attn_batch(LlmModel *m, int l, int nblocks, int max_rows, cudaStream_t st)
{
    AttnBatchArgs a;
    const LlmConfig &c = m->c;
    a.q = m->bt_q;
    a.kc = m->kcache;
    a.vc = m->vcache;
    a.seq_stride = (size_t)c.n_layers * c.seq_len * m->kv_dim;
    a.layer_off = (size_t)l * c.seq_len * m->kv_dim;
    a.tok = m->bt_tok;
    a.blocks = m->bt_blocks;
    a.xb = m->bt_xb;
    a.q_dim = m->q_dim;
    a.kv_dim = m->kv_dim;
    a.hs = m->head_size;
    a.kv_mul = c.n_heads / c.n_kv_heads;
    a.seq_len = c.seq_len;
    a.n_seqs = m->n_seqs;
    // single-token blocks (batched decode): a CTA per (block, query head)
    if (max_rows == a.kv_mul && a.hs <= DEC_MAX_HS_ATT && a.hs % 4 == 0) {
        k_attn_tok<<<dim3(nblocks, m->heads_loc), AK_WARPS * 32, 0, st>>>(a);
        return cudaGetLastError();
    }
    // blocks of 16 query rows or more (prefill) go to the tensor cores
    if (a.hs == MA_HS && max_rows >= 16) {
        const size_t smem = ma_smem_bytes();
        cudaError_t e = cudaFuncSetAttribute(k_attn_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e) return e;
        k_attn_mma<<<dim3(nblocks, m->kv_heads_loc), MA_THREADS, smem, st>>>(a);
        return cudaGetLastError();
    }
    const size_t smem = attn_smem_floats(a.hs) * 4;
    cudaError_t e = cudaFuncSetAttribute(k_attn_batch, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e) return e;
    k_attn_batch<<<dim3(nblocks, m->kv_heads_loc), AT_THREADS, smem, st>>>(a);
    return cudaGetLastError();
}

// Accumulate a row-split product (wo, w2) into the residual stream: directly,
// or, when sharded, through the delta buffer, a sum-allreduce and an add.
// Unsharded, a K split is left to the next rmsnorm (*pend), which adds it.
static cudaError_t residual_product(LlmModel *m, const DevWeight &W, int T, cudaStream_t st, SplitOut *pend)
{
    const LlmConfig &c = m->c;
    *pend = SplitOut{};
    if (c.tp_size <= 1)
        return launch_qgemm_x16(W.L, W.ptr, m->bt_x16, m->bt_x, T, true, m->bt_ws, m->bt_ws_bytes, m->err, st, pend);
    cudaError_t e = launch_qgemm_x16(W.L, W.ptr, m->bt_x16, m->bt_delta, T, false, m->bt_ws, m->bt_ws_bytes, m->err, st);
    if (e) return e;
    m->allreduce(m->comm_ctx, m->bt_delta, (size_t)T * c.dim, st);
    const long long n = (long long)T * c.dim;
    k_add<<<grid_for(n, 256), 256, 0, st>>>(m->bt_x, m->bt_delta, n);
    return cudaGetLastError();
}

cudaError_t llm_batch_enqueue(LlmModel *m, int T, int nblocks, bool advance, int *log, int log_cap)
{
    const LlmConfig &c = m->c;
    cudaStream_t st = m->stream;
    const int Tpad = qgemm_tpad(T);
    cudaError_t e;
    k_embed<<<T, 128, 0, st>>>(m->bt_tok, m->emb, m->bt_x, c.dim, c.vocab, m->err);
    if ((e = cudaGetLastError())) return e;
    const size_t seq_stride = (size_t)c.n_layers * c.seq_len * m->kv_dim;
    // A product split over K leaves its partials to the kernel that reads it
    // next (the split sum folded into RoPE, SwiGLU, rmsnorm or the argmax).
    const long long nd = (long long)T * c.dim, nqkv = (long long)T * (m->q_dim + 2 * m->kv_dim);
    SplitOut so, pend;   // pend: the last residual product's split, added by the next rmsnorm
    for (int l = 0; l < c.n_layers; l++) {
        k_rmsnorm_x16<<<T, 256, 0, st>>>(m->bt_x, m->rms_att + (size_t)l * c.dim, m->bt_x16, c.dim, Tpad,
                                         part_src(m->bt_x, pend, nd));
        if ((e = cudaGetLastError())) return e;
        if ((e = launch_qgemm_x16(m->qkv[l].L, m->qkv[l].ptr, m->bt_x16, m->bt_y, T, false, m->bt_ws,
                                    m->bt_ws_bytes, m->err, st, &so))) return e;
        const long long np = nqkv / 2;
        k_rope_kv<<<grid_for(np, 256), 256, 0, st>>>(part_src(m->bt_y, so, nqkv), T, m->bt_tok, m->bt_q, m->kcache,
                                                     m->vcache, seq_stride, (size_t)l * c.seq_len * m->kv_dim,
                                                     m->q_dim, m->kv_dim, m->head_size, c.seq_len, m->n_seqs, m->err);
        if ((e = cudaGetLastError())) return e;
        if ((e = launch_attn_batch(m, l, nblocks, m->bt_max_rows, st))) return e;
        if ((e = launch_x16(m->bt_xb, m->bt_x16, T, m->q_dim, st))) return e;
        if ((e = residual_product(m, m->wo[l], T, st, &pend))) return e;
        k_rmsnorm_x16<<<T, 256, 0, st>>>(m->bt_x, m->rms_ffn + (size_t)l * c.dim, m->bt_x16, c.dim, Tpad,
                                         part_src(m->bt_x, pend, nd));
        if ((e = cudaGetLastError())) return e;
        if ((e = launch_qgemm_x16(m->w13[l].L, m->w13[l].ptr, m->bt_x16, m->bt_y, T, false, m->bt_ws,
                                    m->bt_ws_bytes, m->err, st, &so))) return e;
        const long long nh = (long long)T * (m->hidden_loc / 8);
        k_swiglu_x16<<<grid_for(nh, 256), 256, 0, st>>>(part_src(m->bt_y, so, (long long)T * 2 * m->hidden_loc), T,
                                                        m->hidden_loc, m->bt_x16, Tpad);
        if ((e = cudaGetLastError())) return e;
        if ((e = residual_product(m, m->w2[l], T, st, &pend))) return e;
    }
    k_rmsnorm_x16<<<T, 256, 0, st>>>(m->bt_x, m->rms_final, m->bt_x16, c.dim, Tpad, part_src(m->bt_x, pend, nd));
    if ((e = cudaGetLastError())) return e;
    float *lg = m->bt_lg + (size_t)c.tp_rank * T * m->vocab_loc;
    // sharded, the slices are gathered first: the classifier's split is summed in place
    if ((e = launch_qgemm_x16(m->cls.L, m->cls.ptr, m->bt_x16, lg, T, false, m->bt_ws, m->bt_ws_bytes, m->err, st,
                              c.tp_size > 1 ? nullptr : &so))) return e;
    if (c.tp_size > 1) {
        m->allgather(m->comm_ctx, m->bt_lg, (size_t)T * m->vocab_loc, c.tp_rank, st);
        so = SplitOut{};
    }
    k_logits_argmax<<<T, 256, 0, st>>>(part_src(m->bt_lg, so, (long long)T * m->vocab_loc), T, m->vocab_loc,
                                       c.tp_size, m->bt_logits, m->bt_next, m->err);
    if ((e = cudaGetLastError())) return e;
    if (advance) {
        k_batch_advance<<<1, 256, 0, st>>>(m->bt_tok, m->bt_next, T, log, log_cap, m->bt_step);
        if ((e = cudaGetLastError())) return e;
    }
    return cudaSuccess;
}

// Validate and upload a batch (tokens, positions, sequences); returns the
// number of attention blocks through *nblocks.
int llm_batch_set(LlmModel *m, const int *tokens, const int *pos, const int *seqs, int T, int *nblocks)
{
    const LlmConfig &c = m->c;
    if (T <= 0 || T > m->bt_cap || !tokens || !pos) return E_ARG;
    for (int t = 0; t < T; t++) {
        const int s = seqs ? seqs[t] : 0;
        if (tokens[t] < 0 || tokens[t] >= c.vocab || pos[t] < 0 || pos[t] >= c.seq_len || s < 0 || s >= m->n_seqs)
            return E_ARG;
    }
    // the pinned staging may still be the source of an earlier copy
    if (cudaStreamSynchronize(m->stream) != cudaSuccess) return E_CUDA;
    for (int t = 0; t < T; t++) m->bt_tok_host[t] = BatchTok{tokens[t], pos[t], seqs ? seqs[t] : 0, 0};
    const int nb = make_blocks(m, m->bt_tok_host, T, m->bt_blocks_host);
    int most = 0;
    for (int b = 0; b < nb; b++) most = std::max(most, m->bt_blocks_host[b].y);
    m->bt_max_rows = most * (c.n_heads / c.n_kv_heads);
    if (cudaMemcpyAsync(m->bt_tok, m->bt_tok_host, (size_t)T * sizeof(BatchTok), cudaMemcpyHostToDevice, m->stream) ||
        cudaMemcpyAsync(m->bt_blocks, m->bt_blocks_host, (size_t)nb * sizeof(int2), cudaMemcpyHostToDevice,
                        m->stream) ||
        cudaMemsetAsync(m->bt_step, 0, 4, m->stream))
        return E_CUDA;
    *nblocks = nb;
    return E_OK;
}

int llm_forward_batch(LlmModel *m, const int *tokens, const int *pos, const int *seqs, int T, int *next_host,
                      float *logits_host)
{
    int nb = 0;
    int rc = llm_batch_set(m, tokens, pos, seqs, T, &nb);
    if (rc) return rc;
    if (llm_batch_enqueue(m, T, nb, false, nullptr, 0) != cudaSuccess) return E_CUDA;
    if (next_host && cudaMemcpyAsync(next_host, m->bt_next, (size_t)T * 4, cudaMemcpyDeviceToHost, m->stream))
        return E_CUDA;
    if (logits_host &&
        cudaMemcpyAsync(logits_host, m->bt_logits, (size_t)T * m->c.vocab * 4, cudaMemcpyDeviceToHost, m->stream))
        return E_CUDA;
    return cudaStreamSynchronize(m->stream) == cudaSuccess ? E_OK : E_CUDA;
}

cudaError_t llm_batch_decode_enqueue(LlmModel *m, int T, int steps)
{
    // one token per sequence (set by llm_batch_set): every attention block is
    // one token; one step is captured once into a graph and replayed
    if (steps <= 0) return cudaSuccess;
    cudaError_t e;
    if (m->bt_log_cap < steps * T) {
        if (m->bt_log) cudaFree(m->bt_log);
        m->bt_log = nullptr;
        m->bt_log_cap = 0;
        if ((e = cudaMalloc(&m->bt_log, (size_t)steps * T * 4))) return e;
        m->bt_log_cap = steps * T;
        if (m->bt_exec) { cudaGraphExecDestroy(m->bt_exec); m->bt_exec = nullptr; }
        if (m->bt_graph) { cudaGraphDestroy(m->bt_graph); m->bt_graph = nullptr; }
        m->bt_graph_T = 0;
    }
    if (m->bt_graph_T != T || !m->bt_exec) {
        if (m->bt_exec) { cudaGraphExecDestroy(m->bt_exec); m->bt_exec = nullptr; }
        if (m->bt_graph) { cudaGraphDestroy(m->bt_graph); m->bt_graph = nullptr; }
        if ((e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal))) return e;
        const cudaError_t e1 = llm_batch_enqueue(m, T, T, true, m->bt_log, m->bt_log_cap / T);
        const cudaError_t e2 = cudaStreamEndCapture(m->stream, &m->bt_graph);
        if (e1) return e1;
        if (e2) return e2;
        if ((e = cudaGraphInstantiate(&m->bt_exec, m->bt_graph, 0))) return e;
        m->bt_graph_T = T;
    }
    for (int s = 0; s < steps; s++)
        if ((e = cudaGraphLaunch(m->bt_exec, m->stream))) return e;
    return cudaSuccess;
}

int llm_generate_batch(LlmModel *m, int T, int steps, int *tokens_host)
{
    if (steps <= 0) return E_OK;
    cudaError_t e = llm_batch_decode_enqueue(m, T, steps);
    if (e) return e == cudaErrorMemoryAllocation ? E_NOMEM : E_CUDA;
    if (tokens_host &&
        cudaMemcpyAsync(tokens_host, m->bt_log, (size_t)steps * T * 4, cudaMemcpyDeviceToHost, m->stream))
        return E_CUDA;
    return cudaStreamSynchronize(m->stream) == cudaSuccess ? E_OK : E_CUDA;
}

cudaError_t llm_time_product(LlmModel *m, int kind, int T, int reps, float *ms_per_launch, double *flop_per_launch,
                             double *weight_bytes_per_launch)
{
    const LlmConfig &c = m->c;
    if (T <= 0 || T > m->bt_cap || reps <= 0 || kind < 0 || kind > 4) return cudaErrorInvalidValue;
    std::vector<const DevWeight *> ws;
    for (int l = 0; l < c.n_layers && kind < 4; l++)
        ws.push_back(kind == 0 ? &m->qkv[l] : kind == 1 ? &m->wo[l] : kind == 2 ? &m->w13[l] : &m->w2[l]);
    if (kind == 4) ws.push_back(&m->cls);
    float *y = kind == 4 ? m->bt_lg : m->bt_y;   // both hold [T][d] of this kind
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    auto run = [&](int passes) -> cudaError_t {
        for (int r = 0; r < passes; r++)
            for (auto w : ws) {
                cudaError_t le = launch_qgemm_x16(w->L, w->ptr, m->bt_x16, y, T, false, m->bt_ws, m->bt_ws_bytes, m->err,
                                                  m->stream);
                if (le) return le;
            }
        return cudaSuccess;
    };
    cudaError_t e = run(1);   // warm-up
    if (!e) e = cudaEventRecord(e0, m->stream);
    if (!e) e = run(reps);
    if (!e) e = cudaEventRecord(e1, m->stream);
    if (!e) e = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (!e) cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    const WeightLayout &L = ws[0]->L;
    *ms_per_launch = ms / (float)(reps * ws.size());
    *flop_per_launch = 2.0 * T * L.n * L.d;
    *weight_bytes_per_launch = (double)gguf_row_bytes(L.type, L.n) * L.d;
    return e;
}

} // namespace cats
