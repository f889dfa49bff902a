// qgemm.cu — batched product of a block-quantized weight with T activation
// vectors on the 5th-generation tensor cores (tcgen05, TMEM accumulators):
//     Y[T][d] = X[T][n] * W[d][n]^T
// i.e. T matmul calls of the llama runtime at once (llm/catseye_llm.h:1531,
// 844-879 for one vector), the dense contraction of a prefill or of a
// batched decode step.  The reference has no batched form; it is defined as
// the same sums with fp16 operands (dequantized weights, rounded activations)
// and fp32 accumulation: relative error <= 1e-3.
//
// CTA: 128 weight rows (the UMMA M) x BN tokens (the UMMA N, 16..256), K in
// slices of 64 (two 32-element blocks); grid (N tiles, M tiles, K splits),
// N tiles fastest so the CTAs that share a weight tile run together and the
// second reads it from L2.
//  * Producers (warps 0-7): thread p owns block p & 1 of weight row p >> 1 in
//    every K slice.  It walks the block's words through the weight's tile
//    layout (the matvec's, so prefill and decode share one copy of the
//    weights in HBM) with a cursor, 8 (Q4_0) or 4 (Q8_0) slices ahead,
//    dequantizes them to fp16 in the x16 element order (qgemm.cuh) and
//    stores them in the K-major 128-byte-swizzled form UMMA reads.  Thread 0
//    also brings the stage's BN activation rows in with one bulk copy: the
//    fp16 operand is stored K-slice-major and pre-swizzled (k_x16_swizzled,
//    or a producing kernel writing x16_chunk order).  Then fence.proxy.async
//    and one arrive per warp on the stage's full barrier.
//  * MMA warp (warp 8, one thread): four K=16 tcgen05.mma per stage into the
//    TMEM accumulator; tcgen05.commit releases the stage when they complete.
//  * Epilogue: after a final commit, warps w and w + 4 read TMEM lanes
//    32w..32w+31 (weight rows), each half of the columns, 8 at a time, and
//    write Y or add to it (accumulate: the residual stream); consecutive lanes
//    are consecutive rows of Y (coalesced).  With a K split each CTA writes
//    its partial sums to a workspace and k_splitk_sum adds the splits in
//    order (deterministic).
// Every wait is bounded; TMEM is freed on every path.
#include "qgemm.cuh"
#include "tc.cuh"
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <array>
#include <map>
#include <mutex>
#include <tuple>

namespace cats {

constexpr int QG_M = 128;
constexpr int QG_K = 64;
// K slices of weight words a producer has in flight: 8 of Q4_0 (5 registers
// a slice) or 4 of Q8_0 (9 registers), the same bytes either way
constexpr int QG_PROD = 256;                 // producer threads (8 warps): one block per K slice each
constexpr int QG_THREADS = QG_PROD + 32;     // + the MMA warp
constexpr int QG_MMA_WARP = QG_PROD / 32;
constexpr uint32_t QG_A_BYTES = QG_M * 128;  // one stage of weight rows (fp16, 64 per row)
constexpr int QG_MAX_SPLITS = 16;

__host__ __device__ constexpr int qg_stages(int bn) { return bn >= 256 ? 3 : 4; }

struct QgemmArgs {
    const uint8_t *w;                 // tile layout (matvec.cuh WeightLayout)
    int type, n, d, R, units, nseg;
    uint32_t full_chunk;
    unsigned long long tile_bytes;
    const __half *x;                  // fp16 activations, [n/64][Tpad][64], rows pre-swizzled
    float *y;                         // [T][d]
    float *ws;                        // K split partials [splits][T][d] (splits > 1)
    int T, Tpad;
    int kper;                         // K slices per split
    int splits;
    int accumulate;                   // y += product instead of y = product
    int *err;
};

// The raw words of one 32-element block of a weight row.
struct RawBlk {
    uint4 w[2];     // Q4_0: w[0] = the 16 nibble bytes; Q8_0: w[0], w[1] = the low and high 16 codes
    uint32_t sc;    // fp16 scale in the low half
};

// Where the next block a producer thread loads sits in the tile layout: its
// code words, its scale, the distance from the low to the high Q8_0 plane,
// and the K slices left in the current 64-unit segment.  Within a segment a
// row's next block (two units on) is 32 bytes further, its scale 4 bytes.
struct BlkCursor {
    const uint8_t *codes, *scale;
    uint32_t hi_off;
    int left;
};

template <int WT>
__device__ __forceinline__ void cursor_at(const QgemmArgs &a, int row, int h, int kb, BlkCursor &c)
{
    const int u = 2 * kb + h, s = u / MV_SEG_UNITS, uu = u % MV_SEG_UNITS;
    const int us = min(MV_SEG_UNITS, a.units - MV_SEG_UNITS * s);
    const int t = row / a.R, rr = row % a.R;
    const uint8_t *ch = a.w + (size_t)t * a.tile_bytes + (size_t)s * a.full_chunk;
    const uint32_t sstride = (uint32_t)round_up((size_t)us * 2, 16);
    const uint32_t ub = WT == W_Q4_0 ? 16 : 32;
    c.scale = ch + (size_t)a.R * us * ub + rr * sstride + uu * 2;
    c.codes = ch + ((size_t)(WT == W_Q4_0 ? rr : 2 * rr) * us + uu) * 16;
    c.hi_off = (uint32_t)us * 16;
    c.left = us / 2 - (uu >> 1);
}

// Issue the loads of the cursor's block, then step the cursor one K slice
// (the loads are not used yet, so several slices are in flight at once).
template <int WT>
__device__ __forceinline__ void fetch_next(const QgemmArgs &a, int row, int h, int kb_next, BlkCursor &c, RawBlk &r)
{
    r.sc = __ldg(reinterpret_cast<const unsigned short *>(c.scale));
    r.w[0] = __ldg(reinterpret_cast<const uint4 *>(c.codes));
    if (WT == W_Q8_0) r.w[1] = __ldg(reinterpret_cast<const uint4 *>(c.codes + c.hi_off));
    if (--c.left > 0) {
        c.codes += 32;
        c.scale += 4;
    } else if (2 * kb_next < a.units) {
        cursor_at<WT>(a, row, h, kb_next, c);   // the next segment
    }
}

__device__ __forceinline__ uint32_t h2u(__half2 v) { return *reinterpret_cast<uint32_t *>(&v); }
__device__ __forceinline__ __half2 u2h(uint32_t v) { return *reinterpret_cast<__half2 *>(&v); }

// Dequantize a fetched block into 32 fp16 in the x16 element order and
// store them as chunks 4h .. 4h+3 of the stage's weight-tile row (byte
// offsets `off`).  Value = code * d, computed as (code pair in fp16, exact)
// times d: the correctly rounded q*d.
//  Q4_0: byte j holds element j (low nibble) and j + 16 (high nibble).  For
//  word i (bytes 4i..4i+3), masking bits 0-3 and 16-19 and OR-ing in the
//  exponent of 1024 gives (1024 + e[4i], 1024 + e[4i+2]) exactly; bits 4-7
//  and 20-23 give 1024 + 16 e[4i+16], 1024 + 16 e[4i+18], scaled back by
//  an fma with 1/16 (exact); the word shifted by 8 gives the odd elements.
//  Q8_0: the int8 codes of bytes (4i, 4i+2) and (4i+1, 4i+3) of each plane
//  with the sign bit flipped are code + 128, exact as 1024 + that.
// One Q4_0 code word (4 bytes: elements 4i..4i+3 in the low nibbles and
// 16+4i.. in the high ones) to its 16-byte chunk of fp16 values in the x16
// element order: the masked nibbles OR-ed into the exponent of 1024 are
// 1024 + q (or 1024 + 16q, scaled back exactly by 1/16), so (q - 8) d is one
// rounding of exact operands.
__device__ __forceinline__ uint4 q4_word_fp16(uint32_t w, __half2 d2)
{
    const __half2 lo_bias = __float2half2_rn(1032.f);      // 1024 + the code offset 8
    const __half2 sixteenth = __float2half2_rn(0.0625f);
    const __half2 hi_bias = __float2half2_rn(-72.f);       // -(64 + 8)
    const uint32_t w8 = w >> 8;
    const uint32_t l02 = (w & 0x000F000Fu) | 0x64006400u, l13 = (w8 & 0x000F000Fu) | 0x64006400u;
    const uint32_t g02 = (w & 0x00F000F0u) | 0x64006400u, g13 = (w8 & 0x00F000F0u) | 0x64006400u;
    return make_uint4(h2u(__hmul2(__hsub2(u2h(l02), lo_bias), d2)), h2u(__hmul2(__hsub2(u2h(l13), lo_bias), d2)),
                      h2u(__hmul2(__hfma2(u2h(g02), sixteenth, hi_bias), d2)),
                      h2u(__hmul2(__hfma2(u2h(g13), sixteenth, hi_bias), d2)));
}

template <int WT>
__device__ __forceinline__ void dequant_store(const RawBlk &raw, uint8_t *tile, const uint32_t (&off)[4])
{
    const uint16_t sb = (uint16_t)(raw.sc & 0xffff);
    const __half2 d2 = __halves2half2(__ushort_as_half(sb), __ushort_as_half(sb));
    if (WT == W_Q4_0) {
        const uint32_t wv[4] = {raw.w[0].x, raw.w[0].y, raw.w[0].z, raw.w[0].w};
#pragma unroll
        for (int i = 0; i < 4; i++) *reinterpret_cast<uint4 *>(tile + off[i]) = q4_word_fp16(wv[i], d2);
    } else {
        const __half2 bias = __float2half2_rn(1152.f);          // 1024 + 128
        const uint32_t lo[4] = {raw.w[0].x, raw.w[0].y, raw.w[0].z, raw.w[0].w};
        const uint32_t hi[4] = {raw.w[1].x, raw.w[1].y, raw.w[1].z, raw.w[1].w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t a02 = (__byte_perm(lo[i], 0, 0x4240) ^ 0x00800080u) | 0x64006400u;
            const uint32_t a13 = (__byte_perm(lo[i], 0, 0x4341) ^ 0x00800080u) | 0x64006400u;
            const uint32_t b02 = (__byte_perm(hi[i], 0, 0x4240) ^ 0x00800080u) | 0x64006400u;
            const uint32_t b13 = (__byte_perm(hi[i], 0, 0x4341) ^ 0x00800080u) | 0x64006400u;
            const uint4 o = make_uint4(h2u(__hmul2(__hsub2(u2h(a02), bias), d2)),
                                       h2u(__hmul2(__hsub2(u2h(a13), bias), d2)),
                                       h2u(__hmul2(__hsub2(u2h(b02), bias), d2)),
                                       h2u(__hmul2(__hsub2(u2h(b13), bias), d2)));
            *reinterpret_cast<uint4 *>(tile + off[i]) = o;
        }
    }
}

template <int WT, int BN>
__global__ void __launch_bounds__(QG_THREADS, 1) k_qgemm(const __grid_constant__ QgemmArgs a)
{
    constexpr int ST = qg_stages(BN);
    constexpr int QG_PF = WT == W_Q8_0 ? 4 : 8;
    constexpr uint32_t B_BYTES = BN * 128;
    constexpr uint32_t STAGE = QG_A_BYTES + B_BYTES;
    constexpr int TCOLS = BN < 32 ? 32 : BN;   // TMEM columns: a power of two >= 32
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + ST * STAGE);
    uint64_t *empty = full + ST;
    uint64_t *done = empty + ST;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *commits = const_cast<int *>(abort_s) + 1;   // [ST] commits issued to each empty barrier

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * BN, m0 = blockIdx.y * QG_M, z = blockIdx.z;
    const int ksteps = a.n / QG_K;
    const int kbeg = z * a.kper, nk = max(0, min(ksteps, kbeg + a.kper) - kbeg);

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; s++) {
            mbar_init(&full[s], QG_PROD / 32);   // one arrive per producer warp
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *abort_s = 0;
        for (int s = 0; s < ST; s++) commits[s] = 0;
        fence_barrier_init();
    }
    if (warp == QG_MMA_WARP) {   // TMEM allocation (warp-wide)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == QG_MMA_WARP) {
        // ---------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = umma_idesc(0, QG_M, BN);
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % ST;
                const uint32_t ph = (uint32_t)(kb / ST) & 1u;
                bool ok = false;
                for (uint32_t i = 0; i < CATS_SPIN_LIMIT; i++) {
                    if (mbar_try_wait(&full[s], ph)) { ok = true; break; }
                    if (*abort_s) break;
                    if (i > 64) __nanosleep(32);
                }
                if (!ok) {
                    if (!*abort_s && a.err) atomicOr(a.err, CATS_DEVERR_MBAR_FULL);
                    *abort_s = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * STAGE), sb = sa + QG_A_BYTES;
#pragma unroll
                for (int kk = 0; kk < QG_K / 16; kk++) {
                    const uint64_t da = umma_desc_sw128(sa + kk * 32), db = umma_desc_sw128(sb + kk * 32);
                    const uint32_t acc = (kb | kk) != 0;
                    asm volatile(
                        "{\n\t.reg .pred p;\n\t"
                        "setp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
                        ::"r"(tmem), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0u)
                        : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                             ::"r"(smem_u32(&empty[s])) : "memory");
                commits[s]++;
            }
            // arrives once every MMA issued above has completed (at once if none was)
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         ::"r"(smem_u32(done)) : "memory");
        }
    } else {
        // ---------------- producers: thread p owns block p & 1 of row p >> 1
        const int p = threadIdx.x, r = p >> 1, h = p & 1, row = m0 + r;
        const bool valid = row < a.d;   // rows past d are left unwritten: they reach only unstored outputs
        uint32_t off[4];
#pragma unroll
        for (int i = 0; i < 4; i++) off[i] = sw128(r, 4 * h + i);
        BlkCursor cur;
        RawBlk rb[QG_PF];
        if (valid && nk > 0) cursor_at<WT>(a, row, h, kbeg, cur);
#pragma unroll
        for (int j = 0; j < QG_PF; j++)
            if (valid && j < nk) fetch_next<WT>(a, row, h, kbeg + j + 1, cur, rb[j]);
        int s = 0;
        uint32_t ph = 0;
        bool stop = false;
        for (int kb0 = 0; kb0 < nk && !stop; kb0 += QG_PF) {
#pragma unroll
            for (int j = 0; j < QG_PF; j++) {
                const int kb = kb0 + j;
                if (kb >= nk || stop) break;
                bool ok = false;
                for (uint32_t i = 0; i < CATS_SPIN_LIMIT; i++) {
                    if (mbar_try_wait(&empty[s], ph ^ 1u)) { ok = true; break; }
                    if (*abort_s) break;
                    if (i > 64) __nanosleep(32);
                }
                if (!ok) {
                    if (!*abort_s && a.err) atomicOr(a.err, CATS_DEVERR_MBAR_EMPTY);
                    *abort_s = 1;
                    stop = true;
                    break;
                }
                uint8_t *sa = smem + s * STAGE, *sb = sa + QG_A_BYTES;
                // the BN activation rows of this K slice: one bulk copy of
                // pre-swizzled rows (the tensor cores read them through the
                // async proxy, like the copy writes them)
                if (p == 0)
                    bulk_g2s_keep(sb, a.x + ((size_t)(kbeg + kb) * a.Tpad + t0) * QG_K, B_BYTES, &full[s]);
                if (valid) {
                    dequant_store<WT>(rb[j], sa, off);
                    if (kb + QG_PF < nk) fetch_next<WT>(a, row, h, kbeg + kb + QG_PF + 1, cur, rb[j]);
                }
                fence_proxy_async_smem();   // the generic-proxy weight writes, before the tensor cores read them
                __syncwarp();
                if (lane == 0) {
                    if (p == 0) mbar_arrive_expect_tx(&full[s], B_BYTES);
                    else mbar_arrive(&full[s]);
                }
                if (++s == ST) { s = 0; ph ^= 1u; }
            }
        }
        // ---------------- epilogue: TMEM lanes 32q..32q+31 are rows m0 + 32q + lane;
        // warps q and q + 4 take the two halves of the columns
        bool ok = false;
        for (uint32_t i = 0; i < CATS_SPIN_LIMIT; i++) {
            if (mbar_try_wait(done, 0)) { ok = true; break; }
            if (i > 64) __nanosleep(32);
        }
        if (!ok && a.err) atomicOr(a.err, CATS_DEVERR_MBAR_FULL);
        tc_fence_after();
        if (ok && !*abort_s && nk > 0) {
            const int q = warp & 3, half = warp >> 2;
            const int orow = m0 + q * 32 + lane;
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
            float *out = a.splits > 1 ? a.ws + (size_t)z * a.T * a.d : a.y;
            const bool acc = a.splits == 1 && a.accumulate;
#pragma unroll 1
            for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 8) {
                uint32_t v[8];
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                             : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                               "=r"(v[7])
                             : "r"(taddr + (uint32_t)c0));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (orow < a.d) {
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int tok = t0 + c0 + j;
                        if (tok < a.T) {
                            float *yp = out + (size_t)tok * a.d + orow;
                            *yp = acc ? *yp + __uint_as_float(v[j]) : __uint_as_float(v[j]);
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == QG_MMA_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS));
    }
    if (threadIdx.x == 0) {
        // a commit's arrive lands when its MMAs complete: wait for each empty
        // barrier's last committed phase before retiring the barriers
        for (int s = 0; s < ST; s++)
            if (commits[s] > 0) mbar_wait_bounded(&empty[s], (uint32_t)(commits[s] - 1) & 1u, nullptr, 0);
        for (int s = 0; s < ST; s++) {
            mbar_inval(&full[s]);
            mbar_inval(&empty[s]);
        }
        mbar_inval(done);
    }
}

// ---------------------------------------------------------------------------
// Q4_0 weights through the tensor-memory-access engine.  The producers above
// fetch weight words with ordinary loads, which cap near 8 GB/s per SM (the
// few bytes one SM keeps in flight at the loaded latency).  Here a warp of
// its own (the TMA warp) brings 4 K slices of a
// 128-row tile at a time straight from the matvec's tile layout into a ring
// of raw stages: the codes with one 4-D tensor-map copy (128 bytes of each
// row's segment x 16 rows x 1 segment x 8 tiles, 128-byte swizzled so the
// producers' reads are conflict-free) and the fp16 scales with another (16
// bytes x 16 x 1 x 8).  A weight whose last segment is short has a second
// pair of maps for that segment; coordinates past its end read zeros.  The
// producers dequantize from shared memory as before; the MMA warp and the
// epilogue are unchanged.  With the weights off the producers' path, a K
// slice is paced by the CTA's own chain (the producers' dequantization, the
// one MMA thread's issue, the commit's return to the producers: ~0.5 us at
// 16 and at 512 tokens, against 0.28 us of tensor work for a 128 x 256 x 64
// slice), which the stage counts below trade against CTAs per SM.
// Producer warps: 16 for the wide tiles (one CTA per SM; each thread takes
// half a block per K slice, which halves the producers' link of a slice's
// chain), 8 for the narrow ones (one block per thread; two or three CTAs per
// SM, whose registers leave no room for more).  Then the MMA warp, then the
// TMA warp.
__host__ __device__ constexpr int qt_prod_warps(int bn) { return bn >= 128 ? 16 : 8; }
__host__ __device__ constexpr int qt_threads(int bn) { return qt_prod_warps(bn) * 32 + 64; }
constexpr int QT_GROUP = 4;                    // K slices per raw stage
constexpr uint32_t QT_CODE_BYTES = QG_M * 128;   // 128 rows x 4 slices x 32 bytes
constexpr uint32_t QT_SCALE_BYTES = QG_M * 16;   // 128 rows x 4 slices x 2 blocks x 2 bytes
constexpr uint32_t QT_RAW_BYTES = QT_CODE_BYTES + QT_SCALE_BYTES;

// Stages of the TMA-fed kernel: fp16 operand stages (weight rows and the
// stage's activation rows) and raw weight stages.  Wide tiles (prefill) run
// one CTA per SM with deep rings; tiles of 32 and 64 tokens are sized so two
// CTAs share an SM (<= 113 KB each), 16-token tiles so three do (~74 KB
// each).  A CTA's K slice is paced by its own chain (producers, then the one
// MMA thread, then the commit's return), so more CTAs per SM beat deeper
// rings: same-box A/B of the batch-16 step, 2 + 2 stages at three CTAs per
// SM against 3 + 3 at two, 3526 -> 3772 tok/s (w1/w3 49.2 -> 40.0 us);
// eight stages at one CTA per SM was slower than either.
__host__ __device__ constexpr int qt_stages(int bn) { return bn >= 128 ? qg_stages(bn) : bn == 16 ? 2 : 3; }
__host__ __device__ constexpr int qt_raw_stages(int bn) { return bn >= 256 ? 3 : bn >= 128 ? 4 : 2; }

struct QgemmTmaArgs {
    CUtensorMap codes, scales;             // full segments
    CUtensorMap codes_tail, scales_tail;   // the short last segment (when there is one)
    int full_segs;                         // segments of MV_SEG_UNITS units
    int n, d, T, Tpad, kper, splits, accumulate;
    const __half *x;
    float *y, *ws;
    int *err;
    unsigned long long *trace;   // QgemmTrace: CTA (0, 0, 0)'s timeline, or null
    int trace_slices;
};

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
          "r"(smem_u32(bar))
        : "memory");
}

template <int BN>
__global__ void __launch_bounds__(qt_threads(BN), 1) k_qgemm_tma(const __grid_constant__ QgemmTmaArgs a)
{
    constexpr int NPW = qt_prod_warps(BN);          // producer warps
    constexpr int MMA_WARP = NPW, TMA_WARP = NPW + 1;
    constexpr int ST = qt_stages(BN);
    constexpr int RS = qt_raw_stages(BN);
    constexpr uint32_t B_BYTES = BN * 128;
    constexpr uint32_t STAGE = QG_A_BYTES + B_BYTES;
    constexpr int TCOLS = BN < 32 ? 32 : BN;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
    uint8_t *rawst = smem + ST * STAGE;                 // RS raw stages: codes then scales
    uint64_t *full = reinterpret_cast<uint64_t *>(rawst + RS * QT_RAW_BYTES);
    uint64_t *empty = full + ST;
    uint64_t *rfull = empty + ST;
    uint64_t *rempty = rfull + RS;
    uint64_t *done = rempty + RS;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *commits = const_cast<int *>(abort_s) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * BN, m0 = blockIdx.y * QG_M, z = blockIdx.z;
    const int ksteps = a.n / QG_K;
    const int kbeg = z * a.kper, nk = max(0, min(ksteps, kbeg + a.kper) - kbeg);
    const int ngroups = (nk + QT_GROUP - 1) / QT_GROUP;
    const bool tr = a.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
    auto stamp = [&](int k, int e) {
        if (tr && k >= 0 && k <= a.trace_slices) a.trace[(size_t)k * QG_TRACE_FIELDS + e] = (unsigned long long)clock64();
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; s++) {
            mbar_init(&full[s], NPW);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < RS; s++) {
            mbar_init(&rfull[s], 1);
            mbar_init(&rempty[s], NPW);   // every producer warp, after its last read of the stage
        }
        mbar_init(done, 1);
        *abort_s = 0;
        for (int s = 0; s < ST; s++) commits[s] = 0;
        fence_barrier_init();
    }
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) stamp(a.trace_slices, 0);

    if (warp == TMA_WARP) {
        // ---------------- raw weight stages through the TMA engine
        if (lane == 0) {
            int issued = 0;
            for (int g = 0; g < ngroups; g++) {
                const int rs = g % RS;
                const uint32_t rph = (uint32_t)(g / RS) & 1u;
                if (!tc_wait(&rempty[rs], rph ^ 1u, abort_s, a.err, CATS_DEVERR_MBAR_EMPTY)) break;
                const int slice = kbeg + g * QT_GROUP;
                const int seg = slice / (MV_SEG_UNITS / 2), in_seg = slice % (MV_SEG_UNITS / 2);
                const bool tail = seg >= a.full_segs;
                uint8_t *dst = rawst + rs * QT_RAW_BYTES;
                mbar_arrive_expect_tx(&rfull[rs], QT_RAW_BYTES);
                tma_load_4d(dst, tail ? &a.codes_tail : &a.codes, in_seg * 32, 0, tail ? 0 : seg, m0 / 16, &rfull[rs]);
                tma_load_4d(dst + QT_CODE_BYTES, tail ? &a.scales_tail : &a.scales, in_seg * 4, 0, tail ? 0 : seg,
                            m0 / 16, &rfull[rs]);
                issued = g + 1;
                if (g * QT_GROUP < a.trace_slices) stamp(g * QT_GROUP, 0);
            }
            // every copy lands before the CTA exits (the last phase of each stage)
            for (int g = max(0, issued - RS); g < issued; g++)
                mbar_wait_bounded(&rfull[g % RS], (uint32_t)(g / RS) & 1u, nullptr, 0);
        }
    } else if (warp == MMA_WARP) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc(0, QG_M, BN);
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % ST;
                const uint32_t ph = (uint32_t)(kb / ST) & 1u;
                if (!tc_wait(&full[s], ph, abort_s, a.err, CATS_DEVERR_MBAR_FULL)) break;
                if (kb < a.trace_slices) stamp(kb, 12);
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * STAGE), sb = sa + QG_A_BYTES;
#pragma unroll
                for (int kk = 0; kk < QG_K / 16; kk++) {
                    const uint64_t da = umma_desc_sw128(sa + kk * 32), db = umma_desc_sw128(sb + kk * 32);
                    const uint32_t acc = (kb | kk) != 0;
                    asm volatile(
                        "{\n\t.reg .pred p;\n\t"
                        "setp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
                        ::"r"(tmem), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0u)
                        : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                             ::"r"(smem_u32(&empty[s])) : "memory");
                commits[s]++;
                if (kb < a.trace_slices) stamp(kb, 13);
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         ::"r"(smem_u32(done)) : "memory");
        }
    } else {
        // ---------------- producers: from the raw stage, thread p dequantizes
        // block h of row r (8 warps), or half qh of it (16 warps: code words
        // 2 qh and 2 qh + 1, the chunks they fill)
        constexpr int NW = NPW == 16 ? 2 : 4;   // code words per thread
        const int p = threadIdx.x;
        const int r = NPW == 16 ? p >> 2 : p >> 1, h = NPW == 16 ? (p >> 1) & 1 : p & 1;
        const int qh = NPW == 16 ? p & 1 : 0;
        uint32_t off[NW];
#pragma unroll
        for (int i = 0; i < NW; i++) off[i] = sw128(r, 4 * h + NW * qh + i);
        int s = 0;
        uint32_t ph = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int g = kb / QT_GROUP, k4 = kb % QT_GROUP, rs = g % RS;
            if (k4 == 0 && !tc_wait(&rfull[rs], (uint32_t)(g / RS) & 1u, abort_s, a.err, CATS_DEVERR_MBAR_FULL)) break;
            if (k4 == 0 && p == 0 && kb < a.trace_slices) stamp(kb, 2);
            if (!tc_wait(&empty[s], ph ^ 1u, abort_s, a.err, CATS_DEVERR_MBAR_EMPTY)) break;
            if (p == 0 && kb < a.trace_slices) stamp(kb, 3);
            uint8_t *sa = smem + s * STAGE;
            if (p == 0) {   // the stage's activation rows, with its weights
                bulk_g2s_keep(sa + QG_A_BYTES, a.x + ((size_t)(kbeg + kb) * a.Tpad + t0) * QG_K, B_BYTES, &full[s]);
                if (kb < a.trace_slices) stamp(kb, 1);
            }
            const uint8_t *rb = rawst + rs * QT_RAW_BYTES;
            // the codes of this slice's block: 16-byte chunk 2 k4 + h of row r, 128-byte swizzled by the copy
            const uint8_t *cw = rb + r * 128 + (((2 * k4 + h) ^ (r & 7)) << 4);
            const unsigned short sb = *reinterpret_cast<const unsigned short *>(rb + QT_CODE_BYTES + r * 16 + k4 * 4 + h * 2);
            const __half2 d2 = __halves2half2(__ushort_as_half(sb), __ushort_as_half(sb));
            if constexpr (NW == 4) {
                const uint4 w = *reinterpret_cast<const uint4 *>(cw);
                const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int i = 0; i < 4; i++) *reinterpret_cast<uint4 *>(sa + off[i]) = q4_word_fp16(wv[i], d2);
            } else {
                const uint2 w = *reinterpret_cast<const uint2 *>(cw + 8 * qh);
                *reinterpret_cast<uint4 *>(sa + off[0]) = q4_word_fp16(w.x, d2);
                *reinterpret_cast<uint4 *>(sa + off[1]) = q4_word_fp16(w.y, d2);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (p == 0) mbar_arrive_expect_tx(&full[s], B_BYTES);
                else mbar_arrive(&full[s]);
                if (k4 == QT_GROUP - 1 || kb == nk - 1) mbar_arrive(&rempty[rs]);   // the warp is done with it
                if (kb < a.trace_slices && warp < 8) stamp(kb, 4 + warp);
            }
            if (++s == ST) { s = 0; ph ^= 1u; }
        }
        bool ok = false;
        for (uint32_t i = 0; i < CATS_SPIN_LIMIT; i++) {
            if (mbar_try_wait(done, 0)) { ok = true; break; }
            if (i > 64) __nanosleep(32);
        }
        if (!ok && a.err) atomicOr(a.err, CATS_DEVERR_MBAR_FULL);
        if (p == 0) stamp(a.trace_slices, 1);
        tc_fence_after();
        if (ok && !*abort_s && nk > 0) {
            // warp w reads TMEM lanes 32 (w & 3) .. + 31 (its quarter of the
            // rows) over part w >> 2 of the columns
            constexpr int PARTS = NPW / 4, PCOLS = BN / PARTS;
            const int q = warp & 3, part = warp >> 2;
            const int orow = m0 + q * 32 + lane;
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
            float *out = a.splits > 1 ? a.ws + (size_t)z * a.T * a.d : a.y;
            const bool acc = a.splits == 1 && a.accumulate;
#pragma unroll 1
            for (int c0 = part * PCOLS; c0 < (part + 1) * PCOLS; c0 += 8) {
                uint32_t v[8];
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                             : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                               "=r"(v[7])
                             : "r"(taddr + (uint32_t)c0));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (orow < a.d) {
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int tok = t0 + c0 + j;
                        if (tok < a.T) {
                            float *yp = out + (size_t)tok * a.d + orow;
                            *yp = acc ? *yp + __uint_as_float(v[j]) : __uint_as_float(v[j]);
                        }
                    }
                }
            }
        }
    }
    if (threadIdx.x == 0) stamp(a.trace_slices, 2);
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS));
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; s++)
            if (commits[s] > 0) mbar_wait_bounded(&empty[s], (uint32_t)(commits[s] - 1) & 1u, nullptr, 0);
        for (int s = 0; s < ST; s++) {
            mbar_inval(&full[s]);
            mbar_inval(&empty[s]);
        }
        for (int s = 0; s < RS; s++) {
            mbar_inval(&rfull[s]);
            mbar_inval(&rempty[s]);
        }
        mbar_inval(done);
    }
}

// y (=, or +=) the sum of the K splits' partials, in split order.
__global__ void k_splitk_sum(const float *__restrict__ ws, int splits, long long count, float *__restrict__ y,
                             int accumulate)
{
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count;
         i += (long long)gridDim.x * blockDim.x) {
        float p = 0.f;
        for (int z = 0; z < splits; z++) p += ws[(size_t)z * count + i];
        y[i] = accumulate ? y[i] + p : p;
    }
}

// x[T][n] fp32 -> fp16 in the order the kernel's bulk copies take: K slice
// major ([n/64][Tpad][64]), each row's eight 16-byte chunks in the x16
// element order and permuted as the 128-byte swizzle places them (chunk c of
// token t at c ^ (t & 7); a CTA's first token is a multiple of 8).  Rows
// t >= T are left as they are.
__global__ void k_x16_swizzled(const float *__restrict__ x, __half *__restrict__ y, int T, int Tpad, int n)
{
    const long long total = (long long)(n / QG_K) * T * 8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(i & 7);
        const long long r = i >> 3;
        const int tok = (int)(r % T), kb = (int)(r / T);
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)tok * n + (size_t)kb * QG_K + x16_src_off(c));
        *reinterpret_cast<uint4 *>(y + x16_chunk(kb, c, tok, Tpad)) = x16_pack(src[0], src[4]);
    }
}

static int pick_bn(int T)
{
    return T > 128 ? 256 : T > 64 ? 128 : T > 32 ? 64 : T > 16 ? 32 : 16;
}

int qgemm_tpad(int T)
{
    return (int)round_up((size_t)std::max(T, 1), (size_t)pick_bn(T));
}

size_t qgemm_x16_bytes(int n, int T)
{
    return (size_t)n * qgemm_tpad(T) * 2;
}

size_t qgemm_smem_bytes(int bn)
{
    // alignment slack, stages, barriers, TMEM slot, abort flag, commit counts
    const int st = qg_stages(bn);
    return 1024 + (size_t)st * (QG_A_BYTES + (size_t)bn * 128) + (2 * st + 1) * 8 + 8 + 4 * st;
}

template <int WT, int BN>
static cudaError_t prepare_t(int *per_sm)
{
    const size_t smem = qgemm_smem_bytes(BN);
    cudaError_t e = cudaFuncSetAttribute(k_qgemm<WT, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k_qgemm<WT, BN>, QG_THREADS, smem);
}

template <int WT>
static cudaError_t prepare_bn(int bn, int *per_sm)
{
    switch (bn) {
    case 256: return prepare_t<WT, 256>(per_sm);
    case 128: return prepare_t<WT, 128>(per_sm);
    case 64: return prepare_t<WT, 64>(per_sm);
    case 32: return prepare_t<WT, 32>(per_sm);
    default: return prepare_t<WT, 16>(per_sm);
    }
}

// CTAs of one kernel instance resident per SM (shared memory and registers),
// queried once per device and instance; the dynamic shared-memory limit is
// raised on the way.
static int resident_per_sm(int type, int bn)
{
    static int cache[2][5][64] = {};   // [type][bn][device], 0 = not queried
    int dev = 0;
    cudaGetDevice(&dev);
    const int ti = type == W_Q4_0 ? 0 : 1;
    const int bi = bn == 256 ? 0 : bn == 128 ? 1 : bn == 64 ? 2 : bn == 32 ? 3 : 4;
    int spare = 0;   // ordinals past the table are queried (and the limit raised) on every call
    int &c = dev >= 0 && dev < 64 ? cache[ti][bi][dev] : spare;
    if (c == 0) {
        int n = 0;
        const cudaError_t e = type == W_Q4_0 ? prepare_bn<W_Q4_0>(bn, &n) : prepare_bn<W_Q8_0>(bn, &n);
        if (e != cudaSuccess || n <= 0) return 1;   // not kept: asked again next time
        c = n;
    }
    return c;
}

// K splits for a product: when the (N tile, M tile) grid leaves SMs idle or
// ends in a partial wave, splitting K gives every SM work.  The estimate
// weighs waves of K slices against the partials' extra traffic.
static int resident_for(const WeightLayout &L, int bn);
static bool tma_layout_ok(const WeightLayout &L);

static int pick_splits(const WeightLayout &L, int T)
{
    const int bn = pick_bn(T);
    const int n = L.n, d = L.d;
    const int ksteps = n / QG_K;
    const long long tiles = (long long)cdiv(d, QG_M) * cdiv(T, bn);
    const long long slots = 148LL * resident_for(L, bn);
    // the tensor-map path starts splits on raw-stage boundaries (4 slices)
    const int kq = tma_layout_ok(L) ? QT_GROUP : 1;
    const double t_k = 0.4e-6 * std::max(bn, 64) / 256.0 + 0.05e-6;   // seconds per K slice of one CTA
    int best = 1;
    double best_t = 1e30;
    for (int s = 1; s <= QG_MAX_SPLITS && (s == 1 || ksteps / s >= 4); s++) {
        const int kper = (int)round_up((size_t)cdiv(ksteps, s), kq);
        if (cdiv(ksteps, kper) != s) continue;   // every split gets work
        const double waves = (double)((tiles * s + slots - 1) / slots);
        const double t = waves * kper * t_k + (s > 1 ? 8.0 * s * T * (double)d / 5e12 : 0.0);
        if (t < best_t * 0.97) { best_t = t; best = s; }
    }
    return best;
}

size_t qgemm_workspace_bytes(const WeightLayout &L, int T)
{
    if (T <= 0 || !qgemm_supported(L)) return 0;
    const int s = pick_splits(L, T);
    return s > 1 ? (size_t)s * T * L.d * 4 : 0;
}

template <int WT, int BN>
static cudaError_t launch_t(const QgemmArgs &a, cudaStream_t st)
{
    resident_per_sm(WT, BN);   // raises the kernel's shared-memory limit once
    dim3 grid(cdiv(a.T, BN), cdiv(a.d, QG_M), a.splits);
    k_qgemm<WT, BN><<<grid, QG_THREADS, qgemm_smem_bytes(BN), st>>>(a);
    return cudaGetLastError();
}

template <int WT>
static cudaError_t launch_bn(const QgemmArgs &a, int bn, cudaStream_t st)
{
    switch (bn) {
    case 256: return launch_t<WT, 256>(a, st);
    case 128: return launch_t<WT, 128>(a, st);
    case 64: return launch_t<WT, 64>(a, st);
    case 32: return launch_t<WT, 32>(a, st);
    default: return launch_t<WT, 16>(a, st);
    }
}

// ---------------------------------------------------------------- TMA path
size_t qgemm_tma_smem_bytes(int bn)
{
    const int st = qt_stages(bn), rs = qt_raw_stages(bn);
    // alignment slack, fp16 stages, raw stages, barriers, TMEM slot, abort flag, commit counts
    return 1024 + (size_t)st * (QG_A_BYTES + (size_t)bn * 128) + (size_t)rs * QT_RAW_BYTES + (2 * st + 2 * rs + 1) * 8 +
           8 + 4 * st;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// The layouts the TMA path reads: Q4_0 in 16-row tiles, and a short last
// segment (if any) of at least 8 units, so every box's inner extent (128
// bytes of codes, 16 of scales) fits the segment's row.  CATS_QGEMM_TMA=0
// keeps the load-fed kernel (tuning).
static bool tma_layout_ok(const WeightLayout &L)
{
    static const bool enabled = [] {
        const char *e = getenv("CATS_QGEMM_TMA");
        return !(e && atoi(e) == 0);
    }();
    if (!enabled || L.type != W_Q4_0 || L.R != 16 || L.units % 2) return false;
    const int tail = L.units % MV_SEG_UNITS;
    return (tail == 0 || tail >= 8) && encode_fn() != nullptr;
}

// 4-D map over the tile layout: dim 0 the bytes of one row's part of a
// segment, dim 1 the 16 rows of a tile, dim 2 the segments, dim 3 the tiles.
static bool encode4(CUtensorMap *m, const void *base, uint64_t d0, uint64_t stride1, uint64_t d2, uint64_t stride2,
                    uint64_t d3, uint64_t stride3, uint32_t box0, bool swizzle)
{
    const cuuint64_t dims[4] = {d0, 16, d2, d3};
    const cuuint64_t strides[3] = {stride1, stride2, stride3};
    const cuuint32_t box[4] = {box0, 16, 1, 8};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void *>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The four maps of a weight, encoded once per (address, layout) and kept.
static bool tma_maps(const WeightLayout &L, const uint8_t *w, QgemmTmaArgs &a)
{
    using Key = std::tuple<const void *, int, int, int, unsigned long long>;
    static std::map<Key, std::array<CUtensorMap, 4>> cache;
    static std::mutex mu;
    const Key key{w, L.n, L.d, L.units, (unsigned long long)L.tile_bytes};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it == cache.end()) {
        std::array<CUtensorMap, 4> m;
        const int full = L.units / MV_SEG_UNITS, tail = L.units % MV_SEG_UNITS;
        const uint64_t fs = (uint64_t)std::max(full, 1);
        const uint32_t code_row = MV_SEG_UNITS * 16, scale_row = (uint32_t)round_up(MV_SEG_UNITS * 2, 16);
        bool ok = encode4(&m[0], w, code_row, code_row, fs, L.full_chunk, L.n_tiles, L.tile_bytes, 128, true) &&
                  encode4(&m[1], w + (size_t)16 * code_row, scale_row, scale_row, fs, L.full_chunk, L.n_tiles,
                          L.tile_bytes, 16, false);
        if (ok && tail) {
            const uint8_t *tb = w + (size_t)full * L.full_chunk;
            const uint32_t crow = (uint32_t)tail * 16, srow = (uint32_t)round_up((size_t)tail * 2, 16);
            ok = encode4(&m[2], tb, crow, crow, 1, L.last_chunk, L.n_tiles, L.tile_bytes, 128, true) &&
                 encode4(&m[3], tb + (size_t)16 * crow, srow, srow, 1, L.last_chunk, L.n_tiles, L.tile_bytes, 16, false);
        } else {
            m[2] = m[0];
            m[3] = m[1];
        }
        if (!ok) return false;
        it = cache.emplace(key, m).first;
    }
    a.codes = it->second[0];
    a.scales = it->second[1];
    a.codes_tail = it->second[2];
    a.scales_tail = it->second[3];
    a.full_segs = L.units / MV_SEG_UNITS;
    return true;
}

template <int BN>
static cudaError_t prepare_tma_t(int *per_sm)
{
    const size_t smem = qgemm_tma_smem_bytes(BN);
    cudaError_t e = cudaFuncSetAttribute(k_qgemm_tma<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, k_qgemm_tma<BN>, qt_threads(BN), smem);
}

static cudaError_t prepare_tma_bn(int bn, int *per_sm)
{
    switch (bn) {
    case 256: return prepare_tma_t<256>(per_sm);
    case 128: return prepare_tma_t<128>(per_sm);
    case 64: return prepare_tma_t<64>(per_sm);
    case 32: return prepare_tma_t<32>(per_sm);
    default: return prepare_tma_t<16>(per_sm);
    }
}

// CTAs of a TMA-fed instance resident per SM, queried once per device and
// instance (raising its shared-memory limit on the way).
static int resident_tma(int bn)
{
    static int cache[5][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int bi = bn == 256 ? 0 : bn == 128 ? 1 : bn == 64 ? 2 : bn == 32 ? 3 : 4;
    int spare = 0;
    int &c = dev >= 0 && dev < 64 ? cache[bi][dev] : spare;
    if (c == 0) {
        int n = 0;
        if (prepare_tma_bn(bn, &n) != cudaSuccess || n <= 0) return 1;   // not kept: asked again next time
        c = n;
    }
    return c;
}

// the residency of the kernel a weight's products run on
static int resident_for(const WeightLayout &L, int bn)
{
    return tma_layout_ok(L) ? resident_tma(bn) : resident_per_sm(L.type, bn);
}

template <int BN>
static cudaError_t launch_tma_t(const QgemmTmaArgs &a, cudaStream_t st)
{
    resident_tma(BN);   // raises the kernel's shared-memory limit once per device
    dim3 grid(cdiv(a.T, BN), cdiv(a.d, QG_M), a.splits);
    k_qgemm_tma<BN><<<grid, qt_threads(BN), qgemm_tma_smem_bytes(BN), st>>>(a);
    return cudaGetLastError();
}

static cudaError_t launch_tma_bn(const QgemmTmaArgs &a, int bn, cudaStream_t st)
{
    switch (bn) {
    case 256: return launch_tma_t<256>(a, st);
    case 128: return launch_tma_t<128>(a, st);
    case 64: return launch_tma_t<64>(a, st);
    case 32: return launch_tma_t<32>(a, st);
    default: return launch_tma_t<16>(a, st);
    }
}

bool qgemm_supported(const WeightLayout &L)
{
    return (L.type == W_Q4_0 || L.type == W_Q8_0) && L.n % QG_K == 0 && L.units % 2 == 0;
}

cudaError_t launch_x16(const float *x, __half *x16, int T, int n, cudaStream_t st)
{
    if (T <= 0) return cudaSuccess;
    if (n % QG_K) return cudaErrorInvalidValue;
    const int Tpad = qgemm_tpad(T);
    const long long chunks = (long long)(n / QG_K) * T * 8;
    k_x16_swizzled<<<(int)std::min<long long>((chunks + 255) / 256, 148LL * 16), 256, 0, st>>>(x, x16, T, Tpad, n);
    return cudaGetLastError();
}

QgemmPlan qgemm_plan(const WeightLayout &L, int T)
{
    QgemmPlan p{};
    if (T <= 0 || !qgemm_supported(L)) return p;
    p.bn = pick_bn(T);
    p.splits = pick_splits(L, T);
    p.resident = resident_for(L, p.bn);
    p.tma = tma_layout_ok(L) ? 1 : 0;
    const int ksteps = L.n / QG_K;
    p.kper = (int)round_up((size_t)cdiv(ksteps, p.splits), p.tma ? QT_GROUP : 1);
    int n = 0;
    p.occupancy_err = (int)(p.tma ? prepare_tma_bn(p.bn, &n)
                                  : L.type == W_Q4_0 ? prepare_bn<W_Q4_0>(p.bn, &n) : prepare_bn<W_Q8_0>(p.bn, &n));
    p.occupancy = n;
    return p;
}

cudaError_t launch_qgemm_x16(const WeightLayout &L, const uint8_t *w, const __half *x16, float *y, int T,
                             bool accumulate, float *ws, size_t ws_bytes, int *err, cudaStream_t st, SplitOut *defer,
                             const QgemmTrace *trace)
{
    if (defer) *defer = SplitOut{};
    if (T <= 0) return cudaSuccess;
    if (!qgemm_supported(L)) return cudaErrorInvalidValue;
    QgemmArgs a;
    a.w = w;
    a.type = L.type;
    a.n = L.n;
    a.d = L.d;
    a.R = L.R;
    a.units = L.units;
    a.nseg = L.nseg;
    a.full_chunk = L.full_chunk;
    a.tile_bytes = L.tile_bytes;
    a.x = x16;
    a.y = y;
    a.T = T;
    a.Tpad = qgemm_tpad(T);
    a.accumulate = accumulate ? 1 : 0;
    a.err = err;
    const int ksteps = L.n / QG_K;
    int splits = pick_splits(L, T);
    if (splits > 1 && (!ws || ws_bytes < (size_t)splits * T * L.d * 4)) splits = 1;   // no room: one pass over K
    a.splits = splits;
    a.kper = cdiv(ksteps, splits);
    a.ws = ws;
    const int bn = pick_bn(T);
    cudaError_t e;
    QgemmTmaArgs ta;
    if (tma_layout_ok(L) && tma_maps(L, w, ta)) {
        // K splits start on raw-stage boundaries (4 slices): the scale copy's
        // first coordinate is then 16-byte aligned
        ta.kper = (int)round_up((size_t)cdiv(ksteps, splits), QT_GROUP);
        ta.splits = splits = cdiv(ksteps, ta.kper);
        ta.n = L.n;
        ta.d = L.d;
        ta.T = T;
        ta.Tpad = a.Tpad;
        ta.accumulate = a.accumulate;
        ta.x = x16;
        ta.y = y;
        ta.ws = ws;
        ta.err = err;
        ta.trace = trace ? trace->buf : nullptr;
        ta.trace_slices = trace ? trace->slices : 0;
        e = launch_tma_bn(ta, bn, st);
    } else {
        e = L.type == W_Q4_0 ? launch_bn<W_Q4_0>(a, bn, st) : launch_bn<W_Q8_0>(a, bn, st);
    }
    if (e || splits == 1) return e;
    if (defer) {   // the caller's next kernel adds the partials
        *defer = SplitOut{ws, splits};
        return cudaSuccess;
    }
    const long long count = (long long)T * L.d;
    k_splitk_sum<<<(int)std::min<long long>((count + 255) / 256, 148LL * 8), 256, 0, st>>>(ws, splits, count, y,
                                                                                          a.accumulate);
    return cudaGetLastError();
}

cudaError_t launch_qgemm(const WeightLayout &L, const uint8_t *w, const float *x, __half *x16, float *y, int T,
                         float *ws, size_t ws_bytes, int *err, cudaStream_t st, const QgemmTrace *trace)
{
    if (T <= 0) return cudaSuccess;
    if (!qgemm_supported(L)) return cudaErrorInvalidValue;
    cudaError_t e = launch_x16(x, x16, T, L.n, st);
    if (e) return e;
    return launch_qgemm_x16(L, w, x16, y, T, false, ws, ws_bytes, err, st, nullptr, trace);
}

} // namespace cats
