// sgemm_tc.cu — fp32 GEMM of the CNN path on the 5th-generation tensor cores
// as 3xTF32 (tcgen05.mma kind::tf32, TMEM accumulators).
//
// C = alpha*op(A)*op(B) + beta*C (gemm_rnn / gemm_rnt / gemm_rtn,
// catseye.h:78-129; beta == 0 never reads C).  Every fp32 operand x is split
// into hi = tf32(x) (round to nearest) and lo = tf32(x - hi); the product is
// hi*hi + hi*lo + lo*hi, within ~3 * 2^-22 of x*y (lo*lo and the rounding of
// lo are what is left out).
//
// Accumulation.  The tensor cores add each instruction's products into the
// TMEM accumulator without rounding to nearest: the bits below the
// accumulator's last place are dropped, a bias that grows with the number of
// additions (one accumulator over a 1664-deep K split measured 1.2e-5
// normwise).  So the hi*hi terms go to an accumulator that is restarted every
// TC_CH slices (64 additions) and added, in fp32 with rounding to nearest, to
// a running sum that also lives in TMEM; the hi*lo and lo*hi terms, 2^-11 of
// the size, share a second accumulator over the whole K range, where what is
// dropped is 2^-11 smaller again.  TMEM columns: hi*hi chunk accumulators
// 0-127 and 128-255 (alternating chunks), corrections 256-383, running sum
// 384-511.
//
// The tensor cores compute the transposed tile, D[n][m] = sum_k B^T[n][k]
// A[m][k]: TMEM lanes are C's columns, so the epilogue writes C's rows
// coalesced.  CTA: 128 (n) x 128 (m) outputs, K in slices of 32 (one 128-byte
// swizzled row of fp32).
//  * Producers (warps 0-7): each slice's A and B^T tiles from global memory,
//    two slices ahead in registers, split into hi and lo and stored 128-byte
//    swizzled in the operand's own major order: K-contiguous operands (A of
//    NN/NT, B of NT) K-major, the others (A of TN, B of NN) MN-major, which the
//    tensor cores read directly (instruction descriptor bits 15/16), so every
//    global load is a coalesced row and every shared store a 16-byte chunk.  TC_ST
//    slices into chunk c + 1 they add chunk c's accumulator into the running
//    sum (the MMA warp is then busy with the stages already filled).
//  * MMA warp (warp 8, one thread): per slice and K=8 step, B^T_hi.A_hi into
//    the chunk accumulator, B^T_hi.A_lo and B^T_lo.A_hi into the correction
//    accumulator; tcgen05.commit releases the stage, and at a chunk's end
//    tells the producers its accumulator is complete.
//  * Epilogue: warps q and q + 4 read TMEM lanes 32q..32q+31 (n), each half of
//    the m columns, sum running sum + unflushed chunks + corrections and write
//    alpha*D (+ beta*C) — or the raw partial sums into the K-split workspace.
// Every wait is bounded; a CTA whose wait timed out writes its tile as NaN
// (and sets the error word when one is given); TMEM is freed on every path.
#include "sgemm.cuh"
#include "tc.cuh"
#include <algorithm>

namespace cats {

constexpr int TC_M = 128;                      // m per CTA (the UMMA N)
constexpr int TC_N = 128;                      // n per CTA (the UMMA M)
constexpr int TC_K = 32;                       // k per slice
constexpr int TC_ST = 3;                       // stages
constexpr int TC_CH = 16;                      // slices per hi*hi chunk (64 accumulator additions)
constexpr int TC_PROD = 256;
constexpr int TC_THREADS = TC_PROD + 32;
constexpr int TC_MMA_WARP = TC_PROD / 32;
constexpr uint32_t TC_TILE = 128 * 128;        // bytes of one 128-row x 32-float tile
constexpr uint32_t TC_STAGE = 4 * TC_TILE;     // B^T hi, B^T lo, A hi, A lo
constexpr uint32_t TC_TCOLS = 512;             // TMEM columns: 2 chunk accumulators, corrections, running sum
constexpr uint32_t TC_COL_CORR = 256, TC_COL_SUM = 384;
static_assert(TC_ST <= TC_CH, "a chunk is flushed TC_ST slices into the next one");

struct SgemmTcArgs {
    int M, N, K;
    float alpha, beta;
    const float *A, *B;
    int lda, ldb;
    float *C;
    int ldc;
    float *work;        // K-split partials [splits][M][N] (splits > 1)
    int k_per_split;
    int *err;
};

// Shared-memory barriers and flags after the stages.
struct TcBars {
    uint64_t full[TC_ST], empty[TC_ST];
    uint64_t chunk_done[2];   // a chunk's hi*hi accumulator is complete (tcgen05.commit)
    uint64_t drained[2];      // the producers have added it into the running sum (8 warp arrivals)
    uint64_t done;            // every MMA of the CTA has completed
    uint32_t tmem;
    int abort;
    int commits[TC_ST], chunk_commits[2];
};

__device__ __forceinline__ uint32_t to_tf32(float x)
{
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

// hi and lo of four floats
__device__ __forceinline__ void split4(float4 v, uint4 &hi, uint4 &lo)
{
    hi.x = to_tf32(v.x); lo.x = to_tf32(v.x - __uint_as_float(hi.x));
    hi.y = to_tf32(v.y); lo.y = to_tf32(v.y - __uint_as_float(hi.y));
    hi.z = to_tf32(v.z); lo.z = to_tf32(v.z - __uint_as_float(hi.z));
    hi.w = to_tf32(v.w); lo.w = to_tf32(v.w - __uint_as_float(hi.w));
}

// One operand tile of a slice: 128 rows (m or n) x 32 k.  K_CONTIG: the
// operand is stored row-major along k (X[row][k], ld) and thread t loads
// f = t + 256 i -> (row f / 8, k 4 (f % 8)): 8 lanes per 128-byte row.  Else
// it is stored along rows (X[k][row], ld) and warp w loads k = w + 8 i, rows
// 4 lane .. 4 lane + 3: one 512-byte row of the tile per warp instruction.
template <bool K_CONTIG>
__device__ __forceinline__ void load_tile(const float *__restrict__ X, int ld, int rows, int K, int r0, int k0,
                                          float4 (&v)[4])
{
    const int t = threadIdx.x;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (K_CONTIG) {
            const int f = t + TC_PROD * i, r = r0 + f / 8, k = k0 + 4 * (f % 8);
            if (r < rows && k < K) v[i] = *reinterpret_cast<const float4 *>(X + (size_t)r * ld + k);
        } else {
            const int k = k0 + (t >> 5) + 8 * i, r = r0 + 4 * (t & 31);
            if (k < K && r < rows) v[i] = *reinterpret_cast<const float4 *>(X + (size_t)k * ld + r);
        }
    }
}

// Byte offset of the 16 bytes holding rows r..r+3 (r a multiple of 4) at
// column k in an MN-major tile of 128 rows x 32 k, in the tensor cores'
// MN-major tf32 layout "128-byte swizzle, 32-byte atomicity" (layout type 1;
// the only MN-major layout they take for 32-bit operands): atoms of 4 k-rows
// x 32 rows (512 bytes; k-row kr at kr * 128, its 32-byte chunk c of 8 rows
// at (c ^ kr) * 32), the four row atoms 512 bytes apart (the descriptor's
// leading offset) and the eight k atoms 2048 bytes apart (its stride offset).
__device__ __forceinline__ uint32_t mn_sw128(int r, int k)
{
    const int kr = k & 3, c = (r >> 3) & 3;
    return (uint32_t)((k >> 2) * 2048 + (r >> 5) * 512 + kr * 128 + ((c ^ kr) * 32) + (r & 4) * 4);
}

// Split a thread's loaded values into hi and lo and store them in the
// tile's layout: K-major for K_CONTIG operands, MN-major for the others.
template <bool K_CONTIG>
__device__ __forceinline__ void store_tile(uint8_t *hi_t, uint8_t *lo_t, const float4 (&v)[4])
{
    const int t = threadIdx.x;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint4 h, l;
        split4(v[i], h, l);
        uint32_t off;
        if (K_CONTIG) {
            const int f = t + TC_PROD * i;
            off = sw128(f / 8, f % 8);
        } else {
            off = mn_sw128(4 * (t & 31), (t >> 5) + 8 * i);
        }
        *reinterpret_cast<uint4 *>(hi_t + off) = h;
        *reinterpret_cast<uint4 *>(lo_t + off) = l;
    }
}

// UMMA shared-memory descriptor of that MN-major tile (version 1, layout
// type 1 = 128-byte swizzle with 32-byte atomicity): leading offset 512 bytes
// between 32-row atoms, stride offset 2048 bytes between 4-k atoms.
__device__ __forceinline__ uint64_t umma_desc_mn_sw128(uint32_t smem_addr)
{
    return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)(512 >> 4) << 16) | ((uint64_t)(2048 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)1 << 61);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
                 ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
                   "r"(v[7])
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// The producers add chunk c's hi*hi accumulator into the running sum (the
// first chunk initialises it), then free the accumulator for chunk c + 2.
__device__ __forceinline__ bool flush_chunk(TcBars *bars, uint32_t tmem, int c, int *err)
{
    const int b = c & 1;
    const bool ok = tc_wait(&bars->chunk_done[b], (uint32_t)(c >> 1) & 1u, &bars->abort, err, CATS_DEVERR_MBAR_FULL);
    if (!__all_sync(0xffffffffu, ok)) return false;
    tc_fence_after();
    const int warp = threadIdx.x >> 5, q = warp & 3, half = warp >> 2;
    const uint32_t lanes = (uint32_t)(q * 32) << 16;
#pragma unroll 1
    for (int c0 = half * (TC_M / 2); c0 < (half + 1) * (TC_M / 2); c0 += 8) {
        uint32_t v[8], r[8];
        tmem_ld8(tmem + lanes + (uint32_t)(b * 128 + c0), v);
        if (c > 0) tmem_ld8(tmem + lanes + TC_COL_SUM + (uint32_t)c0, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; j++)
            r[j] = c > 0 ? __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(v[j])) : v[j];
        tmem_st8(tmem + lanes + TC_COL_SUM + (uint32_t)c0, r);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&bars->drained[b]);
    return true;
}

// One slice kb for the producers: flush the previous chunk when kb is TC_ST
// slices into a new one, wait for the slice's stage to be free, split the
// registers' fp32 values into hi and lo tiles, load slice kb + 2 into the same
// registers and hand the stage to the MMA warp.
template <bool TA, bool TB>
__device__ __forceinline__ bool produce(const SgemmTcArgs &a, uint8_t *smem, TcBars *bars, uint32_t tmem, int kb,
                                        int nk, int kb0, int kend, int m0, int n0, float4 (&va)[4], float4 (&vb)[4])
{
    if (kb % TC_CH == TC_ST && kb >= TC_CH && !flush_chunk(bars, tmem, kb / TC_CH - 1, a.err)) return false;
    const int s = kb % TC_ST;
    // every lane waits (bounded); the warp goes on only if all of them saw the stage free
    const bool ok = tc_wait(&bars->empty[s], ((uint32_t)(kb / TC_ST) & 1u) ^ 1u, &bars->abort, a.err,
                            CATS_DEVERR_MBAR_EMPTY);
    if (!__all_sync(0xffffffffu, ok)) return false;
    uint8_t *st = smem + s * TC_STAGE;
    store_tile<TB>(st, st + TC_TILE, vb);
    store_tile<!TA>(st + 2 * TC_TILE, st + 3 * TC_TILE, va);
    if (kb + 2 < nk) {
        load_tile<!TA>(a.A, a.lda, a.M, kend, m0, kb0 + (kb + 2) * TC_K, va);
        load_tile<TB>(a.B, a.ldb, a.N, kend, n0, kb0 + (kb + 2) * TC_K, vb);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&bars->full[s]);
    return true;
}

__device__ __forceinline__ void umma_tf32(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
        ::"r"(d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

template <bool TA, bool TB>
__global__ void __launch_bounds__(TC_THREADS, 1) k_sgemm_tc(const __grid_constant__ SgemmTcArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
    TcBars *bars = reinterpret_cast<TcBars *>(smem + TC_ST * TC_STAGE);
    volatile int *abort_s = &bars->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * TC_M, n0 = blockIdx.y * TC_N;
    const int kb0 = blockIdx.z * a.k_per_split, kend = min(a.K, kb0 + a.k_per_split);
    const int nk = kend > kb0 ? (kend - kb0 + TC_K - 1) / TC_K : 0;
    const int nc = (nk + TC_CH - 1) / TC_CH;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_ST; s++) {
            mbar_init(&bars->full[s], TC_PROD / 32);
            mbar_init(&bars->empty[s], 1);
            bars->commits[s] = 0;
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&bars->chunk_done[b], 1);
            mbar_init(&bars->drained[b], TC_PROD / 32);
            bars->chunk_commits[b] = 0;
        }
        mbar_init(&bars->done, 1);
        bars->abort = 0;
        fence_barrier_init();
    }
    if (warp == TC_MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&bars->tmem)), "r"(TC_TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem;

    if (warp == TC_MMA_WARP) {
        if (lane == 0) {
            // MMA A = the B^T tile (MN-major when B is not transposed), MMA B = the A tile (MN-major when A is)
            const uint32_t idesc = umma_idesc(2, TC_N, TC_M) | (TB ? 0u : 1u << 15) | (TA ? 1u << 16 : 0u);
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % TC_ST, c = kb / TC_CH, b = c & 1;
                const bool chunk_start = kb % TC_CH == 0;
                // chunk c reuses chunk c - 2's accumulator once the producers have flushed it
                if (chunk_start && c >= 2) {
                    if (!tc_wait(&bars->drained[b], (uint32_t)((c >> 1) - 1) & 1u, abort_s, a.err,
                                 CATS_DEVERR_MBAR_FULL))
                        break;
                    tc_fence_after();
                }
                if (!tc_wait(&bars->full[s], (uint32_t)(kb / TC_ST) & 1u, abort_s, a.err, CATS_DEVERR_MBAR_FULL))
                    break;
                tc_fence_after();
                const uint32_t base = smem_u32(smem + s * TC_STAGE);
                const uint32_t bh = base, bl = base + TC_TILE, ah = base + 2 * TC_TILE, al = base + 3 * TC_TILE;
                const uint32_t d_chunk = tmem + (uint32_t)(b * 128), d_corr = tmem + TC_COL_CORR;
#pragma unroll
                for (int kk = 0; kk < TC_K / 8; kk++) {
                    // a K=8 step is 32 bytes into a K-major tile's rows, two 2048-byte k atoms of an MN-major one
                    const uint64_t d_bh = TB ? umma_desc_sw128(bh + kk * 32) : umma_desc_mn_sw128(bh + kk * 4096);
                    const uint64_t d_bl = TB ? umma_desc_sw128(bl + kk * 32) : umma_desc_mn_sw128(bl + kk * 4096);
                    const uint64_t d_ah = TA ? umma_desc_mn_sw128(ah + kk * 4096) : umma_desc_sw128(ah + kk * 32);
                    const uint64_t d_al = TA ? umma_desc_mn_sw128(al + kk * 4096) : umma_desc_sw128(al + kk * 32);
                    umma_tf32(d_chunk, d_bh, d_ah, idesc, !(chunk_start && kk == 0));
                    umma_tf32(d_corr, d_bh, d_al, idesc, !(kb == 0 && kk == 0));
                    umma_tf32(d_corr, d_bl, d_ah, idesc, 1u);
                }
                umma_commit(&bars->empty[s]);
                bars->commits[s]++;
                if (kb % TC_CH == TC_CH - 1 || kb == nk - 1) {
                    umma_commit(&bars->chunk_done[b]);
                    bars->chunk_commits[b]++;
                }
            }
            umma_commit(&bars->done);
        }
    } else {
        // ---------------- producers: two slices in flight in registers
        float4 va0[4], vb0[4], va1[4], vb1[4];
        if (nk > 0) {
            load_tile<!TA>(a.A, a.lda, a.M, kend, m0, kb0, va0);
            load_tile<TB>(a.B, a.ldb, a.N, kend, n0, kb0, vb0);
        }
        if (nk > 1) {
            load_tile<!TA>(a.A, a.lda, a.M, kend, m0, kb0 + TC_K, va1);
            load_tile<TB>(a.B, a.ldb, a.N, kend, n0, kb0 + TC_K, vb1);
        }
        for (int kb = 0; kb < nk; kb += 2) {
            if (!produce<TA, TB>(a, smem, bars, tmem, kb, nk, kb0, kend, m0, n0, va0, vb0)) break;
            if (kb + 1 < nk && !produce<TA, TB>(a, smem, bars, tmem, kb + 1, nk, kb0, kend, m0, n0, va1, vb1))
                break;
        }
        // ---------------- epilogue: lanes 32q..32q+31 = columns n of C
        const bool ok = mbar_wait_bounded(&bars->done, 0, a.err, CATS_DEVERR_MBAR_FULL);
        tc_fence_after();
        const bool good = __all_sync(0xffffffffu, ok && !*abort_s) && nk > 0;   // tcgen05.ld is warp-collective
        // chunk c was flushed when slice (c + 1) * TC_CH + TC_ST exists
        const bool have_sum = TC_CH + TC_ST < nk;
        const bool prev_open = nc >= 2 && !((nc - 1) * TC_CH + TC_ST < nk);
        const uint32_t last_b = (uint32_t)((nc - 1) & 1), prev_b = last_b ^ 1u;
        const int q = warp & 3, half = warp >> 2;
        const int n = n0 + q * 32 + lane;
        const uint32_t lanes = tmem + ((uint32_t)(q * 32) << 16);
        float *dst = a.work ? a.work + (size_t)blockIdx.z * a.M * a.N : a.C;
        const int ld = a.work ? a.N : a.ldc;
#pragma unroll 1
        for (int c0 = half * (TC_M / 2); c0 < (half + 1) * (TC_M / 2); c0 += 8) {
            float acc[8];
            if (good) {
                uint32_t vc[8], vl[8], vs[8], vp[8];
                tmem_ld8(lanes + TC_COL_CORR + (uint32_t)c0, vc);
                tmem_ld8(lanes + last_b * 128 + (uint32_t)c0, vl);
                if (have_sum) tmem_ld8(lanes + TC_COL_SUM + (uint32_t)c0, vs);
                if (prev_open) tmem_ld8(lanes + prev_b * 128 + (uint32_t)c0, vp);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    float hh = __uint_as_float(vl[j]);
                    if (prev_open) hh += __uint_as_float(vp[j]);
                    if (have_sum) hh += __uint_as_float(vs[j]);
                    acc[j] = hh + __uint_as_float(vc[j]);
                }
            }
            if (n < a.N) {
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int m = m0 + c0 + j;
                    if (m >= a.M) break;
                    float *p = dst + (size_t)m * ld + n;
                    if (!good) *p = __int_as_float(0x7fc00000);   // a timed-out tile reads as NaN
                    else if (a.work) *p = acc[j];
                    else *p = a.beta == 0.f ? a.alpha * acc[j] : fmaf(a.alpha, acc[j], a.beta * *p);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == TC_MMA_WARP) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TCOLS));
    }
    if (threadIdx.x == 0) {
        // each commit's arrive lands when its MMAs complete: wait for the last
        // one on every barrier before invalidating it
        for (int s = 0; s < TC_ST; s++)
            if (bars->commits[s] > 0) mbar_wait_bounded(&bars->empty[s], (uint32_t)(bars->commits[s] - 1) & 1u, nullptr, 0);
        for (int b = 0; b < 2; b++)
            if (bars->chunk_commits[b] > 0)
                mbar_wait_bounded(&bars->chunk_done[b], (uint32_t)(bars->chunk_commits[b] - 1) & 1u, nullptr, 0);
        for (int s = 0; s < TC_ST; s++) {
            mbar_inval(&bars->full[s]);
            mbar_inval(&bars->empty[s]);
        }
        for (int b = 0; b < 2; b++) {
            mbar_inval(&bars->chunk_done[b]);
            mbar_inval(&bars->drained[b]);
        }
        mbar_inval(&bars->done);
    }
}

size_t sgemm_tc_smem_bytes()
{
    return 1024 + (size_t)TC_ST * TC_STAGE + sizeof(TcBars);
}

bool sgemm_tc_usable(bool ta, bool tb, int M, int N, int K, const float *A, int lda, const float *B, int ldb)
{
    // float4 loads along each operand's contiguous extent; big enough to beat the CUDA-core kernel
    if (M <= 0 || N <= 0 || K <= 0) return false;
    if ((uintptr_t)A % 16 || (uintptr_t)B % 16 || lda % 4 || ldb % 4) return false;
    if ((ta ? M % 4 : K % 4) || (tb ? K % 4 : N % 4)) return false;
    return (double)M * N * K >= 16.0 * 1024 * 1024;
}

template <bool TA, bool TB>
static cudaError_t launch_tc_t(dim3 grid, const SgemmTcArgs &a, cudaStream_t st)
{
    static bool attr = false;
    const size_t smem = sgemm_tc_smem_bytes();
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(k_sgemm_tc<TA, TB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e) return e;
        attr = true;
    }
    k_sgemm_tc<TA, TB><<<grid, TC_THREADS, smem, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_sgemm_tc(const SgemmPlan &p, bool ta, bool tb, int M, int N, int K, float alpha, const float *A,
                            int lda, const float *B, int ldb, float beta, float *C, int ldc, float *work, int *err,
                            cudaStream_t st)
{
    if (p.k_per_split % TC_K || (long long)p.k_per_split * p.splits < K) return cudaErrorInvalidValue;
    SgemmTcArgs a;
    a.M = M; a.N = N; a.K = K;
    a.alpha = alpha; a.beta = beta;
    a.A = A; a.B = B; a.lda = lda; a.ldb = ldb;
    a.C = C; a.ldc = ldc;
    a.work = p.splits > 1 ? work : nullptr;
    a.k_per_split = p.k_per_split;
    a.err = err;
    const dim3 grid(cdiv(M, TC_M), cdiv(N, TC_N), p.splits);   // x: m tiles, y: n tiles, z: K splits
    cudaError_t e;
    if (!ta && !tb) e = launch_tc_t<false, false>(grid, a, st);
    else if (!ta && tb) e = launch_tc_t<false, true>(grid, a, st);
    else if (ta && !tb) e = launch_tc_t<true, false>(grid, a, st);
    else e = launch_tc_t<true, true>(grid, a, st);
    if (e || p.splits == 1) return e;
    return launch_splitk_reduce(M, N, p.splits, alpha, work, beta, C, ldc, st);
}

} // namespace cats
