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
// normwise).  So the accumulator is restarted every TC_CH slices (96
// additions) and added, in fp32 with rounding to nearest, to a running sum
// that also lives in TMEM.  TMEM columns: chunk accumulator 0..BM-1, running
// sum BM..2 BM-1.  The MMA warp waits while the producers fold a finished
// chunk into the sum (a few hundred cycles per TC_CH slices).
//
// The tensor cores compute the transposed tile, D[n][m] = sum_k B^T[n][k]
// A[m][k] (UMMA M = 128 n, N = BM m): TMEM lanes are C's columns, so the
// epilogue writes C's rows coalesced.  CTA: 128 (n) x BM (m) outputs, BM 256
// (or 128 when M <= 128), K in slices of 32 (one 128-byte swizzled row of
// fp32).
//  * Producers (warps 0-7): each slice's A and B^T tiles from global memory,
//    two slices ahead in registers, split into hi and lo and stored 128-byte
//    swizzled in the operand's own major order: K-contiguous operands (A of
//    NN/NT, B of NT) K-major, the others (A of TN, B of NN) MN-major, which the
//    tensor cores read directly (instruction descriptor bits 15/16), so every
//    global load is a coalesced row and every shared store a 16-byte chunk.
//    One slice into each new chunk they fold the previous chunk into the sum.
//  * MMA warp (warp 8, one thread): per slice and K=8 step, B^T_hi.A_hi,
//    B^T_hi.A_lo and B^T_lo.A_hi into the chunk accumulator; tcgen05.commit
//    releases the stage, and at a chunk's end tells the producers the
//    accumulator is complete.
//  * Epilogue: warps q and q + 4 read TMEM lanes 32q..32q+31 (n), each half of
//    the m columns, add sum + last chunk and write alpha*D (+ beta*C) — or the
//    raw partial sums into the K-split workspace.
// Every wait is bounded; a CTA whose wait timed out writes its tile as NaN
// (and sets the error word when one is given); TMEM is freed on every path.
#include "sgemm.cuh"
#include "conv.cuh"
#include "tc.cuh"
#include <algorithm>

namespace cats {

constexpr int TC_N = 128;                      // n per CTA (the UMMA M)
constexpr int TC_K = 32;                       // k per slice
constexpr int TC_CH = 8;                       // slices per chunk (8 x 4 K steps x 3 products = 96 additions)
constexpr int TC_PROD = 256;
constexpr int TC_THREADS = TC_PROD + 32;
constexpr int TC_MMA_WARP = TC_PROD / 32;

// Per m-tile width BM (128 or 256): tile bytes and stages.
template <int BM>
struct TcCfg {
    static constexpr uint32_t BT = TC_N * 128;           // one 128-row x 32-float tile (B^T hi or lo)
    static constexpr uint32_t AT = BM * 128;             // one BM-row x 32-float tile (A hi or lo)
    static constexpr uint32_t STAGE = 2 * BT + 2 * AT;   // B^T hi, B^T lo, A hi, A lo
    static constexpr int ST = BM == 256 ? 2 : BM == 128 ? 3 : 4;
    static constexpr uint32_t TCOLS = 2 * BM;            // chunk accumulator + running sum
};

struct SgemmTcArgs {
    int M, N, K;
    float alpha, beta;
    const float *A, *B;
    int lda, ldb;
    float *C;
    int ldc;
    float *work;        // K-split partials [splits][M][N] (splits > 1)
    int k_per_split;
    int tiles_m;        // m tiles (tile t: m tile t % tiles_m, n tile t / tiles_m)
    int main_tiles;     // tiles computed whole; the rest in tail_split K pieces of tail_kps
    int tail_split, tail_kps;
    float *tail_ws;     // tail pieces' partials [piece][TC_N x BM block, m-major]
    int *err;
    // convolution mode: B = im2col(x), k = (ci * ks + ky) * ks + kx, n = (b, oy, ox);
    // C = z[b][m][oy * ow + ox]
    const float *x;
    int ich, h, wd, ks, pad, stride, ow, ohw;
};

// Shared-memory table of the convolution's k index (conv mode, after TcBars):
// the element offset ci * h * wd + ky * wd + kx and (ky << 16) | kx; k >= K
// gets ky = 0x4000, which no bounds test passes.
constexpr int TC_CONV_MAX_K = 2304;

// Shared-memory barriers and flags after the stages.
struct TcBars {
    uint64_t full[4], empty[4];
    uint64_t chunk_done;      // the chunk accumulator is complete (tcgen05.commit)
    uint64_t drained;         // the producers have folded it into the sum (8 warp arrivals)
    uint64_t done;            // every MMA of the CTA has completed
    uint32_t tmem;
    int abort;
    int commits[4], chunk_commits;
};

// Round an fp32 bit pattern to tf32 (10 stored mantissa bits), to nearest
// with ties away from zero: add half of the last kept place to the 13 dropped
// bits and clear them (a carry moves into the exponent, as rounding up
// should).  Two integer operations.  A NaN may come out as a zero or another
// NaN, but x - hi is then NaN, so the product still is.
__device__ __forceinline__ uint32_t tf32_rna(uint32_t b) { return (b + 0x1000u) & 0xFFFFE000u; }

// hi and lo of four floats: hi = tf32(x), lo = tf32(x - hi)
__device__ __forceinline__ void split4(float4 v, uint4 &hi, uint4 &lo)
{
    hi.x = tf32_rna(__float_as_uint(v.x)); lo.x = tf32_rna(__float_as_uint(v.x - __uint_as_float(hi.x)));
    hi.y = tf32_rna(__float_as_uint(v.y)); lo.y = tf32_rna(__float_as_uint(v.y - __uint_as_float(hi.y)));
    hi.z = tf32_rna(__float_as_uint(v.z)); lo.z = tf32_rna(__float_as_uint(v.z - __uint_as_float(hi.z)));
    hi.w = tf32_rna(__float_as_uint(v.w)); lo.w = tf32_rna(__float_as_uint(v.w - __uint_as_float(hi.w)));
}

// One operand tile of a slice: ROWS rows (m or n) x 32 k, ROWS / 32 float4
// per thread.  K_CONTIG: the operand is stored row-major along k (X[row][k],
// ld) and thread t loads f = t + 256 i -> (row f / 8, k 4 (f % 8)): 8 lanes
// per 128-byte row.  Else it is stored along rows (X[k][row], ld) and warp w
// loads k = w + 8 (i % 4), rows 128 (i / 4) + 4 lane .. + 3: 512 contiguous
// bytes of one k-row per warp instruction.
template <bool K_CONTIG, int ROWS, bool SCALAR = false>
__device__ __forceinline__ void load_tile(const float *__restrict__ X, int ld, int rows, int K, int r0, int k0,
                                          float4 (&v)[ROWS / 32])
{
    const int t = threadIdx.x;
#pragma unroll
    for (int i = 0; i < ROWS / 32; i++) {
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (K_CONTIG) {
            const int f = t + TC_PROD * i, r = r0 + f / 8, k = k0 + 4 * (f % 8);
            if (r < rows && k < K) {
                if (!SCALAR) {
                    v[i] = *reinterpret_cast<const float4 *>(X + (size_t)r * ld + k);
                } else {   // rows not 16-byte aligned (a convolution's K = ich * ks^2 not a multiple of 4)
                    const float *p = X + (size_t)r * ld + k;
                    v[i].x = p[0];
                    if (k + 1 < K) v[i].y = p[1];
                    if (k + 2 < K) v[i].z = p[2];
                    if (k + 3 < K) v[i].w = p[3];
                }
            }
        } else {
            const int k = k0 + (t >> 5) + 8 * (i & 3), r = r0 + 128 * (i >> 2) + 4 * (t & 31);
            if (k < K && r < rows) v[i] = *reinterpret_cast<const float4 *>(X + (size_t)k * ld + r);
        }
    }
}

// Byte offset of the 16 bytes holding rows r..r+3 (r a multiple of 4) at
// column k in an MN-major tile of ROWS rows x 32 k, in the tensor cores'
// MN-major tf32 layout "128-byte swizzle, 32-byte atomicity" (layout type 1;
// the only MN-major layout they take for 32-bit operands): atoms of 4 k-rows
// x 32 rows (512 bytes; k-row kr at kr * 128, its 32-byte chunk c of 8 rows
// at (c ^ kr) * 32), the row atoms 512 bytes apart (the descriptor's leading
// offset) and the eight k atoms ROWS * 16 bytes apart (its stride offset).
template <int ROWS>
__device__ __forceinline__ uint32_t mn_sw128(int r, int k)
{
    const int kr = k & 3, c = (r >> 3) & 3;
    return (uint32_t)((k >> 2) * (ROWS * 16) + (r >> 5) * 512 + kr * 128 + ((c ^ kr) * 32) + (r & 4) * 4);
}

// Split a thread's loaded values into hi and lo and store them in the
// tile's layout: K-major for K_CONTIG operands, MN-major for the others.
template <bool K_CONTIG, int ROWS>
__device__ __forceinline__ void store_tile(uint8_t *hi_t, uint8_t *lo_t, const float4 (&v)[ROWS / 32])
{
    const int t = threadIdx.x;
#pragma unroll
    for (int i = 0; i < ROWS / 32; i++) {
        uint4 h, l;
        split4(v[i], h, l);
        uint32_t off;
        if (K_CONTIG) {
            const int f = t + TC_PROD * i;
            off = sw128(f / 8, f % 8);
        } else {
            off = mn_sw128<ROWS>(128 * (i >> 2) + 4 * (t & 31), (t >> 5) + 8 * (i & 3));
        }
        *reinterpret_cast<uint4 *>(hi_t + off) = h;
        *reinterpret_cast<uint4 *>(lo_t + off) = l;
    }
}

// UMMA shared-memory descriptor of an MN-major tile of ROWS rows (version 1,
// layout type 1 = 128-byte swizzle with 32-byte atomicity): leading offset
// 512 bytes between 32-row atoms, stride offset ROWS * 16 bytes between 4-k
// atoms.
template <int ROWS>
__device__ __forceinline__ uint64_t umma_desc_mn_sw128(uint32_t smem_addr)
{
    return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)(512 >> 4) << 16) |
           ((uint64_t)((ROWS * 16) >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)1 << 61);
}

// Descriptor of K step kk (8 k) of an operand tile: 32 bytes into a K-major
// tile's rows, two k atoms (ROWS * 32 bytes) into an MN-major one.
template <bool K_MAJOR, int ROWS>
__device__ __forceinline__ uint64_t operand_desc(uint32_t tile, int kk)
{
    return K_MAJOR ? umma_desc_sw128(tile + kk * 32) : umma_desc_mn_sw128<ROWS>(tile + kk * (ROWS * 32));
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

// The producers fold chunk c's accumulator into the running sum (the first
// chunk initialises it) and hand the accumulator back for chunk c + 1.
template <int BM>
__device__ __forceinline__ bool flush_chunk(TcBars *bars, uint32_t tmem, int c, int *err)
{
    const bool ok = tc_wait(&bars->chunk_done, (uint32_t)c & 1u, &bars->abort, err, CATS_DEVERR_MBAR_FULL);
    if (!__all_sync(0xffffffffu, ok)) return false;
    tc_fence_after();
    const int warp = threadIdx.x >> 5, q = warp & 3, half = warp >> 2;
    const uint32_t lanes = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
    for (int c0 = half * (BM / 2); c0 < (half + 1) * (BM / 2); c0 += 8) {
        uint32_t v[8], r[8];
        tmem_ld8(lanes + (uint32_t)c0, v);
        if (c > 0) tmem_ld8(lanes + BM + (uint32_t)c0, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; j++)
            r[j] = c > 0 ? __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(v[j])) : v[j];
        tmem_st8(lanes + BM + (uint32_t)c0, r);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&bars->drained);
    return true;
}

// Convolution mode: a producer thread's four output pixels n0 + lane + 32 j
// as an element offset (b * ich * h * wd + iy0 * wd + ix0) and the input
// corner (iy0, ix0); pixels past N get a corner no bounds test passes.
struct ConvPix {
    int base[4], iy0[4], ix0[4];
};

__device__ __forceinline__ void conv_pixels(const SgemmTcArgs &a, int n0, ConvPix &cp)
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int n = n0 + lane + 32 * j;
        const int b = n / a.ohw, p = n - b * a.ohw, oy = p / a.ow, ox = p - oy * a.ow;
        cp.iy0[j] = n < a.N ? oy * a.stride - a.pad : -0x40000;
        cp.ix0[j] = ox * a.stride - a.pad;
        cp.base[j] = n < a.N ? (b * a.ich * a.h + cp.iy0[j]) * a.wd + cp.ix0[j] : 0;
    }
}

// The im2col tile of slice k0: thread (warp w, lane) gathers k = k0 + w + 8 i
// for its four pixels into v[i] (component j = pixel lane + 32 j); lanes are
// consecutive pixels, so each load instruction reads a contiguous row span.
__device__ __forceinline__ void gather_tile(const SgemmTcArgs &a, const int2 *ktab, const ConvPix &cp, int k0,
                                            float4 (&v)[4])
{
    const int w = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int2 e = ktab[k0 + w + 8 * i];
        const int ky = e.y >> 16, kx = e.y & 0xffff;
        float r[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int iy = cp.iy0[j] + ky, ix = cp.ix0[j] + kx;
            r[j] = ((unsigned)iy < (unsigned)a.h && (unsigned)ix < (unsigned)a.wd) ? __ldg(a.x + cp.base[j] + e.x) : 0.f;
        }
        v[i] = make_float4(r[0], r[1], r[2], r[3]);
    }
}

// Convolution mode 3 (the input channels a multiple of 32): K in the order
// k' = (ky ks + kx) ich + ci, so slice s is one kernel offset kyx = 32 s / ich
// over channels ci0 = 32 s % ich .. + 31.  A thread's four pixels then need
// one bounds test and one base address per slice, and its four channel rows
// of the slice add ci h wd each.  The weights are permuted into the same
// order first (k_perm_weights); the sums are the same products in another
// order.
__device__ __forceinline__ void gather_tile_cb(const SgemmTcArgs &a, const ConvPix &cp, int slice, float4 (&v)[4])
{
    const int w = threadIdx.x >> 5;
    const int k0 = slice * TC_K, kyx = k0 / a.ich, ci0 = k0 - kyx * a.ich;
    const int ky = kyx / a.ks, kx = kyx - ky * a.ks;
    const int hw = a.h * a.wd;
    int off[4];
    bool ok[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        ok[j] = (unsigned)(cp.iy0[j] + ky) < (unsigned)a.h && (unsigned)(cp.ix0[j] + kx) < (unsigned)a.wd;
        off[j] = cp.base[j] + ky * a.wd + kx;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int co = (ci0 + w + 8 * i) * hw;
        float r[4];
#pragma unroll
        for (int j = 0; j < 4; j++) r[j] = ok[j] ? __ldg(a.x + off[j] + co) : 0.f;
        v[i] = make_float4(r[0], r[1], r[2], r[3]);
    }
}

// Store a gathered tile as hi and lo in the MN-major layout of the B^T
// tile: element (pixel lane + 32 j, k w + 8 i), 4-byte stores; the 32 lanes
// of an instruction fill one 128-byte k-row, each bank once.
__device__ __forceinline__ void store_gathered(uint8_t *hi_t, uint8_t *lo_t, const float4 (&v)[4])
{
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int r = lane + 32 * j;
            const uint32_t off = mn_sw128<TC_N>(r & ~3, w + 8 * i) + (r & 3) * 4;
            const uint32_t hb = tf32_rna(__float_as_uint(e[j]));
            *reinterpret_cast<uint32_t *>(hi_t + off) = hb;
            *reinterpret_cast<uint32_t *>(lo_t + off) = tf32_rna(__float_as_uint(e[j] - __uint_as_float(hb)));
        }
    }
}

// One slice kb for the producers: fold the previous chunk into the sum when
// kb is the second slice of a chunk, wait for the slice's stage to be free,
// split the registers' fp32 values into hi and lo tiles, load slice kb + 2
// into the same registers and hand the stage to the MMA warp.
template <bool TA, bool TB, int BM, int CONV>
__device__ __forceinline__ bool produce(const SgemmTcArgs &a, uint8_t *smem, TcBars *bars, uint32_t tmem, int kb,
                                        int nk, int kb0, int kend, int m0, int n0, int &flushed,
                                        float4 (&va)[BM / 32], float4 (&vb)[TC_N / 32], const int2 *ktab,
                                        const ConvPix &cp)
{
    using Cfg = TcCfg<BM>;
    if (kb % TC_CH == 1 && kb > TC_CH) {
        if (!flush_chunk<BM>(bars, tmem, flushed, a.err)) return false;
        flushed++;
    }
    const int s = kb % Cfg::ST;
    // every lane waits (bounded); the warp goes on only if all of them saw the stage free
    const bool ok = tc_wait(&bars->empty[s], ((uint32_t)(kb / Cfg::ST) & 1u) ^ 1u, &bars->abort, a.err,
                            CATS_DEVERR_MBAR_EMPTY);
    if (!__all_sync(0xffffffffu, ok)) return false;
    uint8_t *st = smem + s * Cfg::STAGE;
    if (CONV) store_gathered(st, st + Cfg::BT, vb);
    else store_tile<TB, TC_N>(st, st + Cfg::BT, vb);
    store_tile<!TA, BM>(st + 2 * Cfg::BT, st + 2 * Cfg::BT + Cfg::AT, va);
    if (kb + 2 < nk) {
        if (CONV == 3) {
            load_tile<true, BM>(a.A, a.lda, a.M, kend, m0, kb0 + (kb + 2) * TC_K, va);
            gather_tile_cb(a, cp, kb + 2, vb);
        } else {
            load_tile<!TA, BM, CONV == 2>(a.A, a.lda, a.M, kend, m0, kb0 + (kb + 2) * TC_K, va);
            if (CONV) gather_tile(a, ktab, cp, kb0 + (kb + 2) * TC_K, vb);
            else load_tile<TB, TC_N>(a.B, a.ldb, a.N, kend, n0, kb0 + (kb + 2) * TC_K, vb);
        }
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

// CONV: 0 GEMM, 1 convolution, 2 convolution whose weight rows are not
// 16-byte aligned (scalar weight loads), 3 convolution in the channel-blocked
// K order (input channels a multiple of 32)
template <bool TA, bool TB, int BM, int CONV = 0>
__global__ void __launch_bounds__(TC_THREADS, 1) k_sgemm_tc(const __grid_constant__ SgemmTcArgs a)
{
    using Cfg = TcCfg<BM>;
    constexpr int ST = Cfg::ST;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
    TcBars *bars = reinterpret_cast<TcBars *>(smem + ST * Cfg::STAGE);
    volatile int *abort_s = &bars->abort;
    int2 *ktab = reinterpret_cast<int2 *>(bars + 1);   // conv mode only

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // work unit blockIdx.x: a whole tile, or K piece of a tail tile
    const int unit = blockIdx.x, piece = unit - a.main_tiles;
    const int tile = piece < 0 ? unit : a.main_tiles + piece / a.tail_split;
    const int m0 = (tile % a.tiles_m) * BM, n0 = (tile / a.tiles_m) * TC_N;
    const int kb0 = piece < 0 ? blockIdx.z * a.k_per_split : (piece % a.tail_split) * a.tail_kps;
    const int kend = min(a.K, kb0 + (piece < 0 ? a.k_per_split : a.tail_kps));
    const int nk = kend > kb0 ? (kend - kb0 + TC_K - 1) / TC_K : 0;
    const int nc = (nk + TC_CH - 1) / TC_CH;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; s++) {
            mbar_init(&bars->full[s], TC_PROD / 32);
            mbar_init(&bars->empty[s], 1);
            bars->commits[s] = 0;
        }
        mbar_init(&bars->chunk_done, 1);
        mbar_init(&bars->drained, TC_PROD / 32);
        mbar_init(&bars->done, 1);
        bars->chunk_commits = 0;
        bars->abort = 0;
        fence_barrier_init();
    }
    if (CONV == 1 || CONV == 2) {
        const int kk2 = a.ks * a.ks, kpad = (a.K + TC_K - 1) / TC_K * TC_K;
        for (int k = threadIdx.x; k < kpad; k += blockDim.x) {
            const int ci = k / kk2, r = k - ci * kk2, ky = r / a.ks, kx = r - ky * a.ks;
            ktab[k] = k < a.K ? make_int2((ci * a.h + ky) * a.wd + kx, (ky << 16) | kx) : make_int2(0, 0x4000 << 16);
        }
    }
    if (warp == TC_MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&bars->tmem)), "r"(Cfg::TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem;

    if (warp == TC_MMA_WARP) {
        if (lane == 0) {
            // MMA A = the B^T tile (MN-major when B is not transposed), MMA B = the A tile (MN-major when A is)
            const uint32_t idesc = umma_idesc(2, TC_N, BM) | (TB ? 0u : 1u << 15) | (TA ? 1u << 16 : 0u);
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % ST, c = kb / TC_CH;
                const bool chunk_start = kb % TC_CH == 0;
                // chunk c reuses the accumulator once the producers have folded chunk c - 1 into the sum
                if (chunk_start && c >= 1) {
                    if (!tc_wait(&bars->drained, (uint32_t)(c - 1) & 1u, abort_s, a.err, CATS_DEVERR_MBAR_FULL))
                        break;
                    tc_fence_after();
                }
                if (!tc_wait(&bars->full[s], (uint32_t)(kb / ST) & 1u, abort_s, a.err, CATS_DEVERR_MBAR_FULL))
                    break;
                tc_fence_after();
                const uint32_t bh = smem_u32(smem + s * Cfg::STAGE), bl = bh + Cfg::BT;
                const uint32_t ah = bh + 2 * Cfg::BT, al = ah + Cfg::AT;
#pragma unroll
                for (int kk = 0; kk < TC_K / 8; kk++) {
                    const uint64_t d_bh = operand_desc<TB, TC_N>(bh, kk), d_bl = operand_desc<TB, TC_N>(bl, kk);
                    const uint64_t d_ah = operand_desc<!TA, BM>(ah, kk), d_al = operand_desc<!TA, BM>(al, kk);
                    umma_tf32(tmem, d_bh, d_ah, idesc, !(chunk_start && kk == 0));
                    umma_tf32(tmem, d_bh, d_al, idesc, 1u);
                    umma_tf32(tmem, d_bl, d_ah, idesc, 1u);
                }
                umma_commit(&bars->empty[s]);
                bars->commits[s]++;
                if (kb % TC_CH == TC_CH - 1 || kb == nk - 1) {
                    umma_commit(&bars->chunk_done);
                    bars->chunk_commits++;
                }
            }
            umma_commit(&bars->done);
        }
    } else {
        // ---------------- producers: two slices in flight in registers
        float4 va0[BM / 32], vb0[TC_N / 32], va1[BM / 32], vb1[TC_N / 32];
        int flushed = 0;   // chunks folded into the sum so far
        ConvPix cp;
        if (CONV) conv_pixels(a, n0, cp);
        if (CONV == 3) {
            if (nk > 0) {
                load_tile<true, BM>(a.A, a.lda, a.M, kend, m0, kb0, va0);
                gather_tile_cb(a, cp, 0, vb0);
            }
            if (nk > 1) {
                load_tile<true, BM>(a.A, a.lda, a.M, kend, m0, kb0 + TC_K, va1);
                gather_tile_cb(a, cp, 1, vb1);
            }
        } else {
            if (nk > 0) {
                load_tile<!TA, BM, CONV == 2>(a.A, a.lda, a.M, kend, m0, kb0, va0);
                if (CONV) gather_tile(a, ktab, cp, kb0, vb0);
                else load_tile<TB, TC_N>(a.B, a.ldb, a.N, kend, n0, kb0, vb0);
            }
            if (nk > 1) {
                load_tile<!TA, BM, CONV == 2>(a.A, a.lda, a.M, kend, m0, kb0 + TC_K, va1);
                if (CONV) gather_tile(a, ktab, cp, kb0 + TC_K, vb1);
                else load_tile<TB, TC_N>(a.B, a.ldb, a.N, kend, n0, kb0 + TC_K, vb1);
            }
        }
        bool live = true;
        for (int kb = 0; kb < nk && live; kb += 2) {
            live = produce<TA, TB, BM, CONV>(a, smem, bars, tmem, kb, nk, kb0, kend, m0, n0, flushed, va0, vb0, ktab,
                                             cp);
            if (live && kb + 1 < nk)
                live = produce<TA, TB, BM, CONV>(a, smem, bars, tmem, kb + 1, nk, kb0, kend, m0, n0, flushed, va1,
                                                 vb1, ktab, cp);
        }
        // a last chunk of a single slice: its predecessor is folded here
        if (live && flushed < nc - 1) live = flush_chunk<BM>(bars, tmem, flushed++, a.err);
        // ---------------- epilogue: lanes 32q..32q+31 = columns n of C
        const bool ok = mbar_wait_bounded(&bars->done, 0, a.err, CATS_DEVERR_MBAR_FULL);
        tc_fence_after();
        const bool good = __all_sync(0xffffffffu, ok && live && !*abort_s) && nk > 0;   // tcgen05.ld is warp-collective
        const int q = warp & 3, half = warp >> 2;
        const int n = n0 + q * 32 + lane;
        const uint32_t lanes = tmem + ((uint32_t)(q * 32) << 16);
        // destination: C, a K split's slab [M][N], or a tail piece's block [m - m0][n - n0];
        // conv mode: z[b][m][p] for pixel n = b * ohw + p
        float *dst = piece >= 0 ? a.tail_ws + (size_t)piece * TC_N * BM
                     : a.work   ? a.work + (size_t)blockIdx.z * a.M * a.N
                                : a.C;
        const int ld = CONV ? a.ohw : piece >= 0 ? TC_N : a.work ? a.N : a.ldc;
        const int mo = piece >= 0 ? m0 : 0;
        size_t noff = (size_t)(n - (piece >= 0 ? n0 : 0));
        if (CONV) {
            const int b = n / a.ohw;
            noff = (size_t)b * a.M * a.ohw + (n - b * a.ohw);
        }
        const bool raw_sum = piece >= 0 || a.work;
#pragma unroll 1
        for (int c0 = half * (BM / 2); c0 < (half + 1) * (BM / 2); c0 += 8) {
            float acc[8];
            if (good) {
                uint32_t vl[8], vs[8];
                tmem_ld8(lanes + (uint32_t)c0, vl);
                if (nc > 1) tmem_ld8(lanes + BM + (uint32_t)c0, vs);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 8; j++)
                    acc[j] = nc > 1 ? __uint_as_float(vs[j]) + __uint_as_float(vl[j]) : __uint_as_float(vl[j]);
            }
            if (n < a.N) {
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int m = m0 + c0 + j;
                    if (m >= a.M) break;
                    float *p = dst + (size_t)(m - mo) * ld + noff;
                    if (!good) *p = __int_as_float(0x7fc00000);   // a timed-out tile reads as NaN
                    else if (raw_sum) *p = acc[j];
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::TCOLS));
    }
    if (threadIdx.x == 0) {
        // each commit's arrive lands when its MMAs complete: wait for the last
        // one on every barrier before invalidating it
        for (int s = 0; s < ST; s++)
            if (bars->commits[s] > 0)
                mbar_wait_bounded(&bars->empty[s], (uint32_t)(bars->commits[s] - 1) & 1u, nullptr, 0);
        if (bars->chunk_commits > 0)
            mbar_wait_bounded(&bars->chunk_done, (uint32_t)(bars->chunk_commits - 1) & 1u, nullptr, 0);
        for (int s = 0; s < ST; s++) {
            mbar_inval(&bars->full[s]);
            mbar_inval(&bars->empty[s]);
        }
        mbar_inval(&bars->chunk_done);
        mbar_inval(&bars->drained);
        mbar_inval(&bars->done);
    }
}

template <int BM>
static size_t smem_bytes(int conv_kpad = 0)
{
    return 1024 + (size_t)TcCfg<BM>::ST * TcCfg<BM>::STAGE + sizeof(TcBars) + (size_t)conv_kpad * sizeof(int2);
}

size_t sgemm_tc_smem_bytes() { return std::max(smem_bytes<128>(), smem_bytes<256>()); }

bool sgemm_tc_usable(bool ta, bool tb, int M, int N, int K, const float *A, int lda, const float *B, int ldb)
{
    // float4 loads along each operand's contiguous extent; big enough to beat the CUDA-core kernel
    if (M <= 0 || N <= 0 || K <= 0) return false;
    if ((uintptr_t)A % 16 || (uintptr_t)B % 16 || lda % 4 || ldb % 4) return false;
    if ((ta ? M % 4 : K % 4) || (tb ? K % 4 : N % 4)) return false;
    return (double)M * N * K >= 16.0 * 1024 * 1024;
}

int sgemm_tc_tile_m(int M) { return M > 128 ? 256 : 128; }

template <bool TA, bool TB, int BM>
static cudaError_t launch_tc_t(dim3 grid, const SgemmTcArgs &a, cudaStream_t st)
{
    static unsigned long long attr = 0;   // one bit per device
    const size_t smem = smem_bytes<BM>();
    cudaError_t e = once_per_device(attr, [smem] {
        return cudaFuncSetAttribute(k_sgemm_tc<TA, TB, BM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    });
    if (e) return e;
    k_sgemm_tc<TA, TB, BM><<<grid, TC_THREADS, smem, st>>>(a);
    return cudaGetLastError();
}

// C = alpha * (sum of a tail tile's K pieces, in piece order) + beta * C
template <int BM>
__global__ void k_tail_reduce(const __grid_constant__ SgemmTcArgs a, int tail_tiles)
{
    constexpr int TE = TC_N * BM;   // one tile's block in the workspace: [m - m0][n - n0]
    const size_t total = (size_t)tail_tiles * TE;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / TE), e = (int)(i % TE);
        const int tile = a.main_tiles + t;
        const int m = (tile % a.tiles_m) * BM + e / TC_N, n = (tile / a.tiles_m) * TC_N + e % TC_N;
        if (m >= a.M || n >= a.N) continue;
        const float *w = a.tail_ws + (size_t)t * a.tail_split * TE + e;
        float sum = 0.f;
        for (int q = 0; q < a.tail_split; q++) sum += w[(size_t)q * TE];
        float *p = a.C + (size_t)m * a.ldc + n;
        *p = a.beta == 0.f ? a.alpha * sum : fmaf(a.alpha, sum, a.beta * *p);
    }
}

template <int BM>
static cudaError_t launch_tc_bm(bool ta, bool tb, const SgemmTcArgs &a, int units, int splits, cudaStream_t st)
{
    const dim3 grid(units, 1, splits);
    if (!ta && !tb) return launch_tc_t<false, false, BM>(grid, a, st);
    if (!ta && tb) return launch_tc_t<false, true, BM>(grid, a, st);
    if (ta && !tb) return launch_tc_t<true, false, BM>(grid, a, st);
    return launch_tc_t<true, true, BM>(grid, a, st);
}

template <int BM>
static cudaError_t launch_tc(const SgemmPlan &p, bool ta, bool tb, SgemmTcArgs &a, cudaStream_t st)
{
    a.tiles_m = cdiv(a.M, BM);
    const int tiles = a.tiles_m * cdiv(a.N, TC_N);
    const bool tail = p.splits == 1 && p.tail_tiles > 0 && p.tail_tiles < tiles;
    a.main_tiles = tail ? tiles - p.tail_tiles : tiles;
    a.tail_split = tail ? p.tail_split : 1;
    a.tail_kps = tail ? p.tail_kps : 0;
    const int units = a.main_tiles + (tail ? p.tail_tiles * p.tail_split : 0);
    cudaError_t e = launch_tc_bm<BM>(ta, tb, a, units, p.splits, st);
    if (e || !tail) return e;
    const size_t total = (size_t)p.tail_tiles * TC_N * BM;
    k_tail_reduce<BM><<<(int)std::min<size_t>((total + 255) / 256, 148 * 8), 256, 0, st>>>(a, p.tail_tiles);
    return cudaGetLastError();
}

cudaError_t launch_sgemm_tc(const SgemmPlan &p, bool ta, bool tb, int M, int N, int K, float alpha, const float *A,
                            int lda, const float *B, int ldb, float beta, float *C, int ldc, float *work, int *err,
                            cudaStream_t st)
{
    if (p.k_per_split % TC_K || (long long)p.k_per_split * p.splits < K) return cudaErrorInvalidValue;
    if (p.tail_tiles > 0 && (p.tail_kps % TC_K || (long long)p.tail_kps * p.tail_split < K || !work))
        return cudaErrorInvalidValue;
    SgemmTcArgs a;
    a.M = M; a.N = N; a.K = K;
    a.alpha = alpha; a.beta = beta;
    a.A = A; a.B = B; a.lda = lda; a.ldb = ldb;
    a.C = C; a.ldc = ldc;
    a.work = p.splits > 1 ? work : nullptr;
    a.k_per_split = p.k_per_split;
    a.tail_ws = work;
    a.err = err;
    const cudaError_t e = sgemm_tc_tile_m(M) == 256 ? launch_tc<256>(p, ta, tb, a, st) : launch_tc<128>(p, ta, tb, a, st);
    if (e || p.splits == 1) return e;
    return launch_splitk_reduce(M, N, p.splits, alpha, work, beta, C, ldc, st);
}

// ---------------------------------------------------------------- convolution

// w[m][ci ks^2 + kyx] -> wp[m][kyx ich + ci], the channel-blocked K order
__global__ void k_perm_weights(const float *__restrict__ w, float *__restrict__ wp, int M, int ich, int kk2)
{
    const long long K = (long long)ich * kk2, total = (long long)M * K;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long m = i / K;
        const int kp = (int)(i - m * K), kyx = kp / ich, ci = kp - kyx * ich;
        wp[i] = w[m * K + (long long)ci * kk2 + kyx];
    }
}

bool conv_tc_usable(const float *w, int batch, int ich, int h, int wd, int ch, int ks, int pad, int stride)
{
    if (batch <= 0 || ich <= 0 || ch <= 0 || ch > 256 || ks <= 0 || stride <= 0) return false;
    const int oh = conv_out(h, ks, pad, stride), ow = conv_out(wd, ks, pad, stride);
    // the k table's invalid entry (ky = 0x4000) must fail every bounds test
    if (oh <= 0 || ow <= 0 || ks >= 0x4000 || h + pad >= 0x4000 || wd >= 0x4000) return false;
    const long long K = (long long)ich * ks * ks, N = (long long)batch * oh * ow;
    // 32-bit offsets into the images; at least three 32-deep slices per tile (a
    // shallower convolution is bound by writing its output, which the CUDA-core
    // kernel does with less fixed cost per tile)
    if (K > TC_CONV_MAX_K || K < 96) return false;
    if ((long long)batch * ich * h * wd >= (1LL << 31) || N >= (1LL << 31) || (long long)ch * N >= (1LL << 31))
        return false;
    return (double)ch * N * K >= 16.0 * 1024 * 1024;
}

template <int BM, int CONV>
static cudaError_t launch_conv_bm(const SgemmTcArgs &a, cudaStream_t st)
{
    static unsigned long long attr = 0;   // one bit per device
    cudaError_t e = once_per_device(attr, [] {
        return cudaFuncSetAttribute(k_sgemm_tc<false, false, BM, CONV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem_bytes<BM>(TC_CONV_MAX_K));
    });
    if (e) return e;
    const int kpad = CONV == 3 ? 0 : (a.K + TC_K - 1) / TC_K * TC_K;   // mode 3 needs no k table
    const int tiles = cdiv(a.M, BM) * cdiv(a.N, TC_N);
    k_sgemm_tc<false, false, BM, CONV><<<tiles, TC_THREADS, smem_bytes<BM>(kpad), st>>>(a);
    return cudaGetLastError();
}

// mode 3 (channel-blocked K order) when the input channels are a multiple of
// 32 and there is room for the permuted weights; else the k-table gather
template <int BM>
static cudaError_t launch_conv_bm(SgemmTcArgs a, bool scalar_w, float *wperm, cudaStream_t st)
{
    if (a.ich % TC_K == 0 && wperm) {
        const long long total = (long long)a.M * a.K;
        k_perm_weights<<<(int)std::min<long long>((total + 255) / 256, 148LL * 8), 256, 0, st>>>(a.A, wperm, a.M, a.ich,
                                                                                               a.ks * a.ks);
        cudaError_t e = cudaGetLastError();
        if (e) return e;
        a.A = wperm;
        return launch_conv_bm<BM, 3>(a, st);
    }
    return scalar_w ? launch_conv_bm<BM, 2>(a, st) : launch_conv_bm<BM, 1>(a, st);
}

cudaError_t launch_conv_tc(const float *x, const float *w, float *z, int batch, int ich, int h, int wd, int ch, int ks,
                           int pad, int stride, int *err, float *wperm, cudaStream_t st)
{
    if (!conv_tc_usable(w, batch, ich, h, wd, ch, ks, pad, stride)) return cudaErrorInvalidValue;
    SgemmTcArgs a = {};
    const int oh = conv_out(h, ks, pad, stride), ow = conv_out(wd, ks, pad, stride);
    a.M = ch;
    a.N = batch * oh * ow;
    a.K = ich * ks * ks;
    a.alpha = 1.f;
    a.beta = 0.f;
    a.A = w;
    a.lda = a.K;
    const bool scalar_w = a.K % 4 != 0 || (uintptr_t)w % 16 != 0;
    a.C = z;
    a.k_per_split = (a.K + TC_K - 1) / TC_K * TC_K;
    a.tail_split = 1;
    a.err = err;
    a.x = x;
    a.ich = ich;
    a.h = h;
    a.wd = wd;
    a.ks = ks;
    a.pad = pad;
    a.stride = stride;
    a.ow = ow;
    a.ohw = oh * ow;
    if (ch <= 64) {
        a.tiles_m = 1;
        a.main_tiles = cdiv(a.N, TC_N);
        return launch_conv_bm<64>(a, scalar_w, wperm, st);
    }
    if (ch <= 128) {
        a.tiles_m = 1;
        a.main_tiles = cdiv(a.N, TC_N);
        return launch_conv_bm<128>(a, scalar_w, wperm, st);
    }
    a.tiles_m = cdiv(ch, 256);
    a.main_tiles = a.tiles_m * cdiv(a.N, TC_N);
    return launch_conv_bm<256>(a, scalar_w, wperm, st);
}

} // namespace cats
