// sgemm.cu — fp32 row-major GEMM on CUDA cores for catseye's CNN layers.
//
// Reference: gemm_rnn / gemm_rnt / gemm_rtn (catseye.h:78-129) and the
// OpenCL/GL backends that replace them (sgemm_ocl2.h:17-90, sgemm_gl1.h:51-217):
// C = alpha*op(A)*op(B) + beta*C, beta == 0 never reads C.  The transposed
// forms need no transpose kernel: each (TA, TB) instantiation loads its tiles
// in the operand's own order and writes them k-major into shared memory.
//
// CTA tile 128x128x8, 256 threads, 8x8 outputs per thread (two 4-wide halves
// per dimension so shared-memory reads are float4 and conflict-free), register
// prefetch of the next k-slab into a second shared buffer.  Skinny problems
// that cannot fill 148 SMs split K across CTAs into a partial-sum workspace
// reduced by a second kernel that applies alpha/beta.
#include "sgemm.cuh"
#include <algorithm>

namespace cats {

constexpr int BM = 128, BN = 128, BK = 8, TM = 8, TN = 8, NT = 256;

template <bool TA, bool TB, bool VEC>
__device__ __forceinline__ void load_tiles(const float *__restrict__ A, int lda, const float *__restrict__ B, int ldb,
                                           int M, int N, int K, int m0, int n0, int k0, float (&ra)[4],
                                           float (&rb)[4])
{
    const int t = threadIdx.x;
    // A tile: 128 (m) x 8 (k)
    if (!TA) {   // A[m][k], 4 consecutive k for one m
        const int m = m0 + (t >> 1), k = k0 + (t & 1) * 4;
        if (VEC) {
            if (m < M && k < K) {
                const float4 v = *reinterpret_cast<const float4 *>(A + (size_t)m * lda + k);
                ra[0] = v.x; ra[1] = v.y; ra[2] = v.z; ra[3] = v.w;
            } else { ra[0] = ra[1] = ra[2] = ra[3] = 0.f; }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) ra[i] = (m < M && k + i < K) ? A[(size_t)m * lda + k + i] : 0.f;
        }
    } else {     // A[k][m], 4 consecutive m for one k
        const int k = k0 + (t >> 5), m = m0 + (t & 31) * 4;
        if (VEC) {
            if (k < K && m < M) {
                const float4 v = *reinterpret_cast<const float4 *>(A + (size_t)k * lda + m);
                ra[0] = v.x; ra[1] = v.y; ra[2] = v.z; ra[3] = v.w;
            } else { ra[0] = ra[1] = ra[2] = ra[3] = 0.f; }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) ra[i] = (k < K && m + i < M) ? A[(size_t)k * lda + m + i] : 0.f;
        }
    }
    // B tile: 8 (k) x 128 (n)
    if (!TB) {   // B[k][n]
        const int k = k0 + (t >> 5), n = n0 + (t & 31) * 4;
        if (VEC) {
            if (k < K && n < N) {
                const float4 v = *reinterpret_cast<const float4 *>(B + (size_t)k * ldb + n);
                rb[0] = v.x; rb[1] = v.y; rb[2] = v.z; rb[3] = v.w;
            } else { rb[0] = rb[1] = rb[2] = rb[3] = 0.f; }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) rb[i] = (k < K && n + i < N) ? B[(size_t)k * ldb + n + i] : 0.f;
        }
    } else {     // B[n][k]
        const int n = n0 + (t >> 1), k = k0 + (t & 1) * 4;
        if (VEC) {
            if (n < N && k < K) {
                const float4 v = *reinterpret_cast<const float4 *>(B + (size_t)n * ldb + k);
                rb[0] = v.x; rb[1] = v.y; rb[2] = v.z; rb[3] = v.w;
            } else { rb[0] = rb[1] = rb[2] = rb[3] = 0.f; }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) rb[i] = (n < N && k + i < K) ? B[(size_t)n * ldb + k + i] : 0.f;
        }
    }
}

template <bool TA, bool TB>
__device__ __forceinline__ void store_tiles(float (*As)[BM], float (*Bs)[BN], const float (&ra)[4], const float (&rb)[4])
{
    const int t = threadIdx.x;
    if (!TA) {
        const int m = t >> 1, k = (t & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) As[k + i][m] = ra[i];
    } else {
        const int k = t >> 5, m = (t & 31) * 4;
        *reinterpret_cast<float4 *>(&As[k][m]) = make_float4(ra[0], ra[1], ra[2], ra[3]);
    }
    if (!TB) {
        const int k = t >> 5, n = (t & 31) * 4;
        *reinterpret_cast<float4 *>(&Bs[k][n]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
    } else {
        const int n = t >> 1, k = (t & 1) * 4;
#pragma unroll
        for (int i = 0; i < 4; i++) Bs[k + i][n] = rb[i];
    }
}

// splits == 1: C = alpha*acc + beta*C.  splits > 1: blockIdx.z owns a K range
// and writes its raw partial tile into work[z][M][N].
template <bool TA, bool TB, bool VEC>
__global__ void __launch_bounds__(NT, 2) k_sgemm(int M, int N, int K, float alpha, const float *__restrict__ A, int lda,
                                                 const float *__restrict__ B, int ldb, float beta, float *__restrict__ C,
                                                 int ldc, int k_per_split, float *__restrict__ work)
{
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int kb = blockIdx.z * k_per_split, ke = min(K, kb + k_per_split);
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = 0.f;

    float ra[4], rb[4];
    int buf = 0;
    if (kb < ke) {
        load_tiles<TA, TB, VEC>(A, lda, B, ldb, M, N, ke, m0, n0, kb, ra, rb);
        store_tiles<TA, TB>(As[0], Bs[0], ra, rb);
    }
    __syncthreads();
    for (int k0 = kb; k0 < ke; k0 += BK) {
        const bool more = k0 + BK < ke;
        if (more) load_tiles<TA, TB, VEC>(A, lda, B, ldb, M, N, ke, m0, n0, k0 + BK, ra, rb);
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float a[TM], b[TN];
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][64 + tx * 4]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w; a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (more) {
            store_tiles<TA, TB>(As[buf ^ 1], Bs[buf ^ 1], ra, rb);
            __syncthreads();
            buf ^= 1;
        }
    }

    float *dst = work ? work + (size_t)blockIdx.z * M * N : C;
    const int ld = work ? N : ldc;
#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (n >= N) continue;
            float *p = dst + (size_t)m * ld + n;
            if (work) *p = acc[i][j];
            else *p = beta == 0.f ? alpha * acc[i][j] : fmaf(alpha, acc[i][j], beta * *p);
        }
    }
}

__global__ void k_splitk_reduce(int M, int N, int splits, float alpha, const float *__restrict__ work, float beta,
                                float *__restrict__ C, int ldc)
{
    const size_t MN = (size_t)M * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < MN; i += (size_t)gridDim.x * blockDim.x) {
        float s = 0.f;
        for (int z = 0; z < splits; z++) s += work[z * MN + i];
        const size_t m = i / N, n = i % N;
        float *p = C + m * ldc + n;
        *p = beta == 0.f ? alpha * s : fmaf(alpha, s, beta * *p);
    }
}

SgemmPlan sgemm_plan(int M, int N, int K, int num_sms, size_t max_work_floats)
{
    SgemmPlan p;
    p.tiles_m = cdiv(M, BM);
    p.tiles_n = cdiv(N, BN);
    // the tensor-core kernel (products of 2^24 multiply-adds and more) has
    // 128 x sgemm_tc_tile_m(M) output tiles: the K split is sized for those
    const bool tc = (double)M * N * K >= 16.0 * 1024 * 1024;
    const int tiles = tc ? cdiv(M, sgemm_tc_tile_m(M)) * cdiv(N, 128) : p.tiles_m * p.tiles_n;
    p.splits = 1;
    if (K <= 0) { p.k_per_split = BK; return p; }
    // split K when the output tiles cannot fill the SMs and K is long enough
    // to give every split a few k-slabs of its own
    if (tiles < num_sms && K >= 512) {
        int s = std::min(cdiv(num_sms * 2, tiles), K / 256);
        s = std::max(1, std::min(s, 32));
        // the workspace cap limits the split (down to none), it never refuses the product
        const size_t fit = max_work_floats / std::max<size_t>(1, (size_t)M * N);
        if ((size_t)s > fit) s = fit >= 2 ? (int)fit : 1;
        p.splits = s;
    } else if (tiles < 16 && K >= 128) {
        // a handful of tiles (a classifier layer): 64-deep splits, so one
        // CTA does not walk K alone (when the workspace fits the cap)
        const int s = std::max(1, std::min(cdiv(num_sms, tiles), K / 64));
        if ((size_t)s * M * N <= max_work_floats) p.splits = s;
    }
    // whole 32-deep slices, the tensor-core kernel's unit (a multiple of BK)
    p.k_per_split = (int)round_up((size_t)cdiv(K, p.splits), 32);
    p.splits = cdiv(K, p.k_per_split);
    p.work_floats = p.splits > 1 ? (size_t)p.splits * M * N : 0;
    // Tensor-core tiles beyond the last full wave: when they would occupy at
    // most half of the SMs, split each into 2-4 K pieces so the last wave is
    // as wide as the others and proportionally shorter.
    if (tc && p.splits == 1 && tiles > num_sms) {
        const int tail = tiles % num_sms;
        const int s = std::min({4, tail > 0 ? num_sms / tail : 0, K / 512});
        const int bm = sgemm_tc_tile_m(M);
        const size_t wf = (size_t)tail * s * 128 * bm;
        if (tail > 0 && 2 * tail <= num_sms && s >= 2 && wf <= max_work_floats) {
            p.tail_tiles = tail;
            p.tail_kps = (int)round_up((size_t)cdiv(K, s), 32);
            p.tail_split = cdiv(K, p.tail_kps);
            p.work_floats = (size_t)tail * p.tail_split * 128 * bm;
        }
    }
    return p;
}

template <bool TA, bool TB>
static cudaError_t launch_t(const SgemmPlan &p, bool vec, int M, int N, int K, float alpha, const float *A, int lda,
                            const float *B, int ldb, float beta, float *C, int ldc, float *work, cudaStream_t st)
{
    dim3 grid(p.tiles_n, p.tiles_m, p.splits);
    float *wk = p.splits > 1 ? work : nullptr;
    if (vec) k_sgemm<TA, TB, true><<<grid, NT, 0, st>>>(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, p.k_per_split, wk);
    else k_sgemm<TA, TB, false><<<grid, NT, 0, st>>>(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, p.k_per_split, wk);
    cudaError_t e = cudaGetLastError();
    if (e || p.splits == 1) return e;
    return launch_splitk_reduce(M, N, p.splits, alpha, work, beta, C, ldc, st);
}

cudaError_t launch_splitk_reduce(int M, int N, int splits, float alpha, const float *work, float beta, float *C,
                                 int ldc, cudaStream_t st)
{
    const size_t MN = (size_t)M * N;
    int rg = (int)std::min<size_t>((MN + 255) / 256, 148 * 8);
    k_splitk_reduce<<<rg, 256, 0, st>>>(M, N, splits, alpha, work, beta, C, ldc);
    return cudaGetLastError();
}

cudaError_t launch_sgemm(const SgemmPlan &p, bool ta, bool tb, int M, int N, int K, float alpha, const float *A, int lda,
                         const float *B, int ldb, float beta, float *C, int ldc, float *work, int *err,
                         cudaStream_t st)
{
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (K <= 0) {   // C = beta*C
        return launch_t<false, false>(p, false, M, N, 0, alpha, A, lda, B, ldb, beta, C, ldc, work, st);
    }
    if (sgemm_tc_usable(ta, tb, M, N, K, A, lda, B, ldb))
        return launch_sgemm_tc(p, ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, work, err, st);
    const bool aligned = ((uintptr_t)A % 16 == 0) && ((uintptr_t)B % 16 == 0) && lda % 4 == 0 && ldb % 4 == 0;
    // the vector path needs the contiguous extent of each loaded row to be a multiple of 4
    const bool vec = aligned && (ta ? M % 4 == 0 : K % 4 == 0) && (tb ? K % 4 == 0 : N % 4 == 0);
    if (!ta && !tb) return launch_t<false, false>(p, vec, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, work, st);
    if (!ta && tb) return launch_t<false, true>(p, vec, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, work, st);
    if (ta && !tb) return launch_t<true, false>(p, vec, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, work, st);
    return launch_t<true, true>(p, vec, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, work, st);
}

} // namespace cats
