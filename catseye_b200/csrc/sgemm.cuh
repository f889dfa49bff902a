// sgemm.cuh — fp32 GEMM launcher (catseye.h gemm_rnn / gemm_rnt / gemm_rtn).
#pragma once
#include "common.cuh"

namespace cats {

struct SgemmPlan {
    int tiles_m = 0, tiles_n = 0, splits = 1, k_per_split = 0;
    // tensor-core path with splits == 1: the last tail_tiles output tiles (the
    // ones a last partial wave of CTAs would run alone) are computed in
    // tail_split K pieces of tail_kps each, after the full tiles
    int tail_tiles = 0, tail_split = 1, tail_kps = 0;
    size_t work_floats = 0;   // partial-sum workspace (0 when nothing is split)
};

// max_work_floats caps the workspace: the tail split is only planned when it fits.
SgemmPlan sgemm_plan(int M, int N, int K, int num_sms, size_t max_work_floats = (size_t)-1);

// C[M][N] (leading dim ldc) = alpha * op(A) * op(B) + beta * C.  `work` must hold
// plan.work_floats floats when plan.splits > 1.  Shapes the tensor cores can
// take (sgemm_tc_usable) run as 3xTF32 on tcgen05 (sgemm_tc.cu), the rest on
// the CUDA cores.  `err` (may be null) receives CATS_DEVERR_* bits when a
// tensor-core wait times out; the tiles of such a CTA are written as NaN.
cudaError_t launch_sgemm(const SgemmPlan &p, bool ta, bool tb, int M, int N, int K, float alpha, const float *A,
                         int lda, const float *B, int ldb, float beta, float *C, int ldc, float *work, int *err,
                         cudaStream_t st);

// C = alpha * sum of the plan's K-split partial slabs + beta * C
cudaError_t launch_splitk_reduce(int M, int N, int splits, float alpha, const float *work, float beta, float *C,
                                 int ldc, cudaStream_t st);

// tensor-core (3xTF32) path
bool sgemm_tc_usable(bool ta, bool tb, int M, int N, int K, const float *A, int lda, const float *B, int ldb);
size_t sgemm_tc_smem_bytes();
int sgemm_tc_tile_m(int M);   // m rows per tensor-core CTA: 256, or 128 when M <= 128
cudaError_t launch_sgemm_tc(const SgemmPlan &p, bool ta, bool tb, int M, int N, int K, float alpha, const float *A,
                            int lda, const float *B, int ldb, float beta, float *C, int ldc, float *work, int *err,
                            cudaStream_t st);

} // namespace cats
