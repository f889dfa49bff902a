// sgemm.cuh — fp32 GEMM launcher (catseye.h gemm_rnn / gemm_rnt / gemm_rtn).
#pragma once
#include "common.cuh"

namespace cats {

struct SgemmPlan {
    int tiles_m = 0, tiles_n = 0, splits = 1, k_per_split = 0;
    size_t work_floats = 0;   // split-K partial-sum workspace (0 when splits == 1)
};

SgemmPlan sgemm_plan(int M, int N, int K, int num_sms);

// C[M][N] (leading dim ldc) = alpha * op(A) * op(B) + beta * C.  `work` must hold
// plan.work_floats floats when plan.splits > 1.
cudaError_t launch_sgemm(const SgemmPlan &p, bool ta, bool tb, int M, int N, int K, float alpha, const float *A,
                         int lda, const float *B, int ldb, float beta, float *C, int ldc, float *work,
                         cudaStream_t st);

} // namespace cats
