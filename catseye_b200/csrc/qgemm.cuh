// qgemm.cuh — batched quantized-weight product on the tensor cores (tcgen05).
#pragma once
#include "matvec.cuh"
#include <cuda_fp16.h>

namespace cats {

// Weights qgemm handles: Q4_0 / Q8_0 in the tile layout, n a multiple of 64.
bool qgemm_supported(const WeightLayout &L);

// Token rows the fp16 operand holds for T tokens (T rounded up to the CTA's
// token tile), and the bytes of that operand for n columns.
int qgemm_tpad(int T);
size_t qgemm_x16_bytes(int n, int T);

// The fp16 operand ("x16"): K-slice-major [n/64][Tpad][64] with token t's
// eight 16-byte chunks of a slice stored at chunk c ^ (t & 7) (the 128-byte
// swizzle the tensor cores read, so one bulk copy brings a stage in).
// Chunk c holds, of the slice's 32-element block b = c >> 2 and i = c & 3,
// the elements 4i, 4i+2, 4i+1, 4i+3, 4i+16, 4i+18, 4i+17, 4i+19: the order
// in which the dequantization extracts a block's codes (the nibbles of
// bytes 4i..4i+3 of a Q4_0 block), so weights and activations share one
// permutation of K and the sums are unchanged.  Rows t >= T are never
// stored from: their contents only reach output columns that are not written.
__host__ __device__ inline size_t x16_chunk(int kb, int c, int t, int Tpad)
{
    return (((size_t)kb * Tpad + t) * 8 + (size_t)(c ^ (t & 7))) * 8;   // in halves
}

#ifdef __CUDACC__
// Pack chunk c's eight elements, given a = elements 4i..4i+3 and b =
// elements 4i+16..4i+19 of its block (i = c & 3), as the x16 order places them.
__device__ __forceinline__ uint4 x16_pack(float4 a, float4 b)
{
    auto h2 = [](float lo, float hi) {
        return (uint32_t)__half_as_ushort(__float2half_rn(lo)) | ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
    };
    return make_uint4(h2(a.x, a.z), h2(a.y, a.w), h2(b.x, b.z), h2(b.y, b.w));
}

// Offset (elements) of chunk c's two source runs within its 64-wide slice.
__host__ __device__ inline int x16_src_off(int c) { return (c >> 2) * 32 + (c & 3) * 4; }
#endif

// x[T][n] fp32 (16-byte aligned rows) -> x16.
cudaError_t launch_x16(const float *x, __half *x16, int T, int n, cudaStream_t st);

// Bytes of the K-split workspace a product of L at T tokens uses (0 when it
// runs as one pass over K).  Deterministic in (L, T) on a given GPU.
size_t qgemm_workspace_bytes(const WeightLayout &L, int T);

// Y[T][d] (=, or += when accumulate) X[T][n] * W[d][n]^T with fp16 operands
// and fp32 accumulation, X given as x16.  ws (ws_bytes) holds the K-split
// partials; with less room than qgemm_workspace_bytes the product runs as
// one pass over K.
// With `defer` set, a product split over K leaves its partials in ws
// ([splits][T][d]) for the caller's next kernel to add (in split order, as
// the sum kernel would, then onto y when accumulating) instead of launching
// the sum: *defer = {ws, splits}; splits == 1 means y holds the result.
struct SplitOut {
    const float *ws = nullptr;
    int splits = 1;
};

// Per-K-slice timeline of CTA (0, 0, 0) of the tensor-map-fed kernel (a
// tuning diagnostic).  buf holds (slices + 1) rows of QG_TRACE_FIELDS SM
// clock64 stamps; row k < slices is the CTA's k-th K slice:
//   0 the raw group copy issued (a group's first slice), 1 the activation
//   rows' copy issued (narrow tiles), 2 producer warp 0 saw the raw group
//   land, 3 producer warp 0 found the fp16 stage free, 4..11 producer warp
//   0..7 arrived on the stage's full barrier, 12 the MMA thread found the
//   operands ready, 13 it issued the slice's commit;
// row `slices`: 0 the CTA's start, 1 producer warp 0 saw the last MMA
// complete, 2 producer warp 0 finished its epilogue.
constexpr int QG_TRACE_FIELDS = 16;
struct QgemmTrace {
    unsigned long long *buf = nullptr;   // device
    int slices = 0;
};

cudaError_t launch_qgemm_x16(const WeightLayout &L, const uint8_t *w, const __half *x16, float *y, int T,
                             bool accumulate, float *ws, size_t ws_bytes, int *err, cudaStream_t st,
                             SplitOut *defer = nullptr, const QgemmTrace *trace = nullptr);

// The same from fp32 x (converted into the x16 scratch, qgemm_x16_bytes, first).
cudaError_t launch_qgemm(const WeightLayout &L, const uint8_t *w, const float *x, __half *x16, float *y, int T,
                         float *ws, size_t ws_bytes, int *err, cudaStream_t st, const QgemmTrace *trace = nullptr);

// The plan a product of L at T tokens runs with: token tile, K splits (before
// any cap by the workspace), CTAs of the chosen kernel resident per SM,
// whether the weights come through tensor-map copies, K slices per split.
struct QgemmPlan {
    int bn, splits, resident, tma, kper;
    int occupancy, occupancy_err;   // the occupancy query asked afresh, and its CUDA error
};
QgemmPlan qgemm_plan(const WeightLayout &L, int T);

size_t qgemm_smem_bytes(int bn);

} // namespace cats
