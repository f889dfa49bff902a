// matvec.cuh — device weight layout and the batch-1 matvec launcher.
//
// The reference's matmul(xout, x, w, n, d) (llm/catseye_llm.h:1519-1533)
// computes xout[i] = sum_j W[i][j] x[j] for a row-major [d][n] weight.  Here a
// weight is re-laid out once, at upload, into "tile chunks": rows are grouped
// into tiles of R rows; each row is cut into segments of 32 units (a unit is a
// 32-element quant block, or 4 floats for F32); the bytes of one (tile,
// segment) pair are contiguous, so one bulk copy (TMA engine) stages it:
//
//   chunk(t,s) = [R rows][units_s x unit payload]  [R rows][scales, 16-B padded]
//
// Q4_0 unit payload: the block's 16 nibble bytes (low nibbles = elements 0-15,
// high = 16-31, as in dequantize_q4_0, llm/catseye_llm.h:427-474).  Q8_0: its
// 32 int8, stored as two 16-byte half planes so lanes read conflict-free.  The
// fp16 block scales follow the payload.  F32: 16 bytes of the row, no scales.
#pragma once
#include "common.cuh"

namespace cats {

constexpr int MV_CONSUMER_WARPS = 8;
constexpr int MV_THREADS = 32 * (MV_CONSUMER_WARPS + 1);   // + one producer warp
constexpr int MV_SEG_UNITS = 64;                            // units per segment (two per lane)
constexpr size_t MV_STAGE_BUDGET = 96 * 1024;               // ring bytes of the standalone matvec

struct WeightLayout {
    int type = 0;        // W_F32 / W_Q4_0 / W_Q8_0
    int n = 0, d = 0;    // input length, rows
    int rpw = 1;         // rows per consumer warp (1 or 2)
    int R = 8;           // rows per tile = 8 * rpw
    int units = 0;       // units per row
    int nseg = 0;        // segments per row
    int n_tiles = 0;
    uint32_t unit_bytes = 0;   // payload bytes per unit
    uint32_t full_chunk = 0;   // bytes of a chunk with a full segment
    uint32_t last_chunk = 0;   // bytes of the chunk of the last segment
    size_t tile_bytes = 0;
    size_t total_bytes = 0;
};

// host-side layout computation (also used by tests through the C API)
WeightLayout make_layout(int type, int n, int d, int rpw);

// source row bytes in the reference's GGUF layout
size_t gguf_row_bytes(int type, int n);

// Activation staging modes
enum XMode : int {
    XM_Q8_RAW = 0,       // x is n/32 reference Q8 blocks {int8 q[32]; float d} (36 B)
    XM_Q8_FROM_F32 = 1,  // x is fp32: optional rmsnorm, then quantize_q8 (AVX rounding) in smem
    XM_F32 = 2,          // x is fp32: optional rmsnorm, staged as fp32 (F32 weights, or quantized
                         // weights dequantized in registers: the matmul_q4_0 binding)
};

// Epilogues
enum Epi : int {
    EPI_STORE = 0,       // out[row] = v
    EPI_ADD = 1,         // out[row] += v            (residual, rows owned by one warp)
    EPI_QKV_ROPE = 2,    // fused [wq;wk;wv] rows -> q, key/value cache at pos, RoPE applied
    EPI_SWIGLU = 3,      // interleaved [w1_i; w3_i] rows -> out[i] = silu(w1 x) * (w3 x)
    EPI_STORE_ARGMAX = 4 // out[row] = v, and the greedy argmax key
};

struct MatvecArgs {
    const uint8_t *w = nullptr;   // repacked weight (WeightLayout)
    int n = 0, d = 0;
    int R = 8, units = 0, nseg = 0, n_tiles = 0;
    uint32_t unit_bytes = 0, full_chunk = 0, last_chunk = 0;
    unsigned long long tile_bytes = 0;
    int stages = 4;

    // activation
    int xmode = XM_Q8_RAW;
    const void *x = nullptr;          // device pointer (fp32 or Q8 blocks)
    const int *x_row = nullptr;       // if set: x += (*x_row) * n floats (embedding lookup)
    const float *norm_w = nullptr;    // if set: rmsnorm with this weight before staging
    float *x_writeback = nullptr;     // if set: CTA 0 stores the (pre-norm) source vector here

    // epilogue
    int epi = EPI_STORE;
    float *out = nullptr;             // STORE/ADD/SWIGLU/ARGMAX target; QKV: q
    float *k_out = nullptr, *v_out = nullptr;  // QKV: cache rows at pos 0 of this layer
    const int *pos = nullptr;         // QKV: device position
    int q_dim = 0, kv_dim = 0, head_size = 0;
    int kv_rows = 0;                  // QKV: rows of the cache (seq_len); pos >= kv_rows is refused
    unsigned long long *argmax = nullptr;
    int argmax_base = 0;              // ARGMAX: index of row 0 (a tensor-parallel rank's vocabulary offset)

    int *err = nullptr;               // device error word
};

// Launch one matvec (PDL attribute set when `pdl`).  Returns a cudaError_t.
cudaError_t launch_matvec(const MatvecArgs &a, int rpw, int type, cudaStream_t st, bool pdl, int grid_override = 0);

// Repack a weight from the reference's GGUF row layout (device memory) into the tile layout.
cudaError_t launch_repack(const uint8_t *src_gguf, uint8_t *dst, const WeightLayout &L, cudaStream_t st);

// Standalone Q8 activation quantizer, bit-exact with the AVX quantize_q8
// (llm/catseye_llm.h:155-225) or, with scalar_mode, the plain-C one (:227-251).
cudaError_t launch_quantize_q8(int8_t *q, const float *x, int n, int scalar_mode, cudaStream_t st);

// Dequantize `rows` rows of a reference-layout weight into fp32.
cudaError_t launch_dequantize(int type, float *y, const uint8_t *w, int n, int rows, cudaStream_t st);

int matvec_num_sms();
size_t matvec_smem_bytes(const MatvecArgs &a, int type);

} // namespace cats
