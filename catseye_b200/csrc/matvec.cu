// matvec.cu — HBM-streaming batch-1 matvec for F32, Q4_0 and Q8_0 weights.
//
// Reference: matmul_f32 / matmul_q4_0_q8 (llm/catseye_llm.h:1519-1533, dots at
// :1449-1465 and :844-879) and the Q8_0 block scheme the runtime enumerates
// (:2566).  One persistent CTA per SM: a producer warp streams (tile, segment)
// chunks of the repacked weight into a ring of shared-memory stages with 1-D
// bulk copies (TMA engine, L2 evict-first); eight consumer warps dot them
// against the activation staged once per CTA in shared memory.  Quantized dots
// are integer (dp4a) per 32-block, scaled by the float product d_w*d_x exactly
// as the reference does.  The producer issues its first copies before the
// programmatic-dependent-launch wait, so weight streaming overlaps the tail of
// the kernel before it.
#include "mv_device.cuh"
#include <algorithm>

namespace cats {

size_t gguf_row_bytes(int type, int n)
{
    switch (type) {
    case W_F32: return (size_t)n * 4;
    case W_Q4_0: return (size_t)(n / 32) * 18;
    case W_Q8_0: return (size_t)(n / 32) * 34;
    case W_Q3_K: return (size_t)(n / 256) * 110;
    case W_Q6_K: return (size_t)(n / 256) * 210;
    }
    return 0;
}

static uint32_t chunk_bytes(int type, int R, int units_s, uint32_t ub)
{
    size_t pay = (size_t)units_s * ub;
    size_t sc = type == W_F32 ? 0 : round_up((size_t)units_s * 2, 16);
    return (uint32_t)(R * (pay + sc));
}

WeightLayout make_layout(int type, int n, int d, int rpw)
{
    WeightLayout L;
    L.type = type;
    L.n = n;
    L.d = d;
    L.rpw = rpw;
    L.R = MV_CONSUMER_WARPS * rpw;
    if (type == W_F32) { L.units = n / 4; L.unit_bytes = 16; }
    else if (type == W_Q4_0) { L.units = n / 32; L.unit_bytes = 16; }
    else { L.units = n / 32; L.unit_bytes = 32; }
    L.nseg = cdiv(L.units, MV_SEG_UNITS);
    L.full_chunk = chunk_bytes(type, L.R, std::min(MV_SEG_UNITS, L.units), L.unit_bytes);
    L.last_chunk = chunk_bytes(type, L.R, L.units - MV_SEG_UNITS * (L.nseg - 1), L.unit_bytes);
    L.tile_bytes = (size_t)(L.nseg - 1) * L.full_chunk + L.last_chunk;
    L.n_tiles = cdiv(d, L.R);
    L.total_bytes = L.tile_bytes * L.n_tiles;
    return L;
}

// ------------------------------------------------------------------ repack
__global__ void k_repack(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, WeightLayout L)
{
    const long long total = (long long)L.d * L.units;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / L.units), u = (int)(i % L.units);
        const int t = row / L.R, rr = row % L.R, s = u / MV_SEG_UNITS, j = u % MV_SEG_UNITS;
        const int us = min(MV_SEG_UNITS, L.units - MV_SEG_UNITS * s);
        uint8_t *base = dst + (size_t)t * L.tile_bytes + (size_t)s * L.full_chunk;
        const size_t sstride = round_up((size_t)us * 2, 16);
        if (L.type == W_F32) {
            const uint8_t *p = src + (size_t)row * L.n * 4 + (size_t)u * 16;
            uint8_t *q = base + ((size_t)rr * us + j) * 16;
            for (int k = 0; k < 16; k++) q[k] = p[k];
        } else if (L.type == W_Q4_0) {
            const uint8_t *p = src + (size_t)row * L.units * 18 + (size_t)u * 18;
            uint8_t *q = base + ((size_t)rr * us + j) * 16;
            for (int k = 0; k < 16; k++) q[k] = p[2 + k];
            uint8_t *sc = base + (size_t)L.R * us * 16 + rr * sstride + j * 2;
            sc[0] = p[0];
            sc[1] = p[1];
        } else {
            const uint8_t *p = src + (size_t)row * L.units * 34 + (size_t)u * 34;
            uint8_t *lo = base + ((size_t)(rr * 2) * us + j) * 16;
            uint8_t *hi = base + ((size_t)(rr * 2 + 1) * us + j) * 16;
            for (int k = 0; k < 16; k++) { lo[k] = p[2 + k]; hi[k] = p[18 + k]; }
            uint8_t *sc = base + (size_t)L.R * us * 32 + rr * sstride + j * 2;
            sc[0] = p[0];
            sc[1] = p[1];
        }
    }
}

cudaError_t launch_repack(const uint8_t *src, uint8_t *dst, const WeightLayout &L, cudaStream_t st)
{
    cudaError_t e = cudaMemsetAsync(dst, 0, L.total_bytes, st);   // padded rows and scale pads = 0
    if (e != cudaSuccess) return e;
    long long total = (long long)L.d * L.units;
    int grid = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
    k_repack<<<grid, 256, 0, st>>>(src, dst, L);
    return cudaGetLastError();
}

// ------------------------------------------------- Q8 quantizer (standalone)
__global__ void k_quantize_q8(int8_t *__restrict__ q, const float *__restrict__ x, int n, int scalar_mode)
{
    const int n4 = n / 4;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;   // float4 index; n4 % 8 == 0
    const int lane = threadIdx.x & 31;
    const unsigned gmask = 0xffu << (lane & 24);
    if (i >= n4) return;                                   // whole 8-lane groups leave together
    float4 v = reinterpret_cast<const float4 *>(x)[i];
    float d;
    int s;
    uint32_t packed = q8_group_quant(v, gmask, scalar_mode != 0, d, s);
    const int b = i >> 3, g = i & 7;
    uint8_t *blk = reinterpret_cast<uint8_t *>(q) + (size_t)b * 36;
    *reinterpret_cast<uint32_t *>(blk + g * 4) = packed;
    if (g == 0) *reinterpret_cast<float *>(blk + 32) = d;
}

cudaError_t launch_quantize_q8(int8_t *q, const float *x, int n, int scalar_mode, cudaStream_t st)
{
    int n4 = n / 4;
    k_quantize_q8<<<cdiv(n4, 256), 256, 0, st>>>(q, x, n, scalar_mode);
    return cudaGetLastError();
}

// ------------------------------------------------------------- dequantize
// dequantize_q4_0 (llm/catseye_llm.h:427-474) and the Q8_0 value q*d; one
// thread per block.  Products of a small integer and an fp16-exact scale are
// exact in fp32, so the result is bit-identical to the reference.
__global__ void k_dequantize(int type, float *__restrict__ y, const uint8_t *__restrict__ w, long long nblocks)
{
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nblocks;
         b += (long long)gridDim.x * blockDim.x) {
        float *o = y + b * 32;
        if (type == W_Q4_0) {
            const uint8_t *p = w + b * 18;
            const float dd = half_bits_to_float((uint16_t)(p[0] | (p[1] << 8)));
            for (int j = 0; j < 16; j++) {
                o[j] = (float)((p[2 + j] & 0x0f) - 8) * dd;
                o[j + 16] = (float)((p[2 + j] >> 4) - 8) * dd;
            }
        } else if (type == W_Q8_0) {
            const uint8_t *p = w + b * 34;
            const float dd = half_bits_to_float((uint16_t)(p[0] | (p[1] << 8)));
            for (int j = 0; j < 32; j++) o[j] = (float)(int8_t)p[2 + j] * dd;
        } else {
            const float *p = reinterpret_cast<const float *>(w) + b * 32;
            for (int j = 0; j < 32; j++) o[j] = p[j];
        }
    }
}

cudaError_t launch_dequantize(int type, float *y, const uint8_t *w, int n, int rows, cudaStream_t st)
{
    long long nb = (long long)rows * (n / 32);
    int grid = (int)std::min<long long>((nb + 127) / 128, 148LL * 8);
    if (grid < 1) grid = 1;
    k_dequantize<<<grid, 128, 0, st>>>(type, y, w, nb);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ matvec
// Shared memory: a 384-byte header at offset 0 (8 full + 8 empty mbarriers,
// then the reduction scratch), the ring of stages, the staged activation.
struct SmemPlan {
    uint32_t stage_stride, ring_off, xs_off, xs_bytes, bar_off, red_off, total;
};

__host__ __device__ inline SmemPlan smem_plan(const MatvecArgs &a, int type)
{
    SmemPlan p;
    p.bar_off = 0;
    p.red_off = 16 * 8;
    p.ring_off = 384;
    p.stage_stride = (uint32_t)round_up(a.full_chunk, 128);
    p.xs_off = p.ring_off + p.stage_stride * a.stages;
    if (type == W_F32 || a.xmode == XM_F32) p.xs_bytes = (uint32_t)round_up((size_t)a.n * 4, 128);
    else p.xs_bytes = (uint32_t)round_up((size_t)a.units * 40, 128);   // lo16 + hi16 + (d, sum)
    p.total = p.xs_off + p.xs_bytes;
    return p;
}

size_t matvec_smem_bytes(const MatvecArgs &a, int type) { return smem_plan(a, type).total; }

// Producer (one thread): weights only, so it does not wait for the upstream
// grid.  Returns after every issued copy has landed and been released.
__device__ __forceinline__ void mv_produce(const MatvecArgs &a, const SmemPlan &sp, uint8_t *smem, uint64_t *full,
                                           uint64_t *empty)
{
    const int stages = a.stages;
    uint8_t *ring = smem + sp.ring_off;
    const uint64_t pol = l2_evict_first_policy();
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x) {
        const uint8_t *tb = a.w + (size_t)t * a.tile_bytes;
        for (int s = 0; s < a.nseg; s++) {
            if (!mbar_wait_bounded(&empty[stage], phase ^ 1, a.err, CATS_DEVERR_MBAR_EMPTY)) {
                ok = false;
                break;
            }
            const uint32_t bytes = (s == a.nseg - 1) ? a.last_chunk : a.full_chunk;
            mbar_arrive_expect_tx(&full[stage], bytes);
            bulk_g2s(ring + (size_t)stage * sp.stage_stride, tb + (size_t)s * a.full_chunk, bytes, &full[stage], pol);
            if (++stage == stages) { stage = 0; phase ^= 1; }
        }
    }
    // drain: every issued copy must have landed and been released before the CTA exits
    for (int k = 0; k < stages; k++) {
        if (!mbar_wait_bounded(&empty[stage], phase ^ 1, a.err, CATS_DEVERR_MBAR_EMPTY)) {
            mbar_wait_bounded(&full[stage], phase, nullptr, 0);
        }
        if (++stage == stages) { stage = 0; phase ^= 1; }
    }
}

// Consumer warps: stage the activation, dot every chunk of this CTA's tiles,
// run the epilogue.
template <int WT, int RPW, bool XF>
__device__ __forceinline__ void mv_consume(const MatvecArgs &a, const SmemPlan &sp, uint8_t *smem, uint64_t *full,
                                           uint64_t *empty, float *red)
{
    constexpr int R = MV_CONSUMER_WARPS * RPW;
    const int stages = a.stages;
    uint8_t *xs = smem + sp.xs_off;
    uint8_t *ring = smem + sp.ring_off;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    constexpr int NC = 32 * MV_CONSUMER_WARPS;
    if (a.xmode == XM_Q8_RAW) {
        stage_q8_raw(static_cast<const uint8_t *>(a.x), a.n, xs, threadIdx.x, NC);
    } else {
        const float *src = static_cast<const float *>(a.x) + (a.x_row ? (size_t)(*a.x_row) * a.n : 0);
        stage_act<XF ? (int)W_F32 : WT>(Float4Src{reinterpret_cast<const float4 *>(src), false}, a.n, a.norm_w,
                                        blockIdx.x == 0 ? a.x_writeback : nullptr, xs, red, threadIdx.x, NC);
    }
    pdl_launch_dependents();

    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    unsigned long long best = 0ull;
    const int pos = (a.epi == EPI_QKV_ROPE) ? *a.pos : 0;
    const bool pos_ok = a.epi != EPI_QKV_ROPE || (pos >= 0 && pos < a.kv_rows);
    if (!pos_ok && threadIdx.x == 0 && blockIdx.x == 0 && a.err) atomicOr(a.err, CATS_DEVERR_POS_RANGE);
    for (int t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x) {
        float acc[RPW];
#pragma unroll
        for (int r = 0; r < RPW; r++) acc[r] = 0.f;
        for (int s = 0; s < a.nseg; s++) {
            if (!mbar_wait_bounded(&full[stage], phase, a.err, CATS_DEVERR_MBAR_FULL)) { ok = false; break; }
            const int us = min(MV_SEG_UNITS, a.units - MV_SEG_UNITS * s);
            consume_chunk<WT, RPW, XF>(ring + (size_t)stage * sp.stage_stride, us, s, warp, lane, a.units, xs, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (++stage == stages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
#pragma unroll
        for (int r = 0; r < RPW; r++) acc[r] = warp_sum(acc[r]);
        if (lane == 0) {
            const int row0 = t * R + warp * RPW;
            if (a.epi == EPI_QKV_ROPE || a.epi == EPI_SWIGLU) {
                if (RPW == 2 && row0 < a.d) {
                    float v0 = acc[0], v1 = acc[RPW - 1];
                    if (a.epi == EPI_SWIGLU) {
                        const float sg = v0 * (1.f / (1.f + expf(-v0)));
                        a.out[row0 >> 1] = sg * v1;
                    } else if (row0 < a.q_dim) {
                        rope_pair(v0, v1, row0, a.head_size, pos);
                        a.out[row0] = v0;
                        a.out[row0 + 1] = v1;
                    } else if (!pos_ok) {
                        // out-of-range position: nothing is written into the cache
                    } else if (row0 < a.q_dim + a.kv_dim) {
                        const int i = row0 - a.q_dim;
                        rope_pair(v0, v1, i, a.head_size, pos);
                        a.k_out[(size_t)pos * a.kv_dim + i] = v0;
                        a.k_out[(size_t)pos * a.kv_dim + i + 1] = v1;
                    } else {
                        const int i = row0 - a.q_dim - a.kv_dim;
                        a.v_out[(size_t)pos * a.kv_dim + i] = v0;
                        a.v_out[(size_t)pos * a.kv_dim + i + 1] = v1;
                    }
                }
            } else {
#pragma unroll
                for (int r = 0; r < RPW; r++) {
                    const int row = row0 + r;
                    if (row >= a.d) break;
                    if (a.epi == EPI_ADD) a.out[row] += acc[r];
                    else a.out[row] = acc[r];
                    if (a.epi == EPI_STORE_ARGMAX) {
                        const unsigned long long k = argmax_key(acc[r], a.argmax_base + row);
                        best = k > best ? k : best;
                    }
                }
            }
        }
    }
    if (a.epi == EPI_STORE_ARGMAX) {
        unsigned long long *keys = reinterpret_cast<unsigned long long *>(red + 16);
        if (lane == 0) keys[warp] = best;
        named_bar_sync(1, 32 * MV_CONSUMER_WARPS);
        if (threadIdx.x == 0) {
            unsigned long long m = 0;
            for (int w = 0; w < MV_CONSUMER_WARPS; w++) m = keys[w] > m ? keys[w] : m;
            if (m) atomicMax(a.argmax, m);
        }
    }
}

template <int WT, int RPW, bool XF>
__global__ void __launch_bounds__(MV_THREADS, 1) k_matvec(const __grid_constant__ MatvecArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const SmemPlan sp = smem_plan(a, WT);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + sp.bar_off);
    uint64_t *empty = full + 8;
    float *red = reinterpret_cast<float *>(smem + sp.red_off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MV_CONSUMER_WARPS);
        }
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    __syncthreads();
    if (warp == MV_CONSUMER_WARPS) {
        if (lane == 0) mv_produce(a, sp, smem, full, empty);
    } else {
        mv_consume<WT, RPW, XF>(a, sp, smem, full, empty, red);
    }
    // No thread returns early: once all copies have landed and every arrive
    // is done, retire the mbarriers so the next kernel on this SM may use
    // these bytes for ordinary data.
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.stages; s++) {
            mbar_inval(&full[s]);
            mbar_inval(&empty[s]);
        }
    }
}

int matvec_num_sms()
{
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

template <int WT, int RPW, bool XF>
static cudaError_t launch_t(const MatvecArgs &a, cudaStream_t st, bool pdl, int grid_override)
{
    const size_t smem = matvec_smem_bytes(a, WT);
    static unsigned long long attr_set = 0;   // one bit per device
    cudaError_t ea = once_per_device(attr_set, [] {
        return cudaFuncSetAttribute(k_matvec<WT, RPW, XF>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    });
    if (ea != cudaSuccess) return ea;
    int grid = grid_override > 0 ? grid_override : std::min(a.n_tiles, matvec_num_sms());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(MV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_matvec<WT, RPW, XF>, a);
}

template <int WT, bool XF>
static cudaError_t launch_rpw(const MatvecArgs &a, int rpw, cudaStream_t st, bool pdl, int grid_override)
{
    return rpw == 2 ? launch_t<WT, 2, XF>(a, st, pdl, grid_override) : launch_t<WT, 1, XF>(a, st, pdl, grid_override);
}

cudaError_t launch_matvec(const MatvecArgs &a, int rpw, int type, cudaStream_t st, bool pdl, int grid_override)
{
    if (a.stages < 2 || a.stages > 8) return cudaErrorInvalidValue;
    if (matvec_smem_bytes(a, type) > 227 * 1024) return cudaErrorInvalidValue;
    // fp32 activations with quantized weights: the matmul_q4_0 binding (dequantize, fp32 dot)
    const bool xf = type != W_F32 && a.xmode == XM_F32;
    switch (type) {
    case W_F32: return launch_rpw<W_F32, false>(a, rpw, st, pdl, grid_override);
    case W_Q4_0: return xf ? launch_rpw<W_Q4_0, true>(a, rpw, st, pdl, grid_override)
                           : launch_rpw<W_Q4_0, false>(a, rpw, st, pdl, grid_override);
    case W_Q8_0: return xf ? launch_rpw<W_Q8_0, true>(a, rpw, st, pdl, grid_override)
                           : launch_rpw<W_Q8_0, false>(a, rpw, st, pdl, grid_override);
    }
    return cudaErrorInvalidValue;
}

} // namespace cats
