// capi.cu — the C ABI of libcatsgpu.so (include/catsgpu.h).
//
// Owns the device, one CUDA stream, the weight registry (host pointer of the
// caller's cats_tensor.data -> re-laid-out device copy), grow-only staging
// buffers for the host-pointer drop-ins, and the sticky error status that the
// void drop-in signatures cannot return.
#include "../../include/catsgpu.h"
#include "loader.cuh"
#include "conv.cuh"
#include "kquant.cuh"
#include "llm.cuh"
#include "qgemm.cuh"
#include "sgemm.cuh"
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <mutex>
#include <unordered_map>

using namespace cats;

namespace {

struct Reg {
    int type = 0, n = 0, d = 0;
    DevWeight W;
};

struct Ctx {
    bool init = false;
    int device = 0;
    cudaStream_t stream = nullptr;
    int last_err = 0;
    bool strict = false;
    unsigned printed = 0;
    int *d_err = nullptr;
    std::unordered_map<const void *, Reg> weights;
    void *d_x = nullptr;
    size_t d_x_cap = 0;
    float *d_out = nullptr;
    size_t d_out_cap = 0;
    float *d_a = nullptr, *d_b = nullptr, *d_c = nullptr, *d_work = nullptr;
    size_t cap_a = 0, cap_b = 0, cap_c = 0, cap_work = 0;
    __half *d_x16 = nullptr;   // fp16 activations of the batched product
    size_t cap_x16 = 0;
    float *d_ws = nullptr;     // its K-split partials
    size_t cap_ws = 0;
    // CNN training: the batched column matrix, the channel-major gradients,
    // and a fourth host-copy staging buffer
    float *d_col = nullptr, *d_tr = nullptr, *d_d = nullptr;
    size_t cap_col = 0, cap_tr = 0, cap_d = 0;
};

Ctx g;

const char *err_name(int c)
{
    switch (c) {
    case CATS_OK: return "ok";
    case CATS_ERR_CUDA: return "CUDA runtime error";
    case CATS_ERR_ARG: return "invalid argument";
    case CATS_ERR_NOMEM: return "device out of memory";
    case CATS_ERR_TIMEOUT: return "device wait timed out";
    case CATS_ERR_UNSUPPORTED: return "unsupported shape or type";
    case CATS_ERR_NOT_INIT: return "library not initialised";
    case CATS_ERR_NCCL: return "collective failed";
    }
    return "unknown";
}

int fail(int code, const char *what, cudaError_t ce = cudaSuccess)
{
    g.last_err = code;
    if (g.strict || !(g.printed & (1u << code))) {
        g.printed |= 1u << code;
        fprintf(stderr, "catsgpu: %s: %s%s%s\n", what, err_name(code), ce ? " / " : "", ce ? cudaGetErrorString(ce) : "");
    }
    if (g.strict) abort();
    return code;
}

int check(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return CATS_OK;
    return fail(e == cudaErrorMemoryAllocation ? CATS_ERR_NOMEM : CATS_ERR_CUDA, what, e);
}

bool ensure_init()
{
    if (g.init) return true;
    if (cats_gpu_init(-1) != CATS_OK) return false;
    return true;
}

int grow(void **p, size_t *cap, size_t bytes)
{
    if (*cap >= bytes) return CATS_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    size_t want = round_up(bytes, 1 << 20);
    if (cudaMalloc(p, want) != cudaSuccess) return fail(CATS_ERR_NOMEM, "staging buffer");
    *cap = want;
    return CATS_OK;
}

int check_device_error(const char *what)
{
    int h = 0;
    if (cudaMemcpy(&h, g.d_err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return fail(CATS_ERR_CUDA, what);
    if (h) {
        cudaMemset(g.d_err, 0, 4);
        return fail(CATS_ERR_TIMEOUT, what);
    }
    return CATS_OK;
}

bool type_ok(int t) { return t == CATS_TYPE_F32 || t == CATS_TYPE_Q4_0 || t == CATS_TYPE_Q8_0; }
bool kquant(int t) { return t == CATS_TYPE_Q3_K || t == CATS_TYPE_Q6_K; }

int validate_shape(int type, int n, int d)
{
    if (n <= 0 || d <= 0) return CATS_ERR_ARG;
    if (!type_ok(type) && !kquant(type)) return CATS_ERR_UNSUPPORTED;
    if (type == CATS_TYPE_F32 ? (n % 4) : kquant(type) ? (n % 256) : (n % 32)) return CATS_ERR_ARG;
    return CATS_OK;
}

Reg *lookup(const void *w, int type, int n, int d)
{
    auto it = g.weights.find(w);
    if (it != g.weights.end()) {
        Reg &r = it->second;
        if (r.type == type && r.n == n && r.d == d) return &r;
        cats_gpu_unregister_weight(w);   // same address, new meaning: re-upload
    }
    if (cats_gpu_register_weight(w, type, n, d) != CATS_OK) return nullptr;
    return &g.weights[w];
}

MatvecArgs args_for(const Reg &r)
{
    MatvecArgs a;
    const WeightLayout &L = r.W.L;
    a.w = r.W.ptr;
    a.n = L.n;
    a.d = L.d;
    a.R = L.R;
    a.units = L.units;
    a.nseg = L.nseg;
    a.n_tiles = L.n_tiles;
    a.unit_bytes = L.unit_bytes;
    a.full_chunk = L.full_chunk;
    a.last_chunk = L.last_chunk;
    a.tile_bytes = L.tile_bytes;
    a.stages = std::max(2, std::min(8, (int)(MV_STAGE_BUDGET / round_up(L.full_chunk, 128))));
    a.err = g.d_err;
    return a;
}

// x_f32: fp32 activations against quantized weights (the matmul_q4_0 binding)
void matmul_host(int type, float *xout, void *x, void *w, int n, int d, const char *what, bool x_f32 = false)
{
    if (!ensure_init()) return;
    if (!xout || !x || !w) { fail(CATS_ERR_ARG, what); return; }
    if (int rc = validate_shape(type, n, d)) { fail(rc, what); return; }
    Reg *r = lookup(w, type, n, d);
    if (!r) return;
    const size_t xb = (type == CATS_TYPE_F32 || x_f32) ? (size_t)n * 4
                      : kquant(type)                  ? (size_t)(n / 256) * 260
                                                      : (size_t)(n / 32) * 36;
    if (grow(&g.d_x, &g.d_x_cap, xb) || grow((void **)&g.d_out, &g.d_out_cap, (size_t)d * 4)) return;
    if (check(cudaMemcpyAsync(g.d_x, x, xb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (kquant(type)) {
        if (check(launch_matvec_kquant(type, g.d_out, (const uint8_t *)g.d_x, r->W.ptr, n, d, g.stream), what))
            return;
    } else {
        MatvecArgs a = args_for(*r);
        a.xmode = (type == CATS_TYPE_F32 || x_f32) ? XM_F32 : XM_Q8_RAW;
        a.x = g.d_x;
        a.epi = EPI_STORE;
        a.out = g.d_out;
        if (check(launch_matvec(a, r->W.L.rpw, type, g.stream, false), what)) return;
    }
    if (check(cudaMemcpyAsync(xout, g.d_out, (size_t)d * 4, cudaMemcpyDeviceToHost, g.stream), what)) return;
    if (check(cudaStreamSynchronize(g.stream), what)) return;
    check_device_error(what);
}

} // namespace

namespace cats {
// the sticky status, for entry points defined in other files
int capi_fail(int code, const char *what) { return fail(code, what); }
int noalloc_device_error(bool clear);   // noalloc.cu: the no-allocation sgemm's status word
// the library's stream (after cats_gpu_init), for entry points in other files
cudaStream_t capi_stream() { return g.stream; }
}

// ===================================================================== C ABI
extern "C" {

int cats_gpu_init(int device)
{
    if (g.init) return CATS_OK;
    const char *s = getenv("CATS_GPU_STRICT");
    g.strict = s && atoi(s) == 1;
    if (device < 0) {
        const char *e = getenv("CATS_GPU_DEVICE");
        device = e ? atoi(e) : 0;
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return fail(CATS_ERR_CUDA, "cats_gpu_init: no CUDA device");
    if (device >= n) return fail(CATS_ERR_ARG, "cats_gpu_init: device index");
    if (check(cudaSetDevice(device), "cats_gpu_init")) return g.last_err;
    cudaDeviceProp prop;
    if (check(cudaGetDeviceProperties(&prop, device), "cats_gpu_init")) return g.last_err;
    if (prop.major != 10) return fail(CATS_ERR_UNSUPPORTED, "cats_gpu_init: libcatsgpu needs an sm_100 (B200) device");
    // A blocking stream: the device-pointer entry points called with stream
    // NULL run here, ordered after the caller's work on the legacy default
    // stream (where the caller's inputs were most likely written) and before
    // its later work there.  A non-blocking stream let a product start before
    // the kernels writing its operands had finished.
    if (check(cudaStreamCreateWithFlags(&g.stream, cudaStreamDefault), "cats_gpu_init")) return g.last_err;
    if (check(cudaMalloc(&g.d_err, 4), "cats_gpu_init")) return g.last_err;
    cudaMemset(g.d_err, 0, 4);
    g.device = device;
    g.init = true;
    return CATS_OK;
}

void cats_gpu_term(void)
{
    if (!g.init) return;
    cudaStreamSynchronize(g.stream);
    for (auto &kv : g.weights) if (kv.second.W.ptr) cudaFree(kv.second.W.ptr);
    g.weights.clear();
    void *bufs[] = {g.d_x, g.d_out, g.d_a, g.d_b, g.d_c, g.d_work, g.d_err, g.d_x16, g.d_ws, g.d_col, g.d_tr, g.d_d};
    for (void *b : bufs) if (b) cudaFree(b);
    g.d_x = nullptr; g.d_out = nullptr; g.d_a = g.d_b = g.d_c = g.d_work = nullptr; g.d_err = nullptr;
    g.d_x16 = nullptr;
    g.d_ws = nullptr;
    g.d_col = g.d_tr = g.d_d = nullptr;
    g.d_x_cap = g.d_out_cap = g.cap_a = g.cap_b = g.cap_c = g.cap_work = g.cap_x16 = g.cap_ws = 0;
    g.cap_col = g.cap_tr = g.cap_d = 0;
    cudaStreamDestroy(g.stream);
    g.stream = nullptr;
    g.init = false;
}

int cats_gpu_last_error(void) { return g.last_err; }
void cats_gpu_clear_error(void)
{
    g.last_err = 0;
    cats::noalloc_device_error(true);
}
const char *cats_gpu_error_string(int code) { return err_name(code); }

int cats_gpu_device_error(void)
{
    int h = 0;
    if (g.init) cudaMemcpy(&h, g.d_err, 4, cudaMemcpyDeviceToHost);
    return h | cats::noalloc_device_error(false);
}

int cats_gpu_register_weight(const void *w, int type, int n, int d)
{
    if (!ensure_init()) return g.last_err;
    if (!w) return fail(CATS_ERR_ARG, "cats_gpu_register_weight: null weight");
    if (int rc = validate_shape(type, n, d)) return fail(rc, "cats_gpu_register_weight");
    auto it = g.weights.find(w);
    if (it != g.weights.end()) {
        if (it->second.type == type && it->second.n == n && it->second.d == d) return CATS_OK;
        cats_gpu_unregister_weight(w);
    }
    const size_t bytes = gguf_row_bytes(type, n) * d;
    Reg r;
    r.type = type; r.n = n; r.d = d;
    if (kquant(type)) {
        // K-quant weights keep the reference's row layout on the device
        r.W.L.type = type;
        r.W.L.n = n;
        r.W.L.d = d;
        r.W.L.total_bytes = bytes;
        if (cudaMalloc(&r.W.ptr, bytes) != cudaSuccess) return fail(CATS_ERR_NOMEM, "cats_gpu_register_weight");
        // on the library's stream and waited for: the matvecs read it from that stream
        int rc = check(cudaMemcpyAsync(r.W.ptr, w, bytes, cudaMemcpyHostToDevice, g.stream), "cats_gpu_register_weight");
        if (!rc) rc = check(cudaStreamSynchronize(g.stream), "cats_gpu_register_weight");
        if (rc) { cudaFree(r.W.ptr); return rc; }
        g.weights[w] = r;
        return CATS_OK;
    }
    uint8_t *stg = nullptr;
    if (cudaMalloc(&stg, bytes) != cudaSuccess) return fail(CATS_ERR_NOMEM, "cats_gpu_register_weight");
    // two rows per warp halves the activation reads per weight byte; use it
    // when there are enough 16-row tiles to give every SM two or more
    r.W.L = make_layout(type, n, d, d >= 2 * 16 * matvec_num_sms() ? 2 : 1);
    int rc = CATS_OK;
    if (cudaMalloc(&r.W.ptr, r.W.L.total_bytes) != cudaSuccess) rc = fail(CATS_ERR_NOMEM, "cats_gpu_register_weight");
    if (!rc) rc = check(cudaMemcpyAsync(stg, w, bytes, cudaMemcpyHostToDevice, g.stream), "cats_gpu_register_weight");
    if (!rc) rc = check(launch_repack(stg, r.W.ptr, r.W.L, g.stream), "cats_gpu_register_weight");
    if (!rc) rc = check(cudaStreamSynchronize(g.stream), "cats_gpu_register_weight");
    cudaFree(stg);
    if (rc) { if (r.W.ptr) cudaFree(r.W.ptr); return rc; }
    g.weights[w] = r;
    return CATS_OK;
}

void cats_gpu_unregister_weight(const void *w)
{
    auto it = g.weights.find(w);
    if (it == g.weights.end()) return;
    cudaStreamSynchronize(g.stream);
    if (it->second.W.ptr) cudaFree(it->second.W.ptr);
    g.weights.erase(it);
}

size_t cats_gpu_weight_device_bytes(const void *w)
{
    auto it = g.weights.find(w);
    return it == g.weights.end() ? 0 : it->second.W.L.total_bytes;
}

void cats_gpu_matmul_f32(float *xout, void *x, void *w, int n, int d)
{ matmul_host(CATS_TYPE_F32, xout, x, w, n, d, "cats_gpu_matmul_f32"); }
void cats_gpu_matmul_q4_0_q8(float *xout, void *x, void *w, int n, int d)
{ matmul_host(CATS_TYPE_Q4_0, xout, x, w, n, d, "cats_gpu_matmul_q4_0_q8"); }
void cats_gpu_matmul_q8_0_q8(float *xout, void *x, void *w, int n, int d)
{ matmul_host(CATS_TYPE_Q8_0, xout, x, w, n, d, "cats_gpu_matmul_q8_0_q8"); }

void cats_gpu_matmul_q4_0_f32(float *xout, void *x, void *w, int n, int d)
{ matmul_host(CATS_TYPE_Q4_0, xout, x, w, n, d, "cats_gpu_matmul_q4_0_f32", true); }
void cats_gpu_matmul_q8_0_f32(float *xout, void *x, void *w, int n, int d)
{ matmul_host(CATS_TYPE_Q8_0, xout, x, w, n, d, "cats_gpu_matmul_q8_0_f32", true); }
void cats_gpu_matmul_q3_K_q8_K(float *xout, void *x, void *w, int n, int d)
{ matmul_host(CATS_TYPE_Q3_K, xout, x, w, n, d, "cats_gpu_matmul_q3_K_q8_K"); }
void cats_gpu_matmul_q6_K_q8_K(float *xout, void *x, void *w, int n, int d)
{ matmul_host(CATS_TYPE_Q6_K, xout, x, w, n, d, "cats_gpu_matmul_q6_K_q8_K"); }

void cats_gpu_quantize_q8_K(int8_t *q, float *x, int n)
{
    const char *what = "cats_gpu_quantize_q8_K";
    if (!ensure_init()) return;
    if (!q || !x || n <= 0 || n % 256) { fail(CATS_ERR_ARG, what); return; }
    const size_t xb = (size_t)n * 4, qb = (size_t)(n / 256) * 260;
    if (grow(&g.d_x, &g.d_x_cap, xb) || grow((void **)&g.d_out, &g.d_out_cap, qb)) return;
    if (check(cudaMemcpyAsync(g.d_x, x, xb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(launch_quantize_q8_K((uint8_t *)g.d_out, (const float *)g.d_x, n, g.stream), what)) return;
    if (check(cudaMemcpyAsync(q, g.d_out, qb, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

void cats_gpu_quantize_q8(int8_t *q, float *x, int n)
{
    const char *what = "cats_gpu_quantize_q8";
    if (!ensure_init()) return;
    if (!q || !x || n <= 0 || n % 32) { fail(CATS_ERR_ARG, what); return; }
    const size_t xb = (size_t)n * 4, qb = (size_t)(n / 32) * 36;
    if (grow(&g.d_x, &g.d_x_cap, xb) || grow((void **)&g.d_out, &g.d_out_cap, qb)) return;
    if (check(cudaMemcpyAsync(g.d_x, x, xb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(launch_quantize_q8((int8_t *)g.d_out, (const float *)g.d_x, n, 0, g.stream), what)) return;
    if (check(cudaMemcpyAsync(q, g.d_out, qb, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

static void *dequant_host(int type, void *y, const void *x, int row, int n, const char *what)
{
    if (!ensure_init()) return 0;
    if (!y || !x || row < 0 || n <= 0 || n % (kquant(type) ? 256 : 32)) { fail(CATS_ERR_ARG, what); return 0; }
    const size_t rb = gguf_row_bytes(type, n);
    if (grow(&g.d_x, &g.d_x_cap, rb) || grow((void **)&g.d_out, &g.d_out_cap, (size_t)n * 4)) return 0;
    const uint8_t *src = static_cast<const uint8_t *>(x) + (size_t)row * rb;
    if (check(cudaMemcpyAsync(g.d_x, src, rb, cudaMemcpyHostToDevice, g.stream), what)) return 0;
    if (check(kquant(type) ? launch_dequantize_kquant(type, g.d_out, (const uint8_t *)g.d_x, n, 1, g.stream)
                           : launch_dequantize(type, g.d_out, (const uint8_t *)g.d_x, n, 1, g.stream),
              what))
        return 0;
    if (check(cudaMemcpyAsync(y, g.d_out, (size_t)n * 4, cudaMemcpyDeviceToHost, g.stream), what)) return 0;
    check(cudaStreamSynchronize(g.stream), what);
    return 0;
}

void *cats_gpu_dequantize_q4_0(void *y, const void *x, int row, int n)
{ return dequant_host(CATS_TYPE_Q4_0, y, x, row, n, "cats_gpu_dequantize_q4_0"); }
void *cats_gpu_dequantize_q8_0(void *y, const void *x, int row, int n)
{ return dequant_host(CATS_TYPE_Q8_0, y, x, row, n, "cats_gpu_dequantize_q8_0"); }
void *cats_gpu_dequantize_q3_K(void *y, const void *x, int row, int n)
{ return dequant_host(CATS_TYPE_Q3_K, y, x, row, n, "cats_gpu_dequantize_q3_K"); }
void *cats_gpu_dequantize_q6_K(void *y, const void *x, int row, int n)
{ return dequant_host(CATS_TYPE_Q6_K, y, x, row, n, "cats_gpu_dequantize_q6_K"); }

int cats_gpu_matvec_dev(const void *w, float *d_out, const void *d_x, int x_is_q8, void *stream)
{
    const char *what = "cats_gpu_matvec_dev";
    if (!ensure_init()) return g.last_err;
    auto it = g.weights.find(w);
    if (it == g.weights.end()) return fail(CATS_ERR_ARG, "cats_gpu_matvec_dev: weight not registered");
    if (!d_out || !d_x || ((uintptr_t)d_x % 16)) return fail(CATS_ERR_ARG, what);
    Reg &r = it->second;
    if (x_is_q8 < 0 || x_is_q8 > 2) return fail(CATS_ERR_ARG, what);
    if (x_is_q8 && r.type == CATS_TYPE_F32) return fail(CATS_ERR_ARG, "cats_gpu_matvec_dev: F32 weight with Q8 input");
    cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
    if (kquant(r.type)) {
        if (x_is_q8 == 2) return fail(CATS_ERR_UNSUPPORTED, what);
        const uint8_t *xq = static_cast<const uint8_t *>(d_x);
        if (!x_is_q8) {   // quantize_q8_K into the library's scratch first
            if (grow((void **)&g.d_out, &g.d_out_cap, (size_t)(r.n / 256) * 260)) return g.last_err;
            if (check(launch_quantize_q8_K((uint8_t *)g.d_out, static_cast<const float *>(d_x), r.n, st), what))
                return g.last_err;
            xq = (const uint8_t *)g.d_out;
        }
        return check(launch_matvec_kquant(r.type, d_out, xq, r.W.ptr, r.n, r.d, st), what);
    }
    MatvecArgs a = args_for(r);
    a.xmode = (r.type == CATS_TYPE_F32 || x_is_q8 == 2) ? XM_F32 : (x_is_q8 ? XM_Q8_RAW : XM_Q8_FROM_F32);
    a.x = d_x;
    a.epi = EPI_STORE;
    a.out = d_out;
    return check(launch_matvec(a, r.W.L.rpw, r.type, st, false), what);
}

int cats_gpu_qgemm_dev(const void *w, const float *d_x, float *d_y, int T, void *stream)
{
    const char *what = "cats_gpu_qgemm_dev";
    if (!ensure_init()) return g.last_err;
    auto it = g.weights.find(w);
    if (it == g.weights.end()) return fail(CATS_ERR_ARG, "cats_gpu_qgemm_dev: weight not registered");
    Reg &r = it->second;
    if (!d_x || !d_y || T <= 0 || ((uintptr_t)d_x % 16)) return fail(CATS_ERR_ARG, what);
    if (!qgemm_supported(r.W.L)) return fail(CATS_ERR_UNSUPPORTED, what);
    cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
    if (grow((void **)&g.d_x16, &g.cap_x16, qgemm_x16_bytes(r.n, T))) return g.last_err;
    const size_t wsb = qgemm_workspace_bytes(r.W.L, T);
    if (wsb && grow((void **)&g.d_ws, &g.cap_ws, wsb)) return g.last_err;
    return check(launch_qgemm(r.W.L, r.W.ptr, d_x, g.d_x16, d_y, T, g.d_ws, g.cap_ws, g.d_err, st), what);
}

int cats_gpu_qgemm_plan(const void *w, int T, int *plan)
{
    const char *what = "cats_gpu_qgemm_plan";
    if (!ensure_init()) return g.last_err;
    auto it = g.weights.find(w);
    if (it == g.weights.end() || !plan || T <= 0) return fail(CATS_ERR_ARG, what);
    if (!qgemm_supported(it->second.W.L)) return fail(CATS_ERR_UNSUPPORTED, what);
    const QgemmPlan p = qgemm_plan(it->second.W.L, T);
    plan[0] = p.bn;
    plan[1] = p.splits;
    plan[2] = p.resident;
    plan[3] = p.tma;
    plan[4] = p.kper;
    plan[5] = p.occupancy;
    plan[6] = p.occupancy_err;
    return CATS_OK;
}

int cats_gpu_qgemm_trace(const void *w, const float *d_x, float *d_y, int T, unsigned long long *trace_host,
                         int trace_slices)
{
    const char *what = "cats_gpu_qgemm_trace";
    if (!ensure_init()) return g.last_err;
    auto it = g.weights.find(w);
    if (it == g.weights.end()) return fail(CATS_ERR_ARG, "cats_gpu_qgemm_trace: weight not registered");
    Reg &r = it->second;
    if (!d_x || !d_y || T <= 0 || ((uintptr_t)d_x % 16) || !trace_host || trace_slices <= 0)
        return fail(CATS_ERR_ARG, what);
    if (!qgemm_supported(r.W.L)) return fail(CATS_ERR_UNSUPPORTED, what);
    if (grow((void **)&g.d_x16, &g.cap_x16, qgemm_x16_bytes(r.n, T))) return g.last_err;
    const size_t wsb = qgemm_workspace_bytes(r.W.L, T);
    if (wsb && grow((void **)&g.d_ws, &g.cap_ws, wsb)) return g.last_err;
    const size_t tb = (size_t)(trace_slices + 1) * QG_TRACE_FIELDS * 8;
    unsigned long long *d_tr = nullptr;
    if (check(cudaMalloc(&d_tr, tb), what)) return g.last_err;
    QgemmTrace tr;
    tr.buf = d_tr;
    tr.slices = trace_slices;
    int rc = check(cudaMemsetAsync(d_tr, 0, tb, g.stream), what);
    if (!rc) rc = check(launch_qgemm(r.W.L, r.W.ptr, d_x, g.d_x16, d_y, T, g.d_ws, g.cap_ws, g.d_err, g.stream, &tr), what);
    if (!rc) rc = check(cudaMemcpyAsync(trace_host, d_tr, tb, cudaMemcpyDeviceToHost, g.stream), what);
    if (!rc) rc = check(cudaStreamSynchronize(g.stream), what);
    cudaFree(d_tr);
    return rc;
}

int cats_gpu_qgemm(const void *w, const float *x, float *y, int T)
{
    const char *what = "cats_gpu_qgemm";
    if (!ensure_init()) return g.last_err;
    auto it = g.weights.find(w);
    if (it == g.weights.end()) return fail(CATS_ERR_ARG, "cats_gpu_qgemm: weight not registered");
    Reg &r = it->second;
    if (!x || !y || T <= 0) return fail(CATS_ERR_ARG, what);
    const size_t xb = (size_t)T * r.n * 4, yb = (size_t)T * r.d * 4;
    if (grow((void **)&g.d_a, &g.cap_a, xb) || grow((void **)&g.d_c, &g.cap_c, yb)) return g.last_err;
    if (check(cudaMemcpyAsync(g.d_a, x, xb, cudaMemcpyHostToDevice, g.stream), what)) return g.last_err;
    if (int rc = cats_gpu_qgemm_dev(w, g.d_a, g.d_c, T, g.stream)) return rc;
    if (check(cudaMemcpyAsync(y, g.d_c, yb, cudaMemcpyDeviceToHost, g.stream), what)) return g.last_err;
    if (check(cudaStreamSynchronize(g.stream), what)) return g.last_err;
    return check_device_error(what);
}

int cats_gpu_quantize_q8_dev(int8_t *d_q, const float *d_x, int n, int scalar_mode, void *stream)
{
    if (!ensure_init()) return g.last_err;
    if (!d_q || !d_x || n <= 0 || n % 32 || ((uintptr_t)d_x % 16) || ((uintptr_t)d_q % 4))
        return fail(CATS_ERR_ARG, "cats_gpu_quantize_q8_dev");
    return check(launch_quantize_q8(d_q, d_x, n, scalar_mode, stream ? (cudaStream_t)stream : g.stream),
                 "cats_gpu_quantize_q8_dev");
}

int cats_gpu_dequantize_dev(int type, float *d_y, const void *d_w, int n, int rows, void *stream)
{
    if (!ensure_init()) return g.last_err;
    if (!d_y || !d_w || n <= 0 || rows <= 0 || (!type_ok(type) && !kquant(type)) || n % (kquant(type) ? 256 : 32))
        return fail(CATS_ERR_ARG, "cats_gpu_dequantize_dev");
    cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
    return check(kquant(type) ? launch_dequantize_kquant(type, d_y, (const uint8_t *)d_w, n, rows, st)
                              : launch_dequantize(type, d_y, (const uint8_t *)d_w, n, rows, st),
                 "cats_gpu_dequantize_dev");
}

// ------------------------------------------------------------------ LLM
struct cats_gpu_llm {
    LlmModel m;
    int engine = CATS_ENGINE_PERSISTENT;
    int *tok_log = nullptr;   // device: argmax ids of generate()
    int bt_T = 0, bt_nb = 0;  // the batch set last (cats_gpu_llm_batch_set)
    cudaEvent_t params_sent = nullptr;   // the last copy out of the pinned step parameters
    int *err_host = nullptr;              // pinned: the device error word, read with the logits
};

cats_gpu_llm *cats_gpu_llm_create(const cats_gpu_llm_config *cfg)
{
    if (!ensure_init()) return nullptr;
    if (!cfg || cfg->dim <= 0 || cfg->n_layers <= 0 || cfg->vocab <= 0 || cfg->seq_len <= 0 || !type_ok(cfg->wtype)) {
        fail(CATS_ERR_ARG, "cats_gpu_llm_create");
        return nullptr;
    }
    LlmConfig c{cfg->dim, cfg->hidden, cfg->n_layers, cfg->n_heads, cfg->n_kv_heads, cfg->vocab, cfg->seq_len,
                cfg->wtype, cfg->tp_size > 1 ? cfg->tp_rank : 0, cfg->tp_size > 0 ? cfg->tp_size : 1};
    if (c.tp_rank < 0 || c.tp_rank >= c.tp_size) { fail(CATS_ERR_ARG, "cats_gpu_llm_create: tp_rank"); return nullptr; }
    cats_gpu_llm *h = new cats_gpu_llm();
    // sharded models run the per-phase graph until cats_gpu_llm_tp_connect has
    // mapped the peers' exchange buffers (then the persistent kernel)
    if (c.tp_size > 1) h->engine = CATS_ENGINE_GRAPH;
    int rc = llm_alloc(&h->m, c);
    if (rc == CATS_OK && cudaMalloc(&h->tok_log, (size_t)(c.seq_len + 1) * 4) != cudaSuccess) rc = CATS_ERR_NOMEM;
    if (rc == CATS_OK && (cudaEventCreateWithFlags(&h->params_sent, cudaEventDisableTiming) != cudaSuccess ||
                          cudaMallocHost(&h->err_host, 4) != cudaSuccess))
        rc = CATS_ERR_CUDA;
    if (rc != CATS_OK) {
        fail(rc, "cats_gpu_llm_create");
        llm_free(&h->m);
        delete h;
        return nullptr;
    }
    return h;
}

void cats_gpu_llm_destroy(cats_gpu_llm *h)
{
    if (!h) return;
    if (h->m.stream) cudaStreamSynchronize(h->m.stream);
    llm_free(&h->m);
    if (h->tok_log) cudaFree(h->tok_log);
    if (h->params_sent) cudaEventDestroy(h->params_sent);
    if (h->err_host) cudaFreeHost(h->err_host);
    delete h;
}

int cats_gpu_llm_file_config(const char *path, cats_gpu_llm_config *cfg)
{
    if (!path || !cfg) return fail(CATS_ERR_ARG, "cats_gpu_llm_file_config");
    ModelFile f;
    std::string why;
    if (model_file_open(path, f, &why) != E_OK) return fail(CATS_ERR_ARG, ("cats_gpu_llm_file_config: " + why).c_str());
    const LlmConfig &c = f.cfg;
    *cfg = cats_gpu_llm_config{c.dim, c.hidden, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab, c.seq_len, c.wtype, 0, 1};
    model_file_close(f);
    return CATS_OK;
}

cats_gpu_llm *cats_gpu_llm_load(const char *path, int tp_rank, int tp_size, int seq_len)
{
    if (!ensure_init()) return nullptr;
    if (!path || tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size || seq_len < 0) {
        fail(CATS_ERR_ARG, "cats_gpu_llm_load");
        return nullptr;
    }
    ModelFile f;
    std::string why;
    if (model_file_open(path, f, &why) != E_OK) {
        fail(CATS_ERR_ARG, ("cats_gpu_llm_load: " + why).c_str());
        return nullptr;
    }
    const LlmConfig &c = f.cfg;
    cats_gpu_llm_config cc{c.dim, c.hidden, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab, seq_len ? seq_len : c.seq_len,
                           c.wtype, tp_rank, tp_size};
    cats_gpu_llm *h = nullptr;
    if (cc.wtype != CATS_TYPE_F32 && cc.wtype != CATS_TYPE_Q4_0 && cc.wtype != CATS_TYPE_Q8_0) {
        fail(CATS_ERR_UNSUPPORTED, "cats_gpu_llm_load: layer weight type (F32, Q4_0 or Q8_0 models run on the device)");
    } else if ((h = cats_gpu_llm_create(&cc)) != nullptr) {
        const int rc = model_file_load(&h->m, f, &why);
        if (rc != E_OK) {
            fail(rc, ("cats_gpu_llm_load: " + why).c_str());
            cats_gpu_llm_destroy(h);
            h = nullptr;
        }
    }
    model_file_close(f);
    return h;
}

int cats_gpu_llm_set_weights(cats_gpu_llm *h, const float *emb, const float *rms_att, const float *rms_ffn,
                             const float *rms_final, const void *wq, const void *wk, const void *wv, const void *wo,
                             const void *w1, const void *w2, const void *w3, const void *wcls)
{
    if (!h || !emb || !rms_att || !rms_ffn || !rms_final || !wq || !wk || !wv || !wo || !w1 || !w2 || !w3 || !wcls)
        return fail(CATS_ERR_ARG, "cats_gpu_llm_set_weights");
    int rc = llm_set_weights(&h->m, emb, rms_att, rms_ffn, rms_final, wq, wk, wv, wo, w1, w2, w3, wcls);
    return rc ? fail(rc, "cats_gpu_llm_set_weights") : CATS_OK;
}

int cats_gpu_llm_init_random(cats_gpu_llm *h, unsigned long long seed, float std)
{
    if (!h) return fail(CATS_ERR_ARG, "cats_gpu_llm_init_random");
    int rc = llm_init_random(&h->m, seed, std);
    return rc ? fail(rc, "cats_gpu_llm_init_random") : CATS_OK;
}

static int ensure_graph(cats_gpu_llm *h)
{
    if (!h->m.weights_ready) return fail(CATS_ERR_ARG, "llm: weights not set");
    if (h->engine == CATS_ENGINE_PERSISTENT) {
        if (h->m.c.tp_size > 1 && !h->m.tp_p2p) return fail(CATS_ERR_ARG, "llm: tensor parallel model not connected");
        int rc = decode_prepare(&h->m);
        return rc ? fail(rc, "llm: persistent decode setup") : CATS_OK;
    }
    if (h->m.exec) return CATS_OK;
    if (h->m.c.tp_size > 1 && !h->m.comm_ctx) return fail(CATS_ERR_ARG, "llm: tensor parallel model not connected");
    return check(llm_build_graph(&h->m), "llm: graph capture");
}

// Enqueue `steps` greedy steps from the device params on the model's stream.
static int run_steps(cats_gpu_llm *h, int steps, int *tok_log_dev, const char *what)
{
    LlmModel &m = h->m;
    if (h->engine == CATS_ENGINE_PERSISTENT)
        return check(decode_launch(&m, steps, tok_log_dev, m.c.seq_len + 1), what);
    for (int s = 0; s < steps; s++) {
        if (check(cudaGraphLaunch(m.exec, m.stream), what)) return g.last_err;
        if (tok_log_dev && check(cudaMemcpyAsync(tok_log_dev + s, &m.params->next, 4, cudaMemcpyDeviceToDevice,
                                                 m.stream), what))
            return g.last_err;
    }
    return CATS_OK;
}

int cats_gpu_llm_set_engine(cats_gpu_llm *h, int engine)
{
    if (!h || (engine != CATS_ENGINE_PERSISTENT && engine != CATS_ENGINE_GRAPH))
        return fail(CATS_ERR_ARG, "cats_gpu_llm_set_engine");
    if (engine == CATS_ENGINE_PERSISTENT && h->m.c.tp_size > 1 && !h->m.tp_p2p)
        return fail(CATS_ERR_UNSUPPORTED,
                    "cats_gpu_llm_set_engine: this sharded model has no mapped peers (not connected, ranks sharing "
                    "a GPU, or CATS_TP_NO_P2P=1): the persistent engine needs them");
    h->engine = engine;
    return CATS_OK;
}

size_t cats_gpu_tp_unique_id_bytes(void) { return tp_unique_id_bytes(); }

int cats_gpu_tp_unique_id(void *id, size_t bytes)
{
    if (!ensure_init()) return g.last_err;
    int rc = tp_unique_id(id, bytes);
    return rc ? fail(rc, "cats_gpu_tp_unique_id") : CATS_OK;
}

int cats_gpu_llm_tp_connect(cats_gpu_llm *h, const void *id)
{
    if (!h || !id || h->m.c.tp_size < 2) return fail(CATS_ERR_ARG, "cats_gpu_llm_tp_connect");
    if (check(cudaSetDevice(g.device), "cats_gpu_llm_tp_connect")) return g.last_err;
    int rc = tp_connect(&h->m, id);
    if (rc) return fail(rc, "cats_gpu_llm_tp_connect");
    if (h->m.tp_p2p) h->engine = CATS_ENGINE_PERSISTENT;   // the exchange inside the persistent kernel
    return CATS_OK;
}

int cats_gpu_llm_tp_loopback(cats_gpu_llm *h)
{
    if (!h || h->m.c.tp_size < 2) return fail(CATS_ERR_ARG, "cats_gpu_llm_tp_loopback");
    int rc = tp_loopback(&h->m);
    if (rc) return fail(rc, "cats_gpu_llm_tp_loopback");
    h->engine = CATS_ENGINE_PERSISTENT;
    return CATS_OK;
}

int cats_gpu_llm_set_position(cats_gpu_llm *h, int token, int pos)
{
    if (!h || token < 0 || token >= h->m.c.vocab || pos < 0 || pos >= h->m.c.seq_len)
        return fail(CATS_ERR_ARG, "cats_gpu_llm_set_position");
    // the pinned staging struct may still be the source of the previous copy
    if (check(cudaEventSynchronize(h->params_sent), "cats_gpu_llm_set_position")) return g.last_err;
    StepParams *p = h->m.params_host;
    p->token = token;
    p->pos = pos;
    p->next = 0;
    p->steps = 0;
    if (check(cudaMemcpyAsync(h->m.params, p, sizeof(StepParams), cudaMemcpyHostToDevice, h->m.stream),
              "cats_gpu_llm_set_position"))
        return g.last_err;
    return check(cudaEventRecord(h->params_sent, h->m.stream), "cats_gpu_llm_set_position");
}

float *cats_gpu_llama2_transformer(int token, int pos, cats_gpu_llm *h, float *logits_host)
{
    const char *what = "cats_gpu_llama2_transformer";
    if (!h) { fail(CATS_ERR_ARG, what); return nullptr; }
    if (ensure_graph(h)) return nullptr;
    if (cats_gpu_llm_set_position(h, token, pos)) return nullptr;
    LlmModel &m = h->m;
    if (run_steps(h, 1, nullptr, what)) return nullptr;
    // the logits and the error word come back in one wait
    if (check(cudaMemcpyAsync(m.logits_host, m.logits, (size_t)m.c.vocab * 4, cudaMemcpyDeviceToHost, m.stream), what))
        return nullptr;
    if (check(cudaMemcpyAsync(h->err_host, m.err, 4, cudaMemcpyDeviceToHost, m.stream), what)) return nullptr;
    if (check(cudaStreamSynchronize(m.stream), what)) return nullptr;
    if (*h->err_host) { cudaMemset(m.err, 0, 4); fail(CATS_ERR_TIMEOUT, what); return nullptr; }
    if (!logits_host) return m.logits_host;   // the model's own copy, as the reference returns s->logits
    memcpy(logits_host, m.logits_host, (size_t)m.c.vocab * 4);
    return logits_host;
}

int cats_gpu_llm_trace_step(cats_gpu_llm *h, int token, int pos, unsigned long long *host, int per_cta, int *ctas)
{
    const char *what = "cats_gpu_llm_trace_step";
    if (!h || !host || per_cta <= 0 || !ctas) return fail(CATS_ERR_ARG, what);
    if (int rc = ensure_graph(h)) return rc;
    if (int rc = decode_prepare(&h->m)) return fail(rc, what);
    if (int rc = cats_gpu_llm_set_position(h, token, pos)) return rc;
    const int grid = matvec_num_sms();
    const size_t bytes = (size_t)2 * grid * per_cta * 8;   // globaltimer plane, then clock64 plane
    unsigned long long *d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) return fail(CATS_ERR_NOMEM, what);
    cudaMemsetAsync(d, 0, bytes, h->m.stream);
    int rc = check(decode_launch(&h->m, 1, nullptr, 0, d, per_cta), what);
    if (!rc) rc = check(cudaMemcpyAsync(host, d, bytes, cudaMemcpyDeviceToHost, h->m.stream), what);
    if (!rc) rc = check(cudaStreamSynchronize(h->m.stream), what);
    cudaFree(d);
    *ctas = grid;
    return rc;
}

int cats_gpu_llm_enqueue(cats_gpu_llm *h, int steps)
{
    if (!h || steps < 0) return fail(CATS_ERR_ARG, "cats_gpu_llm_enqueue");
    if (int rc = ensure_graph(h)) return rc;
    return run_steps(h, steps, nullptr, "cats_gpu_llm_enqueue");
}

int cats_gpu_llm_generate(cats_gpu_llm *h, int token, int pos, int steps, int *tokens_host)
{
    if (!h || steps < 0 || pos + steps > h->m.c.seq_len) return fail(CATS_ERR_ARG, "cats_gpu_llm_generate");
    if (int rc = ensure_graph(h)) return rc;
    if (int rc = cats_gpu_llm_set_position(h, token, pos)) return rc;
    LlmModel &m = h->m;
    if (int rc = run_steps(h, steps, tokens_host ? h->tok_log : nullptr, "cats_gpu_llm_generate")) return rc;
    if (tokens_host &&
        check(cudaMemcpyAsync(tokens_host, h->tok_log, (size_t)steps * 4, cudaMemcpyDeviceToHost, m.stream), "generate"))
        return g.last_err;
    return cats_gpu_llm_synchronize(h);
}

// ---------------------------------------------------- batched step (batch.cu)
static int batch_ready(cats_gpu_llm *h, const char *what)
{
    if (!h->m.weights_ready) return fail(CATS_ERR_ARG, what);
    if (!batch_supported(&h->m)) return fail(CATS_ERR_UNSUPPORTED, what);
    if (h->m.bt_cap == 0) return fail(CATS_ERR_ARG, what);   // cats_gpu_llm_batch_reserve first
    if (h->m.c.tp_size > 1 && !h->m.comm_ctx) return fail(CATS_ERR_ARG, what);
    return CATS_OK;
}

static int device_status(cats_gpu_llm *h, const char *what)
{
    int e = 0;
    if (cudaMemcpy(&e, h->m.err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return fail(CATS_ERR_CUDA, what);
    if (e) {
        cudaMemset(h->m.err, 0, 4);
        return fail(CATS_ERR_TIMEOUT, what);
    }
    return CATS_OK;
}

int cats_gpu_llm_batch_reserve(cats_gpu_llm *h, int max_tokens, int n_seqs)
{
    const char *what = "cats_gpu_llm_batch_reserve";
    if (!h || max_tokens <= 0 || n_seqs <= 0) return fail(CATS_ERR_ARG, what);
    int rc = llm_batch_reserve(&h->m, max_tokens, n_seqs);
    return rc ? fail(rc, what) : CATS_OK;
}

int cats_gpu_llm_batch_set(cats_gpu_llm *h, const int *tokens, const int *pos, const int *seqs, int T)
{
    const char *what = "cats_gpu_llm_batch_set";
    if (!h) return fail(CATS_ERR_ARG, what);
    if (int rc = batch_ready(h, what)) return rc;
    int nb = 0;
    if (int rc = llm_batch_set(&h->m, tokens, pos, seqs, T, &nb)) return fail(rc, what);
    h->bt_T = T;
    h->bt_nb = nb;
    return CATS_OK;
}

int cats_gpu_llm_batch_enqueue(cats_gpu_llm *h)
{
    const char *what = "cats_gpu_llm_batch_enqueue";
    if (!h || h->bt_T <= 0) return fail(CATS_ERR_ARG, what);
    return check(llm_batch_enqueue(&h->m, h->bt_T, h->bt_nb, false, nullptr, 0), what);
}

int cats_gpu_llm_batch_enqueue_decode(cats_gpu_llm *h, int steps)
{
    const char *what = "cats_gpu_llm_batch_enqueue_decode";
    if (!h || h->bt_T <= 0 || steps < 0 || h->bt_nb != h->bt_T) return fail(CATS_ERR_ARG, what);
    return check(llm_batch_decode_enqueue(&h->m, h->bt_T, steps), what);
}

int cats_gpu_llm_time_product(cats_gpu_llm *h, int kind, int T, int reps, float *ms_per_launch,
                              double *flop_per_launch, double *weight_bytes_per_launch)
{
    const char *what = "cats_gpu_llm_time_product";
    if (!h || !ms_per_launch || !flop_per_launch || !weight_bytes_per_launch) return fail(CATS_ERR_ARG, what);
    if (int rc = batch_ready(h, what)) return rc;
    return check(llm_time_product(&h->m, kind, T, reps, ms_per_launch, flop_per_launch, weight_bytes_per_launch),
                 what);
}

int cats_gpu_llm_forward_batch(cats_gpu_llm *h, const int *tokens, const int *pos, const int *seqs, int T,
                               int *next_host, float *logits_host)
{
    const char *what = "cats_gpu_llm_forward_batch";
    if (!h) return fail(CATS_ERR_ARG, what);
    if (int rc = batch_ready(h, what)) return rc;
    if (int rc = llm_forward_batch(&h->m, tokens, pos, seqs, T, next_host, logits_host)) return fail(rc, what);
    h->bt_T = 0;
    return device_status(h, what);
}

int cats_gpu_llm_generate_batch(cats_gpu_llm *h, const int *tokens, const int *pos, int n, int steps,
                                int *tokens_host)
{
    const char *what = "cats_gpu_llm_generate_batch";
    if (!h || !tokens || !pos || n <= 0 || steps < 0 || n > h->m.n_seqs) return fail(CATS_ERR_ARG, what);
    if (int rc = batch_ready(h, what)) return rc;
    for (int i = 0; i < n; i++)
        if (pos[i] < 0 || pos[i] + steps > h->m.c.seq_len) return fail(CATS_ERR_ARG, what);
    std::vector<int> seqs(n);
    for (int i = 0; i < n; i++) seqs[i] = i;
    int nb = 0;
    if (int rc = llm_batch_set(&h->m, tokens, pos, seqs.data(), n, &nb)) return fail(rc, what);
    h->bt_T = 0;
    if (int rc = llm_generate_batch(&h->m, n, steps, tokens_host)) return fail(rc, what);
    return device_status(h, what);
}

int cats_gpu_llm_synchronize(cats_gpu_llm *h)
{
    if (!h) return fail(CATS_ERR_ARG, "cats_gpu_llm_synchronize");
    if (check(cudaStreamSynchronize(h->m.stream), "cats_gpu_llm_synchronize")) return g.last_err;
    int e = 0;
    cudaMemcpy(&e, h->m.err, 4, cudaMemcpyDeviceToHost);
    if (e) return fail(CATS_ERR_TIMEOUT, "llm: a device wait timed out");
    return CATS_OK;
}

void *cats_gpu_llm_stream(cats_gpu_llm *h) { return h ? (void *)h->m.stream : nullptr; }

int cats_gpu_llm_logits(cats_gpu_llm *h, float *logits_host)
{
    if (!h || !logits_host) return fail(CATS_ERR_ARG, "cats_gpu_llm_logits");
    if (check(cudaMemcpyAsync(logits_host, h->m.logits, (size_t)h->m.c.vocab * 4, cudaMemcpyDeviceToHost, h->m.stream),
              "cats_gpu_llm_logits"))
        return g.last_err;
    return check(cudaStreamSynchronize(h->m.stream), "cats_gpu_llm_logits");
}

int cats_gpu_llm_next_token(cats_gpu_llm *h)
{
    if (!h) return -1;
    StepParams p;
    if (cudaMemcpyAsync(&p, h->m.params, sizeof(p), cudaMemcpyDeviceToHost, h->m.stream) != cudaSuccess ||
        cudaStreamSynchronize(h->m.stream) != cudaSuccess)
        return -1;
    return p.next;
}

size_t cats_gpu_llm_weight_bytes(cats_gpu_llm *h)
{
    if (!h) return 0;
    // algorithmic bytes: the reference-layout weight bytes one step reads
    const LlmModel &m = h->m;
    size_t s = 0;
    auto add = [&](const DevWeight &w) { s += gguf_row_bytes(w.L.type, w.L.n) * w.L.d; };
    for (auto &w : m.qkv) add(w);
    for (auto &w : m.wo) add(w);
    for (auto &w : m.w13) add(w);
    for (auto &w : m.w2) add(w);
    add(m.cls);
    return s;
}

int cats_gpu_llm_time_matvec(cats_gpu_llm *h, int kind, int reps, float *ms_per_launch, double *bytes_per_launch)
{
    if (!h || !ms_per_launch || !bytes_per_launch || kind < 0 || kind > 4 || reps <= 0)
        return fail(CATS_ERR_ARG, "cats_gpu_llm_time_matvec");
    if (!h->m.weights_ready) return fail(CATS_ERR_ARG, "cats_gpu_llm_time_matvec: weights not set");
    return check(llm_time_matvec(&h->m, kind, reps, ms_per_launch, bytes_per_launch), "cats_gpu_llm_time_matvec");
}

int cats_gpu_synth_tensor(void *host_dst, int type, int n, int d, unsigned long long seed, int tensor_id, float std,
                          float constant)
{
    if (!ensure_init()) return g.last_err;
    if (!host_dst || !type_ok(type) || n <= 0 || d <= 0 || n % 32) return fail(CATS_ERR_ARG, "cats_gpu_synth_tensor");
    const size_t bytes = gguf_row_bytes(type, n) * d;
    uint8_t *buf = nullptr;
    if (cudaMalloc(&buf, bytes) != cudaSuccess) return fail(CATS_ERR_NOMEM, "cats_gpu_synth_tensor");
    int rc = check(synth_tensor(buf, type, n, d, seed, tensor_id, std, constant, g.stream), "cats_gpu_synth_tensor");
    if (!rc) rc = check(cudaMemcpyAsync(host_dst, buf, bytes, cudaMemcpyDeviceToHost, g.stream), "cats_gpu_synth_tensor");
    if (!rc) rc = check(cudaStreamSynchronize(g.stream), "cats_gpu_synth_tensor");
    cudaFree(buf);
    return rc;
}

// ------------------------------------------------------------------ sgemm
int cats_sgemm_dev(char ta, char tb, int m, int n, int k, float alpha, const float *a, int lda, const float *b,
                   int ldb, float beta, float *c, int ldc, void *stream)
{
    const char *what = "cats_sgemm_dev";
    if (!ensure_init()) return g.last_err;
    const bool at = ta == 'T' || ta == 't', bt = tb == 'T' || tb == 't';
    if ((!at && ta != 'N' && ta != 'n') || (!bt && tb != 'N' && tb != 'n') || m < 0 || n < 0 || k < 0)
        return fail(CATS_ERR_ARG, what);
    if (m == 0 || n == 0) return CATS_OK;
    if (!c || (k > 0 && (!a || !b)) || ldc < n || (k > 0 && (lda < (at ? m : k) || ldb < (bt ? k : n))))
        return fail(CATS_ERR_ARG, what);
    SgemmPlan p = sgemm_plan(m, n, k, matvec_num_sms());
    if (p.work_floats && grow((void **)&g.d_work, &g.cap_work, p.work_floats * 4)) return g.last_err;
    return check(launch_sgemm(p, at, bt, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc, g.d_work, g.d_err,
                              stream ? (cudaStream_t)stream : g.stream),
                 what);
}

void cats_sgemm(char ta, char tb, int m, int n, int k, float alpha, const float *a, const float *b, float beta,
                float *c)
{
    const char *what = "cats_sgemm";
    if (!ensure_init()) return;
    const bool at = ta == 'T' || ta == 't', bt = tb == 'T' || tb == 't';
    if (m < 0 || n < 0 || k < 0 || !c || (k > 0 && (!a || !b))) { fail(CATS_ERR_ARG, what); return; }
    if (m == 0 || n == 0) return;
    const size_t ab = (size_t)m * k * 4, bb = (size_t)k * n * 4, cb = (size_t)m * n * 4;
    if (grow((void **)&g.d_a, &g.cap_a, ab ? ab : 4) || grow((void **)&g.d_b, &g.cap_b, bb ? bb : 4) ||
        grow((void **)&g.d_c, &g.cap_c, cb))
        return;
    if (ab && check(cudaMemcpyAsync(g.d_a, a, ab, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (bb && check(cudaMemcpyAsync(g.d_b, b, bb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (beta != 0.f && check(cudaMemcpyAsync(g.d_c, c, cb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (cats_sgemm_dev(ta, tb, m, n, k, alpha, g.d_a, at ? m : k, g.d_b, bt ? k : n, beta, g.d_c, n, g.stream)) return;
    if (check(cudaMemcpyAsync(c, g.d_c, cb, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

void cats_gemm_rnn(int M, int N, int K, float alpha, float *A, float *B, float beta, float *C)
{ cats_sgemm('N', 'N', M, N, K, alpha, A, B, beta, C); }
void cats_gemm_rnt(int M, int N, int K, float alpha, float *A, float *B, float beta, float *C)
{ cats_sgemm('N', 'T', M, N, K, alpha, A, B, beta, C); }
void cats_gemm_rtn(int M, int N, int K, float alpha, float *A, float *B, float beta, float *C)
{ cats_sgemm('T', 'N', M, N, K, alpha, A, B, beta, C); }

// ---------------------------------------------------------------- CNN forward
static bool conv_geom_ok(int c, int h, int w, int kh, int kw, int ph, int pw, int sh, int sw)
{
    return c > 0 && h > 0 && w > 0 && kh > 0 && kw > 0 && ph >= 0 && pw >= 0 && sh > 0 && sw > 0 &&
           conv_out(h, kh, ph, sh) > 0 && conv_out(w, kw, pw, sw) > 0;
}

int cats_im2col_dev(const float *im, int channels, int height, int width, int kh, int kw, int ph, int pw, int sh,
                    int sw, float *col, void *stream)
{
    const char *what = "cats_im2col_dev";
    if (!ensure_init()) return g.last_err;
    if (!im || !col || !conv_geom_ok(channels, height, width, kh, kw, ph, pw, sh, sw)) return fail(CATS_ERR_ARG, what);
    return check(launch_im2col(im, channels, height, width, kh, kw, ph, pw, sh, sw, col,
                               stream ? (cudaStream_t)stream : g.stream),
                 what);
}

void cats_im2col(const float *im, int channels, int height, int width, int kh, int kw, int ph, int pw, int sh,
                 int sw, float *col)
{
    const char *what = "cats_im2col";
    if (!ensure_init()) return;
    if (!im || !col || !conv_geom_ok(channels, height, width, kh, kw, ph, pw, sh, sw)) { fail(CATS_ERR_ARG, what); return; }
    const size_t ib = (size_t)channels * height * width * 4;
    const size_t cb = (size_t)channels * kh * kw * conv_out(height, kh, ph, sh) * conv_out(width, kw, pw, sw) * 4;
    if (grow((void **)&g.d_a, &g.cap_a, ib) || grow((void **)&g.d_c, &g.cap_c, cb)) return;
    if (check(cudaMemcpyAsync(g.d_a, im, ib, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (cats_im2col_dev(g.d_a, channels, height, width, kh, kw, ph, pw, sh, sw, g.d_c, g.stream)) return;
    if (check(cudaMemcpyAsync(col, g.d_c, cb, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

int cats_conv2d_forward_dev(const float *x, const float *w, float *z, int batch, int ich, int h, int wd, int ch,
                            int ksize, int pad, int stride, void *stream)
{
    const char *what = "cats_conv2d_forward_dev";
    if (!ensure_init()) return g.last_err;
    if (!x || !w || !z || batch <= 0 || ch <= 0 || !conv_geom_ok(ich, h, wd, ksize, ksize, pad, pad, stride, stride))
        return fail(CATS_ERR_ARG, what);
    // scratch for the weights in the tensor-core path's channel-blocked order
    const size_t wpb = (size_t)ch * ich * ksize * ksize * 4;
    if (grow((void **)&g.d_work, &g.cap_work, wpb)) return g.last_err;
    return check(launch_conv2d_forward(x, w, z, batch, ich, h, wd, ch, ksize, pad, stride, g.d_err, g.d_work,
                                       stream ? (cudaStream_t)stream : g.stream),
                 what);
}

void cats_conv2d_forward(const float *x, const float *w, float *z, int batch, int ich, int h, int wd, int ch,
                         int ksize, int pad, int stride)
{
    const char *what = "cats_conv2d_forward";
    if (!ensure_init()) return;
    if (!x || !w || !z || batch <= 0 || ch <= 0 || !conv_geom_ok(ich, h, wd, ksize, ksize, pad, pad, stride, stride)) {
        fail(CATS_ERR_ARG, what);
        return;
    }
    const size_t xb = (size_t)batch * ich * h * wd * 4, wb = (size_t)ch * ich * ksize * ksize * 4;
    const size_t zb = (size_t)batch * ch * conv_out(h, ksize, pad, stride) * conv_out(wd, ksize, pad, stride) * 4;
    if (grow((void **)&g.d_a, &g.cap_a, xb) || grow((void **)&g.d_b, &g.cap_b, wb) ||
        grow((void **)&g.d_c, &g.cap_c, zb))
        return;
    if (check(cudaMemcpyAsync(g.d_a, x, xb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(cudaMemcpyAsync(g.d_b, w, wb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (cats_conv2d_forward_dev(g.d_a, g.d_b, g.d_c, batch, ich, h, wd, ch, ksize, pad, stride, g.stream)) return;
    if (check(cudaMemcpyAsync(z, g.d_c, zb, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

int cats_linear_forward_dev(const float *x, const float *w, float *z, int batch, int in, int out, void *stream)
{
    const char *what = "cats_linear_forward_dev";
    if (!ensure_init()) return g.last_err;
    if (!x || !w || !z || batch <= 0 || in <= 0 || out <= 0) return fail(CATS_ERR_ARG, what);
    cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
    if (check(launch_bias_rows(w + (size_t)in * out, z, batch, out, st), what)) return g.last_err;
    return cats_sgemm_dev('N', 'T', batch, out, in, 1.f, x, in, w, in, 1.f, z, out, st);
}

void cats_linear_forward(const float *x, const float *w, float *z, int batch, int in, int out)
{
    const char *what = "cats_linear_forward";
    if (!ensure_init()) return;
    if (!x || !w || !z || batch <= 0 || in <= 0 || out <= 0) { fail(CATS_ERR_ARG, what); return; }
    const size_t xb = (size_t)batch * in * 4, wb = ((size_t)in * out + out) * 4, zb = (size_t)batch * out * 4;
    if (grow((void **)&g.d_a, &g.cap_a, xb) || grow((void **)&g.d_b, &g.cap_b, wb) ||
        grow((void **)&g.d_c, &g.cap_c, zb))
        return;
    if (check(cudaMemcpyAsync(g.d_a, x, xb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(cudaMemcpyAsync(g.d_b, w, wb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (cats_linear_forward_dev(g.d_a, g.d_b, g.d_c, batch, in, out, g.stream)) return;
    if (check(cudaMemcpyAsync(z, g.d_c, zb, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

// ------------------------------------------------------------- CNN training
int cats_col2im_dev(const float *col, int channels, int height, int width, int kh, int kw, int ph, int pw, int sh,
                    int sw, float *im, void *stream)
{
    const char *what = "cats_col2im_dev";
    if (!ensure_init()) return g.last_err;
    if (!im || !col || !conv_geom_ok(channels, height, width, kh, kw, ph, pw, sh, sw)) return fail(CATS_ERR_ARG, what);
    const long long P = (long long)conv_out(height, kh, ph, sh) * conv_out(width, kw, pw, sw);
    return check(launch_col2im(col, P, 1, channels, height, width, kh, kw, ph, pw, sh, sw, im,
                               stream ? (cudaStream_t)stream : g.stream),
                 what);
}

void cats_col2im(const float *col, int channels, int height, int width, int kh, int kw, int ph, int pw, int sh,
                 int sw, float *im)
{
    const char *what = "cats_col2im";
    if (!ensure_init()) return;
    if (!im || !col || !conv_geom_ok(channels, height, width, kh, kw, ph, pw, sh, sw)) { fail(CATS_ERR_ARG, what); return; }
    const size_t ib = (size_t)channels * height * width * 4;
    const size_t cb = (size_t)channels * kh * kw * conv_out(height, kh, ph, sh) * conv_out(width, kw, pw, sw) * 4;
    if (grow((void **)&g.d_a, &g.cap_a, cb) || grow((void **)&g.d_c, &g.cap_c, ib)) return;
    if (check(cudaMemcpyAsync(g.d_a, col, cb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (cats_col2im_dev(g.d_a, channels, height, width, kh, kw, ph, pw, sh, sw, g.d_c, g.stream)) return;
    if (check(cudaMemcpyAsync(im, g.d_c, ib, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

// The sizes of a convolution layer's batch: K = ich*k*k, P = oh*ow, N = batch*P.
static bool conv_sizes(int batch, int ich, int h, int wd, int ch, int ksize, int pad, int stride, long long *K,
                       long long *P, long long *N)
{
    if (batch <= 0 || ch <= 0 || !conv_geom_ok(ich, h, wd, ksize, ksize, pad, pad, stride, stride)) return false;
    *K = (long long)ich * ksize * ksize;
    *P = (long long)conv_out(h, ksize, pad, stride) * conv_out(wd, ksize, pad, stride);
    *N = *P * batch;
    // the GEMMs take int sizes
    return *K < (1LL << 31) && *N < (1LL << 31) && *K * *N < (1LL << 40);
}

int cats_conv2d_backward_dev(const float *dout, const float *w, float *din, int batch, int ich, int h, int wd, int ch,
                             int ksize, int pad, int stride, void *stream)
{
    const char *what = "cats_conv2d_backward_dev";
    if (!ensure_init()) return g.last_err;
    long long K, P, N;
    if (!dout || !w || !din || !conv_sizes(batch, ich, h, wd, ch, ksize, pad, stride, &K, &P, &N))
        return fail(CATS_ERR_ARG, what);
    cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
    if (grow((void **)&g.d_tr, &g.cap_tr, (size_t)ch * N * 4) || grow((void **)&g.d_col, &g.cap_col, (size_t)K * N * 4))
        return g.last_err;
    // dOut as one [ch][batch*P] operand, then col[k][b*P + p] = sum_c w[c][k] dOut[b][c][p]
    // (every sample's gemm_rtn at once), then col2im of every sample
    if (check(launch_batch_to_channel_major(dout, batch, ch, (int)P, g.d_tr, st), what)) return g.last_err;
    if (int rc = cats_sgemm_dev('T', 'N', (int)K, (int)N, ch, 1.f, w, (int)K, g.d_tr, (int)N, 0.f, g.d_col, (int)N, st))
        return rc;
    return check(launch_col2im(g.d_col, N, batch, ich, h, wd, ksize, ksize, pad, pad, stride, stride, din, st), what);
}

void cats_conv2d_backward(const float *dout, const float *w, float *din, int batch, int ich, int h, int wd, int ch,
                          int ksize, int pad, int stride)
{
    const char *what = "cats_conv2d_backward";
    if (!ensure_init()) return;
    long long K, P, N;
    if (!dout || !w || !din || !conv_sizes(batch, ich, h, wd, ch, ksize, pad, stride, &K, &P, &N)) {
        fail(CATS_ERR_ARG, what);
        return;
    }
    const size_t ob = (size_t)ch * N * 4, wb = (size_t)ch * K * 4, ib = (size_t)batch * ich * h * wd * 4;
    if (grow((void **)&g.d_a, &g.cap_a, ob) || grow((void **)&g.d_b, &g.cap_b, wb) || grow((void **)&g.d_c, &g.cap_c, ib))
        return;
    if (check(cudaMemcpyAsync(g.d_a, dout, ob, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(cudaMemcpyAsync(g.d_b, w, wb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (cats_conv2d_backward_dev(g.d_a, g.d_b, g.d_c, batch, ich, h, wd, ch, ksize, pad, stride, g.stream)) return;
    if (check(cudaMemcpyAsync(din, g.d_c, ib, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

int cats_conv2d_update_dev(const float *dout, const float *x, float *dw, int batch, int ich, int h, int wd, int ch,
                           int ksize, int pad, int stride, void *stream)
{
    const char *what = "cats_conv2d_update_dev";
    if (!ensure_init()) return g.last_err;
    long long K, P, N;
    if (!dout || !x || !dw || !conv_sizes(batch, ich, h, wd, ch, ksize, pad, stride, &K, &P, &N))
        return fail(CATS_ERR_ARG, what);
    cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
    if (grow((void **)&g.d_tr, &g.cap_tr, (size_t)ch * N * 4) || grow((void **)&g.d_col, &g.cap_col, (size_t)K * N * 4))
        return g.last_err;
    // dw[c][k] += (1/batch) * sum over every sample's pixels of dOut[b][c][p] im2col(x[b])[k][p]:
    // the per-sample gemm_rnt calls with alpha = 1/batch (catseye.h:622-640) as one GEMM
    if (check(launch_batch_to_channel_major(dout, batch, ch, (int)P, g.d_tr, st), what)) return g.last_err;
    if (check(launch_im2col_cols(x, batch, ich, h, wd, ksize, ksize, pad, pad, stride, stride, g.d_col, st), what))
        return g.last_err;
    const float alpha = (float)(1.0 / batch);   // the reference's real alpha = 1.0/l->p->batch
    return cats_sgemm_dev('N', 'T', ch, (int)K, (int)N, alpha, g.d_tr, (int)N, g.d_col, (int)N, 1.f, dw, (int)K, st);
}

void cats_conv2d_update(const float *dout, const float *x, float *dw, int batch, int ich, int h, int wd, int ch,
                        int ksize, int pad, int stride)
{
    const char *what = "cats_conv2d_update";
    if (!ensure_init()) return;
    long long K, P, N;
    if (!dout || !x || !dw || !conv_sizes(batch, ich, h, wd, ch, ksize, pad, stride, &K, &P, &N)) {
        fail(CATS_ERR_ARG, what);
        return;
    }
    const size_t ob = (size_t)ch * N * 4, xb = (size_t)batch * ich * h * wd * 4, wb = (size_t)ch * K * 4;
    if (grow((void **)&g.d_a, &g.cap_a, ob) || grow((void **)&g.d_b, &g.cap_b, xb) || grow((void **)&g.d_c, &g.cap_c, wb))
        return;
    if (check(cudaMemcpyAsync(g.d_a, dout, ob, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(cudaMemcpyAsync(g.d_b, x, xb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(cudaMemcpyAsync(g.d_c, dw, wb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (cats_conv2d_update_dev(g.d_a, g.d_b, g.d_c, batch, ich, h, wd, ch, ksize, pad, stride, g.stream)) return;
    if (check(cudaMemcpyAsync(dw, g.d_c, wb, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

int cats_linear_backward_dev(const float *dout, const float *w, float *din, int batch, int in, int out, void *stream)
{
    const char *what = "cats_linear_backward_dev";
    if (!ensure_init()) return g.last_err;
    if (!dout || !w || !din || batch <= 0 || in <= 0 || out <= 0) return fail(CATS_ERR_ARG, what);
    // dIn = dOut * W (gemm_rnn(batch, in, out), catseye.h:466)
    return cats_sgemm_dev('N', 'N', batch, in, out, 1.f, dout, out, w, in, 0.f, din, in,
                          stream ? (cudaStream_t)stream : g.stream);
}

void cats_linear_backward(const float *dout, const float *w, float *din, int batch, int in, int out)
{
    const char *what = "cats_linear_backward";
    if (!ensure_init()) return;
    if (!dout || !w || !din || batch <= 0 || in <= 0 || out <= 0) { fail(CATS_ERR_ARG, what); return; }
    const size_t ob = (size_t)batch * out * 4, wb = (size_t)in * out * 4, ib = (size_t)batch * in * 4;
    if (grow((void **)&g.d_a, &g.cap_a, ob) || grow((void **)&g.d_b, &g.cap_b, wb) || grow((void **)&g.d_c, &g.cap_c, ib))
        return;
    if (check(cudaMemcpyAsync(g.d_a, dout, ob, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(cudaMemcpyAsync(g.d_b, w, wb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (cats_linear_backward_dev(g.d_a, g.d_b, g.d_c, batch, in, out, g.stream)) return;
    if (check(cudaMemcpyAsync(din, g.d_c, ib, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

int cats_linear_update_dev(const float *dout, const float *x, float *w, float *dw, int batch, int in, int out,
                           float eta, void *stream)
{
    const char *what = "cats_linear_update_dev";
    if (!ensure_init()) return g.last_err;
    if (!dout || !x || !w || !dw || batch <= 0 || in <= 0 || out <= 0) return fail(CATS_ERR_ARG, what);
    cudaStream_t st = stream ? (cudaStream_t)stream : g.stream;
    // dw += dOut^T x (gemm_rtn(out, in, batch, 1, dOut, x, 1, dw), catseye.h:490)
    if (int rc = cats_sgemm_dev('T', 'N', out, in, batch, 1.f, dout, out, x, in, 1.f, dw, in, st)) return rc;
    // the bias after the weights: w[in*out + o] -= eta * dOut[b][o], sample after sample (:494-496)
    return check(launch_bias_update(w + (size_t)in * out, dout, batch, out, eta, st), what);
}

void cats_linear_update(const float *dout, const float *x, float *w, float *dw, int batch, int in, int out, float eta)
{
    const char *what = "cats_linear_update";
    if (!ensure_init()) return;
    if (!dout || !x || !w || !dw || batch <= 0 || in <= 0 || out <= 0) { fail(CATS_ERR_ARG, what); return; }
    const size_t ob = (size_t)batch * out * 4, xb = (size_t)batch * in * 4, wb = ((size_t)in * out + out) * 4,
                 db = (size_t)in * out * 4;
    if (grow((void **)&g.d_a, &g.cap_a, ob) || grow((void **)&g.d_b, &g.cap_b, xb) ||
        grow((void **)&g.d_c, &g.cap_c, wb) || grow((void **)&g.d_d, &g.cap_d, db))
        return;
    if (check(cudaMemcpyAsync(g.d_a, dout, ob, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(cudaMemcpyAsync(g.d_b, x, xb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(cudaMemcpyAsync(g.d_c, w, wb, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (check(cudaMemcpyAsync(g.d_d, dw, db, cudaMemcpyHostToDevice, g.stream), what)) return;
    if (cats_linear_update_dev(g.d_a, g.d_b, g.d_c, g.d_d, batch, in, out, eta, g.stream)) return;
    if (check(cudaMemcpyAsync(w, g.d_c, wb, cudaMemcpyDeviceToHost, g.stream), what)) return;
    if (check(cudaMemcpyAsync(dw, g.d_d, db, cudaMemcpyDeviceToHost, g.stream), what)) return;
    check(cudaStreamSynchronize(g.stream), what);
}

} // extern "C"
