/*
 * catsgpu.h — C ABI of libcatsgpu.so, the B200 (sm_100a) matrix-multiply hot
 * path for catseye.  Plain C types only; no CUDA or torch types cross this
 * boundary (streams are passed as void*, a cudaStream_t).
 *
 * Two families of entry points:
 *  - drop-ins with the reference's exact signatures and host pointers, which a
 *    catseye program binds in place of the CPU / OpenCL / OpenGL backends;
 *  - device-pointer ("_dev") entry points with the same arithmetic, for callers
 *    that keep data resident in HBM, plus the device-resident decode step.
 *
 * Errors: the drop-ins return void like the functions they replace.  Every
 * call records a sticky status readable with cats_gpu_last_error(); with
 * CATS_GPU_STRICT=1 in the environment the library prints the error and aborts.
 * Non-void entry points return that status (0 = success).
 *
 * Threading: one host thread drives the library at a time; every host-pointer
 * call is synchronous (outputs are valid on return).
 */
#ifndef CATSGPU_H
#define CATSGPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ggml type numbers, as in llm/catseye_llm.h:2557-2580 */
#define CATS_TYPE_F32  0
#define CATS_TYPE_Q4_0 2
#define CATS_TYPE_Q8_0 8
#define CATS_TYPE_Q3_K 11
#define CATS_TYPE_Q6_K 14

/* status codes */
#define CATS_OK             0
#define CATS_ERR_CUDA       1   /* a CUDA runtime call failed */
#define CATS_ERR_ARG        2   /* bad pointer, size or type, rejected before launch */
#define CATS_ERR_NOMEM      3   /* device allocation failed */
#define CATS_ERR_TIMEOUT    4   /* a bounded device-side wait gave up (kernel returned early) */
#define CATS_ERR_UNSUPPORTED 5  /* shape or type this build does not handle */
#define CATS_ERR_NOT_INIT   6   /* cats_gpu_init was not called */
#define CATS_ERR_NCCL       7   /* a collective failed */

/* ------------------------------------------------------------ lifecycle */

/* Select and initialise a device (-1: $CATS_GPU_DEVICE or 0).  Replaces
 * matmul_gpu_init (llm/gpgpu_matmul.h:24-35, called from cats_llm_malloc,
 * llm/catseye_llm.h:634-636) and sgemm_ocl_init (sgemm_ocl2.h:200-207). */
int cats_gpu_init(int device);
/* Free every device resource.  Replaces matmul_gpu_term (llm/gpgpu_matmul.h:
 * 106-112, called from cats_llm_free :641-643) and sgemm_ocl_finish
 * (sgemm_ocl2.h:262-266). */
void cats_gpu_term(void);
int cats_gpu_last_error(void);           /* sticky status of the last failing call */
void cats_gpu_clear_error(void);
const char *cats_gpu_error_string(int code);
/* device error word OR-ed by kernels whose bounded waits expired (0 = none) */
int cats_gpu_device_error(void);

/* ------------------------------------------------------ weight registry */

/* Upload and re-lay-out a weight the caller keeps alive and unchanged
 * (cats_tensor.data, llm/catseye_llm.h:527-539): [d][n] in the reference's
 * GGUF row layout.  The drop-in matmuls register on first use; calling this
 * up front moves the upload out of the first matmul. */
int cats_gpu_register_weight(const void *w, int type, int n, int d);
void cats_gpu_unregister_weight(const void *w);
/* bytes of the device copy of a registered weight (0 if unknown) */
size_t cats_gpu_weight_device_bytes(const void *w);

/* ------------------------------------------- LLM drop-ins (host pointers) */

/* matmul(xout, x, w, n, d): xout[i] = sum_j W[i][j] x[j], W row-major [d][n]
 * (MATMUL_FUNC, llm/catseye_llm.h:1519-1533; bound through gguf_matmul[] :2583
 * and cats_tensor.matmul :2839-2840, :2985-2990).  x is what the tensor's
 * quantize produced. */
void cats_gpu_matmul_f32(float *xout, void *x, void *w, int n, int d);      /* matmul_f32  :1529 */
void cats_gpu_matmul_q4_0_q8(float *xout, void *x, void *w, int n, int d);  /* matmul_q4_0_q8 :1531 */
void cats_gpu_matmul_q8_0_q8(float *xout, void *x, void *w, int n, int d);  /* GGML_TYPE_Q8_0 (:2566), no
                                                                               reference matmul: same block scheme */
/* quantize_q8 (llm/catseye_llm.h:155-225, AVX build rounding), in place like
 * the reference: n floats -> n/32 blocks of {int8 q[32]; float d}. */
void cats_gpu_quantize_q8(int8_t *q, float *x, int n);
/* _dequantize_q4_0 (llm/catseye_llm.h:483-486): row `row` of a [*][n] Q4_0
 * matrix -> n floats.  Returns 0 like the reference. */
void *cats_gpu_dequantize_q4_0(void *y, const void *x, int row, int n);
void *cats_gpu_dequantize_q8_0(void *y, const void *x, int row, int n);
/* matmul_q4_0 (llm/catseye_llm.h:880-914, MATMUL_FUNC :1530): Q4_0 weights
 * against fp32 x (the binding with quantize_null, :2593-2595): each weight
 * dequantized, products and sums in fp32.  cats_gpu_matmul_q8_0_f32 is the
 * same for Q8_0 weights (no reference counterpart). */
void cats_gpu_matmul_q4_0_f32(float *xout, void *x, void *w, int n, int d);
void cats_gpu_matmul_q8_0_f32(float *xout, void *x, void *w, int n, int d);
/* K-quants (256-element super-blocks; n % 256 == 0): matmul_q3_K_q8_K and
 * matmul_q6_K_q8_K (:1532-1533; dots :1057-1261, 1332-1511) with x as
 * quantize_q8_K made it (n/256 blocks of {int8 q[256]; float d}, 260 B);
 * quantize_q8_K (:262-296, in place like the reference); _dequantize_q3_K /
 * _dequantize_q6_K (:349-426, bound in gguf_dequantize[] :2602-2607). */
void cats_gpu_matmul_q3_K_q8_K(float *xout, void *x, void *w, int n, int d);
void cats_gpu_matmul_q6_K_q8_K(float *xout, void *x, void *w, int n, int d);
void cats_gpu_quantize_q8_K(int8_t *q, float *x, int n);
void *cats_gpu_dequantize_q3_K(void *y, const void *x, int row, int n);
void *cats_gpu_dequantize_q6_K(void *y, const void *x, int row, int n);

/* -------------------------------------- LLM device-pointer entry points */

/* d_out[d] = W x for a registered weight w (host key); d_x is a device
 * pointer to n floats (x_is_q8 = 0: quantized on the device for quantized
 * types, quantize_q8 or quantize_q8_K as the type takes) or to the quantized
 * blocks (x_is_q8 = 1: Q8 or Q8_K); x_is_q8 = 2 takes n floats as they are
 * against Q4_0/Q8_0 weights (the matmul_q4_0 binding).  stream:
 * cudaStream_t or NULL. */
int cats_gpu_matvec_dev(const void *w, float *d_out, const void *d_x, int x_is_q8, void *stream);
/* Batched product for prefill and batched decode: y[T][d] = x[T][n] * W^T
 * for a registered Q4_0 or Q8_0 weight (n a multiple of 64), i.e. T calls of
 * matmul (llm/catseye_llm.h:1531) at once, on the tensor cores: weights are
 * dequantized and activations rounded to fp16, sums accumulate in fp32
 * (normwise relative error <= 1e-3 against the exact dequantized product).
 * The _dev form takes device pointers (d_x 16-byte aligned) and a stream;
 * cats_gpu_qgemm takes host pointers and returns after the copy back. */
int cats_gpu_qgemm_dev(const void *w, const float *d_x, float *d_y, int T, void *stream);
int cats_gpu_qgemm(const void *w, const float *x, float *y, int T);
/* Tuning diagnostics of the batched product for a registered weight at T
 * tokens.  cats_gpu_qgemm_plan: plan[0..6] = token tile, K splits, CTAs of
 * the kernel resident per SM, 1 if the weights come through tensor-map
 * copies, K slices per split, and the occupancy query asked afresh with its
 * CUDA error code.  cats_gpu_qgemm_trace: runs the product once
 * (d_x device, T x n fp32; d_y device, T x d) on the library's stream, with
 * CTA (0, 0, 0) of the tensor-map-fed kernel stamping its SM clock at each
 * step of its first trace_slices K slices; trace_host receives
 * (trace_slices + 1) x 16 values: per slice k, [k*16 + 0] raw weight copy
 * issued, 1 activation copy issued, 2 raw copy seen landed, 3 fp16 stage
 * free, 4..11 producer warps 0..7 done, 12 operands ready at the MMA
 * thread, 13 its commit issued; row trace_slices: 0 start, 1 last MMA seen
 * complete, 2 epilogue done.  Zero = not stamped. */
int cats_gpu_qgemm_plan(const void *w, int T, int *plan);
int cats_gpu_qgemm_trace(const void *w, const float *d_x, float *d_y, int T, unsigned long long *trace_host,
                         int trace_slices);
/* quantize_q8 on device buffers; scalar_mode selects the plain-C build's
 * rounding (llm/catseye_llm.h:227-251). */
int cats_gpu_quantize_q8_dev(int8_t *d_q, const float *d_x, int n, int scalar_mode, void *stream);
/* dequantize `rows` rows of a reference-layout weight on the device */
int cats_gpu_dequantize_dev(int type, float *d_y, const void *d_w, int n, int rows, void *stream);

/* ------------------------------------------ LLM device-resident decode */

typedef struct cats_gpu_llm cats_gpu_llm;

typedef struct {
    int dim, hidden, n_layers, n_heads, n_kv_heads, vocab, seq_len;
    int wtype;              /* CATS_TYPE_F32 / Q4_0 / Q8_0 for wq..w3 and the classifier */
    int tp_rank, tp_size;   /* tensor-parallel shard (1 process per GPU); 0,1 = no TP */
} cats_gpu_llm_config;

/* Allocate a model on the current device (cats_llm_malloc, llm/catseye_llm.h:607-637). */
cats_gpu_llm *cats_gpu_llm_create(const cats_gpu_llm_config *cfg);
void cats_gpu_llm_destroy(cats_gpu_llm *m);
/* Upload weights from host blobs in the reference's layouts (what the
 * loaders bind, llm/catseye_llm.h:2897-2993): emb [vocab][dim] f32; norms f32;
 * wq..w3 the n_layers matrices of a kind stored back to back; wcls [vocab][dim]. */
int cats_gpu_llm_set_weights(cats_gpu_llm *m, const float *emb, const float *rms_att,
                             const float *rms_ffn, const float *rms_final, const void *wq,
                             const void *wk, const void *wv, const void *wo, const void *w1,
                             const void *w2, const void *w3, const void *wcls);
/* Model files straight to the device, the formats the reference's loaders
 * read: GGUF v2/v3 (cats_gguf_load, llm/catseye_llm.h:2678-2895), the legacy
 * llama.cpp 'ggjt' v3 files (cats_ggml_load, :2326-2550) and llama2.c .bin
 * checkpoints (cats_checkpoint_load, :2900-2993).  The file is mapped and
 * every header, metadata and tensor-table read is checked against its size
 * (the reference copies metadata strings into 64-byte buffers, :2653, :2714).
 * cats_gpu_llm_file_config parses only (no GPU) and reports the model's
 * hyperparameters: wtype is the layer matrices' ggml type, tp fields 0 / 1.
 * cats_gpu_llm_load creates the model (tp_rank of tp_size: each rank uploads
 * only its slices; seq_len 0 = the file's context) and uploads the weights a
 * layer at a time.  The device model takes F32, Q4_0 or Q8_0 layer matrices
 * with a classifier of the same type (output.weight, or the embedding when
 * the file has none); the embedding may be F32, F16, Q4_0 or Q8_0 (expanded to
 * fp32 once, exactly); norms F32.  Other mixes fail with CATS_ERR_UNSUPPORTED
 * and a reason printed once. */
int cats_gpu_llm_file_config(const char *path, cats_gpu_llm_config *cfg);
cats_gpu_llm *cats_gpu_llm_load(const char *path, int tp_rank, int tp_size, int seq_len);
/* Synthetic weights generated on the device: N(0, std) (norms = 1), then
 * block-quantized to the model's type; deterministic in seed. */
int cats_gpu_llm_init_random(cats_gpu_llm *m, unsigned long long seed, float std);
/* One decode step, cats_llama2_transformer(token, pos, m) (llm/catseye_llm.h:
 * 1625-1772): token and pos go in, the logits come back in logits_host
 * (vocab floats).  Returns logits_host, or NULL on error.  With logits_host
 * NULL it returns the model's own host copy of the logits (page-locked,
 * overwritten by the model's next step), as the reference returns its state's
 * logits array (:1772), and copies nothing more. */
float *cats_gpu_llama2_transformer(int token, int pos, cats_gpu_llm *m, float *logits_host);
/* Device-resident greedy decoding: run `steps` steps starting at (token, pos),
 * each step's argmax (sample_argmax, :1944-1956) feeding the next, with no
 * host round trip.  tokens_host (may be NULL) receives the steps' argmax ids. */
int cats_gpu_llm_generate(cats_gpu_llm *m, int token, int pos, int steps, int *tokens_host);
/* Decode engines: the persistent cooperative kernel (one launch runs whole
 * tokens; the default) or a CUDA graph of per-phase kernels chained with
 * programmatic dependent launch. */
#define CATS_ENGINE_PERSISTENT 0
#define CATS_ENGINE_GRAPH      1
int cats_gpu_llm_set_engine(cats_gpu_llm *m, int engine);
/* Tensor parallelism, one process per GPU (tp_size > 1 in the config).  The
 * model is sharded as the Megatron split of the llama layer: wq/wk/wv and
 * w1/w3 by rows (whole heads), wo and w2 by input columns on 32-block
 * boundaries, the classifier by vocabulary rows.  One rank makes an NCCL
 * unique id (cats_gpu_tp_unique_id_bytes() bytes) and the caller hands it to
 * every rank; each rank calls cats_gpu_llm_tp_connect with it (the calls of
 * all ranks must overlap: NCCL waits for every rank) before its first step.
 * With every rank on its own GPU of one box (up to 8 ranks), the connect
 * also maps every rank's exchange buffer into every other rank (CUDA IPC) and
 * the model runs the persistent kernel: after wo and after w2 each CTA stores
 * its partial rows into every rank's buffer over NVLink and counts itself in
 * with a system-scope atomic (bounded waits), and every rank adds the partial
 * rows in rank order, so all ranks keep the same residual stream; the
 * classifier rows and the greedy key reach every rank the same way.  Else
 * (ranks sharing a GPU, more than 8 ranks, or CATS_TP_NO_P2P=1 on every rank)
 * it runs the per-phase graph engine: after wo and after w2 an NCCL sum
 * allreduce of dim floats, after the classifier a max allreduce of the
 * greedy key and an allgather of the logits.  cats_gpu_llm_set_engine selects
 * either where both are possible.  Every rank feeds the same tokens and gets
 * the full logits.  The ranks must start each call within the exchange's
 * bounded wait (a few seconds) of one another.  After a bounded wait expires
 * (CATS_ERR_TIMEOUT) a sharded model's ranks are out of step: destroy and
 * recreate them. */
size_t cats_gpu_tp_unique_id_bytes(void);
int cats_gpu_tp_unique_id(void *id, size_t bytes);
int cats_gpu_llm_tp_connect(cats_gpu_llm *m, const void *id);
/* Failure-detection check of the tensor-parallel exchange on one GPU (no
 * counterpart in the reference, which has no multi-GPU path): instead of
 * connecting to other ranks, map every rank's exchange buffer to this rank's
 * own.  No other rank ever arrives, so the first step's first exchange gives
 * up after its bounded wait (seconds) and the step returns CATS_ERR_TIMEOUT
 * with the GPU context intact.  The model is unusable for decoding after it. */
int cats_gpu_llm_tp_loopback(cats_gpu_llm *m);
/* One step of the persistent engine with a phase timeline, the counterpart
 * of the reference's per-layer CATS_CHECK timings (catseye.h:2110-2117):
 * host receives [2][ctas][per_cta] stamps taken by thread 0 of each CTA:
 * globaltimer ns, then the SM's clock64, at the start of the step, after
 * staging an activation, when its first weight chunk of a matvec was ready,
 * after its last dot, after its epilogue, after attention and after each grid
 * barrier; *ctas receives the grid size (host must hold 2*148*per_cta). */
int cats_gpu_llm_trace_step(cats_gpu_llm *m, int token, int pos, unsigned long long *host, int per_cta,
                            int *ctas);
/* Batched step on the tensor cores: prefill of a prompt, and batched decode
 * of several sequences.  T tokens go through cats_llama2_transformer
 * (llm/catseye_llm.h:1625-1772) together, token t at position pos[t] of KV
 * sequence seqs[t] (seqs NULL: sequence 0, the one the single-token engines
 * use), attending to positions 0..pos[t] of its sequence.  Every weight
 * product is one tcgen05 GEMM over the T tokens with fp16 activations: the
 * reference's fp32-activation binding (matmul_q4_0 with quantize_null,
 * :880-914) up to fp16 rounding.  Q4_0/Q8_0 models whose products have
 * n % 64 == 0 and head_size % 8 == 0 (else CATS_ERR_UNSUPPORTED).
 * cats_gpu_llm_batch_reserve: room for max_tokens per step and n_seqs KV
 *   sequences (more sequences reallocate the cache, keeping those present).
 * cats_gpu_llm_forward_batch: one step; next_host (may be NULL) receives the
 *   greedy argmax per token, logits_host (may be NULL) [T][vocab].
 * cats_gpu_llm_generate_batch: greedy decoding of n sequences (sequence i
 *   starts from tokens[i] at pos[i]) for `steps` steps, one token of every
 *   sequence per step, replayed from a captured graph with no host round
 *   trip; tokens_host (may be NULL) receives [steps][n] ids.
 * cats_gpu_llm_batch_set / _batch_enqueue: upload a batch, then enqueue one
 *   step of it on the model's stream (asynchronous, for timing).
 * cats_gpu_llm_batch_enqueue_decode: `steps` greedy steps from a batch of
 *   one token per sequence set last (the loop of _generate_batch, enqueued).
 * cats_gpu_llm_time_product: device time of one kind of batched product
 *   (0 qkv, 1 wo, 2 w13, 3 w2, 4 classifier) at T tokens, `reps` passes over
 *   the layers back to back: ms, FLOPs (2*T*n*d) and weight bytes per launch. */
int cats_gpu_llm_batch_reserve(cats_gpu_llm *m, int max_tokens, int n_seqs);
int cats_gpu_llm_forward_batch(cats_gpu_llm *m, const int *tokens, const int *pos, const int *seqs, int T,
                               int *next_host, float *logits_host);
int cats_gpu_llm_generate_batch(cats_gpu_llm *m, const int *tokens, const int *pos, int n, int steps,
                                int *tokens_host);
int cats_gpu_llm_batch_set(cats_gpu_llm *m, const int *tokens, const int *pos, const int *seqs, int T);
int cats_gpu_llm_batch_enqueue(cats_gpu_llm *m);
int cats_gpu_llm_batch_enqueue_decode(cats_gpu_llm *m, int steps);
int cats_gpu_llm_time_product(cats_gpu_llm *m, int kind, int T, int reps, float *ms_per_launch,
                              double *flop_per_launch, double *weight_bytes_per_launch);
/* Asynchronous form for timing: enqueue `steps` greedy steps on the model's stream. */
int cats_gpu_llm_enqueue(cats_gpu_llm *m, int steps);
int cats_gpu_llm_set_position(cats_gpu_llm *m, int token, int pos);
int cats_gpu_llm_synchronize(cats_gpu_llm *m);
void *cats_gpu_llm_stream(cats_gpu_llm *m);
/* copies of device state for tests: logits (vocab floats) and the last argmax */
int cats_gpu_llm_logits(cats_gpu_llm *m, float *logits_host);
int cats_gpu_llm_next_token(cats_gpu_llm *m);
/* Bytes of weights one decode step streams (for roofline accounting). */
size_t cats_gpu_llm_weight_bytes(cats_gpu_llm *m);
/* Device time of one kind of matvec launch (0 qkv, 1 wo, 2 w13, 3 w2,
 * 4 classifier): `reps` passes over all layers, back to back on the model's
 * stream, timed with CUDA events.  Reports ms per launch and the algorithmic
 * bytes one launch must move (reference-layout weight + x + out). */
int cats_gpu_llm_time_matvec(cats_gpu_llm *m, int kind, int reps, float *ms_per_launch,
                             double *bytes_per_launch);
/* Write synthetic tensor `tensor_id` of the generator in the reference's GGUF
 * layout to host memory (tests regenerate the device model's weights). */
int cats_gpu_synth_tensor(void *host_dst, int type, int n, int d, unsigned long long seed,
                          int tensor_id, float std, float constant);

/* ------------------------------------------------------------ CNN sgemm */

/* C = alpha*op(A)*op(B) + beta*C, row-major, packed (lda = K|M, ldb = N|K,
 * ldc = N); ta/tb in 'N','T'.  beta == 0 does not read C.  Host pointers,
 * copied in and out per call like the reference's GPU backends.
 * Replaces sgemm_ocl (sgemm_ocl2.h:208-261) and sgemm_gl (sgemm_gl1.h:247-273). */
void cats_sgemm(char ta, char tb, int m, int n, int k, float alpha, const float *a,
                const float *b, float beta, float *c);
/* The three forms catseye.h calls (gemm_rnn / gemm_rnt / gemm_rtn, catseye.h:61-75,78-129). */
void cats_gemm_rnn(int M, int N, int K, float alpha, float *A, float *B, float beta, float *C);
void cats_gemm_rnt(int M, int N, int K, float alpha, float *A, float *B, float beta, float *C);
void cats_gemm_rtn(int M, int N, int K, float alpha, float *A, float *B, float beta, float *C);
/* Device pointers with explicit leading dimensions.  stream: the CUDA stream
 * to queue on; NULL = the library's own stream, which is ordered with the
 * legacy default stream (it starts after work queued there and later work
 * there waits for it), as are the other *_dev entry points given NULL. */
int cats_sgemm_dev(char ta, char tb, int m, int n, int k, float alpha, const float *a, int lda,
                   const float *b, int ldb, float beta, float *c, int ldc, void *stream);

/* cats_sgemm_dev for callers that cannot allocate device memory: a process
 * whose device memory another allocator already owns, or a latency-critical
 * loop that must not meet cudaMalloc's implicit device synchronisation.  It
 * has no counterpart in the reference.  Same arguments and arithmetic as
 * cats_sgemm_dev, but it allocates nothing: no cudaMalloc, no cudaFree, and
 * no call to cats_gpu_init (it runs on the current device and the given
 * stream, NULL = the default stream).  Skinny problems split K into a
 * workspace that is a fixed array compiled into the library:
 * CATS_SGEMM_NOALLOC_SCRATCH_FLOATS floats (8 MiB), held by every GPU that
 * loads the library until the process exits.  The K split is fitted to that
 * array (fewer splits, down to none), so no size is refused for it.
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and the SM count; make that first call before any
 * stream capture.  Every call shares the one array, so calls that overlap on
 * the GPU (other streams, other host threads) race on it; serialize them.
 * The call returns before the GPU work ends: a bounded wait of the
 * tensor-core kernel that gave up writes its output tile as NaN and sets a
 * bit in a status word of the current device (also a fixed array), which
 * cats_gpu_device_error() returns OR-ed in and cats_gpu_clear_error() resets. */
#define CATS_SGEMM_NOALLOC_SCRATCH_FLOATS (2 * 1024 * 1024)
int cats_sgemm_dev_noalloc(char ta, char tb, int m, int n, int k, float alpha, const float *a, int lda,
                           const float *b, int ldb, float beta, float *c, int ldc, void *stream);

/* ---- CNN forward callers of the GEMM ---------------------------------------
 * Replace im2col (catseye.h:508-532), CatsEye_convolutional_forward
 * (catseye.h:557-588) and CatsEye_linear_forward (catseye.h:416-444) for a
 * whole batch.  The plain forms take host pointers (copied in and out); the
 * _dev forms take device pointers and enqueue on `stream` (NULL: the
 * library's stream).  Sizes must be positive, ksize/stride >= 1, pad >= 0. */

/* col[(c*kh + i)*kw + j][oh][ow] = im[c][oh*sh - ph + i][ow*sw - pw + j] (0 outside). */
void cats_im2col(const float *im, int channels, int height, int width, int kh, int kw, int ph, int pw,
                 int sh, int sw, float *col);
int cats_im2col_dev(const float *im, int channels, int height, int width, int kh, int kw, int ph, int pw,
                    int sh, int sw, float *col, void *stream);
/* z[b][ch][oh*ow] = sum_k w[ch][k] * im2col(x[b])[k][oh*ow], x = [batch][ich][h][wd],
 * w = [ch][ich*ksize*ksize], no bias; oh = (h + 2*pad - ksize)/stride + 1, ow likewise.
 * One implicit GEMM over the batch (the reference runs im2col + gemm_rnn per sample).
 * The reference's 1x1 convolution multiplies x without im2col, which is the
 * same only for pad 0 and stride 1 (the only 1x1 form its layers build). */
void cats_conv2d_forward(const float *x, const float *w, float *z, int batch, int ich, int h, int wd, int ch,
                         int ksize, int pad, int stride);
int cats_conv2d_forward_dev(const float *x, const float *w, float *z, int batch, int ich, int h, int wd, int ch,
                            int ksize, int pad, int stride, void *stream);
/* z[b][o] = sum_i x[b][i] * w[o][i] + w[in*out + o] (gemm_rnt, then the bias kept after the weights). */
void cats_linear_forward(const float *x, const float *w, float *z, int batch, int in, int out);
int cats_linear_forward_dev(const float *x, const float *w, float *z, int batch, int in, int out, void *stream);

/* ---- CNN training callers of the GEMM ---------------------------------------
 * Replace col2im (catseye.h:533-556), CatsEye_convolutional_backward
 * (catseye.h:589-620), CatsEye_convolutional_update (:622-640),
 * CatsEye_linear_backward (:445-477) and CatsEye_linear_update (:478-505) for a
 * whole batch, in the layouts the reference's layers keep: x, dIn
 * [batch][ich][h][wd]; dOut [batch][ch][oh*ow] (convolution) or
 * [batch][out] (linear); w [ch][ich*k*k] or [out][in] then the out biases.
 * Plain forms take host pointers (copied in and out); _dev forms take device
 * pointers and enqueue on `stream` (NULL: the library's stream). */

/* im[c][y][x] = sum of the col entries covering it, in the reference's order
 * (the inverse gather of cats_im2col; bit-exact). */
void cats_col2im(const float *col, int channels, int height, int width, int kh, int kw, int ph, int pw, int sh,
                 int sw, float *im);
int cats_col2im_dev(const float *col, int channels, int height, int width, int kh, int kw, int ph, int pw, int sh,
                    int sw, float *im, void *stream);
/* dIn[b] = col2im(W^T dOut[b]) for every sample: one GEMM over the batch, then
 * col2im.  (For ksize 1 the reference skips col2im, which equals this only for
 * pad 0 and stride 1, the only 1x1 form its layers build.) */
void cats_conv2d_backward(const float *dout, const float *w, float *din, int batch, int ich, int h, int wd, int ch,
                          int ksize, int pad, int stride);
int cats_conv2d_backward_dev(const float *dout, const float *w, float *din, int batch, int ich, int h, int wd, int ch,
                             int ksize, int pad, int stride, void *stream);
/* dw[c][k] += (1/batch) * sum_b sum_p dOut[b][c][p] * im2col(x[b])[k][p] (the
 * reference's per-sample gemm_rnt with alpha = 1/batch, beta = 1, as one GEMM
 * whose K runs over the whole batch's pixels). */
void cats_conv2d_update(const float *dout, const float *x, float *dw, int batch, int ich, int h, int wd, int ch,
                        int ksize, int pad, int stride);
int cats_conv2d_update_dev(const float *dout, const float *x, float *dw, int batch, int ich, int h, int wd, int ch,
                           int ksize, int pad, int stride, void *stream);
/* dIn[b][i] = sum_o dOut[b][o] * w[o][i] (gemm_rnn(batch, in, out)). */
void cats_linear_backward(const float *dout, const float *w, float *din, int batch, int in, int out);
int cats_linear_backward_dev(const float *dout, const float *w, float *din, int batch, int in, int out, void *stream);
/* dw[o][i] += sum_b dOut[b][o] * x[b][i] (gemm_rtn(out, in, batch), beta = 1);
 * then the biases w[in*out + o] -= eta * dOut[b][o], sample after sample. */
void cats_linear_update(const float *dout, const float *x, float *w, float *dw, int batch, int in, int out, float eta);
int cats_linear_update_dev(const float *dout, const float *x, float *w, float *dw, int batch, int in, int out,
                           float eta, void *stream);

/* ---- the OpenCL backend's host API over this library ----------------------
 * What include/cats_ocl_cuda.h maps ocl.h's calls onto, so catseye's OpenCL
 * sgemm backend (sgemm_ocl2.h) runs unchanged on the GPU
 * (cc -DCATS_OPENCL -include cats_ocl_cuda.h ...).  cats_ocl_setup replaces
 * oclSetup (ocl.h:142-195): initialises the device and returns the size of
 * the backend's one device buffer ($CATS_OCL_BUFFER_BYTES, default 1 GiB).
 * cats_ocl_alloc / _free / _write / _read replace the buffer calls
 * (ocl.h:229-320, blocking).  cats_ocl_run replaces oclRun (ocl.h:322-355)
 * for the backend's kernels by name ("gemm_rnn", "transpose", "im2col";
 * sgemm_ocl2.h:14-169) with their int8 / float4 argument blocks; float
 * offsets into the buffer as the kernels take them. */
unsigned long cats_ocl_setup(int device);
void *cats_ocl_alloc(size_t bytes);
void cats_ocl_free(void *buf);
int cats_ocl_write(void *buf, size_t offset, size_t size, const void *host);
int cats_ocl_read(void *buf, size_t offset, size_t size, void *host);
int cats_ocl_run(const char *kernel, void *buf, const int *info, const float *param);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif
