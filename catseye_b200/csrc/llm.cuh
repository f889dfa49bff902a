// llm.cuh — device-resident llama decode step built on the matvec kernel.
#pragma once
#include "matvec.cuh"
#include <cuda_fp16.h>
#include <vector>

namespace cats {

constexpr int TP_MAX_RANKS = 8;   // tensor-parallel ranks of the persistent kernel's exchange (one box)

struct DevWeight {
    WeightLayout L;
    uint8_t *ptr = nullptr;
};

struct LlmConfig {
    int dim, hidden, n_layers, n_heads, n_kv_heads, vocab, seq_len, wtype;
    int tp_rank, tp_size;   // tensor parallel shard of this process (1 GPU each)
};

// step parameters read by the graph from device memory
struct StepParams {
    int token;     // input token of this step
    int pos;       // position of this step
    int next;      // greedy argmax of the step's logits (written by the advance kernel)
    int steps;     // number of advance() calls (diagnostics)
};

// one token of a batched step (batch.cu): input token, position, KV sequence
struct BatchTok {
    int token, pos, seq, pad;
};

typedef void (*AllreduceFn)(void *ctx, float *buf, size_t count, cudaStream_t st);
typedef void (*ArgmaxReduceFn)(void *ctx, unsigned long long *key, cudaStream_t st);
typedef void (*AllgatherFn)(void *ctx, float *buf, size_t count_per_rank, int rank, cudaStream_t st);

struct LlmModel {
    LlmConfig c{};
    int q_dim = 0, kv_dim = 0, head_size = 0, hidden_loc = 0, vocab_loc = 0, vocab_off = 0;
    int kv_heads_loc = 0, heads_loc = 0, n_splits = 8;
    // weights (device)
    float *emb = nullptr;                 // [vocab][dim] fp32 (replicated)
    float *rms_att = nullptr, *rms_ffn = nullptr, *rms_final = nullptr;
    std::vector<DevWeight> qkv, wo, w13, w2;
    DevWeight cls;
    // state (device)
    float *x = nullptr, *x2 = nullptr, *delta = nullptr, *q = nullptr, *xb = nullptr, *hb = nullptr;
    float *logits = nullptr, *kcache = nullptr, *vcache = nullptr;
    float *part = nullptr;                // attention split partials
    int *counters = nullptr;              // per-head arrival counters
    unsigned long long *argmax = nullptr;
    StepParams *params = nullptr;         // device
    StepParams *params_host = nullptr;    // pinned
    float *logits_host = nullptr;         // pinned staging for the host-pointer API
    int *err = nullptr;
    cudaStream_t stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool weights_ready = false;
    int stages_cache = 0;
    // persistent decode kernel (decode.cu)
    void *wdesc = nullptr;                // device array of weight descriptors in step order
    int n_wdesc = 0;
    float *dec_part = nullptr;            // attention chunk partials [heads][max_splits][hs + 4]
    unsigned int *dec_bar = nullptr;      // [0] grid barrier counter, [1] abort flag
    int dec_stages = 0, dec_max_splits = 32;
    uint32_t dec_slot = 0, dec_xs = 0, dec_push = 0;
    // batched step (batch.cu): prefill and batched decode on the tensor cores
    int n_seqs = 1;                       // KV sequences: kcache is [seq][layer][seq_len][kv_dim]
    int bt_cap = 0;                       // tokens per batched step (0: not reserved)
    BatchTok *bt_tok = nullptr;           // device [cap]
    int2 *bt_blocks = nullptr;            // device [cap]: attention query blocks (first token, count)
    int bt_max_rows = 0;                  // query rows of the largest block of the batch set last
    float *bt_x = nullptr, *bt_delta = nullptr, *bt_y = nullptr, *bt_q = nullptr, *bt_xb = nullptr;
    float *bt_lg = nullptr;               // classifier slices [tp][T][vocab_loc]
    float *bt_logits = nullptr;           // [T][vocab]
    __half *bt_x16 = nullptr;             // the fp16 operand of the products
    float *bt_ws = nullptr;               // K-split partials of the products
    size_t bt_ws_bytes = 0;
    int *bt_next = nullptr;               // [T] greedy argmax
    int *bt_step = nullptr;               // generate loop: steps taken
    int *bt_log = nullptr;                // generate loop: [steps][T] token ids
    int bt_log_cap = 0;
    BatchTok *bt_tok_host = nullptr;      // pinned staging
    int2 *bt_blocks_host = nullptr;
    cudaGraph_t bt_graph = nullptr;
    cudaGraphExec_t bt_exec = nullptr;
    int bt_graph_T = 0;
    // tensor parallel hooks (NCCL, tp.cu), null when tp_size == 1
    AllreduceFn allreduce = nullptr;
    ArgmaxReduceFn argmax_reduce = nullptr;
    AllgatherFn allgather = nullptr;
    void *comm_ctx = nullptr;
    // Tensor parallelism inside the persistent kernel (tp.cu, decode.cu): every
    // rank's exchange buffer mapped into this process (CUDA IPC over NVLink),
    // which the ranks' kernels write with plain stores and signal with
    // system-scope atomics.  Layout of one buffer (TpXchg offsets):
    // arrival counters per source rank, the greedy-argmax key, the partial
    // rows of wo / w2 [2 slots][tp_size][dim], the full logits [vocab].
    uint8_t *tp_xchg = nullptr;           // this rank's buffer (cudaMalloc, exported)
    uint8_t *tp_peer[TP_MAX_RANKS] = {};  // rank r's buffer in this process (tp_peer[tp_rank] = tp_xchg)
    bool tp_p2p = false;                  // ranks on distinct GPUs, buffers mapped: the persistent engine may run
    unsigned int tp_epoch = 0;            // classifier arrivals per source rank counted so far (wraps)
    unsigned int tp_seq = 1;              // tag of the next partial-row exchange (wraps, never 0)
    float *logits_own = nullptr;          // the model's own logits buffer while m->logits points into tp_xchg
};

// offsets into a tensor-parallel exchange buffer (LlmModel::tp_xchg)
struct TpXchg {
    static constexpr size_t bar = 0;         // unsigned int [TP_MAX_RANKS]: classifier arrivals per source rank
    static constexpr size_t argmax = 128;    // unsigned long long: greedy key, max over every rank's rows
    static constexpr size_t recv = 256;      // u64 [2][tp_size][dim]: partial rows of wo / w2, tagged words
    static size_t logits(int tp_size, int dim) { return recv + round_up((size_t)2 * tp_size * dim * 8, 256); }
    static size_t bytes(int tp_size, int dim, int vocab) { return logits(tp_size, dim) + round_up((size_t)vocab * 4, 256); }
};

// tensor parallel (tp.cu): an NCCL unique id (made on one rank, passed to all),
// the communicator of a model's rank, and its release
int tp_unique_id(void *out, size_t bytes);
size_t tp_unique_id_bytes();
int tp_connect(LlmModel *m, const void *id_bytes);
int tp_loopback(LlmModel *m);   // every rank's exchange buffer = this rank's (failure-detection check)
void tp_release(LlmModel *m);

int llm_alloc(LlmModel *m, const LlmConfig &c);
void llm_free(LlmModel *m);
// upload weights from host blobs in the reference's layout (layer matrices back to back)
int llm_set_weights(LlmModel *m, const float *emb, const float *rms_att, const float *rms_ffn,
                    const float *rms_final, const void *wq, const void *wk, const void *wv,
                    const void *wo, const void *w1, const void *w2, const void *w3, const void *wcls);
// the same from one host pointer per tensor: layer_w[7 * l + k] for k = wq, wk,
// wv, wo, w1, w2, w3 of layer l (a loader's memory-mapped file); only this
// rank's slices of each matrix are read
int llm_set_weights_layers(LlmModel *m, const float *emb, const float *rms_att, const float *rms_ffn,
                           const float *rms_final, const void *const *layer_w, const void *wcls);
// synthetic weights generated on the device: N(0, std) then block-quantized
int llm_init_random(LlmModel *m, unsigned long long seed, float std);
// enqueue one decode step (token/pos from m->params) on m->stream (graph if captured)
cudaError_t llm_enqueue_step(LlmModel *m, bool advance);
cudaError_t llm_build_graph(LlmModel *m);
// Persistent cooperative decode: `steps` greedy tokens in one launch on
// m->stream, starting from m->params (token, pos); tok_log (device, may be
// null) receives the argmax ids.
// trace (device, may be null): [grid][trace_stride] globaltimer stamps of each
// CTA's phase boundaries (after staging, after the matvec/attention work,
// after each grid barrier).
cudaError_t decode_launch(LlmModel *m, int steps, int *tok_log, int tok_cap, unsigned long long *trace = nullptr,
                          int trace_stride = 0);
int decode_prepare(LlmModel *m);
// Time `reps` passes over every layer's matvec of one kind (0 qkv, 1 wo, 2 w13,
// 3 w2, 4 classifier) launched back to back with PDL on the model's stream, as
// in the decode step but storing into scratch.  Outputs the mean device time
// per launch (CUDA events) and the algorithmic bytes per launch.
cudaError_t llm_time_matvec(LlmModel *m, int kind, int reps, float *ms_per_launch, double *bytes_per_launch);

// Batched step (batch.cu).  Models of Q4_0/Q8_0 weights whose products the
// tensor-core path takes (batch_supported).  llm_batch_reserve allocates
// room for `cap` tokens per step and `n_seqs` KV sequences (sequence 0 is the
// one the decode engines use; a larger count reallocates the cache, keeping
// the sequences already there).  llm_batch_set validates and uploads T
// tokens (seqs may be null: all sequence 0); llm_batch_enqueue runs one step
// on the model's stream (advance: every token's argmax becomes its next input
// at pos + 1, logged into log[step][T]); llm_forward_batch is set + enqueue +
// the argmax ids (and logits [T][vocab]) copied back; llm_generate_batch
// replays a captured step `steps` times after llm_batch_set of one token per
// sequence.
bool batch_supported(const LlmModel *m);
int llm_batch_reserve(LlmModel *m, int cap, int n_seqs);
void llm_batch_free(LlmModel *m);
int llm_batch_set(LlmModel *m, const int *tokens, const int *pos, const int *seqs, int T, int *nblocks);
cudaError_t llm_batch_enqueue(LlmModel *m, int T, int nblocks, bool advance, int *log, int log_cap);
int llm_forward_batch(LlmModel *m, const int *tokens, const int *pos, const int *seqs, int T, int *next_host,
                      float *logits_host);
int llm_generate_batch(LlmModel *m, int T, int steps, int *tokens_host);
cudaError_t llm_batch_decode_enqueue(LlmModel *m, int T, int steps);
// Device time of one kind of batched product (0 qkv, 1 wo, 2 w13, 3 w2,
// 4 classifier) at T tokens: `reps` passes over every layer's weight of that
// kind, back to back on the model's stream (CUDA events).  Reports ms per
// launch, its 2*T*n*d FLOPs and its weight bytes (reference layout).
cudaError_t llm_time_product(LlmModel *m, int kind, int T, int reps, float *ms_per_launch, double *flop_per_launch,
                             double *weight_bytes_per_launch);

// generate one synthetic tensor in the reference's GGUF layout (device dst)
cudaError_t synth_tensor(uint8_t *dst, int type, int n, int d, unsigned long long seed, int tensor_id,
                         float std, float constant, cudaStream_t st);

} // namespace cats
