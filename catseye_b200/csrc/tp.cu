// tp.cu — tensor-parallel decode across GPUs (one process per GPU) over NCCL.
//
// The sharding follows the Megatron split of the llama layer (the weight
// builder in llm.cu slices per rank): wq/wk/wv and w1/w3 by output rows
// (whole heads, hidden rows), wo and w2 by input columns on 32-block
// boundaries, the classifier by vocabulary rows.  Each rank quantizes its own
// input slice, which holds the same 32-blocks the unsharded quantize_q8
// would (llm/catseye_llm.h:155-225).  The exchange steps: one fp32 sum
// allreduce of dim floats after wo and after w2, a max allreduce of the
// greedy-argmax key, and an allgather of the vocabulary slices of the logits.
//
// The persistent kernel exchanges through peer memory instead (decode.cu):
// at connect time every rank exports one buffer with CUDA IPC, the handles
// travel once over the NCCL communicator (an allgather), and each rank maps
// every peer's buffer.  The kernels then store their partial rows straight
// into the peers' buffers over NVLink and count arrivals with system-scope
// atomics; NCCL is not called again on that path.  The mapping is refused
// (the model stays on the per-phase graph engine) when two ranks share a
// GPU: kernels that wait on each other must run on different devices.
//
// NCCL is opened when a model first connects, not linked: a process that also
// loads a framework with its own libnccl.so.2 (torch bundles a newer one) must
// end up with a single copy, and a link-time dependency loaded first would
// shadow the framework's.  An already loaded libnccl.so.2 is used as is.
#include "llm.cuh"
#include <cstdlib>
#include <cstring>
#include <dlfcn.h>
#include <vector>
#include <mutex>
#include <nccl.h>

namespace cats {

namespace {

struct NcclApi {
    bool ok = false;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
};

const NcclApi &nccl()
{
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.all_gather;
    });
    return api;
}

struct TpComm {
    ncclComm_t comm = nullptr;
};

void nccl_sum(void *ctx, float *buf, size_t n, cudaStream_t st)
{
    nccl().all_reduce(buf, buf, n, ncclFloat, ncclSum, static_cast<TpComm *>(ctx)->comm, st);
}

void nccl_max_key(void *ctx, unsigned long long *key, cudaStream_t st)
{
    nccl().all_reduce(key, key, 1, ncclUint64, ncclMax, static_cast<TpComm *>(ctx)->comm, st);
}

// in place: rank r's count floats sit at buf + r * count
void nccl_gather(void *ctx, float *buf, size_t count, int rank, cudaStream_t st)
{
    nccl().all_gather(buf + (size_t)rank * count, buf, count, ncclFloat, static_cast<TpComm *>(ctx)->comm, st);
}

// What each rank tells the others at connect time (gathered over NCCL).
struct PeerInfo {
    cudaIpcMemHandle_t handle;   // this rank's exchange buffer
    unsigned char uuid[16];      // its GPU
    int sms;                     // the persistent kernel's grid on that GPU
    int rank;
    int ok;                      // the rank allocated and exported its buffer
    int pad;
};

void unmap_peers(LlmModel *m)
{
    for (int r = 0; r < TP_MAX_RANKS; r++) {
        if (m->tp_peer[r] && m->tp_peer[r] != m->tp_xchg) cudaIpcCloseMemHandle(m->tp_peer[r]);
        m->tp_peer[r] = nullptr;
    }
    if (m->logits_own) {
        m->logits = m->logits_own;
        m->logits_own = nullptr;
    }
    if (m->tp_xchg) cudaFree(m->tp_xchg);
    m->tp_xchg = nullptr;
    m->tp_p2p = false;
}

// Export this rank's exchange buffer, gather every rank's handle and GPU, map
// the peers.  Every rank takes the same collective steps whatever happens
// locally (a rank that failed to export still joins the allgather, with
// ok = 0), so all ranks reach the same decision.  Returns E_OK also when the
// peer path is refused (m->tp_p2p stays false).
int tp_map_peers(LlmModel *m, TpComm *t)
{
    const LlmConfig &c = m->c;
    const int n = c.tp_size;
    if (n > TP_MAX_RANKS) return E_OK;   // NCCL path only
    const size_t bytes = TpXchg::bytes(n, c.dim, c.vocab);
    PeerInfo me{};
    me.rank = c.tp_rank;
    me.sms = matvec_num_sms();
    int dev = 0;
    cudaDeviceProp prop{};
    bool ok = cudaGetDevice(&dev) == cudaSuccess && cudaGetDeviceProperties(&prop, dev) == cudaSuccess;
    if (ok) memcpy(me.uuid, &prop.uuid, 16);
    ok = ok && cudaMalloc(&m->tp_xchg, bytes) == cudaSuccess;
    ok = ok && cudaMemset(m->tp_xchg, 0, bytes) == cudaSuccess;
    ok = ok && cudaIpcGetMemHandle(&me.handle, m->tp_xchg) == cudaSuccess;
    me.ok = ok ? 1 : 0;
    PeerInfo *d = nullptr;
    // (if this small allocation fails the connect fails before any collective,
    // and the caller has to tear down every rank: the others wait in NCCL)
    if (cudaMalloc(&d, sizeof(PeerInfo) * n) != cudaSuccess) return E_NOMEM;
    std::vector<PeerInfo> all(n);
    cudaError_t e = cudaMemcpyAsync(d + c.tp_rank, &me, sizeof me, cudaMemcpyHostToDevice, m->stream);
    ncclResult_t nr = nccl().all_gather(d + c.tp_rank, d, sizeof(PeerInfo), ncclUint8, t->comm, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e == cudaSuccess) e = cudaMemcpy(all.data(), d, sizeof(PeerInfo) * n, cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (nr != ncclSuccess) return E_NCCL;
    if (e != cudaSuccess) return E_CUDA;
    bool use = true;
    for (int r = 0; r < n; r++) {
        use = use && all[r].ok && all[r].rank == r && all[r].sms == me.sms;
        for (int q = 0; q < r; q++) use = use && memcmp(all[r].uuid, all[q].uuid, 16) != 0;   // distinct GPUs
    }
    if (use) {
        for (int r = 0; r < n && use; r++) {
            if (r == c.tp_rank) { m->tp_peer[r] = m->tp_xchg; continue; }
            void *p = nullptr;
            use = cudaIpcOpenMemHandle(&p, all[r].handle, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
            m->tp_peer[r] = static_cast<uint8_t *>(p);
        }
        if (!use) cudaGetLastError();
    }
    // The ranks decide together: one that could not map a peer makes all of
    // them stay on NCCL (a sum allreduce of the verdicts over the same comm).
    int *v = nullptr;
    int verdict = use ? 0 : 1;
    if (cudaMalloc(&v, 4) != cudaSuccess) { unmap_peers(m); return E_NOMEM; }
    cudaMemcpyAsync(v, &verdict, 4, cudaMemcpyHostToDevice, m->stream);   // ordered before the collective
    nr = nccl().all_reduce(v, v, 1, ncclInt32, ncclSum, t->comm, m->stream);
    e = cudaStreamSynchronize(m->stream);
    if (e == cudaSuccess) e = cudaMemcpy(&verdict, v, 4, cudaMemcpyDeviceToHost);
    cudaFree(v);
    if (nr != ncclSuccess || e != cudaSuccess || verdict != 0) {
        unmap_peers(m);
        return nr != ncclSuccess ? E_NCCL : (e != cudaSuccess ? E_CUDA : E_OK);
    }
    // the full logits land in the exchange buffer (every rank stores its rows in every peer's)
    m->logits_own = m->logits;
    m->logits = reinterpret_cast<float *>(m->tp_xchg + TpXchg::logits(n, c.dim));
    m->tp_epoch = 0;
    m->tp_seq = 1;
    m->tp_p2p = true;
    return E_OK;
}

} // namespace

// Failure-detection check on one GPU: every rank's exchange buffer is this
// rank's own, and no other rank exists.  The first exchange of a step then
// waits for arrivals that never come, gives up after its bounded wait, sets
// CATS_DEVERR_PEER_WAIT and returns; the host reports CATS_ERR_TIMEOUT.
int tp_loopback(LlmModel *m)
{
    const LlmConfig &c = m->c;
    if (c.tp_size < 2 || c.tp_size > TP_MAX_RANKS || m->comm_ctx || m->tp_xchg) return E_ARG;
    const size_t bytes = TpXchg::bytes(c.tp_size, c.dim, c.vocab);
    if (cudaMalloc(&m->tp_xchg, bytes) != cudaSuccess) return E_NOMEM;
    if (cudaMemset(m->tp_xchg, 0, bytes) != cudaSuccess) { unmap_peers(m); return E_CUDA; }
    for (int r = 0; r < c.tp_size; r++) m->tp_peer[r] = m->tp_xchg;
    m->logits_own = m->logits;
    m->logits = reinterpret_cast<float *>(m->tp_xchg + TpXchg::logits(c.tp_size, c.dim));
    m->tp_epoch = 0;
    m->tp_seq = 1;
    m->tp_p2p = true;
    return E_OK;
}

int tp_unique_id(void *out, size_t bytes)
{
    if (!out || bytes < sizeof(ncclUniqueId)) return E_ARG;
    if (!nccl().ok) return E_NCCL;
    ncclUniqueId id;
    if (nccl().get_unique_id(&id) != ncclSuccess) return E_NCCL;
    memcpy(out, &id, sizeof(id));
    return E_OK;
}

size_t tp_unique_id_bytes() { return sizeof(ncclUniqueId); }

int tp_connect(LlmModel *m, const void *id_bytes)
{
    if (!m || !id_bytes || m->c.tp_size < 2) return E_ARG;
    if (m->comm_ctx) return E_OK;
    if (!nccl().ok) return E_NCCL;
    ncclUniqueId id;
    memcpy(&id, id_bytes, sizeof(id));
    TpComm *t = new TpComm;
    if (nccl().comm_init_rank(&t->comm, m->c.tp_size, id, m->c.tp_rank) != ncclSuccess) {
        delete t;
        return E_NCCL;
    }
    m->comm_ctx = t;
    m->allreduce = nccl_sum;
    m->argmax_reduce = nccl_max_key;
    m->allgather = nccl_gather;
    if (getenv("CATS_TP_NO_P2P") && atoi(getenv("CATS_TP_NO_P2P")) == 1) return E_OK;   // same on every rank
    return tp_map_peers(m, t);
}

// Called after every graph holding NCCL calls has been destroyed.
void tp_release(LlmModel *m)
{
    unmap_peers(m);
    if (!m->comm_ctx) return;
    TpComm *t = static_cast<TpComm *>(m->comm_ctx);
    if (t->comm) nccl().comm_destroy(t->comm);
    delete t;
    m->comm_ctx = nullptr;
    m->allreduce = nullptr;
    m->argmax_reduce = nullptr;
    m->allgather = nullptr;
}

} // namespace cats
