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
// NCCL is opened when a model first connects, not linked: a process that also
// loads a framework with its own libnccl.so.2 (torch bundles a newer one) must
// end up with a single copy, and a link-time dependency loaded first would
// shadow the framework's.  An already loaded libnccl.so.2 is used as is.
#include "llm.cuh"
#include <cstring>
#include <dlfcn.h>
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

} // namespace

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
    return E_OK;
}

// Called after every graph holding NCCL calls has been destroyed.
void tp_release(LlmModel *m)
{
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
