// decode.cu — persistent, cooperative decode kernel: whole tokens in one launch.
//
// Restates cats_llama2_transformer (llm/catseye_llm.h:1625-1772) for one
// B200.  One CTA per SM, launched cooperatively so every CTA is resident.
//
//  * Two producer warps (lane 0 of each) walk the weights of every layer in
//    step order (qkv, wo, w1/w3, w2 per layer, then the classifier; this
//    CTA's tiles of each)
//    and stream their (tile, segment) chunks into shared-memory rings with
//    1-D bulk copies (TMA engine, L2 evict-first).  They never wait for an
//    activation, so HBM keeps streaming through every phase boundary.
//  * Two consumer warp-groups of eight warps run the phases.  The CTA's tiles
//    of a weight are taken in pairs, one per group; each group has a ring of
//    its own (slots plus full/empty mbarriers) fed by its own producer warp,
//    so both groups dot in parallel and every ring has one consumer that
//    waits on each of its chunks in order (a group never polls a slot whose
//    previous chunk belongs to someone else, which could show it a phase that
//    has not started yet).  Between phases all CTAs meet at a grid barrier
//    (release add, acquire polls, bounded); after it each CTA stages the
//    phase's activation (rmsnorm + quantize_q8) in shared memory, with every
//    load of a thread issued before any is used.  The weight descriptors are
//    copied into shared memory at the start: a global load queued behind the
//    SM's weight copies takes microseconds.
//  * Attention (:1677-1723) is split over time into short (head, chunk)
//    items, one per warp, four timesteps' K and V rows in flight at a time,
//    online softmax; the last warp to finish a head merges its chunks.
//  * After the classifier (:1765-1770) CTA 0 turns the greedy argmax
//    (:1944-1956) into the next token and position, so `steps` tokens decode
//    with no host round trip.
//
//  * Tensor parallelism (one process and one GPU per rank): each rank runs
//    this kernel over its weight slices (llm.cu shards them).  wo and w2 give
//    partial sums of every row; a CTA keeps its rows in shared memory and, at
//    the phase's end, stores them straight into every rank's exchange buffer
//    over NVLink (peer memory mapped with CUDA IPC) as 8-byte words that
//    carry the exchange's sequence number beside the value, and moves on: no
//    fence, no flag.  Each CTA then builds its slice of the next residual
//    stream, waiting (bounded) per row until every rank's word is current and
//    adding the ranks' values in rank order, so every rank holds the same
//    residual stream bit for bit; the phase's grid barrier publishes it.  The
//    classifier rows go to every rank's logits with plain stores, the greedy
//    key is a system-scope max on every rank's word, and one counted barrier
//    across the ranks (a system-scope fence, then arrival atomics) ends the
//    token.  No collective library call, no bulk copy from peer memory, no
//    multicast.
//
// Shared memory: a fixed 1 KB header (the mbarriers at offset 0, reduction
// scratch, flags), the weight descriptors, then the two rings (group g's
// slot k at index g * stages + k), then the staged activation, then (with
// tensor parallelism) the CTA's rows to push.  The mbarriers are invalidated
// before the kernel exits.
#include "llm.cuh"
#include "mv_device.cuh"
#include <algorithm>
#include <cstdlib>

namespace cats {

constexpr int DEC_GROUPS = 2;                                 // consumer warp-groups
constexpr int DEC_GW = MV_CONSUMER_WARPS;                     // warps per group (8): R = 16 rows = 8 x 2
constexpr int DEC_WARPS = DEC_GROUPS * DEC_GW;                // 16 consumer warps
constexpr int DEC_NC = 32 * DEC_WARPS;                        // 512 consumer threads
constexpr int DEC_THREADS = DEC_NC + 32 * DEC_GROUPS;         // + one producer warp per ring
constexpr int DEC_MAX_STAGES = 16;                            // per ring (two rings)
constexpr int DEC_DEFAULT_STAGES = 4;                         // slots per ring unless tuned
constexpr int DEC_RPW = 2;                                    // rows per warp in a 16-row tile
constexpr int DEC_MAX_HS = 128;                               // head size held as one float4 per lane
constexpr int DEC_STAGE_V = 4;                                // staging loads in flight per thread (512 threads)
constexpr int DEC_STAGE_V_WIDE = 6;                           // the same without rmsnorm: the hidden vector in one pass
constexpr uint32_t DEC_HEADER = 1024;                         // mbarriers + scratch at the start of smem
constexpr uint32_t GRID_SPIN_LIMIT = 1u << 22;                // polls of ~0.5-1 us each (with a 50 ns pause): seconds at most

// One weight in the tile-chunk layout (16-row tiles, 64-unit segments).
struct WDesc {
    const uint8_t *w;
    unsigned long long tile_bytes;
    int d, units, nseg, n_tiles;
    uint32_t full_chunk, last_chunk;
    int pad[2];
};

struct DecodeArgs {
    const WDesc *wd;   // per layer: qkv, wo, w13, w2; then the classifier
    int n_wd;
    int n_layers, dim, hidden, q_dim, kv_dim, head_size, kv_mul, heads, seq_len, vocab;
    const float *emb, *rms_att, *rms_ffn, *rms_final;
    float *x, *q, *xb, *hb, *logits, *kcache, *vcache, *part;
    int *head_cnt;       // per-head arrival counters of the attention chunks (0 between phases)
    int max_splits;
    StepParams *params;
    unsigned long long *argmax;
    int *tok_log;
    int tok_cap;
    unsigned int *bar;   // grid barrier counter, zeroed before each launch
    int *abort_flag;     // set by any CTA whose bounded wait expired
    int steps;
    int stages;          // slots per ring
    uint32_t slot_bytes, xs_bytes;
    int *err;
    unsigned long long *trace;   // optional per-CTA phase timeline (globaltimer ns), trace_stride records each
    int trace_stride;
    // tensor parallelism (tp_size > 1; see TpXchg for the exchange buffers)
    int tp_size, tp_rank, vocab_off;
    unsigned int tp_epoch;                // classifier arrivals per source rank counted before this launch
    unsigned int tp_seq;                  // tag of this launch's first partial-row exchange (never 0)
    uint8_t *tp_peer[TP_MAX_RANKS];       // rank r's exchange buffer, mapped here (this rank's at tp_rank)
    unsigned long long tp_logits_off;     // byte offset of the logits in an exchange buffer
    float *x_alt;                         // the residual stream alternates between x and x_alt
    uint32_t push_bytes;                  // shared memory for the CTA's rows to push
};

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Thread 0 of each CTA records a timestamp (tracing only): globaltimer ns in
// trace[cta][k], the SM's clock64 in trace[grid + cta][k].
__device__ __forceinline__ void trace_put(const DecodeArgs &a, int &k, unsigned long long ns, long long clk)
{
    if (a.trace && threadIdx.x == 0 && k < a.trace_stride) {
        a.trace[(size_t)blockIdx.x * a.trace_stride + k] = ns;
        a.trace[(size_t)(gridDim.x + blockIdx.x) * a.trace_stride + k] = (unsigned long long)clk;
    }
    k++;
}

__device__ __forceinline__ void trace_mark(const DecodeArgs &a, int &k)
{
    trace_put(a, k, a.trace ? global_ns() : 0ull, a.trace ? clock64() : 0ll);
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_volatile_i32(const int *p)
{
    return *reinterpret_cast<const volatile int *>(p);
}

struct Smem {
    uint8_t *ring, *xs;
    uint64_t *full, *empty;
    float *red;
    volatile int *abort_s;   // hint for bounded waits: stop waiting, the kernel is unwinding
    volatile int *sync_ok;   // grid_sync's decision, written by thread 0 between its two CTA barriers
    WDesc *wd;               // the weight descriptors, copied in at the start (global reads cost microseconds)
    float *push;             // tensor parallelism: this CTA's rows of the phase, 16 per tile it owns
};

__host__ __device__ inline size_t desc_bytes(int n_wd)
{
    return round_up((size_t)n_wd * sizeof(WDesc), 128);
}

__device__ __forceinline__ Smem smem_layout(uint8_t *base, const DecodeArgs &a)
{
    Smem s;
    s.full = reinterpret_cast<uint64_t *>(base);
    s.empty = s.full + DEC_GROUPS * DEC_MAX_STAGES;
    s.red = reinterpret_cast<float *>(s.empty + DEC_GROUPS * DEC_MAX_STAGES);   // 64 floats (16 u64 keys at +32)
    s.abort_s = reinterpret_cast<volatile int *>(s.red + 64);
    s.sync_ok = s.abort_s + 1;
    s.wd = reinterpret_cast<WDesc *>(base + DEC_HEADER);
    s.ring = base + DEC_HEADER + desc_bytes(a.n_wd);
    s.xs = s.ring + (size_t)DEC_GROUPS * a.stages * a.slot_bytes;
    s.push = reinterpret_cast<float *>(s.xs + a.xs_bytes);
    return s;
}
static_assert(2 * DEC_GROUPS * DEC_MAX_STAGES * 8 + 64 * 4 + 8 <= DEC_HEADER, "smem header overflow");
static_assert(sizeof(WDesc) % 16 == 0, "descriptors are copied as 16-byte words");

size_t decode_smem_bytes(int n_wd, int stages, uint32_t slot, uint32_t xs, uint32_t push = 0)
{
    return DEC_HEADER + desc_bytes(n_wd) + (size_t)DEC_GROUPS * stages * slot + xs + push;
}

// Grid barrier among the consumer threads of every CTA.  Returns false when
// this or another CTA gave up waiting; every consumer thread of the CTA gets
// the same answer (thread 0 decides and publishes it between two CTA
// barriers), so the CTA's warps always leave the step loop together.
__device__ __forceinline__ bool grid_sync(const DecodeArgs &a, const Smem &sm, unsigned &target)
{
    named_bar_sync(1, DEC_NC);
    if (threadIdx.x == 0) {
        bool ok = *sm.abort_s == 0;
        if (ok) {
            target += gridDim.x;
            // the release covers the CTA's writes ordered before it by the CTA
            // barrier; the acquire polls make the other CTAs' writes visible
            red_release_add(a.bar, 1u);
            uint32_t i = 0;
            // 148 pollers on one line: a short pause between polls keeps their
            // traffic from slowing the weight stream and the other CTAs'
            // arrivals (measured on B200: no pause 728 tok/s, 50 ns 802, 400 ns 783)
            while (ld_acquire_u32(a.bar) < target) {
                __nanosleep(50);
                if ((++i & 63) == 0 && (i > GRID_SPIN_LIMIT || ld_volatile_i32(a.abort_flag))) {
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) {
            if (a.err) atomicOr(a.err, CATS_DEVERR_PEER_WAIT);
            atomicExch(a.abort_flag, 1);
            *sm.abort_s = 1;
        }
        *sm.sync_ok = ok ? 1 : 0;
    }
    named_bar_sync(1, DEC_NC);
    return *sm.sync_ok != 0;
}

// Tiles of a weight this CTA owns: blockIdx.x, blockIdx.x + grid, ...  They
// are processed in pairs; group g takes tile 2p+g of pair p, through its own
// ring.  The producer issues a pair's chunks alternately into the two rings
// (tile A seg 0, tile B seg 0, tile A seg 1, ...).
__device__ __forceinline__ int my_tiles(const WDesc &W)
{
    return (int)blockIdx.x < W.n_tiles ? (W.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
}

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Tagged words of the partial-row exchange: the fp32 value in the low half,
// the exchange's sequence number in the high half.  One aligned 8-byte store
// is single-copy atomic, so a reader that sees the current sequence number
// holds that exchange's value: no fence and no separate flag.
__device__ __forceinline__ unsigned long long *tp_recv(const DecodeArgs &a, int rank, int slot)
{
    return reinterpret_cast<unsigned long long *>(a.tp_peer[rank] + TpXchg::recv) + (size_t)slot * a.tp_size * a.dim;
}

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// This CTA's slice of the residual-stream rows (all CTAs together: dim).
__device__ __forceinline__ void tp_slice(int dim, int &r0, int &r1)
{
    r0 = (int)((long long)dim * blockIdx.x / gridDim.x);
    r1 = (int)((long long)dim * (blockIdx.x + 1) / gridDim.x);
}

// The exchange after wo or w2 (tensor parallelism).  The CTA's partial rows
// (sm.push, 16 per owned tile) go to every rank's slot `slot` as tagged words
// (16 consecutive threads store a tile's 128 bytes to one rank; nothing
// waits for them).  Then the CTA builds its slice of the next residual
// stream: for each of its rows it waits (bounded) until every rank's word
// carries `seq`, and xnext[row] = xcur[row] + rank 0's value + rank 1's + ...
// in rank order, so every rank computes the same sums.  The caller's grid
// barrier then publishes xnext.  Returns false when a wait gave up.
__device__ __forceinline__ bool tp_exchange(const DecodeArgs &a, const Smem &sm, const WDesc &W, int slot,
                                            unsigned seq, const float *xcur, float *xnext)
{
    constexpr int R = DEC_GW * DEC_RPW;
    named_bar_sync(1, DEC_NC);   // the CTA's rows are in shared memory
    const unsigned long long tag = (unsigned long long)seq << 32;
    if (*sm.abort_s == 0) {
        const int items = my_tiles(W) * a.tp_size * R;
        for (int it = threadIdx.x; it < items; it += DEC_NC) {
            const int q = it % R, rest = it / R;
            const int r = rest % a.tp_size, j = rest / a.tp_size;
            const int row = (blockIdx.x + j * gridDim.x) * R + q;
            if (row >= W.d) continue;
            const unsigned long long w = tag | __float_as_uint(sm.push[j * R + q]);
            tp_recv(a, r, slot)[(size_t)a.tp_rank * a.dim + row] = w;
        }
    }
    named_bar_sync(1, DEC_NC);   // sm.push is free again: it holds the gathered values below
    int r0, r1;
    tp_slice(a.dim, r0, r1);
    const int n = (r1 - r0) * a.tp_size;
    const unsigned long long *recv = tp_recv(a, a.tp_rank, slot);
    bool ok = *sm.abort_s == 0;
    for (int p = threadIdx.x; p < n && ok; p += DEC_NC) {
        const int row = r0 + p / a.tp_size, r = p % a.tp_size;
        const unsigned long long *src = recv + (size_t)r * a.dim + row;
        unsigned long long v = ld_volatile_u64(src);
        for (uint32_t i = 0; (v & 0xffffffff00000000ull) != tag; i++) {
            if ((i & 63) == 63 && (i > GRID_SPIN_LIMIT || ld_volatile_i32(a.abort_flag))) {
                ok = false;
                break;
            }
            __nanosleep(32);
            v = ld_volatile_u64(src);
        }
        sm.push[p] = __uint_as_float((uint32_t)v);
    }
    if (!ok) {
        if (a.err) atomicOr(a.err, CATS_DEVERR_PEER_WAIT);
        atomicExch(a.abort_flag, 1);
        *sm.abort_s = 1;
    }
    named_bar_sync(1, DEC_NC);
    for (int t = threadIdx.x; t < r1 - r0 && *sm.abort_s == 0; t += DEC_NC) {
        float s = __ldcg(xcur + r0 + t);
        for (int r = 0; r < a.tp_size; r++) s = __fadd_rn(s, sm.push[t * a.tp_size + r]);
        xnext[r0 + t] = s;
    }
    return *sm.abort_s == 0;
}

// Store this CTA's classifier rows (sm.push, 16 per owned tile) into every
// rank's logits at this rank's vocabulary offset.  Four consecutive threads
// write one tile's 64 bytes to one rank.
__device__ __forceinline__ void tp_push_logits(const DecodeArgs &a, const Smem &sm, const WDesc &W)
{
    constexpr int R = DEC_GW * DEC_RPW;
    const int items = my_tiles(W) * a.tp_size * (R / 4);
    for (int it = threadIdx.x; it < items; it += DEC_NC) {
        const int q = it & (R / 4 - 1), rest = it / (R / 4);
        const int r = rest % a.tp_size, j = rest / a.tp_size;
        const int row = (blockIdx.x + j * gridDim.x) * R + q * 4;
        if (row >= W.d) continue;
        float *dst = reinterpret_cast<float *>(a.tp_peer[r] + a.tp_logits_off) + a.vocab_off + row;
        const float *src = sm.push + j * R + q * 4;
        if (row + 4 <= W.d && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
            *reinterpret_cast<float4 *>(dst) = *reinterpret_cast<const float4 *>(src);
        } else {
            for (int e = 0; e < 4 && row + e < W.d; e++) dst[e] = src[e];
        }
    }
}

// The classifier's exchange among the ranks (and grid barrier of this rank's
// CTAs): push the CTA's logits rows to every rank, max the CTA's greedy key
// (thread 0's `key`) into every rank's word, publish both with a
// system-scope fence, count in on every rank, then wait until every CTA of
// every rank has counted in.  Bounded like grid_sync, with the same CTA-wide
// decision.  Once per token: the per-layer exchanges use tp_exchange.
__device__ __forceinline__ bool tp_sync(const DecodeArgs &a, const Smem &sm, unsigned &target, const WDesc &W,
                                        unsigned long long key)
{
    named_bar_sync(1, DEC_NC);   // the CTA's rows are in shared memory
    if (*sm.abort_s == 0) tp_push_logits(a, sm, W);
    named_bar_sync(1, DEC_NC);   // every store of the CTA issued
    if (threadIdx.x == 0) {
        bool ok = *sm.abort_s == 0;
        if (ok) {
            target += gridDim.x;
            for (int r = 0; key && r < a.tp_size; r++)
                asm volatile("red.relaxed.sys.global.max.u64 [%0], %1;"
                             ::"l"(a.tp_peer[r] + TpXchg::argmax), "l"(key) : "memory");
            // cumulative: orders the CTA's stores (seen by this thread through
            // the CTA barrier) before the arrivals below, for every GPU
            __threadfence_system();
            for (int r = 0; r < a.tp_size; r++)
                asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;"
                             ::"l"(reinterpret_cast<unsigned *>(a.tp_peer[r] + TpXchg::bar) + a.tp_rank) : "memory");
            const unsigned *bar = reinterpret_cast<const unsigned *>(a.tp_peer[a.tp_rank] + TpXchg::bar);
            uint32_t i = 0;
            for (int r = 0; r < a.tp_size && ok; r++) {
                while ((int)(ld_acquire_sys_u32(bar + r) - target) < 0) {
                    __nanosleep(50);
                    if ((++i & 63) == 0 && (i > GRID_SPIN_LIMIT || ld_volatile_i32(a.abort_flag))) {
                        ok = false;
                        break;
                    }
                }
            }
        }
        if (!ok) {
            if (a.err) atomicOr(a.err, CATS_DEVERR_PEER_WAIT);
            atomicExch(a.abort_flag, 1);
            *sm.abort_s = 1;
        }
        *sm.sync_ok = ok ? 1 : 0;
    }
    named_bar_sync(1, DEC_NC);
    return *sm.sync_ok != 0;
}

// Bounded wait on an mbarrier (producer: one thread) that also gives up when
// the CTA is unwinding.
__device__ __forceinline__ bool ring_wait(uint64_t *bar, uint32_t parity, const Smem &sm, int *err, int code)
{
    // no software pause: try_wait parks the thread until the phase completes
    // or a hardware time limit passes (same-box A/B 821.2 -> 823.3 tok/s)
    for (uint32_t i = 0; i < CATS_SPIN_LIMIT; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*sm.abort_s) return false;
    }
    if (err) atomicOr(err, code);
    *sm.abort_s = 1;
    return false;
}

// Warp-collective form for the consumers: every lane observes the phase (so
// each has the bulk copy's data visible), and the lanes agree on the outcome.
__device__ __forceinline__ bool ring_wait_warp(uint64_t *bar, uint32_t parity, const Smem &sm, int *err, int code)
{
    for (uint32_t i = 0; i < CATS_SPIN_LIMIT; i++) {
        const bool ok = mbar_try_wait(bar, parity);
        if (__all_sync(0xffffffffu, ok)) return true;
        if (__any_sync(0xffffffffu, *sm.abort_s != 0)) return false;
        // no software pause: try_wait already parks the warp until the phase
        // completes or a hardware time limit passes (same-box A/B 818.8 -> 821.2 tok/s)
    }
    if ((threadIdx.x & 31) == 0) {
        if (err) atomicOr(err, code);
        *sm.abort_s = 1;
    }
    __syncwarp();
    return false;
}

// Position of the next chunk in one group's ring (slot and wrap parity).
struct Ring {
    int slot;
    uint32_t phase;
};

__device__ __forceinline__ void ring_adv(Ring &r, int stages)
{
    if (++r.slot == stages) { r.slot = 0; r.phase ^= 1; }
}


// DE_PUSH: tensor parallelism's partial rows of wo / w2, kept in shared
// memory for tp_sync to push (the residual is added when they are summed).
enum DecEpi { DE_QKV, DE_ADD, DE_SWIGLU, DE_CLS, DE_PUSH };

// Residual rows (row0, row0 + 1) of tile t for this warp, read by lane 0.  A
// load queued behind the SM's weight copies takes microseconds, so these are
// issued well before the epilogue needs them: for a warp's first tile before
// the phase's activation staging, for later tiles before their dots.
__device__ __forceinline__ void residual_rows(const DecodeArgs &a, const WDesc &W, int t, float (&xr)[2])
{
    const int lane = threadIdx.x & 31, gw = (threadIdx.x >> 5) % DEC_GW;
    const int row0 = t * DEC_GW * DEC_RPW + gw * DEC_RPW;
    xr[0] = xr[1] = 0.f;
    if (lane == 0 && row0 < W.d) {
        xr[0] = __ldcg(a.x + row0);
        if (row0 + 1 < W.d) xr[1] = __ldcg(a.x + row0 + 1);
    }
}

// The first tile's residual rows of this warp (see residual_rows).
__device__ __forceinline__ void residual_first(const DecodeArgs &a, const WDesc &W, float (&xr)[2])
{
    const int grp = (threadIdx.x >> 5) / DEC_GW;
    xr[0] = xr[1] = 0.f;
    if (grp < my_tiles(W)) residual_rows(a, W, blockIdx.x + grp * gridDim.x, xr);
}

// One matvec phase for the consumer warps; `rg` is this warp's group ring.
// xr_first: the residual rows of the warp's first tile (DE_ADD only).
template <int WT>
__device__ __forceinline__ bool run_matvec(const DecodeArgs &a, const Smem &sm, const WDesc W, Ring &rg, int epi,
                                           int l, int pos, unsigned long long &best, int &tk,
                                           const float (&xr_first)[2])
{
    constexpr int R = DEC_GW * DEC_RPW;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = warp / DEC_GW, gw = warp % DEC_GW;
    const int nt = my_tiles(W);
    bool ok = true;
    // tracing: when thread 0 first had a chunk, and when it finished its last dot
    unsigned long long ns_first = 0, ns_dots = 0;
    long long ck_first = 0, ck_dots = 0;
    for (int p = 0; 2 * p + grp < nt && ok; p++) {
        const int t = blockIdx.x + (2 * p + grp) * gridDim.x;
        {
            // residual rows of a later tile: loaded now, used after the dots
            float xr[2] = {xr_first[0], xr_first[1]};
            if (p > 0 && epi == DE_ADD) residual_rows(a, W, t, xr);
            float acc[DEC_RPW] = {0.f, 0.f};
            for (int s = 0; s < W.nseg; s++) {
                const int k = grp * a.stages + rg.slot;
                if (!ring_wait_warp(&sm.full[k], rg.phase, sm, a.err, CATS_DEVERR_MBAR_FULL)) { ok = false; break; }
                if (a.trace && p == 0 && s == 0) { ns_first = global_ns(); ck_first = clock64(); }
                const int us = min(MV_SEG_UNITS, W.units - MV_SEG_UNITS * s);
                consume_chunk<WT, DEC_RPW>(sm.ring + (size_t)k * a.slot_bytes, us, s, gw, lane, W.units, sm.xs, acc);
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.empty[k]);
                ring_adv(rg, a.stages);
            }
            if (a.trace) { ns_dots = global_ns(); ck_dots = clock64(); }
            if (ok) {
                acc[0] = warp_sum(acc[0]);
                acc[1] = warp_sum(acc[1]);
                const int row0 = t * R + gw * DEC_RPW;
                if (lane == 0 && row0 < W.d) {
                    float v0 = acc[0], v1 = acc[1];
                    if (epi == DE_SWIGLU) {
                        a.hb[row0 >> 1] = v0 * (1.f / (1.f + expf(-v0))) * v1;   // silu(w1 x) * (w3 x), :1744-1752
                    } else if (epi == DE_QKV) {
                        if (row0 < a.q_dim) {
                            rope_pair(v0, v1, row0, a.head_size, pos);
                            a.q[row0] = v0;
                            a.q[row0 + 1] = v1;
                        } else {
                            const bool is_k = row0 < a.q_dim + a.kv_dim;
                            const int i = row0 - a.q_dim - (is_k ? 0 : a.kv_dim);
                            if (is_k) rope_pair(v0, v1, i, a.head_size, pos);
                            float *c = (is_k ? a.kcache : a.vcache) + ((size_t)l * a.seq_len + pos) * a.kv_dim + i;
                            c[0] = v0;
                            c[1] = v1;
                        }
                    } else if (epi == DE_ADD) {   // residual (:1731-1733, :1759-1761)
                        a.x[row0] = xr[0] + v0;
                        if (row0 + 1 < W.d) a.x[row0 + 1] = xr[1] + v1;
                    } else if (epi == DE_PUSH) {
                        float *pr = sm.push + (2 * p + grp) * R + gw * DEC_RPW;
                        pr[0] = v0;
                        pr[1] = v1;
                    } else {
                        // tensor parallelism: this rank's vocabulary rows, pushed to every rank at tp_sync
                        if (a.tp_size > 1) {
                            float *pr = sm.push + (2 * p + grp) * R + gw * DEC_RPW;
                            pr[0] = v0;
                            pr[1] = v1;
                        } else {
                            a.logits[row0] = v0;
                            if (row0 + 1 < W.d) a.logits[row0 + 1] = v1;
                        }
                        unsigned long long k = argmax_key(v0, a.vocab_off + row0);
                        if (row0 + 1 < W.d) {
                            const unsigned long long k1 = argmax_key(v1, a.vocab_off + row0 + 1);
                            k = k1 > k ? k1 : k;
                        }
                        best = k > best ? k : best;
                    }
                }
            }
        }
    }
    if (a.trace && ns_first == 0) {   // no tile for this CTA's first group: zero-length wait and dots
        ns_first = ns_dots = global_ns();
        ck_first = ck_dots = clock64();
    }
    trace_put(a, tk, ns_first, ck_first);
    trace_put(a, tk, ns_dots, ck_dots);
    return ok;
}

__device__ __forceinline__ int attn_splits(int T, int max_splits)
{
    return max(1, min(max_splits, (T + 3) / 4));
}

// Attention items (head h, time chunk s), one per warp: scores q.k/sqrt(hs)
// with K and V rows read as one float4 per lane, four timesteps in flight,
// online softmax, sum p*v; the partial (max, sum, acc) goes to part[h][s].
// The last warp to finish a head merges its chunks into xb (:1706-1722).
__device__ __forceinline__ void attention_phase(const DecodeArgs &a, int l, int pos)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hs = a.head_size, P = hs + 4;
    const bool mine = lane * 4 < hs;                 // lanes holding 4 dims of the head
    const int T = pos + 1;
    const int ns = attn_splits(T, a.max_splits);
    const int chunk = (T + ns - 1) / ns;
    const float rs = sqrtf((float)hs);
    const float *kc = a.kcache + (size_t)l * a.seq_len * a.kv_dim;
    const float *vc = a.vcache + (size_t)l * a.seq_len * a.kv_dim;
    const int nwarps = gridDim.x * DEC_WARPS;
    constexpr int U = 4;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int item = blockIdx.x * DEC_WARPS + warp; item < a.heads * ns; item += nwarps) {
        const int h = item / ns, s = item % ns;
        const int t0 = s * chunk, t1 = min(T, t0 + chunk);
        const int kvo = (h / a.kv_mul) * hs + lane * 4;
        const float4 qv = mine ? __ldcg(reinterpret_cast<const float4 *>(a.q + h * hs) + lane) : z4;
        float4 acc = z4;
        float m = -INFINITY, lsum = 0.f;
        for (int tb = t0; tb < t1; tb += U) {
            float4 kr[U], vr[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int t = min(tb + u, t1 - 1);   // clamped rows are loaded but not used
                kr[u] = mine ? __ldcg(reinterpret_cast<const float4 *>(kc + (size_t)t * a.kv_dim + kvo)) : z4;
                vr[u] = mine ? __ldcg(reinterpret_cast<const float4 *>(vc + (size_t)t * a.kv_dim + kvo)) : z4;
            }
            float dot[U];
#pragma unroll
            for (int u = 0; u < U; u++) dot[u] = qv.x * kr[u].x + qv.y * kr[u].y + qv.z * kr[u].z + qv.w * kr[u].w;
#pragma unroll
            for (int u = 0; u < U; u++) dot[u] = warp_sum(dot[u]);
#pragma unroll
            for (int u = 0; u < U; u++) {
                if (tb + u >= t1) break;
                const float sc = __fdiv_rn(dot[u], rs);
                const float mn = fmaxf(m, sc);
                const float corr = expf(m - mn);
                const float p = expf(sc - mn);
                lsum = lsum * corr + p;
                acc.x = acc.x * corr + p * vr[u].x;
                acc.y = acc.y * corr + p * vr[u].y;
                acc.z = acc.z * corr + p * vr[u].z;
                acc.w = acc.w * corr + p * vr[u].w;
                m = mn;
            }
        }
        float *out = a.part + ((size_t)h * a.max_splits + s) * P;
        if (lane == 0) { out[0] = t1 > t0 ? m : -INFINITY; out[1] = lsum; }
        if (mine) reinterpret_cast<float4 *>(out + 4)[lane] = acc;
        // the last arriver of head h merges the chunks
        __syncwarp();
        int prev = 0;
        if (lane == 0) {
            __threadfence();
            prev = atomicAdd(a.head_cnt + h, 1);
        }
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != ns - 1) continue;
        __threadfence();
        const float *ph = a.part + (size_t)h * a.max_splits * P;
        // chunk maxima and sums: lanes take chunks c = lane, lane + 32
        float mc[2], lc[2];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int c = lane + 32 * k;
            mc[k] = c < ns ? __ldcg(ph + (size_t)c * P) : -INFINITY;
            lc[k] = c < ns ? __ldcg(ph + (size_t)c * P + 1) : 0.f;
        }
        const float M = warp_max(fmaxf(mc[0], mc[1]));
        float L = 0.f;
#pragma unroll
        for (int k = 0; k < 2; k++) L += mc[k] == -INFINITY ? 0.f : expf(mc[k] - M) * lc[k];
        L = warp_sum(L);
        const float inv = 1.f / L;
        float4 v = z4;
        for (int c = 0; c < ns; c++) {
            const float w = __shfl_sync(0xffffffffu, c < 32 ? mc[0] : mc[1], c & 31);
            if (w == -INFINITY || !mine) continue;
            const float e = expf(w - M);
            const float4 ac = __ldcg(reinterpret_cast<const float4 *>(ph + (size_t)c * P + 4) + lane);
            v.x += e * ac.x;
            v.y += e * ac.y;
            v.z += e * ac.z;
            v.w += e * ac.w;
        }
        if (mine)
            reinterpret_cast<float4 *>(a.xb + h * hs)[lane] = make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
        if (lane == 0) a.head_cnt[h] = 0;
    }
}

// Attention for short contexts, one CTA per query head: the CTA's 16 warps
// take four timesteps each per pass (64 per pass), each with its own online
// softmax, and merge in shared memory (scratch: the staged-activation area,
// free between the qkv and wo phases).  No partials go through global memory,
// so the chain is the q/K/V loads, the dots and one CTA barrier.
constexpr int DEC_LOCAL_ATTN_MAX_T = 256;

__host__ __device__ inline uint32_t local_attn_scratch_bytes(int hs)
{
    return (uint32_t)DEC_WARPS * (hs + 4) * 4;
}

__device__ __forceinline__ void attention_local(const DecodeArgs &a, const Smem &sm, int l, int pos)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int h = blockIdx.x;
    if (h >= a.heads) return;   // the whole CTA: no head, nothing to do
    const int hs = a.head_size, P = hs + 4;
    const bool mine = lane * 4 < hs;
    const int T = pos + 1;
    const float rs = sqrtf((float)hs);
    const float *kc = a.kcache + (size_t)l * a.seq_len * a.kv_dim;
    const float *vc = a.vcache + (size_t)l * a.seq_len * a.kv_dim;
    const int kvo = (h / a.kv_mul) * hs + lane * 4;
    constexpr int U = 4;
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 qv = mine ? __ldcg(reinterpret_cast<const float4 *>(a.q + h * hs) + lane) : z4;
    float4 acc = z4;
    float m = -INFINITY, lsum = 0.f;
    for (int tb = warp * U; tb < T; tb += DEC_WARPS * U) {
        float4 kr[U], vr[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int t = min(tb + u, T - 1);   // clamped rows are loaded but not used
            kr[u] = mine ? __ldcg(reinterpret_cast<const float4 *>(kc + (size_t)t * a.kv_dim + kvo)) : z4;
            vr[u] = mine ? __ldcg(reinterpret_cast<const float4 *>(vc + (size_t)t * a.kv_dim + kvo)) : z4;
        }
        float dot[U];
#pragma unroll
        for (int u = 0; u < U; u++) dot[u] = qv.x * kr[u].x + qv.y * kr[u].y + qv.z * kr[u].z + qv.w * kr[u].w;
#pragma unroll
        for (int u = 0; u < U; u++) dot[u] = warp_sum(dot[u]);
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (tb + u >= T) break;
            const float sc = __fdiv_rn(dot[u], rs);
            const float mn = fmaxf(m, sc);
            const float corr = expf(m - mn);
            const float p = expf(sc - mn);
            lsum = lsum * corr + p;
            acc.x = acc.x * corr + p * vr[u].x;
            acc.y = acc.y * corr + p * vr[u].y;
            acc.z = acc.z * corr + p * vr[u].z;
            acc.w = acc.w * corr + p * vr[u].w;
            m = mn;
        }
    }
    // each warp's (max, sum, weighted V) into shared memory, then thread i < hs
    // merges dimension i over the warps (:1706-1722)
    float *scr = reinterpret_cast<float *>(sm.xs);
    float *mine_p = scr + (size_t)warp * P;
    if (lane == 0) { mine_p[0] = m; mine_p[1] = lsum; }
    if (mine) reinterpret_cast<float4 *>(mine_p + 4)[lane] = acc;
    named_bar_sync(1, DEC_NC);
    if (tid < hs) {
        float M = -INFINITY;
        for (int w = 0; w < DEC_WARPS; w++) M = fmaxf(M, scr[w * P]);
        float L = 0.f, v = 0.f;
        for (int w = 0; w < DEC_WARPS; w++) {
            const float mw = scr[w * P];
            if (mw == -INFINITY) continue;
            const float e = expf(mw - M);
            L += e * scr[w * P + 1];
            v += e * scr[w * P + 4 + tid];
        }
        a.xb[h * hs + tid] = v / L;
    }
}

// Producer of group g's ring (lane 0 of producer warp g): streams the chunks
// of the group's tiles (tile 2p + g of every pair p of every weight, step
// after step) into the group's ring, in the order the group takes them.  The
// two producers run independently, so a group that is behind never holds
// back the other's copies.  They are separate warps: as two lanes of one warp
// (diverged, each spinning on its own ring's slots) they took turns, and a
// phase's first chunk waited 0.53 us after staging instead of 0.43 (7B Q4_0
// decode on B200, same-box A/B: 801 -> 818 tok/s).
__device__ __forceinline__ void produce(const DecodeArgs &a, const Smem &sm, int g)
{
    const uint64_t pol = l2_evict_first_policy();
    Ring r{0, 0};
    uint32_t issued = 0, parity = 0;   // per slot of this ring: ever used, parity of its last phase
    bool ok = true;
    for (int step = 0; step < a.steps && ok; step++) {
        for (int wi = 0; wi < a.n_wd && ok; wi++) {
            const WDesc W = sm.wd[wi];
            const int nt = my_tiles(W);
            for (int p = 0; 2 * p + g < nt && ok; p++) {
                const int t = blockIdx.x + (2 * p + g) * gridDim.x;
                for (int s = 0; s < W.nseg; s++) {
                    const uint32_t bytes = s == W.nseg - 1 ? W.last_chunk : W.full_chunk;
                    const int k = g * a.stages + r.slot;
                    if (!ring_wait(&sm.empty[k], r.phase ^ 1, sm, a.err, CATS_DEVERR_MBAR_EMPTY)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&sm.full[k], bytes);
                    bulk_g2s(sm.ring + (size_t)k * a.slot_bytes,
                             W.w + (size_t)t * W.tile_bytes + (size_t)s * W.full_chunk, bytes, &sm.full[k], pol);
                    issued |= 1u << r.slot;
                    parity = (parity & ~(1u << r.slot)) | (r.phase << r.slot);
                    ring_adv(r, a.stages);
                }
            }
        }
    }
    // Every issued copy lands before the CTA exits, also when the consumers
    // stopped early (the last phase of a slot is the only one that can be open).
    for (int s = 0; s < a.stages; s++)
        if (issued & (1u << s)) mbar_wait_bounded(&sm.full[g * a.stages + s], (parity >> s) & 1u, nullptr, 0);
}

// Consumers (16 warps).  Every consumer warp takes the same path through
// stage_act / grid_sync / tp_sync (all hold CTA barriers); only their
// broadcast decision ends it.
//
// With tensor parallelism the residual stream alternates between two buffers:
// the staging after an exchange reads one (plus every rank's partial rows)
// and CTA 0 writes the sum into the other, which no CTA reads until the next
// exchange has completed.  The partial rows alternate between two slots: a
// slot is written again only two exchanges later, after every rank has
// passed the exchange that follows its reading.
template <int WT, bool TP>
__device__ __forceinline__ void consume(const DecodeArgs &a, const Smem &sm)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr bool tp = TP;   // a separate instance: the one-GPU form keeps its registers
    Ring rg{0, 0};
    unsigned target = 0, xtarget = a.tp_epoch;
    unsigned long long best = 0ull;
    const int tid = threadIdx.x;
    const float4 *x4 = reinterpret_cast<const float4 *>(a.x);
    const float no_rows[2] = {0.f, 0.f};
    float *xcur = a.x, *xnext = a.x_alt;   // tensor parallelism: the residual stream's two buffers
    int slot = 0;                          // tensor parallelism: the slot the next partial rows go to
    unsigned seq = a.tp_seq;               // tensor parallelism: the next exchange's tag
    int tk = 0;
    // the exchange after wo / w2, then the grid barrier that publishes the new residual stream
    auto exchange = [&](const WDesc &W) -> bool {
        const bool ok = tp_exchange(a, sm, W, slot, seq, xcur, xnext);
        float *t = xcur;
        xcur = xnext;
        xnext = t;
        slot ^= 1;
        seq++;
        return grid_sync(a, sm, target) && ok;
    };
    trace_mark(a, tk);
    for (int step = 0; step < a.steps; step++) {
        const int pos = ld_volatile_i32(&a.params->pos);
        const int token = ld_volatile_i32(&a.params->token);
        if (pos < 0 || pos >= a.seq_len || token < 0 || token >= a.vocab) {
            // refused before anything is computed or written (every CTA reads the same values)
            if (blockIdx.x == 0 && tid == 0 && a.err) atomicOr(a.err, CATS_DEVERR_POS_RANGE);
            *sm.abort_s = 1;   // the producer stops streaming
            break;
        }
        bool alive = true;
        for (int l = 0; l < a.n_layers && alive; l++) {
            const WDesc *wl = sm.wd + 4 * l;
            // qkv: rmsnorm + quantize, [wq;wk;wv], RoPE, k/v into the cache
            if (l == 0)
                stage_act<WT, DEC_STAGE_V>(Float4Src{reinterpret_cast<const float4 *>(a.emb + (size_t)token * a.dim), false},
                                           a.dim, a.rms_att, blockIdx.x == 0 ? xcur : nullptr, sm.xs, sm.red, tid, DEC_NC);
            else
                stage_act<WT, DEC_STAGE_V>(Float4Src{tp ? reinterpret_cast<const float4 *>(xcur) : x4, true}, a.dim,
                                           a.rms_att + (size_t)l * a.dim, nullptr, sm.xs, sm.red, tid, DEC_NC);
            trace_mark(a, tk);
            run_matvec<WT>(a, sm, wl[0], rg, DE_QKV, l, pos, best, tk, no_rows);
            trace_mark(a, tk);
            if (!(alive = grid_sync(a, sm, target))) break;
            trace_mark(a, tk);
            float xr[2] = {0.f, 0.f};
            if (!tp) residual_first(a, wl[1], xr);   // x is final until the wo epilogue
            // short contexts: one CTA per head, merged in shared memory
            if (pos < DEC_LOCAL_ATTN_MAX_T && a.heads <= (int)gridDim.x &&
                a.xs_bytes >= local_attn_scratch_bytes(a.head_size))
                attention_local(a, sm, l, pos);
            else
                attention_phase(a, l, pos);
            trace_mark(a, tk);
            if (!(alive = grid_sync(a, sm, target))) break;
            trace_mark(a, tk);
            // wo: quantize the attention output, matvec, residual add (tensor
            // parallelism: partial rows exchanged, summed by the next staging)
            stage_act<WT, DEC_STAGE_V, false>(Float4Src{reinterpret_cast<const float4 *>(a.xb), true}, a.q_dim,
                                              nullptr, nullptr, sm.xs, sm.red, tid, DEC_NC);
            trace_mark(a, tk);
            run_matvec<WT>(a, sm, wl[1], rg, tp ? DE_PUSH : DE_ADD, l, pos, best, tk, xr);
            trace_mark(a, tk);
            if (!(alive = tp ? exchange(wl[1]) : grid_sync(a, sm, target))) break;
            trace_mark(a, tk);
            if (!tp) residual_first(a, wl[3], xr);   // x is final until the w2 epilogue
            // w1/w3 + SwiGLU
            stage_act<WT, DEC_STAGE_V>(Float4Src{tp ? reinterpret_cast<const float4 *>(xcur) : x4, true}, a.dim,
                                       a.rms_ffn + (size_t)l * a.dim, nullptr, sm.xs, sm.red, tid, DEC_NC);
            trace_mark(a, tk);
            run_matvec<WT>(a, sm, wl[2], rg, DE_SWIGLU, l, pos, best, tk, no_rows);
            trace_mark(a, tk);
            if (!(alive = grid_sync(a, sm, target))) break;
            trace_mark(a, tk);
            // w2 + residual add (the hidden vector in one pass: 4 * 6 * 512 >= 11008)
            stage_act<WT, DEC_STAGE_V_WIDE, false>(Float4Src{reinterpret_cast<const float4 *>(a.hb), true}, a.hidden,
                                                   nullptr, nullptr, sm.xs, sm.red, tid, DEC_NC);
            trace_mark(a, tk);
            run_matvec<WT>(a, sm, wl[3], rg, tp ? DE_PUSH : DE_ADD, l, pos, best, tk, xr);
            trace_mark(a, tk);
            alive = tp ? exchange(wl[3]) : grid_sync(a, sm, target);
            trace_mark(a, tk);
        }
        if (!alive) break;
        // classifier + greedy argmax
        stage_act<WT, DEC_STAGE_V>(Float4Src{tp ? reinterpret_cast<const float4 *>(xcur) : x4, true}, a.dim,
                                   a.rms_final, nullptr, sm.xs, sm.red, tid, DEC_NC);
        best = 0ull;
        trace_mark(a, tk);
        const WDesc &wc = sm.wd[4 * a.n_layers];
        run_matvec<WT>(a, sm, wc, rg, DE_CLS, 0, pos, best, tk, no_rows);
        trace_mark(a, tk);
        unsigned long long *keys = reinterpret_cast<unsigned long long *>(sm.red + 32);
        if (lane == 0) keys[warp] = best;
        named_bar_sync(1, DEC_NC);
        unsigned long long mk = 0;
        if (tid == 0) {
            for (int w = 0; w < DEC_WARPS; w++) mk = keys[w] > mk ? keys[w] : mk;
            if (mk && !tp) atomicMax(a.argmax, mk);
        }
        // tensor parallelism: the logits rows go to every rank and the key is
        // maxed into every rank's word (thread 0 holds the CTA's key)
        if (!(tp ? tp_sync(a, sm, xtarget, wc, mk) : grid_sync(a, sm, target))) break;
        if (blockIdx.x == 0 && tid == 0) {
            const unsigned long long k = atomicAdd(a.argmax, 0ull);
            int idx = 0x7fffffff - (int)(uint32_t)(k & 0xffffffffu);
            if (k == 0ull || idx < 0 || idx >= a.vocab) {
                idx = 0;
                if (a.err) atomicOr(a.err, CATS_DEVERR_TOKEN_RANGE);
            }
            StepParams *p = a.params;
            const int n = p->steps;
            if (a.tok_log && n >= 0 && n < a.tok_cap) a.tok_log[n] = idx;
            p->next = idx;
            p->token = idx;
            p->pos = pos + 1;
            p->steps = n + 1;
            *a.argmax = 0ull;
            __threadfence();
        }
        if (!grid_sync(a, sm, target)) break;
        trace_mark(a, tk);
    }
}

template <int WT, bool TP>
__global__ void __launch_bounds__(DEC_THREADS, 1) k_decode(const __grid_constant__ DecodeArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const Smem sm = smem_layout(smem, a);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    {
        const int4 *src = reinterpret_cast<const int4 *>(a.wd);
        int4 *dst = reinterpret_cast<int4 *>(sm.wd);
        const int n16 = a.n_wd * (int)(sizeof(WDesc) / 16);
        for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < DEC_GROUPS * a.stages; s++) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], DEC_GW);   // the eight warps of the ring's group
        }
        *sm.abort_s = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    __syncthreads();
    if (warp >= DEC_WARPS) {
        if (lane == 0) produce(a, sm, warp - DEC_WARPS);
    } else {
        consume<WT, TP>(a, sm);
    }
    // Every thread gets here (none returns early) once all copies have landed
    // and every arrive is done: retire the mbarriers so the next kernel on
    // this SM may use these bytes for ordinary data.
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int s = 0; s < DEC_GROUPS * a.stages; s++) {
            mbar_inval(&sm.full[s]);
            mbar_inval(&sm.empty[s]);
        }
    }
}

// ------------------------------------------------------------------- host
static WDesc to_desc(const DevWeight &W)
{
    WDesc d{};
    d.w = W.ptr;
    d.d = W.L.d;
    d.units = W.L.units;
    d.nseg = W.L.nseg;
    d.n_tiles = W.L.n_tiles;
    d.full_chunk = W.L.full_chunk;
    d.last_chunk = W.L.last_chunk;
    d.tile_bytes = W.L.tile_bytes;
    return d;
}

int decode_prepare(LlmModel *m)
{
    if (m->wdesc) return E_OK;
    const LlmConfig &c = m->c;
    if (m->head_size > DEC_MAX_HS || m->head_size % 4 || c.dim > 4 * DEC_STAGE_V * DEC_NC) return E_UNSUPPORTED;
    std::vector<WDesc> v;
    uint32_t slot = 0;
    int maxn = std::max(std::max(c.dim, m->hidden_loc), m->q_dim);
    auto add = [&](const DevWeight &w) -> bool {
        if (w.L.R != DEC_GW * DEC_RPW) return false;   // the persistent kernel consumes 16-row tiles
        v.push_back(to_desc(w));
        slot = std::max(slot, w.L.full_chunk);
        return true;
    };
    for (int l = 0; l < c.n_layers; l++)
        for (const DevWeight *w : {&m->qkv[l], &m->wo[l], &m->w13[l], &m->w2[l]})
            if (!add(*w)) return E_UNSUPPORTED;
    if (!add(m->cls)) return E_UNSUPPORTED;
    slot = (uint32_t)round_up(slot, 128);
    // the staged activations, and room for the one-CTA-per-head attention's
    // scratch (which reuses them): a sharded model's short slices would
    // otherwise leave short contexts on the split attention
    const size_t act = c.wtype == W_F32 ? (size_t)maxn * 4 : (size_t)(maxn / 32) * 40;
    const uint32_t xs = (uint32_t)round_up(std::max(act, (size_t)local_attn_scratch_bytes(m->head_size)), 128);
    // tensor parallelism: the rows of the CTA's tiles of wo / w2 (dim rows) and
    // of the classifier slice, held until they are pushed
    uint32_t push = 0;
    if (c.tp_size > 1) {
        const int R = DEC_GW * DEC_RPW, grid = matvec_num_sms();
        const int rows = std::max(c.dim, m->vocab_loc);
        const size_t tiles = (size_t)cdiv(cdiv(rows, R), grid) * R;                    // rows of the CTA's tiles
        const size_t slice = (size_t)cdiv(c.dim, grid) * c.tp_size;                    // its slice, every rank
        push = (uint32_t)round_up(std::max(tiles, slice) * 4, 128);
    }
    const size_t cap = 227 * 1024;
    const size_t fixed = decode_smem_bytes((int)v.size(), 0, slot, xs, push);
    if (fixed + (size_t)DEC_GROUPS * 2 * slot > cap) return E_UNSUPPORTED;   // at least two slots per ring
    const int fit = (int)std::min<size_t>(DEC_MAX_STAGES, (cap - fixed) / ((size_t)DEC_GROUPS * slot));
    // Four slots per ring by default: with more, the copies queued at a phase
    // boundary lengthen the chain's L2 round trips more than they feed the
    // dots (7B Q4_0 same-box A/B: 5 slots 823 tok/s, 4 slots 836, 3 slots 834;
    // 70B: 5 and 4 slots equal).  CATS_DECODE_RING_STAGES sets 2..fit instead.
    m->dec_stages = std::min(fit, DEC_DEFAULT_STAGES);
    if (const char *e = getenv("CATS_DECODE_RING_STAGES")) {
        const int s = atoi(e);
        if (s >= 2 && s <= fit) m->dec_stages = s;
    }
    m->dec_slot = slot;
    m->dec_xs = xs;
    m->dec_push = push;
    m->dec_max_splits = 64;
    // all or nothing: wdesc is set last, so a failed setup is retried in full
    void *wd = nullptr;
    const size_t part_bytes = (size_t)m->heads_loc * m->dec_max_splits * (m->head_size + 4) * 4;
    bool ok = cudaMalloc(&wd, v.size() * sizeof(WDesc)) == cudaSuccess;
    ok = ok && (m->dec_part || cudaMalloc(&m->dec_part, part_bytes) == cudaSuccess);
    ok = ok && (m->dec_bar || cudaMalloc(&m->dec_bar, 16) == cudaSuccess);
    if (!ok) {
        if (wd) cudaFree(wd);
        return E_NOMEM;
    }
    // on the model's (non-blocking) stream and waited for, before any launch reads it
    if (cudaMemcpyAsync(wd, v.data(), v.size() * sizeof(WDesc), cudaMemcpyHostToDevice, m->stream) != cudaSuccess ||
        cudaStreamSynchronize(m->stream) != cudaSuccess) {
        cudaFree(wd);
        return E_CUDA;
    }
    m->n_wdesc = (int)v.size();
    m->wdesc = wd;
    return E_OK;
}

template <int WT, bool TP>
static cudaError_t launch_decode_t(const DecodeArgs &a, size_t smem, int grid, cudaStream_t st)
{
    // the largest dynamic shared memory a CTA may take, raised once per device
    static unsigned long long attr = 0;
    cudaError_t e = once_per_device(attr, [] {
        return cudaFuncSetAttribute(k_decode<WT, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    });
    if (e) return e;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(DEC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeCooperative;
    attrs[0].val.cooperative = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_decode<WT, TP>, a);
}

cudaError_t decode_launch(LlmModel *m, int steps, int *tok_log, int tok_cap, unsigned long long *trace,
                          int trace_stride)
{
    if (steps <= 0) return cudaSuccess;
    int rc = decode_prepare(m);
    if (rc) return rc == E_NOMEM ? cudaErrorMemoryAllocation : cudaErrorInvalidValue;
    const LlmConfig &c = m->c;
    DecodeArgs a;
    a.wd = static_cast<const WDesc *>(m->wdesc);
    a.n_wd = m->n_wdesc;
    a.n_layers = c.n_layers;
    a.dim = c.dim;
    a.hidden = m->hidden_loc;
    a.q_dim = m->q_dim;
    a.kv_dim = m->kv_dim;
    a.head_size = m->head_size;
    a.kv_mul = c.n_heads / c.n_kv_heads;
    a.heads = m->heads_loc;
    a.seq_len = c.seq_len;
    a.vocab = c.vocab;
    a.emb = m->emb;
    a.rms_att = m->rms_att;
    a.rms_ffn = m->rms_ffn;
    a.rms_final = m->rms_final;
    a.x = m->x;
    a.q = m->q;
    a.xb = m->xb;
    a.hb = m->hb;
    a.logits = m->logits;
    a.kcache = m->kcache;
    a.vcache = m->vcache;
    a.part = m->dec_part;
    a.head_cnt = m->counters;
    a.max_splits = m->dec_max_splits;
    a.params = m->params;
    a.argmax = m->argmax;
    a.tok_log = tok_log;
    a.tok_cap = tok_cap;
    a.bar = m->dec_bar;
    a.abort_flag = reinterpret_cast<int *>(m->dec_bar + 1);
    a.steps = steps;
    a.stages = m->dec_stages;
    a.slot_bytes = m->dec_slot;
    a.xs_bytes = m->dec_xs;
    a.err = m->err;
    a.trace = trace;
    a.trace_stride = trace_stride;
    const int grid = matvec_num_sms();
    a.tp_size = 1;
    a.tp_rank = 0;
    a.vocab_off = 0;
    a.tp_epoch = 0;
    a.tp_seq = 1;
    a.tp_logits_off = 0;
    a.x_alt = m->x2;
    a.push_bytes = m->dec_push;
    for (int r = 0; r < TP_MAX_RANKS; r++) a.tp_peer[r] = nullptr;
    if (c.tp_size > 1) {
        if (!m->tp_p2p) return cudaErrorInvalidValue;   // sharded models need the mapped exchange buffers
        a.tp_size = c.tp_size;
        a.tp_rank = c.tp_rank;
        a.vocab_off = m->vocab_off;
        a.tp_epoch = m->tp_epoch;
        a.tp_seq = m->tp_seq;
        a.tp_logits_off = TpXchg::logits(c.tp_size, c.dim);
        for (int r = 0; r < c.tp_size; r++) a.tp_peer[r] = m->tp_peer[r];
        a.argmax = reinterpret_cast<unsigned long long *>(m->tp_xchg + TpXchg::argmax);
        a.logits = m->logits;   // inside the exchange buffer; written by the pushes
    }
    const size_t smem = decode_smem_bytes(a.n_wd, a.stages, a.slot_bytes, a.xs_bytes, a.push_bytes);
    cudaError_t e = cudaMemsetAsync(m->dec_bar, 0, 16, m->stream);
    if (e) return e;
    const bool tp = c.tp_size > 1;
    switch (c.wtype) {
    case W_F32: e = tp ? launch_decode_t<W_F32, true>(a, smem, grid, m->stream)
                       : launch_decode_t<W_F32, false>(a, smem, grid, m->stream); break;
    case W_Q4_0: e = tp ? launch_decode_t<W_Q4_0, true>(a, smem, grid, m->stream)
                        : launch_decode_t<W_Q4_0, false>(a, smem, grid, m->stream); break;
    case W_Q8_0: e = tp ? launch_decode_t<W_Q8_0, true>(a, smem, grid, m->stream)
                        : launch_decode_t<W_Q8_0, false>(a, smem, grid, m->stream); break;
    default: return cudaErrorInvalidValue;
    }
    // every step of a launch runs 2 tagged exchanges per layer and the
    // classifier's counted barrier (one arrival per CTA of every rank)
    if (e == cudaSuccess && c.tp_size > 1) {
        m->tp_epoch += (unsigned)steps * (unsigned)grid;
        m->tp_seq += (unsigned)steps * (unsigned)(2 * c.n_layers);
        if (m->tp_seq == 0) m->tp_seq = 1;   // the buffer starts zeroed: tag 0 never marks a current word
    }
    return e;
}

} // namespace cats
