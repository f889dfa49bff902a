// loader.cu — model files straight into a device model.
//
// Reads the three formats the reference's runtime loads:
//  * GGUF v2 / v3 (cats_gguf_load, llm/catseye_llm.h:2678-2895): header,
//    key/value metadata, tensor table, data section aligned to
//    general.alignment (32 when absent);
//  * the legacy llama.cpp files, 'ggjt' version 3 (cats_ggml_load,
//    :2326-2550): seven hyperparameters, the vocabulary, then each tensor's
//    header and 32-byte-aligned data;
//  * llama2.c .bin checkpoints (cats_checkpoint_load, :2900-2993): seven
//    int32 hyperparameters, then fp32 tensors of one kind for every layer back
//    to back.
// The file is memory-mapped; every read of the header, metadata and tensor
// table is bounds-checked against the file size, and strings are kept in
// std::string or skipped, so a long metadata string cannot overrun a fixed
// buffer (the reference reads GGUF keys and string values into 64-byte
// arrays, :2653 and :2714).  The weights then go from the mapping to the GPU
// one layer at a time (llm_set_weights_layers): each rank of a
// tensor-parallel model copies only its slices of each matrix.
#include "llm.cuh"
#include "loader.cuh"
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>

namespace cats {

namespace {

constexpr uint32_t MAGIC_GGUF = 0x46554747u;   // "GGUF"
constexpr uint32_t MAGIC_GGML = 0x67676d6cu;   // 'ggml'
constexpr uint32_t MAGIC_GGMF = 0x67676d66u;   // 'ggmf'
constexpr uint32_t MAGIC_GGJT = 0x67676a74u;   // 'ggjt'
constexpr int T_F16 = 1;

// bytes of one row of n elements of a ggml type (0: a type this build cannot size)
uint64_t file_row_bytes(int type, uint64_t n)
{
    switch (type) {
    case W_F32: return n * 4;
    case T_F16: return n * 2;
    case W_Q4_0: return n % 32 ? 0 : n / 32 * 18;
    case W_Q8_0: return n % 32 ? 0 : n / 32 * 34;
    case W_Q3_K: return n % 256 ? 0 : n / 256 * 110;
    case W_Q6_K: return n % 256 ? 0 : n / 256 * 210;
    }
    return 0;
}

struct Reader {
    const uint8_t *p;
    size_t n, at = 0;
    bool ok = true;
    bool take(void *dst, size_t k)
    {
        if (!ok || k > n - at) return ok = false;
        memcpy(dst, p + at, k);
        at += k;
        return true;
    }
    bool skip(uint64_t k)
    {
        if (!ok || k > n - at) return ok = false;
        at += (size_t)k;
        return true;
    }
    template <class T> T get()
    {
        T v{};
        take(&v, sizeof v);
        return v;
    }
    // a string with a 64-bit length, at most max_len bytes
    bool str(std::string &s, uint64_t max_len)
    {
        const uint64_t len = get<uint64_t>();
        if (!ok || len > max_len || len > n - at) return ok = false;
        s.assign(reinterpret_cast<const char *>(p + at), (size_t)len);
        at += (size_t)len;
        return true;
    }
};

// GGUF value types
enum { G_U8, G_I8, G_U16, G_I16, G_U32, G_I32, G_F32, G_BOOL, G_STR, G_ARR, G_U64, G_I64, G_F64 };

int gguf_scalar_bytes(uint32_t t)
{
    switch (t) {
    case G_U8: case G_I8: case G_BOOL: return 1;
    case G_U16: case G_I16: return 2;
    case G_U32: case G_I32: case G_F32: return 4;
    case G_U64: case G_I64: case G_F64: return 8;
    }
    return 0;
}

bool fail_why(std::string *why, const std::string &msg)
{
    if (why) *why = msg;
    return false;
}

bool parse_gguf(ModelFile &f, Reader &r, std::string *why)
{
    r.get<uint32_t>();   // magic
    const uint32_t version = r.get<uint32_t>();
    if (version != 2 && version != 3) return fail_why(why, "GGUF version " + std::to_string(version) + " (2 or 3 read)");
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > (1u << 20) || n_kv > (1u << 20)) return fail_why(why, "GGUF header counts");
    uint64_t alignment = 32;
    long long ctx = 0, dim = 0, layers = 0, hidden = 0, heads = 0, kv_heads = 0;
    for (uint64_t i = 0; i < n_kv && r.ok; i++) {
        std::string key;
        if (!r.str(key, 1 << 16)) break;
        const uint32_t type = r.get<uint32_t>();
        if (type == G_STR) {
            std::string v;
            r.str(v, 1ull << 30);
        } else if (type == G_ARR) {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t cnt = r.get<uint64_t>();
            if (et == G_STR) {
                for (uint64_t k = 0; k < cnt && r.ok; k++) {
                    const uint64_t len = r.get<uint64_t>();
                    r.skip(len);
                }
            } else {
                const int sz = gguf_scalar_bytes(et);
                if (!sz || cnt > (r.n - r.at) / (uint64_t)sz) return fail_why(why, "GGUF array " + key);
                r.skip(cnt * (uint64_t)sz);
            }
        } else {
            const int sz = gguf_scalar_bytes(type);
            if (!sz) return fail_why(why, "GGUF value type of " + key);
            uint64_t u = 0;
            if (type != G_F32 && type != G_F64) {
                if (!r.take(&u, sz)) break;   // little-endian integers of any width
                if ((type == G_I8 || type == G_I16 || type == G_I32) && (u >> (8 * sz - 1)) & 1) u = 0;   // negative: ignored
            } else {
                r.skip(sz);
            }
            if (key == "llama.context_length") ctx = (long long)u;
            else if (key == "llama.embedding_length") dim = (long long)u;
            else if (key == "llama.block_count") layers = (long long)u;
            else if (key == "llama.feed_forward_length") hidden = (long long)u;
            else if (key == "llama.attention.head_count") heads = (long long)u;
            else if (key == "llama.attention.head_count_kv") kv_heads = (long long)u;
            else if (key == "general.alignment") alignment = u;
        }
    }
    if (!r.ok) return fail_why(why, "GGUF metadata runs past the end of the file");
    if (alignment == 0 || alignment > (1u << 20) || (alignment & (alignment - 1))) return fail_why(why, "GGUF alignment");
    std::vector<FileTensor> ts;
    for (uint64_t i = 0; i < n_tensors && r.ok; i++) {
        FileTensor t;
        if (!r.str(t.name, 1 << 16)) break;
        t.n_dims = (int)r.get<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) return fail_why(why, "GGUF tensor dims of " + t.name);
        for (int d = 0; d < t.n_dims; d++) t.ne[d] = r.get<uint64_t>();
        t.type = (int)r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        ts.push_back(t);
    }
    if (!r.ok) return fail_why(why, "GGUF tensor table runs past the end of the file");
    const uint64_t data = (r.at + alignment - 1) / alignment * alignment;
    for (auto &t : ts) t.offset += data;   // absolute
    f.tensors = std::move(ts);
    f.cfg.dim = (int)dim;
    f.cfg.n_layers = (int)layers;
    f.cfg.hidden = (int)hidden;
    f.cfg.n_heads = (int)heads;
    f.cfg.n_kv_heads = (int)(kv_heads ? kv_heads : heads);
    f.cfg.seq_len = (int)ctx;
    f.format = FMT_GGUF;
    return true;
}

bool parse_ggjt(ModelFile &f, Reader &r, std::string *why)
{
    const uint32_t magic = r.get<uint32_t>();
    const uint32_t version = magic == MAGIC_GGML ? 0 : r.get<uint32_t>();
    if (magic != MAGIC_GGJT || version != 3)
        return fail_why(why, "legacy ggml file: only 'ggjt' version 3 is read (its Q4_0 block is the 18-byte GGUF one)");
    uint32_t hp[7];
    for (auto &v : hp) v = r.get<uint32_t>();
    const uint32_t n_vocab = hp[0], n_embd = hp[1], n_mult = hp[2], n_head = hp[3], n_layer = hp[4];
    if (!r.ok || !n_vocab || !n_embd || !n_mult || !n_head || !n_layer) return fail_why(why, "ggjt hyperparameters");
    for (uint32_t i = 0; i < n_vocab && r.ok; i++) {   // word, then score (cats_read_vocab, type 0)
        const uint32_t len = r.get<uint32_t>();
        r.skip(len);
        r.skip(4);
    }
    while (r.ok && r.at < r.n) {
        FileTensor t;
        t.n_dims = (int)r.get<uint32_t>();
        const uint32_t name_len = r.get<uint32_t>();
        t.type = (int)r.get<uint32_t>();
        if (!r.ok || t.n_dims < 1 || t.n_dims > 4 || name_len > (1u << 16)) return fail_why(why, "ggjt tensor header");
        for (int d = 0; d < t.n_dims; d++) t.ne[d] = r.get<uint32_t>();
        if (!r.ok || name_len > r.n - r.at) return fail_why(why, "ggjt tensor header");
        t.name.assign(reinterpret_cast<const char *>(r.p + r.at), name_len);
        r.skip(name_len);
        const size_t aligned = (r.at + 31) & ~(size_t)31;
        if (aligned > r.n) return fail_why(why, "ggjt tensor data");
        r.at = aligned;
        t.offset = r.at;
        const uint64_t rb = file_row_bytes(t.type, t.ne[0]);
        if (!rb) return fail_why(why, "ggjt tensor type of " + t.name);
        uint64_t bytes = rb;
        for (int d = 1; d < t.n_dims; d++) bytes *= t.ne[d];
        if (!r.skip(bytes)) return fail_why(why, "ggjt tensor data of " + t.name + " runs past the end of the file");
        f.tensors.push_back(t);
    }
    f.cfg.dim = (int)n_embd;
    f.cfg.n_layers = (int)n_layer;
    f.cfg.n_heads = (int)n_head;
    f.cfg.n_kv_heads = (int)n_head;
    f.cfg.hidden = (int)((2 * (4 * (uint64_t)n_embd) / 3 + n_mult - 1) / n_mult * n_mult);
    f.cfg.seq_len = 2048;
    f.cfg.vocab = (int)n_vocab;
    f.format = FMT_GGJT;
    return true;
}

// llama2.c .bin: tensors at fixed offsets after the header
bool parse_bin(ModelFile &f, Reader &r, std::string *why)
{
    int32_t h[7];
    for (auto &v : h) v = r.get<int32_t>();
    if (!r.ok) return fail_why(why, "file too short for any model format");
    const long long dim = h[0], hidden = h[1], L = h[2], heads = h[3], kvh = h[4], seq = h[6];
    const long long vocab = h[5] < 0 ? -(long long)h[5] : h[5];
    if (dim <= 0 || hidden <= 0 || L <= 0 || heads <= 0 || kvh <= 0 || vocab <= 0 || seq <= 0 || dim % heads ||
        dim > (1 << 20) || hidden > (1 << 22) || L > 4096 || vocab > (1 << 24))
        return fail_why(why, "not a GGUF, ggjt or llama2.c checkpoint (bad magic or header)");
    const uint64_t kvd = (uint64_t)dim * kvh / heads;
    uint64_t at = 28;
    auto add = [&](const std::string &name, uint64_t n, uint64_t d) {
        FileTensor t;
        t.name = name;
        t.type = W_F32;
        t.n_dims = 2;
        t.ne[0] = n;
        t.ne[1] = d;
        t.offset = at;
        at += n * d * 4;
        f.tensors.push_back(t);
    };
    // the reference's read order (:2950-2978); the classifier follows the
    // final norm directly when it is not shared (vocab < 0)
    add("token_embd.weight", dim, vocab);
    for (long long l = 0; l < L; l++) add("blk." + std::to_string(l) + ".attn_norm.weight", dim, 1);
    for (long long l = 0; l < L; l++) add("blk." + std::to_string(l) + ".attn_q.weight", dim, dim);
    for (long long l = 0; l < L; l++) add("blk." + std::to_string(l) + ".attn_k.weight", dim, kvd);
    for (long long l = 0; l < L; l++) add("blk." + std::to_string(l) + ".attn_v.weight", dim, kvd);
    for (long long l = 0; l < L; l++) add("blk." + std::to_string(l) + ".attn_output.weight", dim, dim);
    for (long long l = 0; l < L; l++) add("blk." + std::to_string(l) + ".ffn_norm.weight", dim, 1);
    for (long long l = 0; l < L; l++) add("blk." + std::to_string(l) + ".ffn_gate.weight", dim, hidden);
    for (long long l = 0; l < L; l++) add("blk." + std::to_string(l) + ".ffn_down.weight", hidden, dim);
    for (long long l = 0; l < L; l++) add("blk." + std::to_string(l) + ".ffn_up.weight", dim, hidden);
    add("output_norm.weight", dim, 1);
    if (h[5] < 0) add("output.weight", dim, vocab);
    if (at > r.n) return fail_why(why, "llama2.c checkpoint shorter than its header says");
    f.cfg.dim = (int)dim;
    f.cfg.hidden = (int)hidden;
    f.cfg.n_layers = (int)L;
    f.cfg.n_heads = (int)heads;
    f.cfg.n_kv_heads = (int)kvh;
    f.cfg.vocab = (int)vocab;
    f.cfg.seq_len = (int)seq;
    f.format = FMT_BIN;
    return true;
}

// the legacy names of a ggjt file, as the GGUF names
std::string gguf_name(const std::string &n)
{
    static const char *pairs[][2] = {{"tok_embeddings.weight", "token_embd.weight"}, {"norm.weight", "output_norm.weight"},
                                     {"output.weight", "output.weight"}};
    for (auto &p : pairs) if (n == p[0]) return p[1];
    if (n.compare(0, 7, "layers.") != 0) return n;
    size_t dot = n.find('.', 7);
    if (dot == std::string::npos) return n;
    const std::string l = n.substr(7, dot - 7), rest = n.substr(dot + 1);
    static const char *parts[][2] = {{"attention.wq.weight", "attn_q.weight"}, {"attention.wk.weight", "attn_k.weight"},
                                     {"attention.wv.weight", "attn_v.weight"}, {"attention.wo.weight", "attn_output.weight"},
                                     {"attention_norm.weight", "attn_norm.weight"},
                                     {"feed_forward.w1.weight", "ffn_gate.weight"},
                                     {"feed_forward.w2.weight", "ffn_down.weight"},
                                     {"feed_forward.w3.weight", "ffn_up.weight"}, {"ffn_norm.weight", "ffn_norm.weight"}};
    for (auto &p : parts) if (rest == p[0]) return "blk." + l + "." + p[1];
    return n;
}

const FileTensor *find(const ModelFile &f, const std::string &name)
{
    for (auto &t : f.tensors) if (t.name == name) return &t;
    return nullptr;
}

uint64_t tensor_bytes(const FileTensor &t)
{
    uint64_t b = file_row_bytes(t.type, t.ne[0]);
    for (int d = 1; d < t.n_dims; d++) b *= t.ne[d];
    return b;
}

} // namespace

void model_file_close(ModelFile &f)
{
    if (f.base) munmap(const_cast<uint8_t *>(f.base), f.size);
    if (f.fd >= 0) close(f.fd);
    f.base = nullptr;
    f.fd = -1;
}

int model_file_open(const char *path, ModelFile &f, std::string *why)
{
    f = ModelFile{};
    f.fd = open(path, O_RDONLY);
    if (f.fd < 0) { if (why) *why = std::string("cannot open ") + path; return E_ARG; }
    struct stat st;
    if (fstat(f.fd, &st) != 0 || st.st_size < 8) { model_file_close(f); if (why) *why = "empty or unreadable file"; return E_ARG; }
    f.size = (size_t)st.st_size;
    void *p = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, f.fd, 0);
    if (p == MAP_FAILED) { f.base = nullptr; model_file_close(f); if (why) *why = "mmap failed"; return E_ARG; }
    f.base = static_cast<const uint8_t *>(p);
    Reader r{f.base, f.size};
    uint32_t magic = 0;
    memcpy(&magic, f.base, 4);
    bool ok = magic == MAGIC_GGUF ? parse_gguf(f, r, why)
              : (magic == MAGIC_GGJT || magic == MAGIC_GGMF || magic == MAGIC_GGML) ? parse_ggjt(f, r, why)
                                                                                 : parse_bin(f, r, why);
    if (ok && f.format == FMT_GGJT)
        for (auto &t : f.tensors) t.name = gguf_name(t.name);
    // every tensor inside the file
    for (auto &t : f.tensors) {
        if (!ok) break;
        const uint64_t b = tensor_bytes(t);
        if (b && (t.offset > f.size || b > f.size - t.offset)) {
            ok = fail_why(why, "tensor " + t.name + " runs past the end of the file");
        }
    }
    // the model's shapes and weight type from its tensors
    if (ok) {
        const FileTensor *emb = find(f, "token_embd.weight"), *q0 = find(f, "blk.0.attn_q.weight");
        if (!emb || !q0) ok = fail_why(why, "no token_embd.weight / blk.0.attn_q.weight tensor");
        else {
            if (f.format == FMT_GGUF) f.cfg.vocab = (int)emb->ne[1];
            f.cfg.wtype = q0->type;
            if (!f.cfg.seq_len) f.cfg.seq_len = 2048;
        }
    }
    if (!ok || f.cfg.dim <= 0 || f.cfg.n_layers <= 0 || f.cfg.hidden <= 0 || f.cfg.n_heads <= 0 ||
        f.cfg.n_kv_heads <= 0 || f.cfg.vocab <= 0) {
        if (ok && why) *why = "model hyperparameters missing from the file";
        model_file_close(f);
        return E_ARG;
    }
    return E_OK;
}

int model_file_load(LlmModel *m, const ModelFile &f, std::string *why)
{
    const LlmConfig &c = m->c;
    const int t = c.wtype, L = c.n_layers;
    if (t != W_F32 && t != W_Q4_0 && t != W_Q8_0) {
        if (why) *why = "layer weight type " + std::to_string(t) + " (F32, Q4_0 or Q8_0 models run on the device)";
        return E_UNSUPPORTED;
    }
    const uint64_t kvd = (uint64_t)c.dim * c.n_kv_heads / c.n_heads;
    auto tensor = [&](const std::string &name, int type, uint64_t n, uint64_t d, const FileTensor **out) -> bool {
        const FileTensor *ft = find(f, name);
        if (!ft) { if (why) *why = "missing tensor " + name; return false; }
        const uint64_t dd = ft->n_dims > 1 ? ft->ne[1] : 1;
        for (int k = 2; k < ft->n_dims; k++) if (ft->ne[k] != 1) { if (why) *why = "shape of " + name; return false; }
        if ((type >= 0 && ft->type != type) || ft->ne[0] != n || dd != d) {
            if (why) *why = "type or shape of " + name;
            return false;
        }
        *out = ft;
        return true;
    };
    // embedding rows as fp32 (the reference dequantizes a row per token, :1652; here once)
    const FileTensor *emb = find(f, "token_embd.weight");
    if (!emb || emb->ne[0] != (uint64_t)c.dim || (emb->n_dims > 1 ? emb->ne[1] : 1) != (uint64_t)c.vocab) {
        if (why) *why = "type or shape of token_embd.weight";
        return E_ARG;
    }
    std::vector<float> emb32;
    const float *embp = nullptr;
    const uint8_t *eb = f.base + emb->offset;
    const size_t ne = (size_t)c.vocab * c.dim;
    if (emb->type == W_F32) {
        embp = reinterpret_cast<const float *>(eb);
    } else if (emb->type == T_F16 || emb->type == W_Q4_0 || emb->type == W_Q8_0) {
        emb32.resize(ne);
        if (emb->type == T_F16) {
            for (size_t i = 0; i < ne; i++) {
                uint16_t hbits;
                memcpy(&hbits, eb + 2 * i, 2);
                emb32[i] = __half2float(__ushort_as_half(hbits));
            }
        } else {
            const size_t bb = emb->type == W_Q4_0 ? 18 : 34;
            for (size_t b = 0; b < ne / 32; b++) {
                const uint8_t *blk = eb + b * bb;
                uint16_t hbits;
                memcpy(&hbits, blk, 2);
                const float d = __half2float(__ushort_as_half(hbits));
                float *o = emb32.data() + b * 32;
                for (int j = 0; j < 16 && emb->type == W_Q4_0; j++) {
                    o[j] = (float)((int)(blk[2 + j] & 0xf) - 8) * d;        // _dequantize_q4_0 (:427-474)
                    o[j + 16] = (float)((int)(blk[2 + j] >> 4) - 8) * d;
                }
                for (int j = 0; j < 32 && emb->type == W_Q8_0; j++) o[j] = (float)(int8_t)blk[2 + j] * d;
            }
        }
        embp = emb32.data();
    } else {
        if (why) *why = "token_embd.weight type " + std::to_string(emb->type);
        return E_UNSUPPORTED;
    }
    std::vector<float> rms_att((size_t)L * c.dim), rms_ffn((size_t)L * c.dim);
    std::vector<const void *> lw((size_t)7 * L);
    static const char *names[7] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_down", "ffn_up"};
    const uint64_t nn[7] = {(uint64_t)c.dim, (uint64_t)c.dim, (uint64_t)c.dim, (uint64_t)c.dim, (uint64_t)c.dim,
                            (uint64_t)c.hidden, (uint64_t)c.dim};
    const uint64_t dd[7] = {(uint64_t)c.dim, kvd, kvd, (uint64_t)c.dim, (uint64_t)c.hidden, (uint64_t)c.dim,
                            (uint64_t)c.hidden};
    for (int l = 0; l < L; l++) {
        const std::string b = "blk." + std::to_string(l) + ".";
        const FileTensor *ft;
        for (int k = 0; k < 7; k++) {
            if (!tensor(b + names[k] + ".weight", t, nn[k], dd[k], &ft)) return E_ARG;
            lw[(size_t)7 * l + k] = f.base + ft->offset;
        }
        if (!tensor(b + "attn_norm.weight", W_F32, c.dim, 1, &ft)) return E_ARG;
        memcpy(rms_att.data() + (size_t)l * c.dim, f.base + ft->offset, (size_t)c.dim * 4);
        if (!tensor(b + "ffn_norm.weight", W_F32, c.dim, 1, &ft)) return E_ARG;
        memcpy(rms_ffn.data() + (size_t)l * c.dim, f.base + ft->offset, (size_t)c.dim * 4);
    }
    const FileTensor *fin;
    if (!tensor("output_norm.weight", W_F32, c.dim, 1, &fin)) return E_ARG;
    // the classifier: output.weight, else the embedding (shared, as llama2.c checkpoints do)
    const void *wcls = nullptr;
    const FileTensor *out = find(f, "output.weight");
    if (out) {
        const FileTensor *ft;
        if (!tensor("output.weight", t, c.dim, c.vocab, &ft)) {
            if (why) *why = "output.weight must have the layers' type (" + std::to_string(t) + ") on the device, not " +
                            std::to_string(out->type);
            return E_UNSUPPORTED;
        }
        wcls = f.base + ft->offset;
    } else if (emb->type == t) {
        wcls = eb;
    } else {
        if (why) *why = "no output.weight and the embedding's type differs from the layers'";
        return E_UNSUPPORTED;
    }
    return llm_set_weights_layers(m, embp, rms_att.data(), rms_ffn.data(),
                                  reinterpret_cast<const float *>(f.base + fin->offset), lw.data(), wcls);
}

} // namespace cats
