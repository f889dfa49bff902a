// loader.cuh — model files (GGUF v2/v3, ggjt v3, llama2.c .bin) to a device model.
#pragma once
#include "llm.cuh"
#include <string>
#include <vector>

namespace cats {

enum { FMT_GGUF = 1, FMT_GGJT = 2, FMT_BIN = 3 };

struct FileTensor {
    std::string name;          // GGUF names (a ggjt file's names are mapped to them)
    int type = 0;              // ggml type
    int n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};   // ne[0]: elements per row (contiguous), ne[1]: rows
    uint64_t offset = 0;       // absolute byte offset in the file
};

struct ModelFile {
    int fd = -1;
    const uint8_t *base = nullptr;   // the whole file, memory-mapped read-only
    size_t size = 0;
    int format = 0;
    LlmConfig cfg{};                 // hyperparameters; wtype = the layer matrices' type; tp fields unset
    std::vector<FileTensor> tensors;
};

// Map and parse a model file (no GPU use).  On failure returns E_ARG and a
// reason in *why; the file is closed.
int model_file_open(const char *path, ModelFile &f, std::string *why);
void model_file_close(ModelFile &f);
// Upload the file's weights into m (allocated with the file's config, any
// tensor-parallel shard): E_UNSUPPORTED for type mixes the device model does
// not run (reason in *why).
int model_file_load(LlmModel *m, const ModelFile &f, std::string *why);

} // namespace cats
