// gguf_loader.h -- native GGUF reader + config resolver for llmdot_cuda_model_load_gguf.
#pragma once
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/llmdot_cuda.h"

namespace llmdot {

struct GgufTensor {
    std::string name;
    uint32_t type = 0, n_dims = 0;
    uint64_t dims[4] = {0, 0, 0, 0};
    uint64_t offset = 0, n_elems = 0, n_bytes = 0;
    const uint8_t *data = nullptr;  // null when the file is truncated (LoadedModel skips it)
};

struct GgufModelFile {
    void *map = nullptr;
    size_t size = 0;
    llmdot_config cfg{};
    std::vector<GgufTensor> tensors;
};

// GgufReader.Read (src/Llmdot.Core/Loading/GgufReader.cs:8-41) + ArchitectureResolver.Resolve
// (src/Llmdot.Core/Loading/ArchitectureResolver.cs:14-112), over a read-only mapping.
int gguf_open(const char *path, GgufModelFile *out);
void gguf_descs(const GgufModelFile &f, std::vector<llmdot_tensor_desc> *out);
void gguf_close(GgufModelFile *f);

}  // namespace llmdot
