// ref_gguf.cpp - C entry points over the reference's own GGUF loader
// (src/models/gguf_loader.cpp of drxddy/MVLM, compiled unmodified from its source tree by
// oracle/Makefile).  TEST INFRASTRUCTURE ONLY: pins the ggml type table and the tensor
// info (dims, type, data_size, offset) that the CUDA weight upload consumes.
#include <cstdint>
#include <cstring>

#include "gguf_loader.h"

extern "C" {

size_t ref_ggml_type_size(uint32_t t) { return mgpu::ggml_type_size((mgpu::GGMLType)t); }

int ref_ggml_type_block_size(uint32_t t) { return mgpu::ggml_type_block_size((mgpu::GGMLType)t); }

size_t ref_tensor_info_size(void) { return sizeof(mgpu::TensorInfo); }

// Open `path`, find tensor `name`, copy its TensorInfo (raw struct bytes) into `info_out`
// and its packed data into `data_out` (capacity `cap` bytes).  Returns data_size, or -1.
long long ref_gguf_read_tensor(const char* path, const char* name, void* info_out, void* data_out,
                               size_t cap) {
    mgpu::GGUFFile f;
    if (!mgpu::gguf_open(&f, path)) return -1;
    const mgpu::TensorInfo* t = mgpu::gguf_find_tensor(&f, name);
    if (!t) { mgpu::gguf_close(&f); return -1; }
    std::memcpy(info_out, t, sizeof(*t));
    long long n = (long long)t->data_size;
    if (data_out && (size_t)n <= cap) std::memcpy(data_out, mgpu::gguf_tensor_data(&f, t), (size_t)n);
    mgpu::gguf_close(&f);
    return n;
}

}  // extern "C"
