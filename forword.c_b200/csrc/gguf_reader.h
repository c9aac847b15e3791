// gguf_reader.h — read-only GGUF v2/v3 view (mmap) and the llama-family
// model configuration derived from it.
//
// Mirrors what forword.c derives on the host: the container parse of
// gguf.c:256-353 (header, metadata, tensor descriptors, general.alignment,
// data offset), the per-type byte sizes of gguf.c:187-253, and the
// model_config_load rules of model_config.c:61-146 (+ transformer.c:43-60 for
// the context clamp and the vocabulary fallback).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace fwb {

struct GgufTensor {
    std::string name;
    uint32_t n_dims = 0, type = 0;
    uint64_t dims[4] = {0, 0, 0, 0};
    uint64_t offset = 0, n_elements = 0, bytes = 0;
    const uint8_t *data = nullptr;  // into the mapping
};

struct ModelConfig {
    std::string arch;
    uint32_t n_vocab = 0, n_ctx = 0, n_embd = 0, n_layer = 0, n_head = 0, n_head_kv = 0;
    uint32_t n_ff = 0, head_dim = 0, n_rot = 0;
    float norm_eps = 1e-5f, rope_freq_base = 10000.f, rope_freq_scale = 1.f;
};

class GgufFile {
public:
    ~GgufFile();
    // Returns false and fills err on failure.
    bool open(const std::string &path, std::string &err);
    const GgufTensor *find(const std::string &name) const;
    bool config(ModelConfig &c, std::string &err) const;

    const std::vector<GgufTensor> &tensors() const { return tensors_; }
    size_t file_size() const { return size_; }

private:
    struct Kv {
        std::string key;
        uint32_t type;
        const uint8_t *val;
    };
    bool u32(const std::string &key, uint32_t &out) const;
    bool f32(const std::string &key, float &out) const;
    const Kv *kv(const std::string &key) const;

    int fd_ = -1;
    void *map_ = nullptr;
    size_t size_ = 0;
    uint32_t alignment_ = 32;
    uint64_t data_offset_ = 0;
    std::string arch_;
    uint64_t n_tokens_ = 0;
    std::vector<Kv> kvs_;
    std::vector<GgufTensor> tensors_;
};

// Bytes of one row block of a ggml type: (values per block, bytes per block);
// false for types this build does not compute with.
bool ggml_block(uint32_t type, uint32_t &values, uint32_t &bytes);

}  // namespace fwb
