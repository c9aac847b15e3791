// gguf_reader.cpp — see gguf_reader.h.
#include "gguf_reader.h"

#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace fwb {

namespace {
constexpr uint32_t kMagic = 0x46554747u;  // "GGUF"
constexpr uint64_t kMaxItems = 10000000u;
constexpr uint64_t kMaxString = 64u << 20;

struct Cursor {
    const uint8_t *p, *end;
    bool bad = false;
    uint64_t take(size_t n) {
        uint64_t v = 0;
        if ((size_t)(end - p) < n) { bad = true; return 0; }
        std::memcpy(&v, p, n);
        p += n;
        return v;
    }
    std::string str() {
        uint64_t n = take(8);
        if (bad || n > kMaxString || n > (uint64_t)(end - p)) { bad = true; return {}; }
        std::string s(reinterpret_cast<const char *>(p), (size_t)n);
        p += n;
        return s;
    }
};

size_t scalar_bytes(uint32_t t) {
    switch (t) {
    case 0: case 1: case 7: return 1;   // u8 i8 bool
    case 2: case 3: return 2;           // u16 i16
    case 4: case 5: case 6: return 4;   // u32 i32 f32
    case 10: case 11: case 12: return 8;  // u64 i64 f64
    default: return 0;
    }
}

void skip_value(Cursor &c, uint32_t t, int depth) {
    if (depth > 8) { c.bad = true; return; }
    if (t == 8) { c.str(); return; }
    if (t == 9) {
        uint32_t et = (uint32_t)c.take(4);
        uint64_t n = c.take(8);
        if (c.bad || n > kMaxItems) { c.bad = true; return; }
        size_t es = scalar_bytes(et);
        if (es) {
            if (n > (uint64_t)(c.end - c.p) / es) { c.bad = true; return; }
            c.p += n * es;
            return;
        }
        for (uint64_t i = 0; i < n && !c.bad; ++i) skip_value(c, et, depth + 1);
        return;
    }
    size_t s = scalar_bytes(t);
    if (!s) { c.bad = true; return; }
    c.take(s);
}

// gguf.c:187-253 byte sizes (the subset of types with known block sizes)
int tensor_size(uint32_t type, const uint64_t *dims, uint32_t n_dims, uint64_t elems, uint64_t &bytes) {
    uint64_t bs = 1, bb = 0;
    switch (type) {
    case 0: bb = 4; break;
    case 1: bb = 2; break;
    case 24: bb = 1; break;
    case 25: bb = 2; break;
    case 26: bb = 4; break;
    case 27: bb = 8; break;
    case 28: bb = 8; break;
    case 30: bb = 2; break;
    case 2: bs = 32; bb = 18; break;
    case 3: bs = 32; bb = 20; break;
    case 6: bs = 32; bb = 22; break;
    case 7: bs = 32; bb = 24; break;
    case 8: bs = 32; bb = 34; break;
    case 9: bs = 32; bb = 40; break;
    case 10: bs = 256; bb = 84; break;
    case 11: bs = 256; bb = 110; break;
    case 12: bs = 256; bb = 144; break;
    case 13: bs = 256; bb = 176; break;
    case 14: bs = 256; bb = 210; break;
    case 15: bs = 256; bb = 292; break;
    default: bytes = 0; return 1;
    }
    if (n_dims == 0) return -1;
    if (elems == 0) { bytes = 0; return 0; }
    if (dims[0] % bs || elems % bs) return -1;
    uint64_t blocks = elems / bs;
    if (blocks > UINT64_MAX / bb) return -1;
    bytes = blocks * bb;
    return 0;
}
}  // namespace

bool ggml_block(uint32_t type, uint32_t &values, uint32_t &bytes) {
    switch (type) {
    case 0: values = 1; bytes = 4; return true;
    case 2: values = 32; bytes = 18; return true;
    case 6: values = 32; bytes = 22; return true;
    case 7: values = 32; bytes = 24; return true;
    case 8: values = 32; bytes = 34; return true;
    case 12: values = 256; bytes = 144; return true;
    case 14: values = 256; bytes = 210; return true;
    default: return false;
    }
}

GgufFile::~GgufFile() {
    if (map_) munmap(map_, size_);
    if (fd_ >= 0) close(fd_);
}

bool GgufFile::open(const std::string &path, std::string &err) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) { err = "open " + path + ": " + std::strerror(errno); return false; }
    struct stat st;
    if (fstat(fd_, &st) || st.st_size < 24) { err = "invalid or too-small file"; return false; }
    size_ = (size_t)st.st_size;
    map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (map_ == MAP_FAILED) { map_ = nullptr; err = std::string("mmap: ") + std::strerror(errno); return false; }
    Cursor c{static_cast<const uint8_t *>(map_), static_cast<const uint8_t *>(map_) + size_};
    uint32_t magic = (uint32_t)c.take(4), version = (uint32_t)c.take(4);
    uint64_t n_t = c.take(8), n_kv = c.take(8);
    if (c.bad || magic != kMagic) { err = "not a valid GGUF header"; return false; }
    if (version < 2 || version > 3 || n_t > kMaxItems || n_kv > kMaxItems) {
        err = "unsupported GGUF version/counts";
        return false;
    }
    for (uint64_t i = 0; i < n_kv; ++i) {
        Kv kv;
        kv.key = c.str();
        kv.type = (uint32_t)c.take(4);
        kv.val = c.p;
        if (c.bad) { err = "malformed metadata entry"; return false; }
        if (kv.key == "general.architecture" && kv.type == 8) {
            Cursor c2 = c;
            arch_ = c2.str();
        }
        if (kv.key == "tokenizer.ggml.tokens" && kv.type == 9) {
            Cursor c2 = c;
            c2.take(4);
            n_tokens_ = c2.take(8);
        }
        skip_value(c, kv.type, 0);
        if (c.bad) { err = "malformed metadata entry"; return false; }
        // (read only after skip_value has checked that the value lies inside the file)
        if (kv.key == "general.alignment" && (kv.type == 4 || kv.type == 5)) {
            uint32_t a;
            std::memcpy(&a, kv.val, 4);
            if (a > 0 && a <= 4096 && (a & (a - 1)) == 0) alignment_ = a;
        }
        kvs_.push_back(std::move(kv));
    }
    tensors_.resize(n_t);
    for (uint64_t i = 0; i < n_t; ++i) {
        GgufTensor &t = tensors_[i];
        t.name = c.str();
        t.n_dims = (uint32_t)c.take(4);
        if (c.bad || t.n_dims == 0 || t.n_dims > 4) { err = "malformed tensor descriptor"; return false; }
        t.n_elements = 1;
        for (uint32_t d = 0; d < t.n_dims; ++d) {
            t.dims[d] = c.take(8);
            if (t.dims[d] && t.n_elements > UINT64_MAX / t.dims[d]) { err = "invalid tensor dimensions"; return false; }
            t.n_elements *= t.dims[d];
        }
        t.type = (uint32_t)c.take(4);
        t.offset = c.take(8);
        if (c.bad) { err = "truncated tensor descriptor"; return false; }
        if (tensor_size(t.type, t.dims, t.n_dims, t.n_elements, t.bytes) < 0) {
            err = "invalid dimensions for tensor '" + t.name + "'";
            return false;
        }
    }
    uint64_t after = (uint64_t)(c.p - static_cast<const uint8_t *>(map_));
    data_offset_ = (after + alignment_ - 1) & ~((uint64_t)alignment_ - 1);
    if (data_offset_ > size_) { err = "tensor data offset outside file"; return false; }
    for (GgufTensor &t : tensors_) {
        if (t.offset > size_ - data_offset_ || t.bytes > size_ - data_offset_ - t.offset) {
            err = "tensor '" + t.name + "' outside file";
            return false;
        }
        t.data = static_cast<const uint8_t *>(map_) + data_offset_ + t.offset;
    }
    return true;
}

const GgufTensor *GgufFile::find(const std::string &name) const {
    for (const GgufTensor &t : tensors_)
        if (t.name == name) return &t;
    return nullptr;
}

const GgufFile::Kv *GgufFile::kv(const std::string &key) const {
    for (const Kv &k : kvs_)
        if (k.key == key) return &k;
    return nullptr;
}

bool GgufFile::u32(const std::string &key, uint32_t &out) const {
    const Kv *k = kv(key);
    if (!k || (k->type != 4 && k->type != 5)) return false;
    std::memcpy(&out, k->val, 4);
    return true;
}

bool GgufFile::f32(const std::string &key, float &out) const {
    const Kv *k = kv(key);
    if (!k || k->type != 6) return false;
    std::memcpy(&out, k->val, 4);
    return true;
}

// model_config.c:61-146 for the architectures configured like llama
// (model_config.c:150-159); others are rejected.
bool GgufFile::config(ModelConfig &c, std::string &err) const {
    c = ModelConfig{};
    if (arch_.empty()) { err = "missing general.architecture"; return false; }
    c.arch = arch_;
    if (arch_ != "llama" && arch_ != "mistral" && arch_ != "phi3" && arch_ != "starcoder") {
        err = "architecture '" + arch_ + "' is outside this build (llama family only)";
        return false;
    }
    const std::string a = arch_ + ".";
    if (!u32(a + "embedding_length", c.n_embd) || !c.n_embd) { err = "missing n_embd"; return false; }
    if (!u32(a + "block_count", c.n_layer) || !c.n_layer) { err = "missing n_layer"; return false; }
    if (!u32(a + "attention.head_count", c.n_head) || !c.n_head) { err = "missing n_head"; return false; }
    if (!u32(a + "attention.head_count_kv", c.n_head_kv)) c.n_head_kv = c.n_head;
    if (!u32(a + "feed_forward_length", c.n_ff)) c.n_ff = 0;
    if (!u32(a + "context_length", c.n_ctx)) c.n_ctx = 2048;
    c.head_dim = c.n_embd / c.n_head;
    if (!u32(a + "rope.dimension_count", c.n_rot)) c.n_rot = c.head_dim;
    if (!f32(a + "attention.layer_norm_rms_epsilon", c.norm_eps)) c.norm_eps = 1e-5f;
    if (c.norm_eps == 1e-5f && !f32(a + "attention.layer_norm_epsilon", c.norm_eps)) c.norm_eps = 1e-5f;
    if (!f32(a + "rope.freq_base", c.rope_freq_base)) c.rope_freq_base = 10000.f;
    if (!f32(a + "rope.scale_linear", c.rope_freq_scale)) c.rope_freq_scale = 1.f;
    if (!u32("tokenizer.ggml.token_type_count", c.n_vocab)) c.n_vocab = 0;
    if (!c.n_vocab) {
        const GgufTensor *ow = find("output.weight");
        if (!ow) ow = find("lm_head.weight");
        if (ow) c.n_vocab = (uint32_t)(ow->n_dims >= 2 ? ow->dims[1] : ow->dims[0]);
    }
    if (!c.n_vocab) c.n_vocab = (uint32_t)n_tokens_;
    if (!c.n_vocab) { err = "invalid vocabulary size"; return false; }
    return true;
}

}  // namespace fwb
