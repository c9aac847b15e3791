// tp_shard.cpp — tensor-parallel slices of the llama block (see tp_shard.h).
#include "tp_shard.h"

#include <algorithm>
#include <cstring>

namespace fwb {


bool tp_check(const ModelConfig &c, uint32_t world, std::string &err) {
    if (world == 0 || world > 8) { err = "tensor parallel: 1 to 8 ranks"; return false; }
    if (c.n_head % world || c.n_head_kv % world || c.n_vocab % world) {
        err = "tensor parallel: heads, KV heads and vocabulary must divide by the rank count";
        return false;
    }
    if ((c.n_ff / world) % 32 || c.n_ff % world || ((c.n_head / world) * c.head_dim) % 32) {
        err = "tensor parallel: per-rank FFN and head widths must be whole 32-blocks";
        return false;
    }
    return true;
}

static bool ends_with(const std::string &s, const char *suf) {
    const size_t n = std::strlen(suf);
    return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

ShardSpec tp_shard_spec(const ModelConfig &c, const std::string &name, uint32_t rows, uint32_t cols,
                        uint32_t rank, uint32_t world, bool as_head) {
    ShardSpec s{0, rows, 0, cols};
    if (world <= 1) return s;
    const uint32_t qw = c.n_head / world * c.head_dim, kw = c.n_head_kv / world * c.head_dim;
    const uint32_t fw = c.n_ff / world, vw = c.n_vocab / world;
    if (as_head) {
        s.r0 = rank * vw; s.r1 = s.r0 + vw;
    } else if (ends_with(name, "attn_q.weight")) {
        s.r0 = rank * qw; s.r1 = s.r0 + qw;
    } else if (ends_with(name, "attn_k.weight") || ends_with(name, "attn_v.weight")) {
        s.r0 = rank * kw; s.r1 = s.r0 + kw;
    } else if (ends_with(name, "attn_output.weight")) {
        s.c0 = rank * qw; s.c1 = s.c0 + qw;
    } else if (ends_with(name, "ffn_gate.weight") || ends_with(name, "ffn_up.weight")) {
        s.r0 = rank * fw; s.r1 = s.r0 + fw;
    } else if (ends_with(name, "ffn_down.weight")) {
        s.c0 = rank * fw; s.c1 = s.c0 + fw;
    }
    return s;
}

uint64_t tp_shard_bytes(const GgufTensor &t, const ShardSpec &s) {
    uint32_t v = 1, b = 4;
    ggml_block(t.type, v, b);
    return (uint64_t)(s.r1 - s.r0) * ((s.c1 - s.c0) / v) * b;
}

void tp_extract(const GgufTensor &t, const ShardSpec &s, uint8_t *dst) {
    uint32_t v = 1, b = 4;
    ggml_block(t.type, v, b);
    const uint64_t cols = t.dims[0];
    const uint64_t row_bytes = cols / v * b;
    const uint64_t off = (uint64_t)s.c0 / v * b, n = (uint64_t)(s.c1 - s.c0) / v * b;
    if (off == 0 && n == row_bytes) {
        std::memcpy(dst, t.data + (uint64_t)s.r0 * row_bytes, (uint64_t)(s.r1 - s.r0) * row_bytes);
        return;
    }
    for (uint32_t r = s.r0; r < s.r1; ++r) std::memcpy(dst + (uint64_t)(r - s.r0) * n, t.data + r * row_bytes + off, n);
}

void tp_extract_range(const GgufTensor &t, const ShardSpec &s, uint64_t off, uint64_t len, uint8_t *dst) {
    uint32_t v = 1, b = 4;
    ggml_block(t.type, v, b);
    const uint64_t row_bytes = t.dims[0] / v * b;
    const uint64_t c_off = (uint64_t)s.c0 / v * b, n = (uint64_t)(s.c1 - s.c0) / v * b;
    if (c_off == 0 && n == row_bytes) {  // whole rows: one contiguous range
        std::memcpy(dst, t.data + (uint64_t)s.r0 * row_bytes + off, len);
        return;
    }
    while (len) {  // packed row r of the slice at r * n
        const uint64_t r = off / n, in = off % n, take = std::min(len, n - in);
        std::memcpy(dst, t.data + ((uint64_t)s.r0 + r) * row_bytes + c_off + in, take);
        dst += take;
        off += take;
        len -= take;
    }
}

}  // namespace fwb
