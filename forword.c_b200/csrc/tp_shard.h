// tp_shard.h — which slice of each tensor a tensor-parallel rank keeps, and
// the extraction of that slice from the GGUF mapping (host only).
//
// Megatron-style split of the llama block for `world` ranks of one box:
//   attn_q / attn_k / attn_v   rows of this rank's query / KV heads
//   attn_output                input columns of those heads
//   ffn_gate / ffn_up          rows [rank*F/world, (rank+1)*F/world)
//   ffn_down                   the same range of input columns
//   output (LM head)           rows [rank*V/world, (rank+1)*V/world)
//   everything else            whole (embedding, norms)
// Column slices are whole 32-blocks, so a shard is again a row-major matrix of
// GGUF blocks: row r of the shard is the byte range of the slice inside row r
// of the tensor, copied unchanged.
#pragma once
#include <cstdint>
#include <string>

#include "gguf_reader.h"

namespace fwb {

struct ShardSpec {
    uint32_t r0 = 0, r1 = 0;  // rows kept
    uint32_t c0 = 0, c1 = 0;  // columns kept (multiples of the block size)
};

// The split needs n_head, n_head_kv, n_vocab divisible by world, and
// n_ff / world and n_head / world * head_dim multiples of 32.
bool tp_check(const ModelConfig &c, uint32_t world, std::string &err);

// Slice of a 2-D tensor `name` with `rows` x `cols` for `rank` of `world`
// (`as_head`: the tensor is used as the LM head, e.g. tied embeddings).
ShardSpec tp_shard_spec(const ModelConfig &c, const std::string &name, uint32_t rows, uint32_t cols,
                        uint32_t rank, uint32_t world, bool as_head);

// Bytes of the packed slice, and the copy itself.
uint64_t tp_shard_bytes(const GgufTensor &t, const ShardSpec &s);
void tp_extract(const GgufTensor &t, const ShardSpec &s, uint8_t *dst);
// Bytes [off, off + len) of the packed slice (tp_extract's output) into dst.
void tp_extract_range(const GgufTensor &t, const ShardSpec &s, uint64_t off, uint64_t len, uint8_t *dst);

}  // namespace fwb
