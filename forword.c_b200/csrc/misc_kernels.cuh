// misc_kernels.cuh — embedding row lookup and bit-exact block dequantisation.
#pragma once
#include "common.cuh"

namespace fwb {

// One 32-value block -> fp32, exactly as the reference decoders compute it:
// Q8_0 quant.c:232-263, Q5_0 linear.c:40-56 (d * (float)(q - 16)), Q4_0 the
// GGML layout (d * (float)(nibble - 8)).  One fp32 multiply per value, so the
// result is bit-identical to the CPU decoders.
__device__ __forceinline__ float decode_value(const uint8_t *blk, uint32_t type, uint32_t j) {
    const float d = f16_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
    int q;
    if (type == 8) {
        q = (int)(int8_t)blk[2 + j];
    } else if (type == 6) {
        const uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) |
                            ((uint32_t)blk[5] << 24);
        const uint32_t byte = blk[6 + (j & 15)];
        const uint32_t nib = j < 16 ? (byte & 15u) : (byte >> 4);
        q = (int)(nib | (((qh >> j) & 1u) << 4)) - 16;
    } else {  // Q4_0
        const uint32_t byte = blk[2 + (j & 15)];
        q = (int)(j < 16 ? (byte & 15u) : (byte >> 4)) - 8;
    }
    return __fmul_rn(d, (float)q);
}

// out[i] = value i of the block stream (n values), grid-stride
__global__ void dequant_kernel(const uint8_t *w, uint32_t type, uint32_t bb, float *out, uint64_t n) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = decode_value(w + (i >> 5) * bb, type, (uint32_t)(i & 31));
}

// x = row `step[0]` of the embedding table (linear_get_row, linear.c:60-151).
__global__ void embed_kernel(const uint8_t *table, uint32_t type, uint32_t cols, uint64_t row_bytes,
                             const uint32_t *step, float *x) {
    pdl_launch();
    pdl_wait();
    const uint32_t tok = step[0];
    const uint8_t *row = table + (uint64_t)tok * row_bytes;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += gridDim.x * blockDim.x) {
        if (type == 0)
            x[i] = reinterpret_cast<const float *>(row)[i];
        else
            x[i] = decode_value(row + (i >> 5) * (type == 2 ? 18 : type == 6 ? 22 : 34), type, i & 31);
    }
}

}  // namespace fwb
