// misc_kernels.cuh — embedding row lookup and bit-exact block dequantisation.
#pragma once
#include "common.cuh"

namespace fwb {

__device__ __forceinline__ uint32_t rd16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// Block geometry of the quantised types: values per block, bytes per block.
__host__ __device__ constexpr uint32_t qblock_values(uint32_t type) { return type == 12 || type == 14 ? 256u : 32u; }
__host__ __device__ constexpr uint32_t qblock_bytes(uint32_t type) {
    return type == 2 ? 18u : type == 6 ? 22u : type == 7 ? 24u : type == 8 ? 34u : type == 12 ? 144u : 210u;
}

// Value i of a row of quantised blocks -> fp32, exactly as the reference's
// decoders compute it, operation by operation in fp32 (no contraction):
//   Q8_0 d * q                      quant.c:232-263
//   Q5_0 d * (q - 16)               linear.c:40-56
//   Q5_1 d * q + m                  quant.c:190-230
//   Q4_K (d * sc) * q - dmin * m    quant.c:85-131 (get_scale_min_k4, quant.c:63-82)
//   Q6_K (d * sc) * (q - 32)        quant.c:133-189
//   Q4_0 d * (q - 8)                GGML's layout (the reference has no Q4_0 decoder)
__device__ __forceinline__ float decode_elem(const uint8_t *row, uint32_t type, uint32_t i) {
    const uint8_t *blk = row + (i / qblock_values(type)) * qblock_bytes(type);
    const uint32_t j = i % qblock_values(type);
    if (type == 12) {
        const float d = f16_bits_to_f32(rd16(blk)), dmin = f16_bits_to_f32(rd16(blk + 2));
        const uint8_t *sc = blk + 4;
        const uint32_t g = j >> 5;
        uint32_t scale, mn;
        if (g < 4) {
            scale = sc[g] & 63u;
            mn = sc[g + 4] & 63u;
        } else {
            scale = (sc[g + 4] & 15u) | ((sc[g - 4] >> 6) << 4);
            mn = (sc[g + 4] >> 4) | ((sc[g] >> 6) << 4);
        }
        const uint32_t byte = blk[16 + (g >> 1) * 32 + (j & 31)];
        const uint32_t v = (g & 1) ? (byte >> 4) : (byte & 15u);
        const float ds = __fmul_rn(d, (float)scale), dm = __fmul_rn(dmin, (float)mn);
        return __fsub_rn(__fmul_rn(ds, (float)v), dm);
    }
    if (type == 14) {
        const uint32_t half = j >> 7, r = j & 127, quarter = r >> 5, l = r & 31;
        const uint8_t *ql = blk + 64 * half, *qh = blk + 128 + 32 * half;
        const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * half);
        const uint32_t lowb = ql[l + ((quarter & 1) ? 32 : 0)];
        const uint32_t low = quarter < 2 ? (lowb & 15u) : (lowb >> 4);
        const uint32_t high = (qh[l] >> (2 * quarter)) & 3u;
        const int q = (int)(low | (high << 4)) - 32;
        const float d = f16_bits_to_f32(rd16(blk + 208));
        return __fmul_rn(__fmul_rn(d, (float)sc[l / 16 + 2 * quarter]), (float)q);
    }
    const float d = f16_bits_to_f32(rd16(blk));
    if (type == 8) return __fmul_rn(d, (float)(int8_t)blk[2 + j]);
    if (type == 6 || type == 7) {
        const uint32_t o = type == 7 ? 4 : 2;
        const uint32_t qh = (uint32_t)blk[o] | ((uint32_t)blk[o + 1] << 8) | ((uint32_t)blk[o + 2] << 16) |
                            ((uint32_t)blk[o + 3] << 24);
        const uint32_t byte = blk[o + 4 + (j & 15)];
        const uint32_t q = (j < 16 ? (byte & 15u) : (byte >> 4)) | (((qh >> j) & 1u) << 4);
        if (type == 6) return __fmul_rn(d, (float)((int)q - 16));
        return __fadd_rn(__fmul_rn(d, (float)q), f16_bits_to_f32(rd16(blk + 2)));
    }
    const uint32_t byte = blk[2 + (j & 15)];  // Q4_0
    return __fmul_rn(d, (float)((int)(j < 16 ? (byte & 15u) : (byte >> 4)) - 8));
}

// out[i] = value i of the block stream (n values), grid-stride
__global__ void dequant_kernel(const uint8_t *w, uint32_t type, uint32_t bb, float *out, uint64_t n) {
    const uint32_t bv = qblock_values(type);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = decode_elem(w + (i / bv) * bb, type, (uint32_t)(i % bv));
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
            x[i] = decode_elem(row, type, i);
    }
}

}  // namespace fwb
