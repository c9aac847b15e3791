/*
 * ref_q4_0_addon.c — TEST INFRASTRUCTURE (oracle).  Linked only into
 * oracle/_ref/libforword_ref.so and oracle/_ref/forword, never into the
 * product.
 *
 * The reference cannot run GGML Q4_0 (type 2): quant_matvec's block_layout
 * has no entry for it (quant_matvec.c:52-62) and dot_quant_block has no
 * decoder (quant_matvec.c:231-261).  This file adds Q4_0 without editing the
 * reference sources: the Makefile compiles quant_matvec.c with its public
 * symbol renamed to forword_ref_quant_matvec_impl, and the quant_matvec below
 * (the symbol linear.c:209 calls) handles type 2 itself and forwards every
 * other type unchanged.
 *
 * The Q4_0 path follows the reference's own Q5_0 path exactly: decode one
 * 32-value block into floats the way linear.c:40-56 does (fp16 scale, quant
 * bytes after it, value = d * (q - offset)), then simd_dot_f32 against the
 * input slice (quant_matvec.c:243-247), summed row by row in block order
 * (quant_matvec.c:291-307).  Only the block layout differs: Q4_0 has no
 * high-bit plane, its 16 quant bytes start at byte 2, element j is the low
 * nibble of byte j and element j+16 the high nibble, and the offset is 8
 * (GGML's Q4_0 definition; the reference names only its 18-byte size, at
 * gguf.c:211).
 */
#include "quant_matvec.h"
#include "simd.h"

#include <stdint.h>
#include <string.h>

int forword_ref_quant_matvec_impl(const void *weights, size_t weights_size,
                                  uint32_t ggml_type, const float *input,
                                  float *output, size_t input_size,
                                  size_t output_size);

/* Same fp16 -> fp32 conversion as quant_matvec.c:18-46 (subnormal-correct). */
static float addon_half_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 31u;
    uint32_t mant = h & 1023u;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = -14;
            while ((mant & 1024u) == 0) { mant <<= 1; --e; }
            mant &= 1023u;
            bits = sign | ((uint32_t)(e + 127) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* Decode one 18-byte Q4_0 block into 32 floats. */
void forword_ref_q4_0_decode_block(const uint8_t *p, float *out)
{
    float d = addon_half_to_float((uint16_t)(p[0] | (p[1] << 8)));
    const uint8_t *qs = p + 2;
    for (int j = 0; j < 16; ++j) {
        out[j] = d * (float)((qs[j] & 15) - 8);
        out[j + 16] = d * (float)((qs[j] >> 4) - 8);
    }
}

int quant_matvec(const void *weights, size_t weights_size, uint32_t ggml_type,
                 const float *input, float *output, size_t input_size,
                 size_t output_size)
{
    if (ggml_type != 2)
        return forword_ref_quant_matvec_impl(weights, weights_size, ggml_type,
                                             input, output, input_size,
                                             output_size);

    /* Argument checks of quant_matvec.c:270-289 with Q4_0's 32 values / 18 B. */
    const size_t block_values = 32, block_bytes = 18;
    if (!weights || !input || !output || input_size == 0 || output_size == 0 ||
        input_size % block_values != 0)
        return -1;
    size_t blocks_per_row = input_size / block_values;
    if (blocks_per_row > SIZE_MAX / block_bytes)
        return -1;
    size_t bytes_per_row = blocks_per_row * block_bytes;
    if (output_size > SIZE_MAX / bytes_per_row ||
        weights_size < output_size * bytes_per_row)
        return -1;

    const uint8_t *raw = (const uint8_t *)weights;
    float decoded[32];
    for (size_t row = 0; row < output_size; ++row) {
        float sum = 0.0f;
        const uint8_t *row_weights = raw + row * bytes_per_row;
        for (size_t b = 0; b < blocks_per_row; ++b) {
            forword_ref_q4_0_decode_block(row_weights + b * block_bytes, decoded);
            sum += simd_dot_f32(decoded, input + b * block_values, 32);
        }
        output[row] = sum;
    }
    return 0;
}
