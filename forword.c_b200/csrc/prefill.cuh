// prefill.cuh — the prompt path: T tokens per layer at once.
//
// forword.c feeds a prompt one token at a time (main.c:145-151 calls
// transformer_forward per token).  Here the prompt's tokens go through each
// layer together: the linear layers become dense dequant-GEMMs on the tensor
// cores (gemm_tc.cuh) and the small kernels below do the per-token work
// around them, with the same arithmetic as the decode step (rms_norm,
// norm.c:7-16; RoPE, rope.c:28-53; causal softmax attention,
// attention.c:142-164; SwiGLU, ffn.c:17-25,82-106).  Activations that feed a
// GEMM are rounded to fp16; everything else is fp32.
#pragma once
#include "common.cuh"

namespace fwb {

// x[t] = row tokens[t] of the embedding table (linear_get_row, linear.c:60-151)
__global__ void pf_embed_kernel(const uint8_t *table, uint32_t type, uint32_t cols, uint64_t row_bytes,
                                const uint32_t *tokens, float *x) {
    const uint32_t t = blockIdx.x;
    const uint8_t *row = table + (uint64_t)tokens[t] * row_bytes;
    for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x)
        x[(size_t)t * cols + i] = type == 0 ? reinterpret_cast<const float *>(row)[i] : decode_elem(row, type, i);
}

__device__ __forceinline__ float pf_block_sum(float v, float *red) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (uint32_t w = 0; w < nw; ++w) t += red[w];  // same order in every thread
    return t;
}

__device__ __forceinline__ float pf_block_max(float v, float *red) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = -INFINITY;
    for (uint32_t w = 0; w < nw; ++w) t = fmaxf(t, red[w]);
    return t;
}

// out[t] = fp16(x[t] * w * (1 / sqrtf(mean(x[t]^2) + eps))), one block per token
__global__ void pf_rmsnorm_f16_kernel(const float *x, const float *w, float eps, uint32_t n, __half *out) {
    __shared__ float red[32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = pf_block_sum(ss, red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    __half *o = out + (size_t)blockIdx.x * n;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) o[i] = __float2half_rn(__fmul_rn(__fmul_rn(xr[i], w[i]), scale));
}

// Rows [q | k | v] of the QKV GEMM output for token t at position p0 + t: RoPE
// on q and k (adjacent pairs, rope.c:37-43), q to qf, k and v appended to the
// layer's cache ([kv_head][kv_ctx][hd]).  One block per token.
__global__ void pf_rope_kv_kernel(const float *qkv, uint32_t p0, uint32_t n_q, uint32_t n_kv, uint32_t hd,
                                  const float *rope_cos, const float *rope_sin, float *qf, float *kcache,
                                  float *vcache, uint32_t kv_ctx) {
    const uint32_t t = blockIdx.x, pos = p0 + t, half = hd >> 1;
    const uint32_t nrow = n_q + 2 * n_kv;
    const float *r = qkv + (size_t)t * nrow;
    for (uint32_t g = 2 * threadIdx.x; g < nrow; g += 2 * blockDim.x) {
        const float v0 = r[g], v1 = r[g + 1];
        if (g < n_q + n_kv) {
            const uint32_t gg = g < n_q ? g : g - n_q, d = gg % hd;
            const float c = rope_cos[(size_t)pos * half + d / 2], s = rope_sin[(size_t)pos * half + d / 2];
            const float r0 = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
            const float r1 = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
            if (g < n_q) {
                qf[(size_t)t * n_q + g] = r0;
                qf[(size_t)t * n_q + g + 1] = r1;
            } else {
                float *dst = kcache + ((size_t)(gg / hd) * kv_ctx + pos) * hd + d;
                dst[0] = r0;
                dst[1] = r1;
            }
        } else {
            const uint32_t gv = g - n_q - n_kv, d = gv % hd;
            float *dst = vcache + ((size_t)(gv / hd) * kv_ctx + pos) * hd + d;
            dst[0] = v0;
            dst[1] = v1;
        }
    }
}

// Causal attention of token t (position p0 + t) and query head h over
// positions 0..p0+t, one block of 128 threads per (t, h): scores
// q.k * 1/sqrtf(hd) into shared memory, softmax with expf, probabilities
// normalised before the weighted sum of the value rows (attention.c:150-163).
// Output rounded to fp16 for the o-proj GEMM.
__global__ void pf_attn_kernel(const float *qf, const float *kcache, const float *vcache, uint32_t p0, uint32_t n_head,
                               uint32_t gq, uint32_t hd, uint32_t kv_ctx, float scale, __half *out) {
    extern __shared__ float pf_sc[];  // [positions]
    __shared__ float red[32];
    const uint32_t t = blockIdx.x, h = blockIdx.y, kvh = h / gq;
    const uint32_t n_pos = p0 + t + 1;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const uint32_t nq = n_head * hd;
    const float *q = qf + (size_t)t * nq + (size_t)h * hd;
    const float *kb = kcache + (size_t)kvh * kv_ctx * hd, *vb = vcache + (size_t)kvh * kv_ctx * hd;
    // lane l holds dims 4l..4l+3 (hd <= 128, hd % 4 == 0)
    const bool act = 4 * lane < hd;
    float4 qv = act ? *reinterpret_cast<const float4 *>(q + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t i = warp; i < n_pos; i += nw) {
        float dot = 0.f;
        if (act) {
            const float4 k = __ldg(reinterpret_cast<const float4 *>(kb + (size_t)i * hd + 4 * lane));
            dot = fmaf(qv.w, k.w, fmaf(qv.z, k.z, fmaf(qv.y, k.y, qv.x * k.x)));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (lane == 0) pf_sc[i] = __fmul_rn(dot, scale);
    }
    __syncthreads();
    float m = -INFINITY;
    for (uint32_t i = threadIdx.x; i < n_pos; i += blockDim.x) m = fmaxf(m, pf_sc[i]);
    m = pf_block_max(m, red);
    float s = 0.f;
    for (uint32_t i = threadIdx.x; i < n_pos; i += blockDim.x) {
        const float e = expf(pf_sc[i] - m);
        pf_sc[i] = e;
        s += e;
    }
    s = pf_block_sum(s, red);  // (its barriers order every e written above)
    // softmax (attention.c:18-33): probabilities times 1/sum, unless the sum
    // is not a positive finite number
    const bool norm = s > 0.0f && isfinite(s);
    const float inv = __fdiv_rn(1.0f, s);
    if (norm)
        for (uint32_t i = threadIdx.x; i < n_pos; i += blockDim.x) pf_sc[i] = __fmul_rn(pf_sc[i], inv);
    __syncthreads();
    for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.f;
        for (uint32_t i = 0; i < n_pos; ++i) o = fmaf(pf_sc[i], vb[(size_t)i * hd + d], o);
        out[(size_t)t * nq + (size_t)h * hd + d] = __float2half_rn(o);
    }
}

// The same attention for all GQ query heads of one KV head per block (grid
// (T, n_kv), 128 threads, hd <= 128): each K row is read once for the GQ
// heads and each V row once for GQ outputs; positions are split over the
// four warps in both passes.  Scores of head g at pf_sc2[g * n_pos + i].
template <int GQ>
__global__ void pf_attn_gqa_kernel(const float *qf, const float *kcache, const float *vcache, uint32_t p0,
                                   uint32_t n_head, uint32_t hd, uint32_t kv_ctx, float scale, __half *out) {
    extern __shared__ float pf_sc2[];  // [GQ][positions]
    __shared__ float red[32];
    const uint32_t t = blockIdx.x, kvh = blockIdx.y;
    const uint32_t n_pos = p0 + t + 1;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const uint32_t nq = n_head * hd;
    const float *kb = kcache + (size_t)kvh * kv_ctx * hd, *vb = vcache + (size_t)kvh * kv_ctx * hd;
    const bool act = 4 * lane < hd;
    float4 qv[GQ];
#pragma unroll
    for (int g = 0; g < GQ; ++g)
        qv[g] = act ? *reinterpret_cast<const float4 *>(qf + (size_t)t * nq + (size_t)(kvh * GQ + g) * hd + 4 * lane)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t i = warp; i < n_pos; i += nw) {
        const float4 k = act ? __ldg(reinterpret_cast<const float4 *>(kb + (size_t)i * hd + 4 * lane))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
            float dot = fmaf(qv[g].w, k.w, fmaf(qv[g].z, k.z, fmaf(qv[g].y, k.y, qv[g].x * k.x)));
#pragma unroll
            for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (lane == 0) pf_sc2[g * n_pos + i] = __fmul_rn(dot, scale);
        }
    }
    __syncthreads();
    for (int g = 0; g < GQ; ++g) {  // softmax of head g (attention.c:18-33)
        float *sc = pf_sc2 + g * n_pos;
        float m = -INFINITY;
        for (uint32_t i = threadIdx.x; i < n_pos; i += blockDim.x) m = fmaxf(m, sc[i]);
        m = pf_block_max(m, red);
        float s = 0.f;
        for (uint32_t i = threadIdx.x; i < n_pos; i += blockDim.x) {
            const float e = expf(sc[i] - m);
            sc[i] = e;
            s += e;
        }
        s = pf_block_sum(s, red);
        const float inv = __fdiv_rn(1.0f, s);
        if (s > 0.0f && isfinite(s))
            for (uint32_t i = threadIdx.x; i < n_pos; i += blockDim.x) sc[i] = __fmul_rn(sc[i], inv);
    }
    __syncthreads();
    // weighted sum of the value rows: warp w takes positions w, w + nw, ...
    // (lanes own 4 dims each), then the warps' partial sums are added
    __shared__ float part[4][GQ][128];
    float4 acc[GQ];
#pragma unroll
    for (int g = 0; g < GQ; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t i = warp; i < n_pos; i += nw) {
        const float4 v = act ? __ldg(reinterpret_cast<const float4 *>(vb + (size_t)i * hd + 4 * lane))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
            const float p = pf_sc2[g * n_pos + i];
            acc[g].x = fmaf(p, v.x, acc[g].x);
            acc[g].y = fmaf(p, v.y, acc[g].y);
            acc[g].z = fmaf(p, v.z, acc[g].z);
            acc[g].w = fmaf(p, v.w, acc[g].w);
        }
    }
    if (act)
#pragma unroll
        for (int g = 0; g < GQ; ++g) *reinterpret_cast<float4 *>(&part[warp][g][4 * lane]) = acc[g];
    __syncthreads();
    for (uint32_t j = threadIdx.x; j < GQ * hd; j += blockDim.x) {
        const uint32_t g = j / hd, d = j % hd;
        float o = 0.f;
        for (uint32_t w = 0; w < nw; ++w) o += part[w][g][d];
        out[(size_t)t * nq + (size_t)(kvh * GQ + g) * hd + d] = __float2half_rn(o);
    }
}

// h = fp16(silu(gate) * up) (ffn.c:17-25, 90-106)
__global__ void pf_swiglu_kernel(const float *g, const float *u, size_t n, __half *h) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = g[i];
        const float sig = v >= 0.0f ? __fdiv_rn(1.0f, 1.0f + expf(-v)) : __fdiv_rn(expf(v), 1.0f + expf(v));
        h[i] = __float2half_rn(__fmul_rn(__fmul_rn(v, sig), u[i]));
    }
}

}  // namespace fwb
