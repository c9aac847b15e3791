// prefill.cuh — the prompt path: T tokens per layer at once.
//
// forword.c feeds a prompt one token at a time (main.c:145-151 calls
// transformer_forward per token).  Here the prompt's tokens go through each
// layer together: the linear layers become dense dequant-GEMMs on the tensor
// cores (gemm_tc.cuh) and the small kernels below do the per-token work
// around them, with the same arithmetic as the decode step (rms_norm,
// norm.c:7-16; RoPE, rope.c:28-53; causal softmax attention,
// attention.c:142-164; SwiGLU, ffn.c:17-25,82-106).  Activations that feed a
// GEMM are rounded to fp16, and so are q, k, v and the probabilities in the
// tensor-core attention (head_dim 128); everything else is fp32.
#pragma once
#include "common.cuh"
#include "gemm_tc.cuh"

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

// out[t] = fp16(x[t] * w * (1 / sqrtf(mean(x[t]^2) + eps))), one block per
// token.  n % 4 == 0 and n <= 16 * 4 * blockDim.x: the row is read once, as
// float4, and kept in registers for the scaling pass.
constexpr int kPfNormVec = 16;  // float4 per thread at most
__global__ void pf_rmsnorm_f16_kernel(const float *x, const float *w, float eps, uint32_t n, __half *out) {
    __shared__ float red[32];
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)blockIdx.x * n);
    const float4 *wr = reinterpret_cast<const float4 *>(w);
    const uint32_t n4 = n / 4;
    float4 v[kPfNormVec];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kPfNormVec; ++k) {
        const uint32_t i = threadIdx.x + k * blockDim.x;
        v[k] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < kPfNormVec; ++k)
        ss = fmaf(v[k].w, v[k].w, fmaf(v[k].z, v[k].z, fmaf(v[k].y, v[k].y, fmaf(v[k].x, v[k].x, ss))));
    ss = pf_block_sum(ss, red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    uint2 *o = reinterpret_cast<uint2 *>(out + (size_t)blockIdx.x * n);
#pragma unroll
    for (int k = 0; k < kPfNormVec; ++k) {
        const uint32_t i = threadIdx.x + k * blockDim.x;
        if (i < n4) {
            const float4 g = __ldg(wr + i);
            const __half2 a = __floats2half2_rn(__fmul_rn(__fmul_rn(v[k].x, g.x), scale),
                                                __fmul_rn(__fmul_rn(v[k].y, g.y), scale));
            const __half2 b = __floats2half2_rn(__fmul_rn(__fmul_rn(v[k].z, g.z), scale),
                                                __fmul_rn(__fmul_rn(v[k].w, g.w), scale));
            o[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
        }
    }
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

// Causal attention of the prompt, tiled (flash form) on the CUDA cores in
// fp32.  A block owns R query rows -- QT = R / GQ consecutive tokens x the
// GQ query heads of one KV head (row r: token r / GQ, head r % GQ) -- and
// walks the positions 0 .. p0 + (its last token) in tiles of KT K / V rows
// staged in shared memory (rows padded by 4 floats: conflict-free 16-byte
// reads).  Per tile: scores S = q.k * scale (attention.c:150-154; each
// thread SR rows x SK positions, dot products in dimension order), causal
// mask, online softmax (running row maximum and sum, expf as
// attention.c:18-33), O += P V (each thread R*16/threads rows x HD/16
// dimensions).
// The output is O / l, rounded to fp16 for the o-proj GEMM.  Grid
// (ceil(nqt/2), n_kv): block b takes query tiles b and nqt-1-b, so every
// block walks about the same number of key tiles.
constexpr int kPfRows = 64, kPfKeys = 64, kPfSR = 4, kPfSK = 4, kPfThreads = 256;
template <int HD>
__host__ __device__ constexpr uint32_t pf_flash_smem() {
    return (uint32_t)((kPfRows + 2 * kPfKeys) * (HD + 4) + kPfRows * kPfKeys + 2 * kPfRows) * 4u;
}

template <int HD, int GQ>
__global__ void __launch_bounds__(kPfThreads) pf_flash_kernel(const float *qf, const float *kcache,
                                                              const float *vcache, uint32_t T, uint32_t p0,
                                                              uint32_t n_head, uint32_t kv_ctx, float scale,
                                                              __half *out) {
    static_assert(HD == 64 || HD == 128, "head_dim");
    constexpr int R = kPfRows, KT = kPfKeys, LD = HD + 4, QT = R / GQ, DV = HD / 16;
    constexpr int SR = kPfSR, SK = kPfSK, NC = KT / SK, RO = R * 16 / kPfThreads;
    static_assert((R / SR) * NC == kPfThreads && NC <= 32 && R % GQ == 0 && RO >= 1 && RO * kPfThreads == R * 16,
                  "thread mapping");
    extern __shared__ float4 pf_flash_raw[];
    float *Qs = reinterpret_cast<float *>(pf_flash_raw);
    float *Ks = Qs + R * LD, *Vs = Ks + KT * LD, *Ps = Vs + KT * LD;  // Ps [R][KT]
    float *alpha_s = Ps + R * KT, *linv_s = alpha_s + R;
    const uint32_t tid = threadIdx.x, kvh = blockIdx.y;
    const uint32_t nq = n_head * HD, nqt = (T + QT - 1) / QT;
    const float *kb = kcache + (size_t)kvh * kv_ctx * HD, *vb = vcache + (size_t)kvh * kv_ctx * HD;
    // score mapping: rows SR tr + a; positions tc + NC j (the NC lanes of a row group are adjacent)
    const uint32_t tr = tid / NC, tc = tid % NC;
    // output mapping: rows RO ro + r; dimensions 4 dg .. 4 dg + 3 (and 64 + 4 dg .. for HD 128)
    const uint32_t ro = tid >> 4, dg = tid & 15;

    for (uint32_t pass = 0; pass < 2; ++pass) {
        const uint32_t qt = pass == 0 ? blockIdx.x : nqt - 1 - blockIdx.x;
        if (pass == 1 && qt <= blockIdx.x) break;  // odd count: the middle tile once
        const uint32_t t0 = qt * QT;
        __syncthreads();  // the previous pass's reads of Qs are done
        // query rows (rows of tokens >= T are zeros and produce no output)
        for (uint32_t i = tid; i < (uint32_t)(R * HD / 4); i += kPfThreads) {
            const uint32_t r = i / (HD / 4), c4 = i % (HD / 4), tq = t0 + r / GQ;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (tq < T)
                v = *reinterpret_cast<const float4 *>(qf + (size_t)tq * nq + (size_t)(kvh * GQ + r % GQ) * HD + 4 * c4);
            *reinterpret_cast<float4 *>(Qs + r * LD + 4 * c4) = v;
        }
        float m[SR], l[SR];
#pragma unroll
        for (int a = 0; a < SR; ++a) { m[a] = -INFINITY; l[a] = 0.f; }
        float o[RO][DV];
#pragma unroll
        for (int r = 0; r < RO; ++r)
#pragma unroll
            for (int d = 0; d < DV; ++d) o[r][d] = 0.f;
        const uint32_t t_last = min(T, t0 + QT) - 1;
        const uint32_t n_keys = p0 + t_last + 1;
        for (uint32_t k0 = 0; k0 < n_keys; k0 += KT) {
            __syncthreads();  // previous tile's K / V / P reads are done
            for (uint32_t i = tid; i < (uint32_t)(KT * HD / 4); i += kPfThreads) {
                const uint32_t r = i / (HD / 4), c4 = i % (HD / 4), j = k0 + r;
                float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
                if (j < n_keys) {
                    kv = *reinterpret_cast<const float4 *>(kb + (size_t)j * HD + 4 * c4);
                    vv = *reinterpret_cast<const float4 *>(vb + (size_t)j * HD + 4 * c4);
                }
                *reinterpret_cast<float4 *>(Ks + r * LD + 4 * c4) = kv;
                *reinterpret_cast<float4 *>(Vs + r * LD + 4 * c4) = vv;
            }
            __syncthreads();
            float sc[SR][SK];
#pragma unroll
            for (int a = 0; a < SR; ++a)
#pragma unroll
                for (int j = 0; j < SK; ++j) sc[a][j] = 0.f;
#pragma unroll 2
            for (int d = 0; d < HD; d += 4) {
                float4 q[SR];
#pragma unroll
                for (int a = 0; a < SR; ++a) q[a] = *reinterpret_cast<const float4 *>(Qs + (SR * tr + a) * LD + d);
#pragma unroll
                for (int j = 0; j < SK; ++j) {
                    const float4 k = *reinterpret_cast<const float4 *>(Ks + (tc + NC * j) * LD + d);
#pragma unroll
                    for (int a = 0; a < SR; ++a)
                        sc[a][j] = fmaf(q[a].w, k.w, fmaf(q[a].z, k.z, fmaf(q[a].y, k.y, fmaf(q[a].x, k.x, sc[a][j]))));
                }
            }
            // causal mask, online softmax (the NC lanes of a row group share its rows)
#pragma unroll
            for (int a = 0; a < SR; ++a) {
                const uint32_t pos = p0 + t0 + (SR * tr + a) / GQ;
                float mx = -INFINITY;
#pragma unroll
                for (int j = 0; j < SK; ++j) {
                    const uint32_t key = k0 + tc + NC * j;
                    sc[a][j] = key <= pos ? __fmul_rn(sc[a][j], scale) : -INFINITY;
                    mx = fmaxf(mx, sc[a][j]);
                }
#pragma unroll
                for (int off = 1; off < NC; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                const float mn = fmaxf(m[a], mx);
                const float al = mn == -INFINITY ? 1.f : expf(m[a] - mn);
                float sum = 0.f;
#pragma unroll
                for (int j = 0; j < SK; ++j) {
                    const float e = sc[a][j] == -INFINITY ? 0.f : expf(sc[a][j] - mn);
                    Ps[(SR * tr + a) * KT + tc + NC * j] = e;
                    sum += e;
                }
#pragma unroll
                for (int off = 1; off < NC; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                l[a] = fmaf(l[a], al, sum);
                m[a] = mn;
                if (tc == 0) alpha_s[SR * tr + a] = al;
            }
            __syncthreads();
            // O = O * alpha + P V for rows RO ro + r
#pragma unroll
            for (int r = 0; r < RO; ++r) {
                const float al = alpha_s[RO * ro + r];
#pragma unroll
                for (int d = 0; d < DV; ++d) o[r][d] *= al;
            }
            const uint32_t kn = min((uint32_t)KT, n_keys - k0);
#pragma unroll 4
            for (uint32_t j = 0; j < kn; ++j) {
                const float4 v0 = *reinterpret_cast<const float4 *>(Vs + j * LD + 4 * dg);
                float4 v1 = v0;
                if (DV == 8) v1 = *reinterpret_cast<const float4 *>(Vs + j * LD + 64 + 4 * dg);
#pragma unroll
                for (int r = 0; r < RO; ++r) {
                    const float p = Ps[(RO * ro + r) * KT + j];
                    o[r][0] = fmaf(p, v0.x, o[r][0]);
                    o[r][1] = fmaf(p, v0.y, o[r][1]);
                    o[r][2] = fmaf(p, v0.z, o[r][2]);
                    o[r][3] = fmaf(p, v0.w, o[r][3]);
                    if (DV == 8) {
                        o[r][DV - 4] = fmaf(p, v1.x, o[r][DV - 4]);
                        o[r][DV - 3] = fmaf(p, v1.y, o[r][DV - 3]);
                        o[r][DV - 2] = fmaf(p, v1.z, o[r][DV - 2]);
                        o[r][DV - 1] = fmaf(p, v1.w, o[r][DV - 1]);
                    }
                }
            }
        }
        if (tc == 0)
#pragma unroll
            for (int a = 0; a < SR; ++a) linv_s[SR * tr + a] = l[a];
        __syncthreads();
#pragma unroll
        for (int r = 0; r < RO; ++r) {
            const uint32_t row = RO * ro + r, tq = t0 + row / GQ;
            if (tq >= T) continue;
            const float L = linv_s[row];
            __half *dst = out + (size_t)tq * nq + (size_t)(kvh * GQ + row % GQ) * HD;
#pragma unroll
            for (int d = 0; d < DV; ++d) {
                const uint32_t dim = d < 4 ? 4 * dg + d : 64 + 4 * dg + (d - 4);
                dst[dim] = __float2half_rn(__fdiv_rn(o[r][d], L));
            }
        }
    }
}

// Causal attention of the prompt on the tensor cores (head_dim 128).  A
// block owns 128 query rows -- 128 / GQ consecutive tokens x the GQ query
// heads of one KV head (row r: token r / GQ, head r % GQ) -- one row per
// thread and TMEM lane, and walks the positions 0 .. p0 + (its last token)
// in tiles of 64.  Per tile:
//  * the K tile (64 x 128) and the V tile, rounded to fp16 once per layer by
//    pf_kv16_kernel (V transposed: dims x positions), arrive by 16-byte
//    cp.async copies into the K-major 128-byte-swizzled layout, double
//    buffered: tile t+1 is in flight while tile t computes; q is rounded to
//    fp16 once per block the same way (two 64-dim halves);
//  * one thread issues S = q k^T as tcgen05.mma.kind::f16 (M 128, N 64,
//    K 8 x 16; fp32 in TMEM columns 0..63) and commits to an mbarrier;
//  * each thread reads its row's 64 scores (tcgen05.ld), scales by
//    1/sqrt(head_dim) (attention.c:150-154), masks the causal future, and
//    updates its running maximum and sum (online softmax, expf as
//    attention.c:18-33).  The output accumulator is rescaled in TMEM only
//    when the row maximum grows by more than 5 (a factor e^5 keeps the
//    probabilities of the tile within fp16), so the reference point m_used
//    changes rarely; p = expf(s - m_used) is rounded to fp16 into the P tile
//    and the row sum adds those rounded values;
//  * one thread issues O += P V (M 128, N 128, K 4 x 16; TMEM columns
//    128..255) and commits to the second mbarrier, which the next tile waits
//    on before it overwrites K, V and P.
// The output is O / l rounded to fp16 for the o-proj GEMM.  Every wait is
// bounded; a failed wait sets the error word, the block stops issuing MMAs,
// and a final commit is waited for before TMEM is released.
constexpr uint32_t kAtRows = 128, kAtKeys = 64, kAtHd = 128, kAtThreads = 128;
constexpr uint32_t kAtQBytes = kAtRows * kAtHd * 2;   // two 64-dim halves of 16 KB
constexpr uint32_t kAtKBytes = kAtKeys * kAtHd * 2;   // two halves of 8 KB
constexpr uint32_t kAtVBytes = kAtHd * kAtKeys * 2;   // 128 dims x 64 positions
constexpr uint32_t kAtPBytes = kAtRows * kAtKeys * 2; // 128 rows x 64 positions
constexpr uint32_t kAtSmem = kAtQBytes + 2 * (kAtKBytes + kAtVBytes) + kAtPBytes + 1024 + 128;  // K, V twice
constexpr float kAtRescale = 5.0f;

// The layer's K and V rows 0 .. n_pos-1 rounded to fp16 once, for every
// query tile of the tensor-core attention: K16[kv][pos][128] and V
// transposed, Vt16[kv][dim][pos] (row stride ctx_pad, a multiple of 64);
// positions n_pos .. the end of the last 64-row tile are zeros.  Grid
// (ceil(n_pos / 64), n_kv), 256 threads; the transpose goes through shared
// memory so that both writes are coalesced.
__global__ void __launch_bounds__(256) pf_kv16_kernel(const float *kcache, const float *vcache, uint32_t n_pos,
                                                      uint32_t kv_ctx, uint32_t ctx_pad, __half *k16,
                                                      __half *vt16) {
    __shared__ float vs[64][129];
    const uint32_t j0 = blockIdx.x * 64, kvh = blockIdx.y, tid = threadIdx.x;
    const float *kb = kcache + (size_t)kvh * kv_ctx * 128, *vb = vcache + (size_t)kvh * kv_ctx * 128;
    __half *kd = k16 + (size_t)kvh * ctx_pad * 128, *vd = vt16 + (size_t)kvh * 128 * ctx_pad;
    for (uint32_t i = tid; i < 64 * 32; i += 256) {
        const uint32_t r = i >> 5, c4 = i & 31, j = j0 + r;
        float4 k = make_float4(0.f, 0.f, 0.f, 0.f), v = k;
        if (j < n_pos) {
            k = *reinterpret_cast<const float4 *>(kb + (size_t)j * 128 + 4 * c4);
            v = *reinterpret_cast<const float4 *>(vb + (size_t)j * 128 + 4 * c4);
        }
        *reinterpret_cast<uint2 *>(kd + (size_t)j * 128 + 4 * c4) = make_uint2(pack_h2(k.x, k.y), pack_h2(k.z, k.w));
        vs[r][4 * c4] = v.x; vs[r][4 * c4 + 1] = v.y; vs[r][4 * c4 + 2] = v.z; vs[r][4 * c4 + 3] = v.w;
    }
    __syncthreads();
    // warp w writes dims 16 w .. 16 w + 15; lane l the positions 2 l, 2 l + 1 of each
    const uint32_t warp = tid >> 5, lane = tid & 31;
#pragma unroll 4
    for (uint32_t i = 0; i < 16; ++i) {
        const uint32_t d = warp * 16 + i;
        *reinterpret_cast<uint32_t *>(vd + (size_t)d * ctx_pad + j0 + 2 * lane) =
            pack_h2(vs[2 * lane][d], vs[2 * lane + 1][d]);
    }
}

__device__ __forceinline__ void at_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
// kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, both
// K-major, M 128, N n
__host__ __device__ constexpr uint32_t at_idesc(uint32_t n) {
    return (1u << 4) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}
__device__ __forceinline__ void at_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

template <int GQ>
__global__ void __launch_bounds__(kAtThreads) pf_attn_tc_kernel(const float *qf, const __half *k16,
                                                                const __half *vt16, uint32_t T, uint32_t p0,
                                                                uint32_t n_head, uint32_t ctx_pad, float scale,
                                                                __half *out, uint32_t *err) {
    constexpr uint32_t QT = kAtRows / GQ, HD = kAtHd;
    extern __shared__ uint8_t at_smem_raw[];
    const uint32_t base = (smem_u32(at_smem_raw) + 1023u) & ~1023u;
    uint8_t *sm = at_smem_raw + (base - smem_u32(at_smem_raw));
    uint8_t *Qs = sm, *Kb = Qs + kAtQBytes, *Vb = Kb + 2 * kAtKBytes, *Ps = Vb + 2 * kAtVBytes;
    uint64_t *bar = reinterpret_cast<uint64_t *>(Ps + kAtPBytes);  // [0] S done, [1] PV done, [2] final
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 3);
    uint32_t *bad = tmem_slot + 1;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, kvh = blockIdx.y;
    const uint32_t nq = n_head * HD, nqt = (T + QT - 1) / QT;
    const uint32_t qt = nqt - 1 - blockIdx.x;  // the longest key ranges start first
    const uint32_t t0 = qt * QT;
    const __half *kg = k16 + (size_t)kvh * ctx_pad * HD, *vg = vt16 + (size_t)kvh * HD * ctx_pad;
    // 16-byte asynchronous copies of key tile `it` into buffer it & 1, placed in
    // the swizzled layouts: K rows (two 64-dim halves), V^T rows (dims)
    auto fetch_tile = [&](uint32_t it) {
        const uint32_t k0 = it * kAtKeys, b = it & 1u;
        uint8_t *Ks = Kb + b * kAtKBytes, *Vt = Vb + b * kAtVBytes;
#pragma unroll
        for (uint32_t q = 0; q < 8; ++q) {
            const uint32_t i = tid + q * kAtThreads;  // 1024 chunks of each
            const uint32_t j = i >> 4, c = i & 15;     // K: row j, 16-byte chunk c of its 128 dims
            cp_async16(Ks + (c >> 3) * (kAtKeys * 128) + tc_sw128(j, c & 7), kg + (size_t)(k0 + j) * HD + 8 * c);
            const uint32_t d = i >> 3, e = i & 7;      // V^T: row d, chunk e of its 64 positions
            cp_async16(Vt + tc_sw128(d, e), vg + (size_t)d * ctx_pad + k0 + 8 * e);
        }
        cp_async_commit();
    };

    if (tid == 0) {
        for (int i = 0; i < 3; ++i) mbar_init(&bar[i], 1);
        *bad = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(256u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // this thread's query row -> fp16, swizzled (rows of tokens >= T are zeros)
    const uint32_t r = tid, tq = t0 + r / GQ;
    const bool live = tq < T;
    {
        const float *q = qf + (size_t)tq * nq + (size_t)(kvh * GQ + r % GQ) * HD;
#pragma unroll 4
        for (uint32_t c = 0; c < HD / 8; ++c) {
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
            if (live) {
                a = *reinterpret_cast<const float4 *>(q + 8 * c);
                b = *reinterpret_cast<const float4 *>(q + 8 * c + 4);
            }
            uint4 o;
            o.x = pack_h2(a.x, a.y); o.y = pack_h2(a.z, a.w); o.z = pack_h2(b.x, b.y); o.w = pack_h2(b.z, b.w);
            *reinterpret_cast<uint4 *>(Qs + (c / 8) * (kAtRows * 128) + tc_sw128(r, c % 8)) = o;
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot, tS = tmem, tO = tmem + 128;
    const uint32_t lane_off = (warp * 32u) << 16;

    const uint32_t t_last = min(T, t0 + QT) - 1;
    const uint32_t n_keys = p0 + t_last + 1, n_tiles = (n_keys + kAtKeys - 1) / kAtKeys;
    const uint32_t pos = p0 + tq;
    float m_used = -INFINITY, l = 0.f;
    fetch_tile(0);
    for (uint32_t it = 0; it < n_tiles; ++it) {
        const uint32_t k0 = it * kAtKeys;
        uint8_t *Ks = Kb + (it & 1u) * kAtKBytes, *Vt = Vb + (it & 1u) * kAtVBytes;
        // the previous tile's MMAs are done with its K / V buffer (the next
        // tile's), P and O
        if (it > 0 && !mbar_wait(&bar[1], (it - 1) & 1u, err, ERR_WAIT_FULL)) atomicExch(bad, 1u);
        tc_fence_after();
        if (it + 1 < n_tiles) {
            fetch_tile(it + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");  // this thread's copies of tile it
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncthreads();
        const bool go = *(volatile uint32_t *)bad == 0;
        if (tid == 0 && go) {
            tc_fence_after();
#pragma unroll
            for (uint32_t h = 0; h < 2; ++h) {
                const uint64_t da = tc_desc(smem_u32(Qs + h * (kAtRows * 128)));
                const uint64_t db = tc_desc(smem_u32(Ks + h * (kAtKeys * 128)));
#pragma unroll
                for (uint32_t k = 0; k < 4; ++k) at_mma(tS, da + 2 * k, db + 2 * k, at_idesc(kAtKeys), (h | k) != 0);
            }
            tc_commit(&bar[0]);
        }
        if (go && !mbar_wait(&bar[0], it & 1u, err, ERR_WAIT_FULL)) atomicExch(bad, 1u);
        tc_fence_after();
        // this row's scores, mask, online softmax
        float sc[64];
        {
            float a[32], b[32];
            tc_ld32(tS + lane_off, a);
            tc_ld32(tS + lane_off + 32, b);
#pragma unroll
            for (int j = 0; j < 32; ++j) { sc[j] = a[j]; sc[32 + j] = b[j]; }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
            const uint32_t key = k0 + j;
            sc[j] = (key <= pos && key < n_keys && live) ? __fmul_rn(sc[j], scale) : -INFINITY;
            mx = fmaxf(mx, sc[j]);
        }
        const bool grow = mx > m_used + kAtRescale || (m_used == -INFINITY && mx != -INFINITY);
        const float al = !grow ? 1.f : (m_used == -INFINITY ? 0.f : expf(m_used - mx));
        if (grow) {
            l *= al;
            m_used = mx;
        }
        // O row *= al in TMEM (the previous PV MMA is complete); TMEM loads and
        // stores are warp-wide, so a warp rescales when any of its rows grew
        if (it > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll 1
            for (uint32_t c0 = 0; c0 < 128; c0 += 32) {
                float o[32];
                tc_ld32(tO + lane_off + c0, o);
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] *= al;
                at_st32(tO + lane_off + c0, o);
            }
        }
        float sum = 0.f;
#pragma unroll
        for (uint32_t c = 0; c < 8; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float pa = sc[8 * c + 2 * e] == -INFINITY ? 0.f : expf(sc[8 * c + 2 * e] - m_used);
                const float pb = sc[8 * c + 2 * e + 1] == -INFINITY ? 0.f : expf(sc[8 * c + 2 * e + 1] - m_used);
                const __half2 hp = __floats2half2_rn(pa, pb);
                const float2 back = __half22float2(hp);
                sum += back.x + back.y;
                w[e] = *reinterpret_cast<const uint32_t *>(&hp);
            }
            *reinterpret_cast<uint4 *>(Ps + tc_sw128(r, c)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        l += sum;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncthreads();
        if (tid == 0 && *(volatile uint32_t *)bad == 0) {
            tc_fence_after();
            const uint64_t da = tc_desc(smem_u32(Ps)), db = tc_desc(smem_u32(Vt));
#pragma unroll
            for (uint32_t k = 0; k < 4; ++k) at_mma(tO, da + 2 * k, db + 2 * k, at_idesc(HD), (it | k) != 0);
            tc_commit(&bar[1]);
        }
    }
    // every MMA issued by thread 0 is covered by one more commit
    if (tid == 0) tc_commit(&bar[2]);
    const bool fin = mbar_wait(&bar[2], 0u, err, ERR_WAIT_DRAIN);
    tc_fence_after();
    if (__all_sync(0xffffffffu, fin && *(volatile uint32_t *)bad == 0) && n_tiles > 0) {  // warp-uniform
        __half *dst = out + (size_t)tq * nq + (size_t)(kvh * GQ + r % GQ) * HD;
        const float inv_ok = l;
#pragma unroll 1
        for (uint32_t c0 = 0; c0 < 128; c0 += 32) {
            float o[32];
            tc_ld32(tO + lane_off + c0, o);
            if (live) {
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const __half2 hv = __floats2half2_rn(__fdiv_rn(o[j], inv_ok), __fdiv_rn(o[j + 1], inv_ok));
                    *reinterpret_cast<__half2 *>(dst + c0 + j) = hv;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256u) : "memory");
    }
}

// h = fp16(silu(gate) * up) (ffn.c:17-25, 90-106); n % 4 == 0, four values
// per thread and step (float4 loads, one 8-byte store)
__device__ __forceinline__ float pf_silu_mul(float v, float u) {
    const float sig = v >= 0.0f ? __fdiv_rn(1.0f, 1.0f + expf(-v)) : __fdiv_rn(expf(v), 1.0f + expf(v));
    return __fmul_rn(__fmul_rn(v, sig), u);
}
__global__ void pf_swiglu_kernel(const float *g, const float *u, size_t n, __half *h) {
    const size_t n4 = n / 4;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 a = __ldcs(reinterpret_cast<const float4 *>(g) + i);
        const float4 b = __ldcs(reinterpret_cast<const float4 *>(u) + i);
        const __half2 lo = __floats2half2_rn(pf_silu_mul(a.x, b.x), pf_silu_mul(a.y, b.y));
        const __half2 hi = __floats2half2_rn(pf_silu_mul(a.z, b.z), pf_silu_mul(a.w, b.w));
        reinterpret_cast<uint2 *>(h)[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&lo),
                                                     *reinterpret_cast<const uint32_t *>(&hi));
    }
}

}  // namespace fwb
