// attention.cuh — batch-1 decode attention over the device KV cache.
//
// Replaces the per-head score / softmax / value loop of attention_forward
// (attention.c:142-164): scores q.k_t * 1/sqrt(head_dim) for t in [0, pos],
// softmax, sum_t p_t v_t, with the GQA map kv_h = h / (n_head / n_kv)
// (attention.c:142,147).
//
// Split-K flash decode.  Grid (n_kv, n_split): CTA (h, s) owns a contiguous
// slice of positions of KV head h and serves all GQ = n_head/n_kv query
// heads of that group, so each K/V row is read from HBM once per step.  The
// KV cache layout is [kv_head][ctx][head_dim] fp32, so a slice is one
// contiguous range.  Each warp runs an online softmax over tiles of
// min(8, 32/GQ) positions: lanes own 4 dims, the (position, head) partial
// dots of a tile are finished with one butterfly reduce-scatter.  Warps are merged in shared memory, each CTA writes one
// (max, sum, o[]) partial per query head, and the last CTA of a KV head to
// finish (atomic ticket) merges the n_split partials and writes the output.
#pragma once
#include "common.cuh"

namespace fwb {

struct AttnArgs {
    const float *q;        // [n_head][HD], RoPE applied
    const float *kc, *vc;  // this layer: [n_kv][kv_ctx][HD]
    float *out;            // [n_head][HD]
    float *part;           // scratch [n_kv][n_split][GQ][HD + 2]
    uint32_t *ticket;      // [n_kv], zero between launches
    uint32_t kv_ctx, n_split;
    float scale;           // 1/sqrtf(head_dim), attention.c:143
    const uint32_t *step;  // [1] = pos
    uint32_t *err;
};

constexpr int kAttnWarps = 4;

template <int HD, int GQ>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
    static_assert(HD % 4 == 0 && HD <= 128, "head_dim");
    static_assert(GQ == 1 || GQ == 2 || GQ == 4 || GQ == 8, "group");
    constexpr int TILE = (32 / GQ) < 8 ? (32 / GQ) : 8;  // positions per tile
    constexpr int NVAL = TILE * GQ;                       // partial dots per tile (8..32)
    constexpr int REP = 32 / NVAL;                        // lanes holding each finished value
    constexpr int LA = HD / 4;                            // active lanes
    __shared__ float pbuf[kAttnWarps][32];
    __shared__ float wm[kAttnWarps][GQ], wl[kAttnWarps][GQ];
    __shared__ float wo[kAttnWarps][GQ][HD];
    __shared__ uint32_t last_flag;

    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t h = blockIdx.x, sp = blockIdx.y;
    pdl_launch();
    pdl_wait();

    const uint32_t n_pos = a.step[1] + 1;
    const uint32_t chunk = (n_pos + a.n_split - 1) / a.n_split;
    const uint32_t c0 = min(n_pos, sp * chunk), c1 = min(n_pos, c0 + chunk);
    const uint32_t wchunk = (c1 - c0 + kAttnWarps - 1) / kAttnWarps;
    const uint32_t w0 = min(c1, c0 + warp * wchunk), w1 = min(c1, w0 + wchunk);

    const bool lact = lane < LA;
    float qv[GQ][4], o[GQ][4], m[GQ], l[GQ];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        const float4 t = lact ? *reinterpret_cast<const float4 *>(a.q + (size_t)(h * GQ + g) * HD + 4 * lane)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        qv[g][0] = t.x; qv[g][1] = t.y; qv[g][2] = t.z; qv[g][3] = t.w;
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int d = 0; d < 4; ++d) o[g][d] = 0.f;
    }
    const float *kb = a.kc + (size_t)h * a.kv_ctx * HD + 4 * lane;
    const float *vb = a.vc + (size_t)h * a.kv_ctx * HD + 4 * lane;

    for (uint32_t t0 = w0; t0 < w1; t0 += TILE) {
        float4 kt[TILE], vt[TILE];
#pragma unroll
        for (int p = 0; p < TILE; ++p) {
            const bool ok = lact && t0 + p < w1;
            kt[p] = ok ? *reinterpret_cast<const float4 *>(kb + (size_t)(t0 + p) * HD) : make_float4(0.f, 0.f, 0.f, 0.f);
            vt[p] = ok ? *reinterpret_cast<const float4 *>(vb + (size_t)(t0 + p) * HD) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float v[NVAL];
#pragma unroll
        for (int p = 0; p < TILE; ++p)
#pragma unroll
            for (int g = 0; g < GQ; ++g) {
                float s = qv[g][0] * kt[p].x;
                s = fmaf(qv[g][1], kt[p].y, s);
                s = fmaf(qv[g][2], kt[p].z, s);
                s = fmaf(qv[g][3], kt[p].w, s);
                v[p * GQ + g] = s;
            }
        // butterfly reduce-scatter: lane l ends with the full sum of value l / REP
#pragma unroll
        for (int st = 0; (NVAL >> st) > 1; ++st) {
            const int o_ = 16 >> st, c = NVAL >> st;
            const bool up = lane & o_;
#pragma unroll
            for (int i = 0; i < c / 2; ++i) {
                const float send = up ? v[i] : v[i + c / 2], keep = up ? v[i + c / 2] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o_);
            }
        }
#pragma unroll
        for (int o_ = REP / 2; o_ >= 1; o_ >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o_);
        const uint32_t vi = lane / REP;
        const uint32_t my_p = vi / GQ, my_g = vi % GQ;
        const float sc = (t0 + my_p < w1) ? v[0] * a.scale : -INFINITY;
        // per-head tile max / sum over the lanes holding that head
        float tm = sc;
#pragma unroll
        for (int o_ = 32 / TILE; o_ < 32; o_ <<= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o_));
        float mg = m[0];
#pragma unroll
        for (int g = 1; g < GQ; ++g) if (my_g == (uint32_t)g) mg = m[g];
        const float mn = fmaxf(mg, tm);
        const float pe = expf(sc - mn);
        float ts = pe;
#pragma unroll
        for (int o_ = 32 / TILE; o_ < 32; o_ <<= 1) ts += __shfl_xor_sync(0xffffffffu, ts, o_);
        const float alpha = expf(mg - mn);
        pbuf[warp][vi] = pe;  // the REP lanes of a value write the same number
#pragma unroll
        for (int g = 0; g < GQ; ++g) {
            const float al = __shfl_sync(0xffffffffu, alpha, g * REP);
            const float mng = __shfl_sync(0xffffffffu, mn, g * REP);
            const float tsg = __shfl_sync(0xffffffffu, ts, g * REP);
            l[g] = fmaf(l[g], al, tsg);
            m[g] = mng;
#pragma unroll
            for (int d = 0; d < 4; ++d) o[g][d] *= al;
        }
        __syncwarp();
#pragma unroll
        for (int p = 0; p < TILE; ++p)
#pragma unroll
            for (int g = 0; g < GQ; ++g) {
                const float w = pbuf[warp][p * GQ + g];
                o[g][0] = fmaf(w, vt[p].x, o[g][0]);
                o[g][1] = fmaf(w, vt[p].y, o[g][1]);
                o[g][2] = fmaf(w, vt[p].z, o[g][2]);
                o[g][3] = fmaf(w, vt[p].w, o[g][3]);
            }
        __syncwarp();
    }

    // merge the warps of this CTA
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        if (lane == 0) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
        if (lact)
#pragma unroll
            for (int d = 0; d < 4; ++d) wo[warp][g][4 * lane + d] = o[g][d];
    }
    __syncthreads();
    float *pp = a.part + ((size_t)h * a.n_split + sp) * GQ * (HD + 2);
    for (uint32_t i = tid; i < (uint32_t)(GQ * HD); i += blockDim.x) {
        const uint32_t g = i / HD, d = i % HD;
        float M = wm[0][g];
        for (int w = 1; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][g]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = wm[w][g] == -INFINITY ? 0.f : expf(wm[w][g] - M);
            L = fmaf(wl[w][g], f, L);
            O = fmaf(wo[w][g][d], f, O);
        }
        pp[g * (HD + 2) + 2 + d] = O;
        if (d == 0) { pp[g * (HD + 2)] = M; pp[g * (HD + 2) + 1] = L; }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last_flag = (atomicAdd(&a.ticket[h], 1u) == a.n_split - 1) ? 1u : 0u;
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    const volatile float *P = a.part + (size_t)h * a.n_split * GQ * (HD + 2);
    for (uint32_t i = tid; i < (uint32_t)(GQ * HD); i += blockDim.x) {
        const uint32_t g = i / HD, d = i % HD;
        float M = -INFINITY;
        for (uint32_t s = 0; s < a.n_split; ++s) M = fmaxf(M, P[(s * GQ + g) * (HD + 2)]);
        float L = 0.f, O = 0.f;
        for (uint32_t s = 0; s < a.n_split; ++s) {
            const float ms = P[(s * GQ + g) * (HD + 2)];
            const float f = ms == -INFINITY ? 0.f : expf(ms - M);
            L = fmaf(P[(s * GQ + g) * (HD + 2) + 1], f, L);
            O = fmaf(P[(s * GQ + g) * (HD + 2) + 2 + d], f, O);
        }
        a.out[(size_t)(h * GQ + g) * HD + d] = __fdiv_rn(O, L);
    }
    if (tid == 0) a.ticket[h] = 0;
}

}  // namespace fwb
