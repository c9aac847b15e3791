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
// contiguous range.  Each warp runs an online softmax over tiles of 16/GQ
// positions (8 when GQ = 1): lanes own 4 dims, the (position, head) partial
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
    uint32_t kv_ctx, n_split, n_kv;
    float scale;           // 1/sqrtf(head_dim), attention.c:143
    const uint32_t *step;  // [1] = pos
    uint32_t *err;
    unsigned long long *trace;  // optional (tracing): every CTA's timeline of its item, [cta][8]
};

__device__ __forceinline__ void attn_stamp(const AttnArgs &a, int i) {
    if (a.trace && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
        a.trace[blockIdx.x * 8 + i] = t;
    }
}

constexpr int kAttnWarps = 4;          // warps per CTA of the standalone kernel
constexpr uint32_t kMinSplitPos = 32;   // positions per split at least
constexpr uint32_t kMaxSplits = 64;

// Splits in use at n_pos positions (short contexts merge few partials).
__device__ __forceinline__ uint32_t attn_splits_in_use(const AttnArgs &a, uint32_t n_pos) {
    return min(a.n_split, (n_pos + kMinSplitPos - 1) / kMinSplitPos);
}

// Shared scratch of one attention item for NW warps.
template <int HD, int GQ, int NW>
struct AttnSmem {
    float pbuf[NW][32];
    float wm[NW][GQ], wl[NW][GQ];
    float wo[NW][GQ][HD];
    float wf[NW][GQ], wM[GQ];  // per-warp rescale factors exp(m_w - M) and the CTA maximum
    float mw[GQ][kMaxSplits], mL[GQ];  // split merge: per-split weights and the total per head
    uint32_t last_flag;
};

// Merge the n_use split partials of KV head h into the output (the last CTA
// of the head to finish runs this; all its threads).  Warp g (one per query
// head) loads the (max, sum) pairs of the splits, one split per lane, and
// turns them into the weights f_s = exp(m_s - M) and the total L in shared
// memory; meanwhile every thread has its element's split values in flight
// (one coalesced load per split).  After one CTA barrier each thread sums its
// values in split order with the weights read from shared memory.
template <int HD, int GQ, int NW>
__device__ __noinline__ void attn_merge(const AttnArgs &a, uint32_t h, uint32_t n_use, AttnSmem<HD, GQ, NW> &sh) {
    constexpr uint32_t NE = (uint32_t)(GQ * HD), ST = HD + 2;
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned FULL = 0xffffffffu;
    const float *P = a.part + (size_t)h * a.n_split * GQ * ST;
    const long long c0 = clock64();
    // this thread's element (the first of them when NE > blockDim.x)
    const uint32_t i_first = min(tid, NE - 1), g_first = i_first / HD, d_first = i_first % HD;
    const uint32_t n_a = min(n_use, 32u);
    float v[32];
#pragma unroll
    for (uint32_t k = 0; k < 32; ++k)
        v[k] = k < n_a ? __ldcg(P + ((size_t)k * GQ + g_first) * ST + 2 + d_first) : 0.f;
    for (uint32_t g = warp; g < (uint32_t)GQ; g += blockDim.x >> 5) {
        float2 ml[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t s = lane + 32u * k;
            ml[k] = s < n_use ? __ldcg(reinterpret_cast<const float2 *>(P + ((size_t)s * GQ + g) * ST))
                              : make_float2(-INFINITY, 0.f);
        }
        float M = fmaxf(ml[0].x, ml[1].x);
#pragma unroll
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, o));
        float f[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) f[k] = ml[k].x == -INFINITY ? 0.f : expf(ml[k].x - M);
        float L = fmaf(ml[1].y, f[1], ml[0].y * f[0]);
#pragma unroll
        for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(FULL, L, o);
        sh.mw[g][lane] = f[0];
        sh.mw[g][lane + 32] = f[1];
        if (lane == 0) sh.mL[g] = L;
    }
    __syncthreads();
    if (a.trace && tid == 0) a.trace[blockIdx.x * 8 + 6] = clock64() - c0;  // weights ready (SM clocks)
    for (uint32_t i = tid; i < NE; i += blockDim.x) {
        const uint32_t g = i / HD, d = i % HD;
        float O = 0.f;
        if (i == tid) {
#pragma unroll
            for (uint32_t k = 0; k < 32; ++k)
                if (k < n_a) O = fmaf(v[k], sh.mw[g][k], O);
        } else {  // a further element of this thread (small CTAs)
            for (uint32_t k = 0; k < n_a; ++k) O = fmaf(__ldcg(P + ((size_t)k * GQ + g) * ST + 2 + d), sh.mw[g][k], O);
        }
        for (uint32_t s0 = 32; s0 < n_use; s0 += 16) {  // beyond 32 splits: 16 more per round trip
            float u[16];
#pragma unroll
            for (uint32_t k = 0; k < 16; ++k) u[k] = s0 + k < n_use ? __ldcg(P + ((size_t)(s0 + k) * GQ + g) * ST + 2 + d) : 0.f;
#pragma unroll
            for (uint32_t k = 0; k < 16; ++k)
                if (s0 + k < n_use) O = fmaf(u[k], sh.mw[g][s0 + k], O);
        }
        a.out[(size_t)(h * GQ + g) * HD + d] = __fdiv_rn(O, sh.mL[g]);
    }
    if (a.trace && tid == 0) a.trace[blockIdx.x * 8 + 7] = clock64() - c0;
    if (tid == 0) a.ticket[h] = 0;
}

// One work item: KV head h, split sp of n_use.  All NW warps of the CTA take
// part.  K/V, q and the partials are read with L2-only loads (other CTAs of
// the persistent kernel wrote them in this very step).
template <int HD, int GQ, int NW>
__device__ void attn_item(const AttnArgs &a, uint32_t h, uint32_t sp, uint32_t n_pos, uint32_t n_use,
                          AttnSmem<HD, GQ, NW> &sh) {
    static_assert(HD % 4 == 0 && HD <= 128, "head_dim");
    static_assert(GQ == 1 || GQ == 2 || GQ == 4 || GQ == 8, "group");
    // positions per tile: 16 (position, head) dots per tile for GQ >= 2
    // (8 for GQ = 1), keeping the K/V tile in registers within the budget
    constexpr int TILE = GQ == 1 ? 8 : 16 / GQ;
    constexpr int NVAL = TILE * GQ;                       // partial dots per tile (8 or 16)
    constexpr int REP = 32 / NVAL;                        // lanes holding each finished value
    constexpr int LA = HD / 4;                            // active lanes
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const uint32_t chunk = (n_pos + n_use - 1) / n_use;
    const uint32_t c0 = min(n_pos, sp * chunk), c1 = min(n_pos, c0 + chunk);
    const uint32_t wchunk = (c1 - c0 + NW - 1) / NW;
    const uint32_t w0 = min(c1, c0 + warp * wchunk), w1 = min(c1, w0 + wchunk);

    const bool lact = lane < LA;
    float qv[GQ][4], o[GQ][4], m[GQ], l[GQ];
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        const float4 t = lact ? __ldcg(reinterpret_cast<const float4 *>(a.q + (size_t)(h * GQ + g) * HD + 4 * lane))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        qv[g][0] = t.x; qv[g][1] = t.y; qv[g][2] = t.z; qv[g][3] = t.w;
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int d = 0; d < 4; ++d) o[g][d] = 0.f;
    }
    const float *kb = a.kc + (size_t)h * a.kv_ctx * HD + 4 * lane;
    const float *vb = a.vc + (size_t)h * a.kv_ctx * HD + 4 * lane;

    attn_stamp(a, 0);
    for (uint32_t t0 = w0; t0 < w1; t0 += TILE) {
        float4 kt[TILE], vt[TILE];
#pragma unroll
        for (int p = 0; p < TILE; ++p) {
            const bool ok = lact && t0 + p < w1;
            kt[p] = ok ? __ldcg(reinterpret_cast<const float4 *>(kb + (size_t)(t0 + p) * HD)) : make_float4(0.f, 0.f, 0.f, 0.f);
            vt[p] = ok ? __ldcg(reinterpret_cast<const float4 *>(vb + (size_t)(t0 + p) * HD)) : make_float4(0.f, 0.f, 0.f, 0.f);
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
        sh.pbuf[warp][vi] = pe;  // the REP lanes of a value write the same number
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
                const float w = sh.pbuf[warp][p * GQ + g];
                o[g][0] = fmaf(w, vt[p].x, o[g][0]);
                o[g][1] = fmaf(w, vt[p].y, o[g][1]);
                o[g][2] = fmaf(w, vt[p].z, o[g][2]);
                o[g][3] = fmaf(w, vt[p].w, o[g][3]);
            }
        __syncwarp();
    }

    attn_stamp(a, 1);  // warp 0's positions done
    // merge the warps of this CTA
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
        if (lane == 0) { sh.wm[warp][g] = m[g]; sh.wl[warp][g] = l[g]; }
        if (lact)
#pragma unroll
            for (int d = 0; d < 4; ++d) sh.wo[warp][g][4 * lane + d] = o[g][d];
    }
    __syncthreads();
    // rescale factor of every (warp, head), once: exp(m_w - M)
    if (tid < (uint32_t)(NW * GQ)) {
        const uint32_t w = tid / GQ, g = tid % GQ;
        float M = sh.wm[0][g];
        for (int v = 1; v < NW; ++v) M = fmaxf(M, sh.wm[v][g]);
        sh.wf[w][g] = sh.wm[w][g] == -INFINITY ? 0.f : expf(sh.wm[w][g] - M);
        if (w == 0) sh.wM[g] = M;
    }
    __syncthreads();
    if (n_use == 1) {  // the only split: normalise and write the output directly
        for (uint32_t i = tid; i < (uint32_t)(GQ * HD); i += blockDim.x) {
            const uint32_t g = i / HD, d = i % HD;
            float L = 0.f, O = 0.f;
            for (int w = 0; w < NW; ++w) {
                L = fmaf(sh.wl[w][g], sh.wf[w][g], L);
                O = fmaf(sh.wo[w][g][d], sh.wf[w][g], O);
            }
            a.out[(size_t)(h * GQ + g) * HD + d] = __fdiv_rn(O, L);
        }
        __syncthreads();
        return;
    }
    float *pp = a.part + ((size_t)h * a.n_split + sp) * GQ * (HD + 2);
    for (uint32_t i = tid; i < (uint32_t)(GQ * HD); i += blockDim.x) {
        const uint32_t g = i / HD, d = i % HD;
        float L = 0.f, O = 0.f;
        for (int w = 0; w < NW; ++w) {
            L = fmaf(sh.wl[w][g], sh.wf[w][g], L);
            O = fmaf(sh.wo[w][g][d], sh.wf[w][g], O);
        }
        pp[g * (HD + 2) + 2 + d] = O;
        if (d == 0) { pp[g * (HD + 2)] = sh.wM[g]; pp[g * (HD + 2) + 1] = L; }
    }
    attn_stamp(a, 2);  // partial written
    // The CTA barrier orders every thread's partial before thread 0's release
    // fence (cumulativity); the fence after the ticket makes the other CTAs'
    // partials visible to this CTA's loads after the next barrier.
    __syncthreads();
    attn_stamp(a, 3);
    if (tid == 0) {
        fence_acq_rel_gpu();
        const bool last = atomicAdd(&a.ticket[h], 1u) == n_use - 1;
        if (last) fence_acq_rel_gpu();
        sh.last_flag = last ? 1u : 0u;
    }
    __syncthreads();
    attn_stamp(a, 4);  // ticket
    if (sh.last_flag) attn_merge<HD, GQ, NW>(a, h, n_use, sh);
    attn_stamp(a, 5);  // merged (last CTA) / done
    __syncthreads();  // the scratch may be reused by the next item
}

// Standalone kernel: grid (n_kv, n_split), one item per CTA.
template <int HD, int GQ>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
    __shared__ AttnSmem<HD, GQ, kAttnWarps> sh;
    pdl_launch();
    pdl_wait();
    const uint32_t n_pos = a.step[1] + 1;
    const uint32_t n_use = attn_splits_in_use(a, n_pos);
    if (blockIdx.y >= n_use) return;
    attn_item<HD, GQ, kAttnWarps>(a, blockIdx.x, blockIdx.y, n_pos, n_use, sh);
}

}  // namespace fwb
