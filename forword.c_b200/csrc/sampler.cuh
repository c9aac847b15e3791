// sampler.cuh — the reference's token sampling on the device logits.
//
// main.c:176-188 with sampler.c:46-100: repetition penalty over the token
// history, then either the greedy argmax (temperature <= 0) or temperature +
// softmax + top-p (nucleus) sampling with one uniform draw.  Replaces the
// 0.5 MB logits copy to the host and the host qsort of the whole vocabulary.
//
// One CTA.  The nucleus is found without sorting: the reference sorts the
// probabilities in descending order (ties by index) and takes the shortest
// prefix whose running sum reaches top_p; the same prefix is located by a
// radix select over the probabilities' float bits (non-negative floats order
// like their bit patterns), 8 bits per pass, with per-digit counts and sums
// in 256 bins; the draw is located the same way inside the nucleus.  Sums
// are kept in 40-bit fixed point (u64), so they do not depend on the order
// of the atomic adds: the result is deterministic.  It can differ from the
// reference only where the draw or top_p falls within the rounding drift of
// the reference's fp32 running sum (~1e-6 of the total over a nucleus of
// thousands of tokens) of a cumulative boundary.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "common.cuh"

namespace fwb {

constexpr uint32_t kSampleThreads = 1024;
constexpr double kFix = 1099511627776.0;  // 2^40

struct SampleArgs {
    const float *lg[kMaxRanks];  // logits slices (one per rank; world 1: lg[0] holds all)
    uint32_t n, slice, world;    // vocabulary size, entries per slice
    float *w;                    // scratch [n]: penalised / scaled logits, then probabilities
    uint32_t *cnt;               // scratch [n], zero on entry and on exit
    const uint32_t *hist;        // [n_hist] token history (prompt and generated tokens)
    uint32_t n_hist;
    float temp, top_p, pen;
    float u;                     // uniform draw: (xorshift64 >> 11) / (UINT64_MAX >> 11), as sampler.c:93
    uint32_t *out;               // chosen token
};

struct SampleSmem {
    unsigned long long sum[256];
    uint32_t count[256];
    float red_f[32];
    uint32_t red_u[32];
    unsigned long long acc;       // fixed-point sum of the elements above the current prefix
    uint32_t prefix, mask, sel, ties;
    uint32_t tie_prefix[kSampleThreads / 32];
};
// per-warp digit histograms (dynamic shared memory): counts [32][256], then sums [32][256]
constexpr uint32_t kSampleDynSmem = (kSampleThreads / 32) * 256 * (4 + 8);

__device__ __forceinline__ unsigned long long umin64(unsigned long long x, unsigned long long y) { return x < y ? x : y; }

__device__ __forceinline__ float sample_logit(const SampleArgs &a, uint32_t i) {
    return a.world == 1 ? a.lg[0][i] : __ldcg(a.lg[i / a.slice] + i % a.slice);
}

// block-wide reductions (fixed order)
__device__ __forceinline__ float block_max(float v, SampleSmem &sh) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) sh.red_f[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = sh.red_f[0];
    for (uint32_t k = 1; k < blockDim.x / 32; ++k) r = fmaxf(r, sh.red_f[k]);
    __syncthreads();
    return r;
}
__device__ __forceinline__ float block_sum(float v, SampleSmem &sh) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sh.red_f[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = sh.red_f[0];
    for (uint32_t k = 1; k < blockDim.x / 32; ++k) r += sh.red_f[k];
    __syncthreads();
    return r;
}

// Radix select over keys = probability bits, in descending order: returns
// (in sh.prefix) the key of the element where the running sum of the
// probabilities, taken in descending order, first reaches `target` (fixed
// point), with sh.acc = the sum of all elements with a larger key.  Only
// keys >= floor_key take part (the nucleus restriction of the draw).
__device__ void radix_select(const SampleArgs &a, SampleSmem &sh, uint32_t *wcount, unsigned long long *wsum,
                             unsigned long long target, uint32_t floor_key) {
    const uint32_t tid = threadIdx.x, warp = tid >> 5, nw = blockDim.x >> 5;
    uint32_t *wc = wcount + warp * 256;
    unsigned long long *ws = wsum + warp * 256;
    if (tid == 0) { sh.prefix = 0; sh.mask = 0; sh.acc = 0; sh.ties = 0; }
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (uint32_t b = tid & 31; b < 256; b += 32) { wc[b] = 0; ws[b] = 0; }
        __syncthreads();
        const uint32_t prefix = sh.prefix, mask = sh.mask;
        for (uint32_t i = tid; i < a.n; i += blockDim.x) {
            const float p = a.w[i];
            const uint32_t k = __float_as_uint(p);
            if (k < floor_key || (k & mask) != prefix) continue;
            const uint32_t d = (k >> shift) & 0xffu;
            atomicAdd(&wc[d], 1u);
            atomicAdd(&ws[d], __double2ull_rn((double)p * kFix));
        }
        __syncthreads();
        for (uint32_t b = tid; b < 256; b += blockDim.x) {  // the warps' histograms, in warp order
            uint32_t c = 0;
            unsigned long long t = 0;
            for (uint32_t w = 0; w < nw; ++w) { c += wcount[w * 256 + b]; t += wsum[w * 256 + b]; }
            sh.count[b] = c;
            sh.sum[b] = t;
        }
        __syncthreads();
        if (tid == 0) {
            // digits from the largest down: the first whose sum reaches the
            // target; if none does (rounding at the end of the range), the
            // smallest non-empty digit, as the reference falls back to the
            // last element of its sorted range
            unsigned long long acc = sh.acc, acc_last = sh.acc;
            int sel = -1, last = -1;
            for (int b = 255; b >= 0; --b) {
                if (!sh.count[b]) continue;
                if (acc + sh.sum[b] >= target) { sel = b; break; }
                last = b;
                acc_last = acc;
                acc += sh.sum[b];
            }
            if (sel < 0) {
                sel = last < 0 ? 0 : last;
                acc = acc_last;
            }
            sh.acc = acc;
            sh.prefix = prefix | ((uint32_t)sel << shift);
            sh.mask = mask | (0xffu << shift);
            sh.ties = sh.count[sel];
        }
        __syncthreads();
    }
}

// Index of the m-th (1-based) element with key == key (index order), or the
// last such element if fewer exist.  Every thread scans a contiguous chunk.
__device__ uint32_t nth_with_key(const SampleArgs &a, SampleSmem &sh, uint32_t key, uint32_t m) {
    const uint32_t tid = threadIdx.x, nt = blockDim.x;
    const uint32_t chunk = (a.n + nt - 1) / nt, b = tid * chunk, e = min(a.n, b + chunk);
    uint32_t c = 0;
    for (uint32_t i = b; i < e; ++i) c += __float_as_uint(a.w[i]) == key;
    // exclusive scan over threads (warp scan, then warp totals)
    uint32_t x = c;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if ((tid & 31) >= (uint32_t)o) x += y;
    }
    if ((tid & 31) == 31) sh.tie_prefix[tid >> 5] = x;
    __syncthreads();
    if (tid == 0) {
        uint32_t run = 0;
        for (uint32_t w = 0; w < nt / 32; ++w) { const uint32_t t = sh.tie_prefix[w]; sh.tie_prefix[w] = run; run += t; }
        sh.sel = 0xffffffffu;
        sh.red_u[0] = run;  // total count
    }
    __syncthreads();
    const uint32_t total = sh.red_u[0];
    const uint32_t want = min(m, total);
    const uint32_t before = sh.tie_prefix[tid >> 5] + x - c;
    if (want && before < want && before + c >= want) {
        uint32_t k = before;
        for (uint32_t i = b; i < e; ++i)
            if (__float_as_uint(a.w[i]) == key && ++k == want) { sh.sel = i; break; }
    }
    __syncthreads();
    return sh.sel;
}

__global__ void __launch_bounds__(kSampleThreads, 1) sample_kernel(const __grid_constant__ SampleArgs a) {
    __shared__ SampleSmem sh;
    extern __shared__ __align__(16) uint8_t dyn[];
    unsigned long long *wsum = reinterpret_cast<unsigned long long *>(dyn);
    uint32_t *wcount = reinterpret_cast<uint32_t *>(dyn + (kSampleThreads / 32) * 256 * 8);
    const uint32_t tid = threadIdx.x, nt = blockDim.x;
    // logits -> scratch; repetition penalty (sampler.c:86-100): every
    // occurrence of a token in the history applies the penalty once more
    for (uint32_t i = tid; i < a.n; i += nt) a.w[i] = sample_logit(a, i);
    __syncthreads();
    if (a.pen != 1.0f) {
        for (uint32_t j = tid; j < a.n_hist; j += nt)
            if (a.hist[j] < a.n) atomicAdd(&a.cnt[a.hist[j]], 1u);
        __syncthreads();
        for (uint32_t j = tid; j < a.n_hist; j += nt) {
            const uint32_t id = a.hist[j];
            if (id >= a.n) continue;
            const uint32_t c = atomicExch(&a.cnt[id], 0u);
            if (!c) continue;
            float x = a.w[id];
            for (uint32_t k = 0; k < c; ++k) x = x > 0.0f ? __fdiv_rn(x, a.pen) : __fmul_rn(x, a.pen);
            a.w[id] = x;
        }
        __syncthreads();
    }
    if (a.temp <= 0.0f) {  // sampler_argmax (sampler.c:28-32) on the penalised logits
        float bv = -INFINITY;
        uint32_t bi = 0xffffffffu;
        for (uint32_t i = tid; i < a.n; i += nt) {
            const float v = a.w[i];
            if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
        }
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if ((tid & 31) == 0) { sh.red_f[tid >> 5] = bv; sh.red_u[tid >> 5] = bi; }
        __syncthreads();
        if (tid == 0) {
            bv = sh.red_f[0];
            bi = sh.red_u[0];
            for (uint32_t k = 1; k < nt / 32; ++k)
                if (sh.red_f[k] > bv || (sh.red_f[k] == bv && sh.red_u[k] < bi)) { bv = sh.red_f[k]; bi = sh.red_u[k]; }
            // a NaN at index 0 is never beaten; all NaN: index 0
            *a.out = (isnan(a.w[0]) || bi == 0xffffffffu) ? 0u : bi;
        }
        return;
    }
    // temperature (sampler.c:12-16), softmax (sampler.c:18-26)
    if (a.temp != 1.0f) {
        const float inv = __fdiv_rn(1.0f, a.temp);
        for (uint32_t i = tid; i < a.n; i += nt) a.w[i] = __fmul_rn(a.w[i], inv);
        __syncthreads();
    }
    float mx = -INFINITY;
    for (uint32_t i = tid; i < a.n; i += nt) mx = fmaxf(mx, a.w[i]);
    mx = block_max(mx, sh);
    float s = 0.f;
    for (uint32_t i = tid; i < a.n; i += nt) {
        const float e = expf(a.w[i] - mx);
        a.w[i] = e;
        s += e;
    }
    const float inv = __fdiv_rn(1.0f, block_sum(s, sh));
    for (uint32_t i = tid; i < a.n; i += nt) a.w[i] = __fmul_rn(a.w[i], inv);
    __syncthreads();

    // nucleus (sampler.c:76-82): the shortest descending prefix with sum >= top_p
    const unsigned long long tp = __double2ull_rn((double)a.top_p * kFix);
    radix_select(a, sh, wcount, wsum, tp, 0u);
    const uint32_t kn = sh.prefix, ties_n = max(1u, sh.ties);
    const unsigned long long above_n = sh.acc;
    const unsigned long long pn = __double2ull_rn((double)__uint_as_float(kn) * kFix);
    // equal probabilities at the boundary: the first m_n of them (index order)
    uint32_t m_n = ties_n;
    if (pn > 0 && tp > above_n) m_n = (uint32_t)umin64((unsigned long long)ties_n, (tp - above_n + pn - 1) / pn);
    if (m_n == 0) m_n = 1;
    const double norm = ((double)above_n + (double)m_n * (double)pn) / kFix;
    // the draw (sampler.c:85-92): r = u * norm; the first element whose running
    // sum reaches r, within the nucleus
    const float r = __fmul_rn(a.u, (float)norm);
    const unsigned long long rt = __double2ull_rn((double)r * kFix);
    radix_select(a, sh, wcount, wsum, rt, kn);
    const uint32_t kd = sh.prefix, ties_d = max(1u, sh.ties);
    const unsigned long long above_d = sh.acc;
    const unsigned long long pd = __double2ull_rn((double)__uint_as_float(kd) * kFix);
    uint32_t m_d = ties_d;
    if (pd > 0 && rt > above_d) m_d = (uint32_t)umin64((unsigned long long)ties_d, (rt - above_d + pd - 1) / pd);
    if (m_d == 0) m_d = 1;
    if (kd == kn && m_d > m_n) m_d = m_n;  // stay inside the nucleus
    const uint32_t idx = nth_with_key(a, sh, kd, m_d);
    if (tid == 0) *a.out = idx == 0xffffffffu ? 0u : idx;
}

}  // namespace fwb
