// gemv.cuh — batch-1 dequant-fused GEMV over GGUF Q4_0 / Q5_0 / Q8_0 rows.
//
// Replaces quant_matvec (quant_matvec.c:263-312) and every linear_forward
// call of the decode step (attention.c:124-127,166; ffn.c:82-86,106;
// transformer.c:322), with the neighbouring elementwise work fused in.
//
// Work split.  A grid of one CTA per SM; CTA c owns a contiguous range of
// output rows, so its weights are one contiguous byte range of the GGUF
// tensor (the bytes are used in their GGUF layout, never repacked).
//
// Data movement.  A producer warp streams that range through a ring of
// shared-memory stages with 1-D bulk async copies (cp.async.bulk, no
// multicast) completing on mbarriers; it starts before griddepcontrol.wait,
// so under programmatic dependent launch the weights of this GEMV stream in
// while the previous kernel of the decode step is still running.
//
// Arithmetic.  Consumer thread (slot s, unit u) owns columns [64u, 64u+64)
// of one row per round.  Its 64 inputs are held in registers as 22-bit
// fixed-point integers per 32-block (scale s_b = max|x_b| / (2^21-1)), split
// into three byte planes, so each quant byte feeds dp4a directly:
//   block dot = d * s_b * (256*(256*A + B) + C - off * sum(xi))
// with A, B, C exact integer dot products of the quants with the high
// (signed), middle and low byte planes.  The products and sums are exact; the
// only rounding is the input's fixed-point representation (relative 2.4e-7
// of the block maximum) and three final float operations per block.
//
// Reduction.  Rows are processed in batches of 8 rounds; the 8 partial sums
// per thread are reduced across the unit lanes with a butterfly
// reduce-scatter (7 + log2(G/8) shuffles per 8 rows), then across warps in
// shared memory, and the epilogue runs on the finished rows.
#pragma once
#include "common.cuh"

namespace fwb {

enum QType : int { QT_Q4_0 = 2, QT_Q5_0 = 6, QT_Q8_0 = 8 };
template <int QT> struct QTraits;
template <> struct QTraits<QT_Q4_0> { static constexpr int BB = 18, OFF = 8; };
template <> struct QTraits<QT_Q5_0> { static constexpr int BB = 22, OFF = 16; };
template <> struct QTraits<QT_Q8_0> { static constexpr int BB = 34, OFF = 0; };

enum GemvMode : int {
    GM_STORE = 0,   // y[r]  = (W x)[r]
    GM_RESID = 1,   // y[r] += (W x)[r]                 (residual stream)
    GM_QKV = 2,     // rows [q | k | v]: RoPE on q, k; k, v appended to the KV cache
    GM_SWIGLU = 3,  // y[i]  = silu((Wg x)[i]) * (Wu x)[i]
    GM_LOGITS = 4,  // y[r]  = (W x)[r], plus the grid-wide greedy argmax
};
enum InMode : int { IN_PLAIN = 0, IN_RMSNORM = 1 };

constexpr int kRB = 8;              // rows per reduction batch (per slot)
constexpr int kMaxStages = 8;
constexpr uint32_t kHeaderBytes = 4096;
constexpr uint32_t kStageSlack = 128;  // alignment + half-unit over-read room
constexpr int kXMax = 2097151;      // 2^21 - 1, fixed-point range of the inputs

struct GemvArgs {
    const uint8_t *w;    // rows of the weight matrix (SWIGLU: gate)
    const uint8_t *w2;   // SWIGLU: up
    uint32_t n_out;      // output rows (SWIGLU: pairs)
    uint32_t K;          // input width, multiple of 32
    uint32_t row_bytes;  // K/32 * block bytes
    uint32_t gran;       // row granule of the CTA split (2 for QKV / SWIGLU pairs)
    uint32_t U, Upad, S, NC;  // units per row, padded to pow2 >= 8, slots, consumer threads
    uint32_t R;          // local rows per stage (multiple of S; even for pair modes)
    uint32_t NS;         // ring stages
    uint32_t stage_bytes;
    const float *x;      // input [K]
    const float *norm_w; // RMSNorm weight [K]
    float eps;
    float *y;            // output
    // GM_QKV
    uint32_t n_q, n_kv, head_dim, kv_ctx;
    const float *rope_cos, *rope_sin;  // [kv_ctx][head_dim/2]
    float *q_out, *kcache, *vcache;    // this layer's cache, [n_head_kv][kv_ctx][head_dim]
    // GM_LOGITS
    float *am_val;
    uint32_t *am_idx, *ticket, *out_token;
    const uint32_t *step;  // [0] token, [1] pos
    uint32_t *err;
};

// ---------------------------------------------------------------------------
// input planes
// ---------------------------------------------------------------------------
struct XBlock {
    uint32_t hi[8], mid[8], lo[8];  // 4 elements per word, element order 4k..4k+3
    int nx;                         // -OFF * sum(xi)
    float s;                        // s_b
};

template <int OFF>
__device__ __forceinline__ void quantize_block(const float *v, XBlock &b) {
    float m = 0.f;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        m = fmaxf(m, fabsf(v[j]));
        bad |= !isfinite(v[j]);
    }
    const float inv = m > 0.f ? (float)kXMax / m : 0.f;
    b.s = bad ? __int_as_float(0x7fc00000) : m * (1.0f / (float)kXMax);
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        int xi[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int t = __float2int_rn(v[4 * k + e] * inv);
            xi[e] = max(-kXMax, min(kXMax, t));
            sum += xi[e];
        }
        b.lo[k] = __byte_perm(__byte_perm(xi[0], xi[1], 0x0040), __byte_perm(xi[2], xi[3], 0x0040), 0x5410);
        b.mid[k] = __byte_perm(__byte_perm(xi[0], xi[1], 0x0051), __byte_perm(xi[2], xi[3], 0x0051), 0x5410);
        b.hi[k] = __byte_perm(__byte_perm(xi[0], xi[1], 0x0062), __byte_perm(xi[2], xi[3], 0x0062), 0x5410);
    }
    b.nx = -OFF * sum;
}

// ---------------------------------------------------------------------------
// block dots
// ---------------------------------------------------------------------------
__device__ __forceinline__ float finish_block(int A, int B, int C, const XBlock &x, uint32_t dbits) {
    const int U = A * 256 + B;
    const float T = fmaf((float)U, 256.0f, (float)(C + x.nx));
    return (f16_bits_to_f32(dbits) * x.s) * T;
}

// Q4_0: 4 quant words (elements 4k..4k+3 in the low nibbles, 16+4k.. in the high)
__device__ __forceinline__ float dot_q4_0(const uint32_t (&q)[4], uint32_t dbits, const XBlock &x) {
    int A = 0, B = 0, C = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t lo = q[k] & 0x0F0F0F0Fu, hi = (q[k] >> 4) & 0x0F0F0F0Fu;
        A = dp4a_us(lo, (int)x.hi[k], A);
        A = dp4a_us(hi, (int)x.hi[k + 4], A);
        B = dp4a_uu(lo, x.mid[k], B);
        B = dp4a_uu(hi, x.mid[k + 4], B);
        C = dp4a_uu(lo, x.lo[k], C);
        C = dp4a_uu(hi, x.lo[k + 4], C);
    }
    return finish_block(A, B, C, x, dbits);
}

// spread 4 bits into bit 4 of each byte
__device__ __forceinline__ uint32_t spread4(uint32_t b) { return ((b & 0xFu) * 0x02040810u) & 0x10101010u; }

// Q5_0: qh = 32-bit high-bit plane (bit j of element j), 4 low-nibble words
__device__ __forceinline__ float dot_q5_0(uint32_t qh, const uint32_t (&q)[4], uint32_t dbits, const XBlock &x) {
    int A = 0, B = 0, C = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t lo = (q[k] & 0x0F0F0F0Fu) | spread4(qh >> (4 * k));
        const uint32_t hi = ((q[k] >> 4) & 0x0F0F0F0Fu) | spread4(qh >> (16 + 4 * k));
        A = dp4a_us(lo, (int)x.hi[k], A);
        A = dp4a_us(hi, (int)x.hi[k + 4], A);
        B = dp4a_uu(lo, x.mid[k], B);
        B = dp4a_uu(hi, x.mid[k + 4], B);
        C = dp4a_uu(lo, x.lo[k], C);
        C = dp4a_uu(hi, x.lo[k + 4], C);
    }
    return finish_block(A, B, C, x, dbits);
}

// Q8_0: 8 signed quant words
__device__ __forceinline__ float dot_q8_0(const uint32_t (&q)[8], uint32_t dbits, const XBlock &x) {
    int A = 0, B = 0, C = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        A = dp4a_ss((int)q[k], (int)x.hi[k], A);
        B = dp4a_su((int)q[k], x.mid[k], B);
        C = dp4a_su((int)q[k], x.lo[k], C);
    }
    return finish_block(A, B, C, x, dbits);
}

// Words of one unit (two blocks, 2*BB bytes) starting at p (2-byte aligned;
// 4-byte aligned when A4).
template <int NWORDS, bool A4>
__device__ __forceinline__ void load_unit_words(const uint8_t *p, uint32_t (&w)[NWORDS]) {
    if (A4) {
        const uint32_t *q = reinterpret_cast<const uint32_t *>(p);
#pragma unroll
        for (int i = 0; i < NWORDS; ++i) w[i] = q[i];
    } else {
        const uintptr_t a = reinterpret_cast<uintptr_t>(p);
        const uint32_t *q = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
        const uint32_t sh = (uint32_t)(a & 3) * 8;
        uint32_t r[NWORDS + 1];
#pragma unroll
        for (int i = 0; i <= NWORDS; ++i) r[i] = q[i];
#pragma unroll
        for (int i = 0; i < NWORDS; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
    }
}

// Partial dot of one unit: block A always, block B when `two`.
template <int QT, bool A4>
__device__ __forceinline__ float unit_dot(const uint8_t *p, const XBlock &xa, const XBlock &xb, bool two) {
    if constexpr (QT == QT_Q4_0) {
        uint32_t w[9];
        load_unit_words<9, A4>(p, w);
        uint32_t qa[4] = {__funnelshift_r(w[0], w[1], 16), __funnelshift_r(w[1], w[2], 16),
                          __funnelshift_r(w[2], w[3], 16), __funnelshift_r(w[3], w[4], 16)};
        float r = dot_q4_0(qa, w[0], xa);
        if (two) {
            uint32_t qb[4] = {w[5], w[6], w[7], w[8]};
            r += dot_q4_0(qb, w[4] >> 16, xb);
        }
        return r;
    } else if constexpr (QT == QT_Q5_0) {
        uint32_t w[11];
        load_unit_words<11, A4>(p, w);
        uint32_t qa[4] = {__funnelshift_r(w[1], w[2], 16), __funnelshift_r(w[2], w[3], 16),
                          __funnelshift_r(w[3], w[4], 16), __funnelshift_r(w[4], w[5], 16)};
        float r = dot_q5_0(__funnelshift_r(w[0], w[1], 16), qa, w[0], xa);
        if (two) {
            uint32_t qb[4] = {w[7], w[8], w[9], w[10]};
            r += dot_q5_0(w[6], qb, w[5] >> 16, xb);
        }
        return r;
    } else {
        uint32_t w[17];
        load_unit_words<17, A4>(p, w);
        uint32_t qa[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) qa[k] = __funnelshift_r(w[k], w[k + 1], 16);
        float r = dot_q8_0(qa, w[0], xa);
        if (two) {
            uint32_t qb[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) qb[k] = w[9 + k];
            r += dot_q8_0(qb, w[8] >> 16, xb);
        }
        return r;
    }
}

// ---------------------------------------------------------------------------
// reduction: 8 partials per lane -> one row per lane group position
// ---------------------------------------------------------------------------
__device__ __forceinline__ float reduce8(float (&v)[kRB], uint32_t lane, uint32_t G, uint32_t &jj) {
    const uint32_t o1 = G >> 1, o2 = G >> 2, o3 = G >> 3;
    const unsigned FULL = 0xffffffffu;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const bool up = lane & o1;
        const float send = up ? v[i] : v[i + 4], keep = up ? v[i + 4] : v[i];
        v[i] = keep + __shfl_xor_sync(FULL, send, o1);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const bool up = lane & o2;
        const float send = up ? v[i] : v[i + 2], keep = up ? v[i + 2] : v[i];
        v[i] = keep + __shfl_xor_sync(FULL, send, o2);
    }
    {
        const bool up = lane & o3;
        const float send = up ? v[0] : v[1], keep = up ? v[1] : v[0];
        v[0] = keep + __shfl_xor_sync(FULL, send, o3);
    }
    for (uint32_t o = o3 >> 1; o >= 1; o >>= 1) v[0] += __shfl_xor_sync(FULL, v[0], o);
    jj = ((lane & o1) ? 4u : 0u) + ((lane & o2) ? 2u : 0u) + ((lane & o3) ? 1u : 0u);
    return v[0];
}

__device__ __forceinline__ float silu_ref(float v) {
    // ffn.c:17-25: two-sided sigmoid, then v * sig
    const float sig = v >= 0.0f ? __fdiv_rn(1.0f, 1.0f + expf(-v)) : __fdiv_rn(expf(v), 1.0f + expf(v));
    return __fmul_rn(v, sig);
}

// CTA row range [b, e) with granule g
__device__ __forceinline__ void cta_rows(uint32_t n_out, uint32_t g, uint32_t &b, uint32_t &e) {
    const uint32_t n = n_out / g;
    b = (uint32_t)((uint64_t)blockIdx.x * n / gridDim.x) * g;
    e = (uint32_t)((uint64_t)(blockIdx.x + 1) * n / gridDim.x) * g;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int QT, int MODE, int IN, bool A4, int MAXT, int MINB>
__global__ void __launch_bounds__(MAXT, MINB) gemv_kernel(const __grid_constant__ GemvArgs a) {
    constexpr int BB = QTraits<QT>::BB;
    constexpr int OFF = QTraits<QT>::OFF;
    constexpr bool PAIRED = (MODE == GM_SWIGLU);
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMaxStages;
    float *red = reinterpret_cast<float *>(smem + 256);       // [8][32]
    float *out_tile = red + kRB * 32;                         // [<= 8 * 64 pairs...] 512
    float *misc = out_tile + 512;                             // 64
    uint32_t *misc_u = reinterpret_cast<uint32_t *>(misc + 64);  // 64
    uint8_t *ring = smem + kHeaderBytes;

    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t NC = a.NC, NCW = NC >> 5;

    uint32_t rb, re;  // CTA range in output rows (pairs for SWIGLU)
    cta_rows(a.n_out, a.gran, rb, re);
    const uint32_t n_loc = PAIRED ? 2 * (re - rb) : (re - rb);  // local rows
    const uint32_t R = a.R, NS = a.NS;
    const uint32_t n_st = (n_loc + R - 1) / R;

    if (tid == 0) {
        for (uint32_t i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NCW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch();

    // ------------------------------------------------------------ producer
    if (warp == NCW) {
        if (lane != 0) return;
        uint32_t issued = 0;
        bool failed = false;
        for (uint32_t k = 0; k < n_st; ++k) {
            const uint32_t s = k % NS;
            if (k >= NS && !mbar_wait(&empty[s], ((k / NS) - 1) & 1, a.err, ERR_WAIT_EMPTY)) {
                failed = true;
                break;
            }
            uint8_t *dst = ring + (size_t)s * a.stage_bytes;
            if (!PAIRED) {
                const uint32_t r0 = k * R, nr = min(R, n_loc - r0);
                const uintptr_t src = reinterpret_cast<uintptr_t>(a.w) + (uint64_t)(rb + r0) * a.row_bytes;
                const uintptr_t s0 = src & ~uintptr_t(15);
                const uint32_t bytes = (uint32_t)(((src + (uint64_t)nr * a.row_bytes + 15) & ~uintptr_t(15)) - s0);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(dst, reinterpret_cast<const void *>(s0), bytes, &full[s]);
            } else {
                const uint32_t p0 = k * (R / 2), np = min(R / 2, (re - rb) - p0);
                const uint64_t off = (uint64_t)(rb + p0) * a.row_bytes;
                const uintptr_t g = reinterpret_cast<uintptr_t>(a.w) + off;
                const uintptr_t u = reinterpret_cast<uintptr_t>(a.w2) + off;
                const uintptr_t g0 = g & ~uintptr_t(15), u0 = u & ~uintptr_t(15);
                const uint32_t gb = (uint32_t)(((g + (uint64_t)np * a.row_bytes + 15) & ~uintptr_t(15)) - g0);
                const uint32_t ub = (uint32_t)(((u + (uint64_t)np * a.row_bytes + 15) & ~uintptr_t(15)) - u0);
                mbar_arrive_expect_tx(&full[s], gb + ub);
                bulk_g2s(dst, reinterpret_cast<const void *>(g0), gb, &full[s]);
                bulk_g2s(dst + a.stage_bytes / 2, reinterpret_cast<const void *>(u0), ub, &full[s]);
            }
            ++issued;
        }
        if (failed) {  // drain copies still in flight before the CTA may exit
            const uint32_t k0 = issued > NS ? issued - NS : 0;
            for (uint32_t k = k0; k < issued; ++k)
                mbar_wait(&full[k % NS], (k / NS) & 1, a.err, ERR_WAIT_DRAIN);
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    const uint32_t Upad = a.Upad, S = a.S, U = a.U;
    const uint32_t slot = tid / Upad, unit = tid % Upad;
    const uint32_t nb = a.K >> 5;
    const bool active = slot < S && unit < U;
    const bool two = active && (2 * unit + 1 < nb);
    const uint32_t G = Upad < 32 ? Upad : 32;

    pdl_wait();  // inputs of this GEMV are outputs of the previous kernel

    // input vector -> fixed-point planes
    float scale = 1.0f;
    if (IN == IN_RMSNORM) {
        // rms_norm, norm.c:7-16: scale = 1/sqrtf(sum(x^2)/n + eps); out = (x*w)*scale
        float ss = 0.f;
        for (uint32_t i = tid; i < a.K; i += NC) ss = fmaf(a.x[i], a.x[i], ss);
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) misc[warp] = ss;
        bar_sync(1, NC);
        if (warp == 0) {
            float t = lane < NCW ? misc[lane] : 0.f;
#pragma unroll
            for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
            if (lane == 0) misc[32] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)a.K), a.eps)));
        }
        bar_sync(1, NC);
        scale = misc[32];
    }
    XBlock xa, xb;
    {
        float v[32];
        const uint32_t c0 = unit * 64;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            float t = 0.f;
            if (active) {
                t = a.x[c0 + j];
                if (IN == IN_RMSNORM) t = __fmul_rn(__fmul_rn(t, a.norm_w[c0 + j]), scale);
            }
            v[j] = t;
        }
        quantize_block<OFF>(v, xa);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            float t = 0.f;
            if (two) {
                t = a.x[c0 + 32 + j];
                if (IN == IN_RMSNORM) t = __fmul_rn(__fmul_rn(t, a.norm_w[c0 + 32 + j]), scale);
            }
            v[j] = t;
        }
        quantize_block<OFF>(v, xb);
    }

    const uint32_t n_rounds = (n_loc + S - 1) / S;
    const uint32_t RPS = R / S;
    uint32_t pos = 0;
    if (MODE == GM_QKV) pos = a.step[1];
    bool failed = false;

    float best_v = -INFINITY;
    uint32_t best_i = 0xffffffffu;

    uint32_t stage = 0, in_stage = 0;  // stage index, round within stage
    const uint8_t *sbase = ring;
    uint32_t delta_a = 0, delta_b = 0;

    for (uint32_t r0 = 0; r0 < n_rounds; r0 += kRB) {
        float acc[kRB];
#pragma unroll
        for (int j = 0; j < kRB; ++j) {
            acc[j] = 0.f;
            const uint32_t r = r0 + j;
            if (r < n_rounds) {
                if (in_stage == 0) {
                    const uint32_t s = stage % NS;
                    if (!failed) failed = !mbar_wait(&full[s], (stage / NS) & 1, a.err, ERR_WAIT_FULL);
                    sbase = ring + (size_t)s * a.stage_bytes;
                    if (!PAIRED) {
                        const uintptr_t src = reinterpret_cast<uintptr_t>(a.w) +
                                              (uint64_t)(rb + stage * R) * a.row_bytes;
                        delta_a = (uint32_t)(src & 15);
                    } else {
                        const uint64_t off = (uint64_t)(rb + stage * (R / 2)) * a.row_bytes;
                        delta_a = (uint32_t)((reinterpret_cast<uintptr_t>(a.w) + off) & 15);
                        delta_b = (uint32_t)((reinterpret_cast<uintptr_t>(a.w2) + off) & 15);
                    }
                }
                const uint32_t l = r * S + slot;  // local row
                if (active && l < n_loc && !failed) {
                    const uint32_t ls = l - stage * R;  // row within stage
                    const uint8_t *rowp;
                    if (!PAIRED) {
                        rowp = sbase + delta_a + (size_t)ls * a.row_bytes;
                    } else {
                        const uint32_t pr = ls >> 1;
                        rowp = (ls & 1) ? sbase + a.stage_bytes / 2 + delta_b + (size_t)pr * a.row_bytes
                                        : sbase + delta_a + (size_t)pr * a.row_bytes;
                    }
                    acc[j] = unit_dot<QT, A4>(rowp + unit * (2 * BB), xa, xb, two);
                }
                if (++in_stage == RPS || r + 1 == n_rounds) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[stage % NS]);
                    in_stage = 0;
                    ++stage;
                }
            }
        }

        // ---- reduce the batch
        uint32_t jj;
        const float v = reduce8(acc, lane, G, jj);
        const uint32_t nbr = min((uint32_t)kRB, n_rounds - r0);
        if (Upad <= 32) {
            if ((lane & ((G >> 3) - 1)) == 0 && slot < S) out_tile[jj * S + slot] = v;
        } else {
            if ((lane & 3) == 0) red[jj * 32 + warp] = v;
            bar_sync(1, NC);
            const uint32_t W = Upad >> 5;
            if (tid < kRB * S) {
                const uint32_t j = tid % kRB, s = tid / kRB;
                float t = 0.f;
                for (uint32_t w = 0; w < W; ++w) t += red[j * 32 + s * W + w];
                out_tile[j * S + s] = t;
            }
        }
        bar_sync(1, NC);

        // ---- epilogue on local rows [r0*S, r0*S + nbr*S) ∩ [0, n_loc)
        const uint32_t l0 = r0 * S;
        const uint32_t cnt = min(nbr * S, n_loc - l0);
        if (!failed) {
            if (MODE == GM_STORE || MODE == GM_RESID || MODE == GM_LOGITS) {
                for (uint32_t i = tid; i < cnt; i += NC) {
                    const uint32_t g = rb + l0 + i;
                    const float t = out_tile[i];
                    if (MODE == GM_STORE) a.y[g] = t;
                    if (MODE == GM_RESID) a.y[g] = __fadd_rn(a.y[g], t);
                    if (MODE == GM_LOGITS) {
                        a.y[g] = t;
                        if (t > best_v || (t == best_v && g < best_i)) { best_v = t; best_i = g; }
                    }
                }
            } else if (MODE == GM_SWIGLU) {
                for (uint32_t i = tid; 2 * i < cnt; i += NC) {
                    const uint32_t p = rb + (l0 >> 1) + i;
                    a.y[p] = __fmul_rn(silu_ref(out_tile[2 * i]), out_tile[2 * i + 1]);
                }
            } else if (MODE == GM_QKV) {
                const uint32_t half = a.head_dim >> 1;
                for (uint32_t i = tid; 2 * i < cnt; i += NC) {
                    const uint32_t g = rb + l0 + 2 * i;
                    const float v0 = out_tile[2 * i], v1 = out_tile[2 * i + 1];
                    if (g < a.n_q + a.n_kv) {
                        const uint32_t gg = g < a.n_q ? g : g - a.n_q;
                        const uint32_t d = gg % a.head_dim;
                        const float c = a.rope_cos[pos * half + d / 2], s = a.rope_sin[pos * half + d / 2];
                        // rope.c:37-43 (adjacent pairs)
                        const float r0v = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
                        const float r1v = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
                        if (g < a.n_q) {
                            a.q_out[g] = r0v;
                            a.q_out[g + 1] = r1v;
                        } else {
                            const uint32_t h = gg / a.head_dim;
                            float *dst = a.kcache + ((size_t)h * a.kv_ctx + pos) * a.head_dim + d;
                            dst[0] = r0v;
                            dst[1] = r1v;
                        }
                    } else {
                        const uint32_t gv = g - a.n_q - a.n_kv;
                        const uint32_t h = gv / a.head_dim, d = gv % a.head_dim;
                        float *dst = a.vcache + ((size_t)h * a.kv_ctx + pos) * a.head_dim + d;
                        dst[0] = v0;
                        dst[1] = v1;
                    }
                }
            }
        }
        bar_sync(1, NC);
    }

    if (MODE == GM_LOGITS) {
        // CTA argmax, then the last CTA to finish reduces the per-CTA results
        // (sampler.c:28-32 semantics: the lowest index wins among equal maxima)
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ov > best_v || (ov == best_v && oi < best_i)) { best_v = ov; best_i = oi; }
        }
        if (lane == 0) { misc[warp] = best_v; misc_u[warp] = best_i; }
        bar_sync(1, NC);
        if (tid == 0) {
            float bv = misc[0];
            uint32_t bi = misc_u[0];
            for (uint32_t w = 1; w < NCW; ++w)
                if (misc[w] > bv || (misc[w] == bv && misc_u[w] < bi)) { bv = misc[w]; bi = misc_u[w]; }
            a.am_val[blockIdx.x] = bv;
            a.am_idx[blockIdx.x] = bi;
            __threadfence();
            const uint32_t t = atomicAdd(a.ticket, 1u);
            if (t == gridDim.x - 1) {
                __threadfence();
                float gv = -INFINITY;
                uint32_t gi = 0xffffffffu;
                for (uint32_t c = 0; c < gridDim.x; ++c) {
                    const float cv = *(volatile float *)&a.am_val[c];
                    const uint32_t ci = *(volatile uint32_t *)&a.am_idx[c];
                    if (cv > gv || (cv == gv && ci < gi)) { gv = cv; gi = ci; }
                }
                // all logits NaN: the reference keeps index 0
                *a.out_token = gi == 0xffffffffu ? 0u : gi;
                *a.ticket = 0;
            }
        }
    }
}

}  // namespace fwb
