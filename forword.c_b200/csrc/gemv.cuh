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
// Data movement.  The range streams through a ring of shared-memory stages
// with 1-D bulk async copies (cp.async.bulk, no multicast) completing on
// mbarriers.  There is no producer warp: all 16 warps compute, and the last
// warp to finish with a stage (a shared-memory counter per stage) issues the
// copy that refills it.  The first NS stages are issued before
// griddepcontrol.wait, so under programmatic dependent launch the weights of
// this GEMV stream in while the previous kernel is still running (in the
// persistent decode kernel the ring runs on across phases instead).
//
// Arithmetic.  Consumer thread (slot s, unit u) owns columns [64u, 64u+64)
// of RPT rows per round (independent instruction streams).  Its 64 inputs are
// held in registers as 24-bit fixed-point integers per 32-block
// (X = rint(x / s_b) rounded once from the exact quotient, scale
// s_b = max|x_b| / (2^23 - 1)), split into three byte planes
// (X = 65536*H + 256*M + L; H signed, M and L unsigned), so each quant byte
// feeds dp4a directly.  Per plane p the block sum
//   A_p = sum_i (q_i - off) * X_p,i
// is exact in integers: dp4a adds q_i * X_p,i to an accumulator that starts
// at the bit pattern of 1.5*2^23 minus off * sum_i X_p,i (a per-block
// constant of the input), so reading it as a float and subtracting 1.5*2^23
// converts it exactly (|A_p| < 2^22) without an int-to-float instruction.
//   block dot = d * s_b * ((256*A_H + A_M)*256 + A_L)
// where 256*A_H + A_M is exact in fp32 and the outer fma rounds once.  So
// the only roundings are the input's 24-bit representation (half a unit of
// 2^-23 of the block maximum per value, the fp32 precision of the block's
// largest input), one rounding of the block dot, its scale and the sum over
// blocks -- fewer than the per-element fp32 roundings of the reference's
// decode-then-dot (quant_matvec.c:243-247); tests/test_gpu_precision.py
// compares both against an exact product.
//
// Reduction.  Rows are processed in batches of 8 per thread; the 8 partial
// sums are reduced across the unit lanes of a warp with a butterfly
// reduce-scatter (7 + log2(G/8) shuffles per 8 rows) and parked in shared
// memory per warp, with no CTA-wide barrier inside the row loop.  After the
// last round one barrier, then the sums across the warps of a slot and the
// fused epilogue over all of the CTA's rows, whose operands (residual, RoPE
// factors) were fetched before the loop.
#pragma once
#include "common.cuh"

namespace fwb {

enum QType : int { QT_Q4_0 = 2, QT_Q5_0 = 6, QT_Q5_1 = 7, QT_Q8_0 = 8, QT_Q4_K = 12, QT_Q6_K = 14 };
template <int QT> struct QTraits;
// BB block bytes (superblock bytes for the K-quants), OFF quant offset folded
// into the accumulator starts, RPT rows per thread per round: four
// independent rows (the per-round ring wait, release and reduction are paid
// once per four rows; measured 5 % faster per decode step than two), two for
// the types whose units need more registers.  SUMX: the block dot needs the
// block's sum of inputs (a min term: Q5_1 d*q + m, Q4_K d*sc*q - dmin*m).
// SUPER: 256-value superblocks, a thread's 64-value unit is a quarter of one.
template <> struct QTraits<QT_Q4_0> { static constexpr int BB = 18, OFF = 8, RPT = 4; static constexpr bool SUMX = false, SUPER = false; };
template <> struct QTraits<QT_Q5_0> { static constexpr int BB = 22, OFF = 16, RPT = 4; static constexpr bool SUMX = false, SUPER = false; };
template <> struct QTraits<QT_Q5_1> { static constexpr int BB = 24, OFF = 0, RPT = 2; static constexpr bool SUMX = true, SUPER = false; };
template <> struct QTraits<QT_Q8_0> { static constexpr int BB = 34, OFF = 0, RPT = 2; static constexpr bool SUMX = false, SUPER = false; };
template <> struct QTraits<QT_Q4_K> { static constexpr int BB = 144, OFF = 0, RPT = 2; static constexpr bool SUMX = true, SUPER = true; };
template <> struct QTraits<QT_Q6_K> { static constexpr int BB = 210, OFF = 0, RPT = 2; static constexpr bool SUMX = false, SUPER = true; };

// half: the halved row count (2, 1 for two-row types) that the persistent
// kernel uses when the ring of full stages does not fit its shared memory
__host__ __device__ constexpr uint32_t rows_per_thread(int qt, bool half = false) {
    return (qt == QT_Q4_0 || qt == QT_Q5_0 ? 4u : 2u) >> (half ? 1 : 0);
}

// Byte offset of unit u (values [64u, 64u + 64)) within a row; for the
// K-quants the start of its superblock.
template <int QT>
__host__ __device__ constexpr uint32_t unit_bytes(uint32_t u) {
    return QTraits<QT>::SUPER ? (u >> 2) * (uint32_t)QTraits<QT>::BB : u * 2u * (uint32_t)QTraits<QT>::BB;
}

enum GemvMode : int {
    GM_STORE = 0,   // y[r]  = (W x)[r]
    GM_RESID = 1,   // y[r] += (W x)[r]                 (residual stream)
    GM_QKV = 2,     // rows [q | k | v]: RoPE on q, k; k, v appended to the KV cache
    GM_SWIGLU = 3,  // y[i]  = silu((Wg x)[i]) * (Wu x)[i]
    GM_LOGITS = 4,  // y[r]  = (W x)[r], plus the grid-wide greedy argmax
    GM_PUSH = 5,    // (W x)[r] sent to every rank as a tagged word (tensor-parallel partial sums)
};
enum InMode : int { IN_PLAIN = 0, IN_RMSNORM = 1 };

constexpr int kRB = 8;              // rows per reduction batch (per slot): 8 / RPT rounds x RPT rows
constexpr int kMaxStages = 8;
constexpr uint32_t kMaxConsumers = 512;  // threads per GEMV CTA (all consumers)
constexpr uint32_t kHeaderBytes = 1024;  // barriers, stage counters, small scratch
constexpr uint32_t kStageSlack = 128;  // alignment + half-unit over-read room
constexpr uint32_t kPosUnknown = 0xffffffffu;  // gemv_consume reads the position from step[1]
constexpr uint32_t kProfSlots = 8;  // GEMV profile values per CTA and phase
constexpr int kXMax = 8388607;      // fixed-point range of the inputs (24 bits per value: 2^23 - 1)
constexpr int kPlanes = 3;          // byte planes of the fixed-point inputs (H, M, L)
constexpr int kPlaneWords = 8 * kPlanes + 4;  // plane words, 3 accumulator starts and the scale per block

struct GemvArgs {
    uint32_t mode;       // GemvMode (the row loop is shared; only prologue/epilogue differ)
    uint32_t norm;       // 1: RMSNorm the input (IN_RMSNORM)
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
    uint32_t red_bytes;  // shared partial row sums: (Upad/32 or 1) floats per local row
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
    uint32_t *step_rw, *hist;  // GM_LOGITS: advance step[0..1], record hist[pos]
    uint32_t idx_base;     // GM_LOGITS: vocabulary index of row 0 (a tensor-parallel rank's slice)
    float *tp_cand;        // GM_LOGITS under tensor parallelism: (value, index) of this rank's
                           // maximum goes here instead of advancing the step
    // GM_PUSH: row r goes to ll_out[q][r] of every rank q (tag: *ll_epoch + ll_k + 1)
    unsigned long long *ll_out[kMaxRanks];
    const uint32_t *ll_epoch;
    uint32_t ll_k, world;
    uint32_t *err;
    // optional profile: thread 0 of each CTA adds ns spent in
    // [0] prologue (norm + planes), [1] waiting for stages, [2] the row loop, [3] tail,
    // and from the phase start to [4] its first input loads landing, [5] the input
    // planes' barrier; [6] from its own loop end until every warp's (kProfSlots per CTA)
    unsigned long long *prof;
};

__device__ __forceinline__ unsigned long long gtime_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// input planes
// ---------------------------------------------------------------------------
struct XBlock {
    uint32_t hi[8], mid[8], lo[8];  // 4 elements per word, element order 4k..4k+3
    int ih, im, il;                 // accumulator starts: kMagicBits - OFF * (sum of the plane's digits);
                                    // SUMX types: ih holds the float bits of sum(X), im = il = kMagicBits
    float s;                        // s_b
};

constexpr int kMagicBits = 0x4B400000;      // 1.5 * 2^23 as fp32 bits
constexpr float kMagic = 12582912.0f;

// ---------------------------------------------------------------------------
// block dots
// ---------------------------------------------------------------------------
// A (high plane), M, B (low plane) carry the kMagicBits bias and already
// hold the -OFF * sum(X_p) term (see the header comment): the block's integer
// dot (before the scales) with one rounding.
__device__ __forceinline__ float finish_block(int A, int M, int B) {
    const float Af = __int_as_float(A) - kMagic, Mf = __int_as_float(M) - kMagic;
    const float Bf = __int_as_float(B) - kMagic;
    return fmaf(fmaf(Af, 256.0f, Mf), 256.0f, Bf);
}

// Q4_0: 4 quant words (elements 4k..4k+3 in the low nibbles, 16+4k.. in the high)
__device__ __forceinline__ float dot_q4_0(const uint32_t (&q)[4], const XBlock &x) {
    int A = x.ih, M = x.im, B = x.il;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t lo = q[k] & 0x0F0F0F0Fu, hi = (q[k] >> 4) & 0x0F0F0F0Fu;
        A = dp4a_us(lo, (int)x.hi[k], A);
        A = dp4a_us(hi, (int)x.hi[k + 4], A);
        M = dp4a_uu(lo, x.mid[k], M);
        M = dp4a_uu(hi, x.mid[k + 4], M);
        B = dp4a_uu(lo, x.lo[k], B);
        B = dp4a_uu(hi, x.lo[k + 4], B);
    }
    return finish_block(A, M, B);
}

// spread 4 bits into bit 4 of each byte
__device__ __forceinline__ uint32_t spread4(uint32_t b) { return ((b & 0xFu) * 0x02040810u) & 0x10101010u; }

// Q5_0: qh = 32-bit high-bit plane (bit j of element j), 4 low-nibble words
__device__ __forceinline__ float dot_q5_0(uint32_t qh, const uint32_t (&q)[4], const XBlock &x) {
    int A = x.ih, M = x.im, B = x.il;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t lo = (q[k] & 0x0F0F0F0Fu) | spread4(qh >> (4 * k));
        const uint32_t hi = ((q[k] >> 4) & 0x0F0F0F0Fu) | spread4(qh >> (16 + 4 * k));
        A = dp4a_us(lo, (int)x.hi[k], A);
        A = dp4a_us(hi, (int)x.hi[k + 4], A);
        M = dp4a_uu(lo, x.mid[k], M);
        M = dp4a_uu(hi, x.mid[k + 4], M);
        B = dp4a_uu(lo, x.lo[k], B);
        B = dp4a_uu(hi, x.lo[k + 4], B);
    }
    return finish_block(A, M, B);
}

// Q8_0: 8 signed quant words
__device__ __forceinline__ float dot_q8_0(const uint32_t (&q)[8], const XBlock &x) {
    int A = x.ih, M = x.im, B = x.il;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        A = dp4a_ss((int)q[k], (int)x.hi[k], A);
        M = dp4a_su((int)q[k], x.mid[k], M);
        B = dp4a_su((int)q[k], x.lo[k], B);
    }
    return finish_block(A, M, B);
}

// d_b * s_b of a block (fp16 scale bits in the low half of dbits)
__device__ __forceinline__ float block_scale(uint32_t dbits, const XBlock &x) {
    return f16_bits_to_f32(dbits) * x.s;
}

// the three plane dots of 4 quant bytes with input word k: unsigned and
// signed quants
__device__ __forceinline__ void acc3_u(uint32_t q, const XBlock &x, int k, int &A, int &M, int &B) {
    A = dp4a_us(q, (int)x.hi[k], A);
    M = dp4a_uu(q, x.mid[k], M);
    B = dp4a_uu(q, x.lo[k], B);
}
__device__ __forceinline__ void acc3_s(uint32_t q, const XBlock &x, int k, int &A, int &M, int &B) {
    A = dp4a_ss((int)q, (int)x.hi[k], A);
    M = dp4a_su((int)q, x.mid[k], M);
    B = dp4a_su((int)q, x.lo[k], B);
}

// Q5_1 block (6 words: d | m << 16, qh, 4 nibble words): s * (d * sum(q X) + m * sum(X))
__device__ __forceinline__ float dot_q5_1(const uint32_t *w, const XBlock &x) {
    int A = kMagicBits, M = kMagicBits, B = kMagicBits;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        acc3_u((w[2 + k] & 0x0F0F0F0Fu) | spread4(w[1] >> (4 * k)), x, k, A, M, B);
        acc3_u(((w[2 + k] >> 4) & 0x0F0F0F0Fu) | spread4(w[1] >> (16 + 4 * k)), x, k + 4, A, M, B);
    }
    const float T = finish_block(A, M, B);
    return x.s * fmaf(f16_bits_to_f32(w[0]), T, f16_bits_to_f32(w[0] >> 16) * __int_as_float(x.ih));
}

// Q4_K 6-bit scale and min of group g from the 12 scale bytes (words y, z,
// w of the superblock's header): get_scale_min_k4, quant.c:63-82
__device__ __forceinline__ void k4_scale_min(const uint4 &h, uint32_t g, float &sc, float &mn) {
    auto byte = [&](uint32_t i) -> uint32_t {
        const uint32_t wv = i < 4 ? h.y : (i < 8 ? h.z : h.w);
        return (wv >> (8 * (i & 3))) & 0xffu;
    };
    uint32_t a, b;
    if (g < 4) {
        a = byte(g) & 63u;
        b = byte(g + 4) & 63u;
    } else {
        a = (byte(g + 4) & 15u) | ((byte(g - 4) >> 6) << 4);
        b = (byte(g + 4) >> 4) | ((byte(g) >> 6) << 4);
    }
    sc = (float)a;
    mn = (float)b;
}

// Q4_K unit sub of a superblock (16-byte aligned): groups 2 sub (low nibbles
// of the 32 quant bytes, block a) and 2 sub + 1 (high nibbles, block b);
// block dot = s * (d * sc * sum(q X) - dmin * m * sum(X))
__device__ __forceinline__ float dot_q4_k_unit(const uint8_t *sb, uint32_t sub, const XBlock &xa,
                                               const XBlock &xb) {
    const uint4 h = *reinterpret_cast<const uint4 *>(sb);
    const uint4 qa = *reinterpret_cast<const uint4 *>(sb + 16 + 32 * sub);
    const uint4 qb = *reinterpret_cast<const uint4 *>(sb + 32 + 32 * sub);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int A = kMagicBits, M = kMagicBits, B = kMagicBits;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc3_u(q[k] & 0x0F0F0F0Fu, xa, k, A, M, B);
    const float Ta = finish_block(A, M, B);
    A = M = B = kMagicBits;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc3_u((q[k] >> 4) & 0x0F0F0F0Fu, xb, k, A, M, B);
    const float Tb = finish_block(A, M, B);
    const float d = f16_bits_to_f32(h.x), dmin = f16_bits_to_f32(h.x >> 16);
    float sa, ma, sb_, mb;
    k4_scale_min(h, 2 * sub, sa, ma);
    k4_scale_min(h, 2 * sub + 1, sb_, mb);
    const float va = xa.s * fmaf(d * sa, Ta, -(dmin * ma) * __int_as_float(xa.ih));
    return fmaf(xb.s, fmaf(d * sb_, Tb, -(dmin * mb) * __int_as_float(xb.ih)), va);
}

// Q6_K: 6-bit quants as signed bytes q - 32 (byte-wise: set bit 7, subtract
// 32, flip bit 7; no borrow crosses a byte since every byte is >= 128 + 0)
__device__ __forceinline__ uint32_t q6_signed(uint32_t low4, uint32_t high2) {
    return (((low4 | (high2 << 4)) | 0x80808080u) - 0x20202020u) ^ 0x80808080u;
}

template <int NWORDS, bool A4>
__device__ __forceinline__ void load_unit_words(const uint8_t *p, uint32_t (&w)[NWORDS]);

// Q6_K unit sub of a superblock at sb (2-byte aligned): half = sub / 2 of
// the superblock, its values [0, 32) + 64 * (sub & 1) (block a: low/high
// nibbles of ql[0..32) by sub & 1, high bits qh bits 0-1 / 4-5) and
// [32, 64) + 64 * (sub & 1) (block b: ql[32..64), qh bits 2-3 / 6-7), with an
// int8 scale per 16 values: block dot = s * d * sum_halves sc * sum((q - 32) X)
__device__ __forceinline__ float dot_q6_k_unit(const uint8_t *sb, uint32_t sub, const XBlock &xa,
                                               const XBlock &xb) {
    const uint32_t half = sub >> 1, sl = 4 * (sub & 1);
    uint32_t qh[8], scw[1], dw[1];
    load_unit_words<8, false>(sb + 128 + 32 * half, qh);
    load_unit_words<1, false>(sb + 192 + 8 * half + 4 * (sub & 1), scw);
    load_unit_words<1, false>(sb + 208, dw);
    const float d = f16_bits_to_f32(dw[0]);
    float v[2];
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
        const XBlock &x = blk ? xb : xa;
        uint32_t ql[8];
        load_unit_words<8, false>(sb + 64 * half + 32 * blk, ql);
        float T[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            int A = kMagicBits, M = kMagicBits, B = kMagicBits;
#pragma unroll
            for (int k = 4 * hh; k < 4 * hh + 4; ++k)
                acc3_s(q6_signed((ql[k] >> sl) & 0x0F0F0F0Fu, (qh[k] >> (sl + 2 * blk)) & 0x03030303u), x, k, A, M, B);
            T[hh] = finish_block(A, M, B);
        }
        const float s0 = (float)(int8_t)(scw[0] >> (16 * blk)), s1 = (float)(int8_t)(scw[0] >> (16 * blk + 8));
        v[blk] = x.s * fmaf(s0, T[0], s1 * T[1]);
    }
    return d * (v[0] + v[1]);
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

// Partial dot of one unit: block A, plus block B when `two` (computed either
// way and selected, so the row loop has no divergent branch; the bytes read
// past the end of a row with an odd block count stay inside the stage slack).
template <int QT, bool A4>
__device__ __forceinline__ float unit_dot(const uint8_t *p, const XBlock &xa, const XBlock &xb, bool two,
                                          uint32_t sub) {
    if constexpr (QT == QT_Q4_K) {
        return dot_q4_k_unit(p, sub, xa, xb);
    } else if constexpr (QT == QT_Q6_K) {
        return dot_q6_k_unit(p, sub, xa, xb);
    } else if constexpr (QT == QT_Q5_1) {
        uint32_t w[12];
        load_unit_words<12, true>(p, w);
        const float r = dot_q5_1(w, xa);
        const float r2 = dot_q5_1(w + 6, xb);
        return two ? r + r2 : r;
    } else if constexpr (QT == QT_Q4_0) {
        uint32_t w[9];
        load_unit_words<9, A4>(p, w);
        uint32_t qa[4] = {__funnelshift_r(w[0], w[1], 16), __funnelshift_r(w[1], w[2], 16),
                          __funnelshift_r(w[2], w[3], 16), __funnelshift_r(w[3], w[4], 16)};
        const float r = block_scale(w[0], xa) * dot_q4_0(qa, xa);
        const uint32_t qb[4] = {w[5], w[6], w[7], w[8]};
        const float r2 = fmaf(block_scale(w[4] >> 16, xb), dot_q4_0(qb, xb), r);
        return two ? r2 : r;
    } else if constexpr (QT == QT_Q5_0) {
        uint32_t w[11];
        load_unit_words<11, A4>(p, w);
        uint32_t qa[4] = {__funnelshift_r(w[1], w[2], 16), __funnelshift_r(w[2], w[3], 16),
                          __funnelshift_r(w[3], w[4], 16), __funnelshift_r(w[4], w[5], 16)};
        const float r = block_scale(w[0], xa) * dot_q5_0(__funnelshift_r(w[0], w[1], 16), qa, xa);
        const uint32_t qb[4] = {w[7], w[8], w[9], w[10]};
        const float r2 = fmaf(block_scale(w[5] >> 16, xb), dot_q5_0(w[6], qb, xb), r);
        return two ? r2 : r;
    } else {
        uint32_t w[17];
        load_unit_words<17, A4>(p, w);
        uint32_t qa[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) qa[k] = __funnelshift_r(w[k], w[k + 1], 16);
        const float r = block_scale(w[0], xa) * dot_q8_0(qa, xa);
        uint32_t qb[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) qb[k] = w[9 + k];
        const float r2 = fmaf(block_scale(w[8] >> 16, xb), dot_q8_0(qb, xb), r);
        return two ? r2 : r;
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
// Shared memory of one GEMV.  Stage k of the CTA lives in ring slot
// kring % NS, phase parity (kring / NS) & 1, where kring counts stages from
// the start of the ring, so several GEMVs can run back to back through one
// ring.
// ---------------------------------------------------------------------------
struct GemvSmem {
    uint64_t *full;   // [kMaxStages] stage landed (transaction count)
    uint32_t *done;   // [kMaxStages] warps finished with the slot, then the refill cursor
    float *misc;      // [64]
    uint32_t *misc_u; // [64]
    uint32_t *planes; // quantised input: word (p*8+k)*nbp + b (p 0 = high, 1 = middle, 2 = low),
                      // accumulator starts (high, middle, low) at (24+p)*nbp + b, s at 27*nbp + b
    uint32_t nbp;     // blocks of the input, rounded up to even
    float *red;       // partial row sums [local row][warp of the slot]
    uint8_t *ring;
};

// Bytes of the plane area for an input of K values.
__host__ __device__ constexpr uint32_t plane_bytes(uint32_t K) {
    return (((uint32_t)kPlaneWords * (((K / 32) + 1) & ~1u) * 4u) + 127u) & ~127u;
}

// Partial-sum area for n_loc local rows with slots `Upad` threads wide.
__host__ __device__ constexpr uint32_t red_bytes_for(uint32_t Upad, uint32_t n_loc) {
    return (((Upad > 32 ? Upad / 32 : 1u) * n_loc * 4u) + 127u) & ~127u;
}

__device__ __forceinline__ GemvSmem gemv_smem(uint8_t *smem, uint32_t K, uint32_t red_bytes) {
    GemvSmem g;
    g.full = reinterpret_cast<uint64_t *>(smem);
    g.done = reinterpret_cast<uint32_t *>(g.full + kMaxStages);
    g.misc = reinterpret_cast<float *>(smem + 256);        // [64]
    g.misc_u = reinterpret_cast<uint32_t *>(smem + 512);   // [64]
    g.planes = reinterpret_cast<uint32_t *>(smem + kHeaderBytes);
    g.nbp = ((K / 32) + 1) & ~1u;
    g.red = reinterpret_cast<float *>(smem + kHeaderBytes + plane_bytes(K));
    g.ring = smem + kHeaderBytes + plane_bytes(K) + red_bytes;
    return g;
}

// Issue the bulk copy of local stage k of this CTA's rows into ring slot
// `slot` (one thread).  Rows are copied as 16-byte-aligned supersets; the
// consumer recomputes the same offset (delta) from the row address.
template <bool PAIRED>
__device__ __forceinline__ void issue_stage(const GemvArgs &a, const GemvSmem &sm, uint32_t rb, uint32_t re,
                                            uint32_t k, uint32_t slot) {
    const uint32_t R = a.R;
    uint8_t *dst = sm.ring + (size_t)slot * a.stage_bytes;
    if (!PAIRED) {
        const uint32_t n_loc = re - rb;
        const uint32_t r0 = k * R, nr = min(R, n_loc - r0);
        const uintptr_t src = reinterpret_cast<uintptr_t>(a.w) + (uint64_t)(rb + r0) * a.row_bytes;
        const uintptr_t s0 = src & ~uintptr_t(15);
        const uint32_t bytes = (uint32_t)(((src + (uint64_t)nr * a.row_bytes + 15) & ~uintptr_t(15)) - s0);
        mbar_arrive_expect_tx(&sm.full[slot], bytes);
        bulk_g2s(dst, reinterpret_cast<const void *>(s0), bytes, &sm.full[slot]);
    } else {
        const uint32_t p0 = k * (R / 2), np = min(R / 2, (re - rb) - p0);
        const uint64_t off = (uint64_t)(rb + p0) * a.row_bytes;
        const uintptr_t g = reinterpret_cast<uintptr_t>(a.w) + off;
        const uintptr_t u = reinterpret_cast<uintptr_t>(a.w2) + off;
        const uintptr_t g0 = g & ~uintptr_t(15), u0 = u & ~uintptr_t(15);
        const uint32_t gb = (uint32_t)(((g + (uint64_t)np * a.row_bytes + 15) & ~uintptr_t(15)) - g0);
        const uint32_t ub = (uint32_t)(((u + (uint64_t)np * a.row_bytes + 15) & ~uintptr_t(15)) - u0);
        mbar_arrive_expect_tx(&sm.full[slot], gb + ub);
        bulk_g2s(dst, reinterpret_cast<const void *>(g0), gb, &sm.full[slot]);
        bulk_g2s(dst + a.stage_bytes / 2, reinterpret_cast<const void *>(u0), ub, &sm.full[slot]);
    }
}

// Stages of this CTA: one per round of R = RPT * S local rows.
template <bool PAIRED>
__device__ __forceinline__ uint32_t n_stages_of(const GemvArgs &a, uint32_t rb, uint32_t re) {
    const uint32_t n_loc = PAIRED ? 2 * (re - rb) : (re - rb);
    return (n_loc + a.R - 1) / a.R;
}

// Ring position of the next stage a consumer will read: slot, phase parity,
// and the stage's index j (local to one GEMV in the standalone kernel, global
// across all phases in the persistent decode kernel).
struct RingState {
    uint32_t slot, par, j;
};

// Called by lane 0 of every warp when it is done with stage rs.j: the last
// warp to finish hands the slot to `refill`, which issues stage j + NS into
// it (if such a stage exists).  The proxy fence orders the warps' generic
// reads of the slot before the bulk copy (async proxy) that overwrites it.
template <class Refill>
__device__ __forceinline__ void ring_release(const GemvSmem &sm, const RingState &rs, uint32_t nwarps,
                                             const Refill &refill) {
    __threadfence_block();
    if (atomicAdd(&sm.done[rs.slot], 1u) == nwarps - 1) {
        sm.done[rs.slot] = 0;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        refill(rs.j, rs.slot);
    }
}

__device__ __forceinline__ void ring_advance(RingState &rs, uint32_t NS) {
    ++rs.j;
    if (++rs.slot == NS) { rs.slot = 0; rs.par ^= 1u; }
}

// Quantise the input once per CTA into the shared plane area, in one pass
// over x: a group of 4 lanes per 32-block, 8 values per lane, and up to 4
// blocks per thread loaded before any is used so that their L2 round trips
// overlap.  With RMSNorm (rms_norm, norm.c:7-16) the values are multiplied by
// the norm weight here; the 1/rms factor is a common scale of every block, so
// it is applied to the block scales afterwards instead of to the values, and
// x is read once.  Float -> int: X = rint(v / s_b) of the exact quotient
// (up to ties within an ulp), clamped to +-(2^23 - 1).
// Ends with a CTA barrier.  Returns the 1/rms factor
// 1/sqrtf(sum(x^2)/K + eps) (IEEE division and square root; every thread
// sums the warp partials in the same order), or 1 without the norm.
// NP passes of build_planes (below) starting at block b0: every pass's loads
// are issued before any is used, and the passes have no early exit, so their
// dependency chains (block maximum, shuffles, rounding) overlap.  Blocks at
// or beyond nb are predicated off.
template <int QT, int NP>
__device__ __forceinline__ void plane_passes(const GemvArgs &a, const GemvSmem &sm, uint32_t tid, uint32_t b0,
                                             uint32_t per, bool norm, float &ss, bool prof,
                                             unsigned long long &t_x) {
    constexpr int OFF = QTraits<QT>::OFF;
    const uint32_t nb = a.K >> 5, nbp = sm.nbp;
    const uint32_t q = tid & 3;
    {
        float v[NP][8], wn[NP][8];
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const uint32_t b = b0 + p * per + (tid >> 2);
            const bool on = b < nb;
            const uint32_t c = b * 32 + q * 8;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float4 t = make_float4(0.f, 0.f, 0.f, 0.f), u = make_float4(1.f, 1.f, 1.f, 1.f);
                if (on) {
                    t = __ldcg(reinterpret_cast<const float4 *>(a.x + c + 4 * h));  // written by other CTAs
                    if (norm) u = __ldg(reinterpret_cast<const float4 *>(a.norm_w + c + 4 * h));
                }
                v[p][4 * h] = t.x; v[p][4 * h + 1] = t.y; v[p][4 * h + 2] = t.z; v[p][4 * h + 3] = t.w;
                wn[p][4 * h] = u.x; wn[p][4 * h + 1] = u.y; wn[p][4 * h + 2] = u.z; wn[p][4 * h + 3] = u.w;
            }
        }
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const uint32_t b = b0 + p * per + (tid >> 2);
            const bool on = b < nb;
            if (norm) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    ss = fmaf(v[p][j], v[p][j], ss);
                    v[p][j] = __fmul_rn(v[p][j], wn[p][j]);
                }
            }
            float m = 0.f, chk = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                m = fmaxf(m, fabsf(v[p][j]));
                chk += v[p][j];  // NaN / inf propagate here (fmaxf would drop NaN)
            }
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
            if (prof && b0 == 0 && p == 0) t_x = gtime_ns();  // the first loads have landed
            const bool bad = !isfinite(chk) || !isfinite(m);
            const bool zero = !(m > 1e-30f) || bad;
            // scale slightly above max/kXMax, so |v / sb| <= kXMax
            const float sb = zero ? 0.f : m * (1.0f / (float)(kXMax - 1));
            const float inv = zero ? 0.f : __frcp_rn(sb), hsb = 0.5f * sb;
            int xi[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                // rint(v / sb) of the exact quotient: a first guess from the
                // rounded product, then the exact remainder v - X * sb (one
                // fma) moves it by one where the guess is off
                int X = __float2int_rn(v[p][j] * inv);
                const float e = fmaf(-(float)X, sb, v[p][j]);
                X += (e > hsb) - (e < -hsb);
                xi[j] = zero ? 0 : min(kXMax, max(-kXMax, X));
            }
            uint32_t pw[3][2];  // plane words (high, middle, low) of this lane's two groups of 4
            int sh = 0, sm_ = 0, sl = 0;
#pragma unroll
            for (int w = 0; w < 2; ++w) {
                const int *x4 = xi + 4 * w;
                // |xi| < 2^23: byte 0 is the low plane, byte 1 the middle, byte 2 the signed high
                const uint32_t t01 = __byte_perm(x4[0], x4[1], 0x5140), t23 = __byte_perm(x4[2], x4[3], 0x5140);
                pw[2][w] = __byte_perm(t01, t23, 0x5410);
                pw[1][w] = __byte_perm(t01, t23, 0x7632);
                const uint32_t u01 = __byte_perm(x4[0], x4[1], 0x0062), u23 = __byte_perm(x4[2], x4[3], 0x0062);
                pw[0][w] = __byte_perm(u01, u23, 0x5410);
                // digit sums of the three planes (dp4a with ones)
                sh = dp4a_ss((int)pw[0][w], 0x01010101, sh);
                sm_ = dp4a_uu(pw[1][w], 0x01010101u, sm_);
                sl = dp4a_uu(pw[2][w], 0x01010101u, sl);
            }
#pragma unroll
            for (int o = 1; o <= 2; o <<= 1) {
                sh += __shfl_xor_sync(0xffffffffu, sh, o);
                sm_ += __shfl_xor_sync(0xffffffffu, sm_, o);
                sl += __shfl_xor_sync(0xffffffffu, sl, o);
            }
            if (on) {
#pragma unroll
                for (int w = 0; w < 2; ++w) {
                    const uint32_t k = 2 * q + w;
                    sm.planes[(0 * 8 + k) * nbp + b] = pw[0][w];
                    sm.planes[(1 * 8 + k) * nbp + b] = pw[1][w];
                    sm.planes[(2 * 8 + k) * nbp + b] = pw[2][w];
                }
                if (q == 0) {
                    if constexpr (QTraits<QT>::SUMX) {  // sum(X) for the min term, exact in int32
                        sm.planes[24 * nbp + b] = __float_as_uint((float)(65536 * sh + 256 * sm_ + sl));
                        sm.planes[25 * nbp + b] = (uint32_t)kMagicBits;
                        sm.planes[26 * nbp + b] = (uint32_t)kMagicBits;
                    } else {
                        sm.planes[24 * nbp + b] = (uint32_t)(kMagicBits - OFF * sh);
                        sm.planes[25 * nbp + b] = (uint32_t)(kMagicBits - OFF * sm_);
                        sm.planes[26 * nbp + b] = (uint32_t)(kMagicBits - OFF * sl);
                    }
                    sm.planes[27 * nbp + b] = __float_as_uint(bad ? __int_as_float(0x7fc00000) : sb);
                }
            }
        }
        }
}

template <int QT>
__device__ float build_planes(const GemvArgs &a, const GemvSmem &sm, uint32_t tid, uint32_t NC, bool prof,
                              unsigned long long &t_x, unsigned long long &t_b) {
    const bool norm = a.norm != 0;
    const uint32_t nb = a.K >> 5;
    const uint32_t lane = tid & 31, warp = tid >> 5;
    const uint32_t per = NC >> 2;  // blocks per pass
    float ss = 0.f;
    for (uint32_t b0 = 0; b0 < nb;) {
        const uint32_t left = (nb - b0 + per - 1) / per;  // passes still needed
        if (left >= 3) {
            plane_passes<QT, 4>(a, sm, tid, b0, per, norm, ss, prof, t_x);
            b0 += 4 * per;
        } else if (left == 2) {
            plane_passes<QT, 2>(a, sm, tid, b0, per, norm, ss, prof, t_x);
            b0 += 2 * per;
        } else {
            plane_passes<QT, 1>(a, sm, tid, b0, per, norm, ss, prof, t_x);
            b0 += per;
        }
    }
    if (norm) {
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) sm.misc[warp] = ss;
    }
    bar_sync(1, NC);
    if (prof) t_b = gtime_ns();
    if (!norm) return 1.0f;
    float t = 0.f;
    for (uint32_t w = 0; w < (NC >> 5); ++w) t += sm.misc[w];
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)a.K), a.eps)));
}

// This thread's two input blocks (2u, 2u+1) from the plane area, block
// scales multiplied by `scale`.
__device__ __forceinline__ void load_planes(const GemvSmem &sm, uint32_t unit, float scale, XBlock &xa, XBlock &xb) {
    const uint32_t nbp = sm.nbp, b = 2 * unit;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint2 h = *reinterpret_cast<const uint2 *>(sm.planes + (0 * 8 + k) * nbp + b);
        const uint2 md = *reinterpret_cast<const uint2 *>(sm.planes + (1 * 8 + k) * nbp + b);
        const uint2 l = *reinterpret_cast<const uint2 *>(sm.planes + (2 * 8 + k) * nbp + b);
        xa.hi[k] = h.x; xb.hi[k] = h.y;
        xa.mid[k] = md.x; xb.mid[k] = md.y;
        xa.lo[k] = l.x; xb.lo[k] = l.y;
    }
    const uint2 ih = *reinterpret_cast<const uint2 *>(sm.planes + 24 * nbp + b);
    const uint2 im = *reinterpret_cast<const uint2 *>(sm.planes + 25 * nbp + b);
    const uint2 il = *reinterpret_cast<const uint2 *>(sm.planes + 26 * nbp + b);
    const uint2 sv = *reinterpret_cast<const uint2 *>(sm.planes + 27 * nbp + b);
    xa.ih = (int)ih.x; xb.ih = (int)ih.y;
    xa.im = (int)im.x; xb.im = (int)im.y;
    xa.il = (int)il.x; xb.il = (int)il.y;
    xa.s = __fmul_rn(__uint_as_float(sv.x), scale);
    xb.s = __fmul_rn(__uint_as_float(sv.y), scale);
}

// RoPE of one adjacent pair (rope.c:37-43).
__device__ __forceinline__ void rope_pair(float v0, float v1, float c, float s, float &r0, float &r1) {
    r0 = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
    r1 = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
}

// One GEMV over this CTA's rows.  Returns false if a bounded wait failed
// (results then invalid).
//
// Structure: prologue (input planes; epilogue operands fetched early), the
// row loop (no CTA-wide barrier: each warp reduces its partial sums of a batch
// of 8 rows per slot with shuffles and parks them in shared memory), one CTA
// barrier, then the epilogue over all local rows.
template <int QT, bool A4, class Refill, bool HALF = false>
__device__ bool gemv_consume(const GemvArgs &a, const GemvSmem &sm, uint32_t tid, RingState &rs,
                             const Refill &refill, uint32_t pos_known = kPosUnknown) {
    // run-time: the mode only changes the prologue / epilogue, pairing only the
    // per-thread row offsets (one copy of the row loop per quant type)
    const uint32_t MODE = a.mode;
    const bool PAIRED = MODE == GM_SWIGLU;
    constexpr uint32_t RPT = (uint32_t)QTraits<QT>::RPT >> (HALF ? 1 : 0);
    constexpr int RND = kRB / (int)RPT;  // rounds per reduction batch
    const uint32_t NC = blockDim.x, lane = tid & 31, warp = tid >> 5, NCW = NC >> 5;
    uint32_t rb, re;
    cta_rows(a.n_out, a.gran, rb, re);
    const uint32_t n_loc = PAIRED ? 2 * (re - rb) : (re - rb);
    const uint32_t Upad = a.Upad, S = a.S, U = a.U;
    const uint32_t slot = tid / Upad, unit = tid % Upad;
    const uint32_t nb = a.K >> 5;
    const bool active = slot < S && unit < U;
    const uint32_t slot_c = min(slot, S - 1), unit_c = min(unit, U - 1);  // in-bounds for inactive threads
    const bool two = 2 * unit_c + 1 < nb;
    const uint32_t G = Upad < 32 ? Upad : 32;
    const uint32_t Wg = Upad > 32 ? Upad >> 5 : 1u;  // warps per slot
    const uint32_t wg = Upad > 32 ? warp % Wg : 0u;
    const uint32_t RS = RPT * S;  // local rows per round

    const bool prof = a.prof != nullptr && tid == 0;
    const unsigned long long t0 = prof ? gtime_ns() : 0ull;

    // epilogue operands, fetched now so that their latency hides behind the loop
    float pre_y = 0.f;
    uint32_t pos = 0;
    if (MODE == GM_RESID && tid < n_loc) pre_y = __ldcg(&a.y[rb + tid]);
    if (MODE == GM_QKV) pos = pos_known != kPosUnknown ? pos_known : __ldcg(&a.step[1]);
    uint32_t ll_tag = 0;
    if (MODE == GM_PUSH) ll_tag = __ldcg(a.ll_epoch) + a.ll_k + 1;

    unsigned long long t_x = 0ull, t_b = 0ull;
    const float rscale = build_planes<QT>(a, sm, tid, NC, prof, t_x, t_b);
    XBlock xa, xb;
    load_planes(sm, unit_c, rscale, xa, xb);

    float rc = 1.f, rsn = 0.f;  // GM_QKV: RoPE factors of this thread's first pair
    const uint32_t half = a.head_dim >> 1;
    if (MODE == GM_QKV && 2 * tid < n_loc) {
        const uint32_t g = rb + 2 * tid;
        if (g < a.n_q + a.n_kv) {
            const uint32_t d = (g < a.n_q ? g : g - a.n_q) % a.head_dim;
            rc = __ldg(&a.rope_cos[pos * half + d / 2]);
            rsn = __ldg(&a.rope_sin[pos * half + d / 2]);
        }
    }
    const unsigned long long t1 = prof ? gtime_ns() : 0ull;
    if (prof) {  // (folded in now: no timer stays live through the row loop; no-return adds)
        atomicAdd(&a.prof[(size_t)blockIdx.x * kProfSlots + 4], t_x - t0);
        atomicAdd(&a.prof[(size_t)blockIdx.x * kProfSlots + 5], t_b - t0);
    }

    // One ring stage per round: local stage k holds local rows [k*RS, (k+1)*RS).
    const uint32_t n_rounds = (n_loc + RS - 1) / RS;
    const uint32_t NS = a.NS, rbytes = a.row_bytes, sbytes = a.stage_bytes;
    // Stage k's rows start (src(k) & 15) bytes into its slot, src(k) = base +
    // k * sstep; the offset is the same for every stage unless sstep % 16 != 0.
    const uintptr_t base_a = reinterpret_cast<uintptr_t>(a.w) + (uint64_t)rb * rbytes;
    const uintptr_t base_b = PAIRED ? reinterpret_cast<uintptr_t>(a.w2) + (uint64_t)rb * rbytes : 0;
    const uint32_t sstep = PAIRED ? (RS / 2) * rbytes : RS * rbytes;
    const bool var_delta = (sstep & 15u) != 0;
    // byte offset inside a stage of this thread's unit in each of its RPT
    // local rows slot*RPT + e; paired stages hold the gate rows in the first
    // half and the up rows in the second, local rows (gate, up, gate, up, ...)
    uint32_t off[RPT], cur[RPT];
    bool upper[RPT];
    const uint32_t sub = unit_c & 3;  // K-quants: quarter of the superblock
#pragma unroll
    for (uint32_t e = 0; e < RPT; ++e) {
        const uint32_t ls = slot_c * RPT + e;
        if (!PAIRED) {
            off[e] = ls * rbytes + unit_bytes<QT>(unit_c);
            upper[e] = false;
        } else {
            off[e] = (ls >> 1) * rbytes + unit_bytes<QT>(unit_c) + ((ls & 1) ? sbytes / 2 : 0u);
            upper[e] = ls & 1;
        }
    }
    auto set_delta = [&](uint32_t k) {
        const uint32_t da = (uint32_t)(base_a + (uint64_t)k * sstep) & 15u;
        const uint32_t db = (uint32_t)(base_b + (uint64_t)k * sstep) & 15u;
#pragma unroll
        for (uint32_t e = 0; e < RPT; ++e) cur[e] = off[e] + (upper[e] ? db : da);
    };
    set_delta(0);

    bool ok = true;
    unsigned long long t_wait = 0ull;
    if (prof && n_rounds) {  // time until the phase's first stage has landed
        const unsigned long long w0 = gtime_ns();
        ok = mbar_wait(&sm.full[rs.slot], rs.par, a.err, ERR_WAIT_FULL);
        t_wait = gtime_ns() - w0;
    }
    const uint8_t *ring = sm.ring;
    for (uint32_t r0 = 0; r0 < n_rounds; r0 += RND) {
        float acc[kRB];
#pragma unroll
        for (int jj = 0; jj < RND; ++jj) {
            const uint32_t r = r0 + jj;
            if (r < n_rounds) {
                if (ok) ok = mbar_wait(&sm.full[rs.slot], rs.par, a.err, ERR_WAIT_FULL);
                if (var_delta) set_delta(r);
                // every thread computes (inactive ones on clamped, in-bounds
                // addresses) so the body has no divergent branch
                const uint8_t *sb = ring + rs.slot * sbytes;
#pragma unroll
                for (uint32_t e = 0; e < RPT; ++e) {
                    const float d = unit_dot<QT, A4>(sb + cur[e], xa, xb, two, sub);
                    acc[RPT * jj + e] = active ? d : 0.f;
                }
                __syncwarp();
                if (lane == 0) ring_release(sm, rs, NCW, refill);
                ring_advance(rs, NS);
            } else {
#pragma unroll
                for (uint32_t e = 0; e < RPT; ++e) acc[RPT * jj + e] = 0.f;
            }
        }
        // acc[i] belongs to local row (r0 + i/RPT)*RS + slot*RPT + i%RPT; the
        // reduce-scatter leaves row jj8 of the batch (summed over this warp's
        // lanes of the slot) on every (G/8)-th lane
        uint32_t jj8;
        const float v = reduce8(acc, lane, G, jj8);
        const uint32_t lrow = (r0 + jj8 / RPT) * RS + slot * RPT + jj8 % RPT;
        if ((lane & ((G >> 3) - 1)) == 0 && slot < S && lrow < n_loc) sm.red[lrow * Wg + wg] = v;
    }

    const unsigned long long t2 = prof ? gtime_ns() : 0ull;
    bar_sync(1, NC);  // every partial sum is parked
    if (prof) atomicAdd(&a.prof[(size_t)blockIdx.x * kProfSlots + 6], gtime_ns() - t2);

    // ---- epilogue over all local rows
    float best_v = -INFINITY;
    uint32_t best_i = 0xffffffffu;
    auto row_sum = [&](uint32_t i) {
        float t = 0.f;
        for (uint32_t w = 0; w < Wg; ++w) t += sm.red[i * Wg + w];
        return t;
    };
    if (ok) {
        if (MODE == GM_STORE || MODE == GM_RESID || MODE == GM_LOGITS) {
            for (uint32_t i = tid; i < n_loc; i += NC) {
                const uint32_t g = rb + i;
                const float t = row_sum(i);
                if (MODE == GM_STORE) a.y[g] = t;
                if (MODE == GM_RESID) a.y[g] = __fadd_rn(i == tid ? pre_y : __ldcg(&a.y[g]), t);
                if (MODE == GM_LOGITS) {
                    a.y[g] = t;
                    const uint32_t gi = a.idx_base + g;
                    if (t > best_v || (t == best_v && gi < best_i)) { best_v = t; best_i = gi; }
                }
            }
        } else if (MODE == GM_PUSH) {
            for (uint32_t i = tid; i < n_loc; i += NC) {
                const float t = row_sum(i);
                for (uint32_t q = 0; q < a.world; ++q) st_tagged(a.ll_out[q] + rb + i, t, ll_tag);
            }
        } else if (MODE == GM_SWIGLU) {
            for (uint32_t i = tid; 2 * i < n_loc; i += NC)
                a.y[rb + i] = __fmul_rn(silu_ref(row_sum(2 * i)), row_sum(2 * i + 1));
        } else if (MODE == GM_QKV) {
            for (uint32_t i = tid; 2 * i < n_loc; i += NC) {
                const uint32_t g = rb + 2 * i;
                const float v0 = row_sum(2 * i), v1 = row_sum(2 * i + 1);
                if (g < a.n_q + a.n_kv) {
                    const uint32_t gg = g < a.n_q ? g : g - a.n_q;
                    const uint32_t d = gg % a.head_dim;
                    const float c = i == tid ? rc : __ldg(&a.rope_cos[pos * half + d / 2]);
                    const float sn = i == tid ? rsn : __ldg(&a.rope_sin[pos * half + d / 2]);
                    float r0v, r1v;
                    rope_pair(v0, v1, c, sn, r0v, r1v);
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

    if (MODE == GM_LOGITS) {
        // CTA argmax, then the last CTA to finish reduces the per-CTA results
        // (sampler.c:28-32: the lowest index wins among equal maxima)
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ov > best_v || (ov == best_v && oi < best_i)) { best_v = ov; best_i = oi; }
        }
        if (lane == 0) { sm.misc[warp] = best_v; sm.misc_u[warp] = best_i; }
        bar_sync(1, NC);
        if (tid == 0) {
            float bv = sm.misc[0];
            uint32_t bi = sm.misc_u[0];
            for (uint32_t w = 1; w < NCW; ++w)
                if (sm.misc[w] > bv || (sm.misc[w] == bv && sm.misc_u[w] < bi)) { bv = sm.misc[w]; bi = sm.misc_u[w]; }
            a.am_val[blockIdx.x] = bv;
            a.am_idx[blockIdx.x] = bi;
            __threadfence();
            sm.misc_u[63] = atomicAdd(a.ticket, 1u) == gridDim.x - 1 ? 1u : 0u;
        }
        bar_sync(1, NC);
        if (sm.misc_u[63]) {
            // the last CTA reduces the per-CTA results in parallel
            __threadfence();
            float bv = -INFINITY;
            uint32_t bi = 0xffffffffu;
            for (uint32_t c = tid; c < gridDim.x; c += NC) {
                const float cv = __ldcg(&a.am_val[c]);
                const uint32_t ci = __ldcg(&a.am_idx[c]);
                if (cv > bv || (cv == bv && ci < bi)) { bv = cv; bi = ci; }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            bar_sync(1, NC);
            if (lane == 0) { sm.misc[warp] = bv; sm.misc_u[warp] = bi; }
            bar_sync(1, NC);
            if (tid == 0) {
                bv = sm.misc[0];
                bi = sm.misc_u[0];
                for (uint32_t w = 1; w < NCW; ++w)
                    if (sm.misc[w] > bv || (sm.misc[w] == bv && sm.misc_u[w] < bi)) { bv = sm.misc[w]; bi = sm.misc_u[w]; }
                // sampler_argmax (sampler.c:28-32) starts from index 0 and
                // moves only on a strict '>': a NaN logit 0 is never beaten,
                // so the token is 0 (as +inf at index 0 for the ranks' merge)
                if (a.idx_base == 0 && isnan(__ldcg(&a.y[0]))) { bv = INFINITY; bi = 0; }
                if (a.tp_cand) {  // the ranks' candidates are combined after a global barrier
                    a.tp_cand[0] = bv;
                    reinterpret_cast<uint32_t *>(a.tp_cand)[1] = bi;
                } else {
                    // every logit NaN: the reference keeps index 0
                    const uint32_t nxt = bi == 0xffffffffu ? 0u : bi;
                    *a.out_token = nxt;
                    if (a.hist) {  // feed the greedy token into the next step
                        const uint32_t p = __ldcg(&a.step_rw[1]);
                        a.hist[p] = nxt;
                        a.step_rw[0] = nxt;
                        a.step_rw[1] = p + 1;
                    }
                }
                *a.ticket = 0;
            }
        }
        bar_sync(1, NC);
    }
    if (prof) {
        unsigned long long *pp = a.prof + (size_t)blockIdx.x * kProfSlots;
        atomicAdd(&pp[0], t1 - t0);
        atomicAdd(&pp[1], t_wait);
        atomicAdd(&pp[2], t2 - t1);
        atomicAdd(&pp[3], gtime_ns() - t2);
    }
    return ok;
}

// ---------------------------------------------------------------------------
// standalone kernel: one GEMV per launch (quant_matvec_dev and the per-kernel
// decode path)
// ---------------------------------------------------------------------------
// After a failed wait: before the CTA may exit, wait (bounded) for the last
// NS stages issued into the ring, the only copies that can be in flight.
__device__ void ring_drain(const GemvSmem &sm, uint32_t n_issued, uint32_t NS, uint32_t *err) {
    for (uint32_t k = n_issued > NS ? n_issued - NS : 0; k < n_issued; ++k)
        mbar_wait(&sm.full[k % NS], (k / NS) & 1, err, ERR_WAIT_DRAIN);
}

template <int QT, bool A4>
__global__ void __launch_bounds__(kMaxConsumers, 1) gemv_kernel(const __grid_constant__ GemvArgs a) {
    const bool PAIRED = a.mode == GM_SWIGLU;
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvSmem sm = gemv_smem(smem, a.K, a.red_bytes);
    const uint32_t tid = threadIdx.x;
    uint32_t rb, re;
    cta_rows(a.n_out, a.gran, rb, re);
    const uint32_t n_st = PAIRED ? n_stages_of<true>(a, rb, re) : n_stages_of<false>(a, rb, re);
    if (tid == 0) {
        for (uint32_t i = 0; i < a.NS; ++i) {
            mbar_init(&sm.full[i], 1);
            sm.done[i] = 0;
        }
        fence_mbar_init();
        // weights do not depend on the previous kernel: start streaming them
        for (uint32_t k = 0; k < min(a.NS, n_st); ++k) {
            if (PAIRED) issue_stage<true>(a, sm, rb, re, k, k);
            else issue_stage<false>(a, sm, rb, re, k, k);
        }
    }
    __syncthreads();
    pdl_launch();
    pdl_wait();  // inputs of this GEMV are outputs of the previous kernel
    RingState rs{0, 0, 0};
    auto refill = [&](uint32_t j, uint32_t slot) {
        if (j + a.NS < n_st) {
            if (PAIRED) issue_stage<true>(a, sm, rb, re, j + a.NS, slot);
            else issue_stage<false>(a, sm, rb, re, j + a.NS, slot);
        }
    };
    const bool ok = gemv_consume<QT, A4>(a, sm, tid, rs, refill);
    if (!ok && tid == 0) ring_drain(sm, n_st, a.NS, a.err);
}

}  // namespace fwb
