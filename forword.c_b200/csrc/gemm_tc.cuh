// gemm_tc.cuh — batched dequant-GEMM on the 5th-generation tensor cores
// (tcgen05 / TMEM) for the prompt (prefill) path.
//
// Computes Y[m][n] = sum_k X[m][k] * W[n][k] for M tokens at once, W a GGUF
// Q4_0 tensor (rows of 18-byte blocks, used in place: never repacked in HBM)
// and X fp16 activations, accumulating in fp32 in tensor memory.  This is the
// batched form of linear_forward / quant_matvec (linear.c:155-223,
// quant_matvec.c:263-312): the prompt's tokens share each weight tile, so the
// contraction is dense enough for the tensor cores, unlike batch-1 decode.
//
// Tile: 128 tokens (TMEM lanes) x 128 weight rows (TMEM columns) per CTA, K
// in steps of 64 (two Q4_0 blocks) through a ring of kTcStages shared-memory
// stages, two CTAs per SM.  Warp-specialised, six warps:
//  * warps 0-3 (producers): thread t dequantises weight row t's two blocks
//    of the step, (q - 8) * d rounded once to fp16 with half2 arithmetic
//    (bit-identical to rounding the exact fp32 product), into the K-major
//    128-byte-swizzled B tile, and the warp arrives on the stage's `full`
//    mbarrier.  The weight row streams through registers a 256-wide K chunk
//    (144 bytes, 16-byte loads when the rows allow) ahead;
//  * warp 5, one thread: the stage's activation tile (128 tokens x 64 fp16)
//    by TMA (cp.async.bulk.tensor, 2-D map with the 128-byte swizzle, no
//    multicast; rows past M read as zeros) onto the stage's `afull`
//    mbarrier, as far ahead as the ring allows;
//  * warp 4, one thread: waits for both barriers, issues four
//    tcgen05.mma.kind::f16 (K = 16 each) and commits them to the stage's
//    `empty` mbarrier, which the producers and the TMA thread wait on before
//    refilling the stage.
// After the last MMA a commit to `done` releases the epilogue: the producer
// warps read the accumulator with tcgen05.ld (warp w owns TMEM lanes
// 32w..32w+31) and store, or add into, Y.  The F16W instance takes weights
// already expanded to fp16 (q4_0_to_f16_kernel, the same values): the TMA
// thread then loads both tiles of a stage and the producers only run the
// epilogue.
//
// Numerics: fp16 weights carry (q - 8) * d to 11 significant bits and fp16
// activations x to 11 bits; products and sums are fp32.  Every wait is
// bounded and sets an error bit; the MMA thread always makes the final
// commit, so the TMEM columns are released only after every issued MMA.
#pragma once
#include <cuda.h>  // CUtensorMap

#include "common.cuh"

namespace fwb {

constexpr uint32_t kTcM = 128;        // tokens per tile
constexpr uint32_t kTcN = 128;        // weight rows per tile
constexpr uint32_t kTcK = 64;         // K per stage
constexpr uint32_t kTcStages = 3;     // ring depth (two CTAs per SM)
constexpr uint32_t kTcProducers = 128;  // four producer warps; a fifth issues the MMAs, a sixth the TMA
constexpr uint32_t kTcThreads = kTcProducers + 64;
constexpr uint32_t kTcTileBytes = 128 * 128;  // 128 rows of 64 fp16 (128 B)
constexpr uint32_t kTcSmem = kTcStages * 2 * kTcTileBytes + 1024 + 256;  // stages x (A, B), alignment, barriers

enum TcMode : uint32_t { TC_STORE = 0, TC_ADD = 1 };

struct TcArgs {
    CUtensorMap xmap;     // the activations as a 2-D tensor map: box 64 x 128, 128-byte swizzle
    CUtensorMap wmap;     // F16W: the weights already expanded to fp16 [N][K], the same box and swizzle
    const uint8_t *w;     // Q4_0 rows [N][K/32 blocks]
    uint32_t row_bytes;   // K/32 * 18
    const __half *x;      // [M][K] fp16, row-major
    float *y;             // [M][ldy] fp32
    uint32_t M, N, K, ldy;
    uint32_t mode;        // TcMode
    uint32_t *err;
};

// Byte offset of 16-byte chunk c of row r in a K-major tile with 128-byte
// rows and the 128-byte swizzle (chunk index XOR row within the 8-row atom).
__device__ __forceinline__ uint32_t tc_sw128(uint32_t r, uint32_t c) {
    return (r >> 3) * 1024u + (r & 7u) * 128u + ((c ^ (r & 7u)) << 4);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 bytes apart (SBO), LBO 1 (unused inside one swizzle atom), version 1.
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator, fp16 A and B, both
// K-major, N = 128, M = 128.
constexpr uint32_t kTcIdesc = (1u << 4) | ((kTcN >> 3) << 17) | ((kTcM >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(kTcIdesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// (q - 8) * d for a pair of fp16 values whose bits are 0x6400 | q (that is,
// 1024 + q): minus 1032, then times d -- each step exact but the last,
// which rounds the exact product once.
__device__ __forceinline__ uint32_t q4_scale(uint32_t p, __half2 d2) {
    const __half2 k1032 = __halves2half2(__ushort_as_half((unsigned short)0x6408u),
                                         __ushort_as_half((unsigned short)0x6408u));
    const __half2 v = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&p), k1032), d2);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// Weight row t of one K step (two Q4_0 blocks in 9 words, the first block's
// scale in the low half of w[0], the second's in the high half of w[4]) into
// the swizzled B tile: 8 chunks of 8 fp16.  Element j < 16 of a block is the
// low nibble of quant byte j, element 16 + j the high nibble; a word of
// nibbles (4 bytes) becomes two fp16 pairs 0x64qq by one byte permutation
// each.
__device__ __forceinline__ void tc_dequant_row(const uint32_t (&w)[9], uint8_t *sb, uint32_t t) {
#pragma unroll
    for (uint32_t blk = 0; blk < 2; ++blk) {
        const uint32_t dbits = blk ? (w[4] >> 16) : (w[0] & 0xffffu);
        const __half dh = __ushort_as_half((unsigned short)dbits);
        const __half2 d2 = __halves2half2(dh, dh);
        uint32_t nib[8];  // [0..3]: low nibbles of quant words 0..3, [4..7]: high nibbles
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t q = blk ? w[5 + i] : __funnelshift_r(w[i], w[i + 1], 16);
            nib[i] = q & 0x0F0F0F0Fu;
            nib[4 + i] = (q >> 4) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (uint32_t c = 0; c < 4; ++c) {  // chunk c: elements 8c .. 8c + 7 = nibble words 2c, 2c + 1
            const uint32_t x0 = nib[2 * c], x1 = nib[2 * c + 1];
            uint4 o;
            o.x = q4_scale(__byte_perm(x0, 0x64646464u, 0x4140u), d2);
            o.y = q4_scale(__byte_perm(x0, 0x64646464u, 0x4342u), d2);
            o.z = q4_scale(__byte_perm(x1, 0x64646464u, 0x4140u), d2);
            o.w = q4_scale(__byte_perm(x1, 0x64646464u, 0x4342u), d2);
            *reinterpret_cast<uint4 *>(sb + tc_sw128(t, blk * 4 + c)) = o;
        }
    }
}

// One activation tile (64 K values x 128 tokens from (k0, m0)) by TMA into
// a 1024-byte-aligned stage, completing on `bar`.
__device__ __forceinline__ void tc_tma_x(uint8_t *dst, const CUtensorMap *map, uint32_t k0, uint32_t m0,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(k0), "r"(m0), "r"(smem_u32(bar))
        : "memory");
}

// 4 K steps (one 256-wide chunk, 36 words) of this producer's weight row
// (zeros -- scale 0 -- outside N or beyond the last K step).  V16: the row's
// chunks are 16-byte aligned (row bytes and base multiples of 16).
template <bool V16>
__device__ __forceinline__ void tc_fetch_w(const TcArgs &a, uint32_t n, uint32_t step0, uint32_t steps,
                                           uint32_t (&w)[36]) {
    const uint8_t *row = a.w + (size_t)n * a.row_bytes + (size_t)step0 * 36u;
    if (n < a.N && V16 && step0 + 4 <= steps) {
#pragma unroll
        for (int i = 0; i < 9; ++i) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(row) + i);
            w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 36; ++i)
            w[i] = (n < a.N && step0 + (uint32_t)i / 9u < steps) ? __ldg(reinterpret_cast<const uint32_t *>(row) + i)
                                                                 : 0u;
    }
}

// Q4_0 rows [rows][cols] -> fp16 [rows][cols]: (q - 8) * d rounded once to
// fp16 (the fp32 product of the 4-bit integer and the fp16 scale is exact),
// the same values the producers of gemm_q4_0_tc_kernel write into the B
// tile.  One thread per 32-value block.
__global__ void q4_0_to_f16_kernel(const uint8_t *w, uint64_t n_blocks, __half *out) {
    for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < n_blocks;
         b += (uint64_t)gridDim.x * blockDim.x) {
        const uint8_t *blk = w + b * 18;
        const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
        uint4 o[4];
        uint32_t *ow = reinterpret_cast<uint32_t *>(o);
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const uint32_t q0 = blk[2 + j], q1 = blk[3 + j];
            ow[j / 2] = pack_h2((float)((int)(q0 & 15) - 8) * d, (float)((int)(q1 & 15) - 8) * d);
            ow[8 + j / 2] = pack_h2((float)((int)(q0 >> 4) - 8) * d, (float)((int)(q1 >> 4) - 8) * d);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(out + b * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = o[i];
    }
}

// V16: the Q4_0 rows allow 16-byte loads.  F16W: the weights come as fp16
// through wmap (expanded once by q4_0_to_f16_kernel): the TMA thread loads
// both operands of every stage and the producer warps only run the epilogue.
template <bool V16, bool F16W = false>
__global__ void __launch_bounds__(kTcThreads, 2) gemm_q4_0_tc_kernel(const __grid_constant__ TcArgs a) {
    extern __shared__ uint8_t tc_smem_raw[];
    const uint32_t base = (smem_u32(tc_smem_raw) + 1023u) & ~1023u;
    uint8_t *smem = tc_smem_raw + (base - smem_u32(tc_smem_raw));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kTcStages * 2 * kTcTileBytes);
    uint64_t *afull = full + kTcStages, *empty = afull + kTcStages, *done = empty + kTcStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t n0 = blockIdx.x * kTcN, m0 = blockIdx.y * kTcM;
    const uint32_t steps = a.K / kTcK;

    if (tid == 0) {
        for (uint32_t s = 0; s < kTcStages; ++s) {
            mbar_init(&full[s], kTcProducers / 32);
            mbar_init(&afull[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 0) {  // 128 fp32 accumulator columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTcN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == kTcProducers / 32) {
        // ---- MMA issue: one thread
        if (lane == 0) {
            uint32_t i = 0;
            for (; i < steps; ++i) {
                const uint32_t s = i % kTcStages;
                if ((!F16W && !mbar_wait(&full[s], (i / kTcStages) & 1u, a.err, ERR_WAIT_FULL)) ||
                    !mbar_wait(&afull[s], (i / kTcStages) & 1u, a.err, ERR_WAIT_FULL)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint8_t *sa = smem + s * 2u * kTcTileBytes, *sb = sa + kTcTileBytes;
                const uint64_t da = tc_desc(smem_u32(sa)), db = tc_desc(smem_u32(sb));
#pragma unroll
                for (uint32_t k = 0; k < kTcK / 16; ++k)  // 16 fp16 = 32 bytes = 2 descriptor units
                    tc_mma(tmem, da + 2u * k, db + 2u * k, (i | k) != 0u);
                tc_commit(&empty[s]);
            }
            tc_commit(done);  // covers every MMA issued above, also after a failed wait
        }
        __syncwarp();
    } else if (warp == kTcProducers / 32 + 1) {
        // ---- activation tiles by TMA: one thread
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.xmap)) : "memory");
            if (F16W) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.wmap)) : "memory");
            uint32_t i = 0;
            for (; i < steps; ++i) {
                const uint32_t s = i % kTcStages;
                if (i >= kTcStages &&
                    !mbar_wait(&empty[s], ((i / kTcStages) - 1) & 1u, a.err, ERR_WAIT_EMPTY))
                    break;
                mbar_arrive_expect_tx(&afull[s], F16W ? 2 * kTcTileBytes : kTcTileBytes);
                tc_tma_x(smem + s * 2u * kTcTileBytes, &a.xmap, i * kTcK, m0, &afull[s]);
                if (F16W) tc_tma_x(smem + s * 2u * kTcTileBytes + kTcTileBytes, &a.wmap, i * kTcK, n0, &afull[s]);
            }
            // before the CTA may exit, the copies still in flight land (the
            // MMA thread consumed every stage unless a wait failed)
            for (uint32_t k = i > kTcStages ? i - kTcStages : 0; k < i; ++k)
                mbar_wait(&afull[k % kTcStages], (k / kTcStages) & 1u, a.err, ERR_WAIT_DRAIN);
        }
        __syncwarp();
    } else {
        // ---- producers: thread t fills weight row t of each stage
        const uint32_t t = tid, n = n0 + t;
        uint32_t wc[36];
        if (steps && !F16W) tc_fetch_w<V16>(a, n, 0, steps, wc);
        for (uint32_t c0 = 0; c0 < steps && ok && !F16W; c0 += 4) {
            uint32_t wn[36];
            tc_fetch_w<V16>(a, n, c0 + 4, steps, wn);  // zeros past the last step
#pragma unroll
            for (uint32_t j = 0; j < 4; ++j) {  // fully unrolled: wc is indexed by constants only
                const uint32_t i = c0 + j;
                if (i < steps && ok) {
                    const uint32_t s = i % kTcStages;
                    if (i >= kTcStages)  // the MMAs that read this stage kTcStages steps ago are done
                        ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ((i / kTcStages) - 1) & 1u, a.err,
                                                               ERR_WAIT_EMPTY));
                    if (ok) {
                        uint8_t *sb = smem + s * 2u * kTcTileBytes + kTcTileBytes;
                        const uint32_t w9[9] = {wc[9 * j], wc[9 * j + 1], wc[9 * j + 2], wc[9 * j + 3], wc[9 * j + 4],
                                                wc[9 * j + 5], wc[9 * j + 6], wc[9 * j + 7], wc[9 * j + 8]};
                        tc_dequant_row(w9, sb, t);
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic -> tensor core
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&full[s]);
                    }
                }
            }
#pragma unroll
            for (uint32_t q = 0; q < 36; ++q) wc[q] = wn[q];
        }
        // ---- epilogue: the accumulator, once every MMA is done
        const bool fin = __all_sync(0xffffffffu, mbar_wait(done, 0u, a.err, ERR_WAIT_FULL));
        tc_fence_after();
        if (ok && fin && steps > 0) {
            const uint32_t mm = m0 + warp * 32 + lane;
            const bool vec = (a.ldy & 3u) == 0u && ((uintptr_t)a.y & 15u) == 0u;
#pragma unroll 1
            for (uint32_t c0 = 0; c0 < kTcN; c0 += 32) {
                float v[32];
                tc_ld32(tmem + ((warp * 32u) << 16) + c0, v);  // warp w reads TMEM lanes 32w..32w+31
                if (mm >= a.M) continue;
                float *yr = a.y + (size_t)mm * a.ldy + n0 + c0;
                if (vec && n0 + c0 + 32 <= a.N) {  // the thread's 128 contiguous bytes as 8 float4
#pragma unroll
                    for (uint32_t i = 0; i < 32; i += 4) {
                        float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                        if (a.mode == TC_ADD) {
                            const float4 y0 = *reinterpret_cast<const float4 *>(yr + i);
                            o.x = __fadd_rn(y0.x, o.x); o.y = __fadd_rn(y0.y, o.y);
                            o.z = __fadd_rn(y0.z, o.z); o.w = __fadd_rn(y0.w, o.w);
                        }
                        *reinterpret_cast<float4 *>(yr + i) = o;
                    }
                } else {
#pragma unroll
                    for (uint32_t i = 0; i < 32; ++i)
                        if (n0 + c0 + i < a.N) yr[i] = a.mode == TC_ADD ? __fadd_rn(yr[i], v[i]) : v[i];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        // normally complete already; after a failed wait, the MMAs the final
        // commit covers must finish before their columns are freed
        mbar_wait(done, 0u, a.err, ERR_WAIT_FULL);
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcN) : "memory");
    }
}

}  // namespace fwb
