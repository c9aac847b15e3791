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
// in steps of 64 (two Q4_0 blocks).  Four warps load the step's activation
// rows and dequantise the weight rows ((q - 8) * d in fp32, as the reference
// decoders, then rounded to fp16) into shared memory in the K-major 128-byte
// swizzled layout the MMA reads; one thread issues four
// tcgen05.mma.kind::f16 (K = 16 each) and commits them to an mbarrier.  Two
// stages: the loads of step i+1 overlap the MMAs of step i, and each thread
// has step i+1's global bytes in flight while it writes step i's tiles.  The epilogue
// reads the accumulator with tcgen05.ld (warp w owns TMEM lanes 32w..32w+31)
// and stores, or adds into, Y.
//
// Numerics: fp16 weights carry (q - 8) * d to 11 significant bits and fp16
// activations x to 11 bits; products and sums are fp32.  Every wait is
// bounded and sets an error bit; the TMEM columns are released on every path.
#pragma once
#include "common.cuh"

namespace fwb {

constexpr uint32_t kTcM = 128;        // tokens per tile
constexpr uint32_t kTcN = 128;        // weight rows per tile
constexpr uint32_t kTcK = 64;         // K per stage
constexpr uint32_t kTcThreads = 128;
constexpr uint32_t kTcTileBytes = 128 * 128;  // 128 rows of 64 fp16 (128 B)
constexpr uint32_t kTcSmem = 4 * kTcTileBytes + 1024 + 256;  // 2 stages x (A, B), alignment, barriers

enum TcMode : uint32_t { TC_STORE = 0, TC_ADD = 1 };

struct TcArgs {
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

// The global bytes of one stage for this thread: its activation row (64 fp16)
// and its weight row's two Q4_0 blocks (36 bytes, 4-byte aligned).  Fetched
// one stage ahead so that their latency hides behind the current stage.
struct TcRaw {
    uint4 a[8];
    uint32_t q[9];
};

__device__ __forceinline__ void tc_fetch(const TcArgs &a, uint32_t m0, uint32_t n0, uint32_t k0, TcRaw &r) {
    const uint32_t t = threadIdx.x, m = m0 + t, n = n0 + t;
    if (m < a.M) {
        const uint4 *src = reinterpret_cast<const uint4 *>(a.x + (size_t)m * a.K + k0);
#pragma unroll
        for (int i = 0; i < 8; ++i) r.a[i] = __ldg(src + i);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) r.a[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    if (n < a.N) {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(a.w + (size_t)n * a.row_bytes + (k0 >> 5) * 18u);
#pragma unroll
        for (int i = 0; i < 9; ++i) r.q[i] = __ldg(src + i);
    } else {
#pragma unroll
        for (int i = 0; i < 9; ++i) r.q[i] = 0u;  // d = 0: every value 0
    }
}

// One stage into the swizzled A / B tiles: the activation row as is, the
// weight row dequantised (rows outside M / N are zero).
__device__ __forceinline__ void tc_store_stage(const TcRaw &r, uint8_t *sa, uint8_t *sb) {
    const uint32_t t = threadIdx.x;
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) *reinterpret_cast<uint4 *>(sa + tc_sw128(t, i)) = r.a[i];
    // block 0: d in q[0] low half, quants in bytes 2..17; block 1: d in q[4]
    // high half, quants in bytes 20..35 = q[5..8]
    const float d0 = __half2float(__ushort_as_half((unsigned short)(r.q[0] & 0xffffu)));
    const float d1 = __half2float(__ushort_as_half((unsigned short)(r.q[4] >> 16)));
    uint32_t qs0[4], qs1[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        qs0[i] = __funnelshift_r(r.q[i], r.q[i + 1], 16);
        qs1[i] = r.q[5 + i];
    }
#pragma unroll
    for (uint32_t blk = 0; blk < 2; ++blk) {
        const uint32_t *qs = blk ? qs1 : qs0;
        const float d = blk ? d1 : d0;
        // element j (< 16): low nibble of byte j; element j + 16: high nibble
#pragma unroll
        for (uint32_t half = 0; half < 2; ++half) {
#pragma unroll
            for (uint32_t cc = 0; cc < 2; ++cc) {  // 8 elements per chunk
                uint32_t o[4];
#pragma unroll
                for (uint32_t e = 0; e < 4; ++e) {
                    float v[2];
#pragma unroll
                    for (uint32_t u = 0; u < 2; ++u) {
                        const uint32_t j = cc * 8 + e * 2 + u;  // byte index 0..15
                        const uint32_t byte = (qs[j >> 2] >> ((j & 3) * 8)) & 0xffu;
                        const int qv = (int)(half ? (byte >> 4) : (byte & 15u)) - 8;
                        v[u] = __fmul_rn((float)qv, d);
                    }
                    o[e] = pack_h2(v[0], v[1]);
                }
                const uint32_t chunk = blk * 4 + half * 2 + cc;
                *reinterpret_cast<uint4 *>(sb + tc_sw128(t, chunk)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
    }
}

__global__ void __launch_bounds__(kTcThreads, 1) gemm_q4_0_tc_kernel(const __grid_constant__ TcArgs a) {
    extern __shared__ uint8_t tc_smem_raw[];
    const uint32_t base = (smem_u32(tc_smem_raw) + 1023u) & ~1023u;
    uint8_t *smem = tc_smem_raw + (base - smem_u32(tc_smem_raw));
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + 4 * kTcTileBytes);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + 4 * kTcTileBytes + 64);
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t n0 = blockIdx.x * kTcN, m0 = blockIdx.y * kTcM;

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
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

    const uint32_t steps = a.K / kTcK;
    bool ok = true;
    TcRaw raw;
    if (steps > 0) tc_fetch(a, m0, n0, 0, raw);
    for (uint32_t it = 0; it < steps; ++it) {
        const uint32_t s = it & 1u;
        uint8_t *sa = smem + s * 2u * kTcTileBytes, *sb = sa + kTcTileBytes;  // stage s: A then B
        TcRaw next = raw;
        if (it + 1 < steps) tc_fetch(a, m0, n0, (it + 1) * kTcK, next);
        if (it >= 2 && ok)  // the MMAs that read this stage two steps ago are done
            ok = mbar_wait(&bar[s], ((it - 2) >> 1) & 1u, a.err, ERR_WAIT_FULL);
        tc_store_stage(raw, sa, sb);
        raw = next;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint64_t da = tc_desc(smem_u32(sa)), db = tc_desc(smem_u32(sb));
#pragma unroll
            for (uint32_t k = 0; k < kTcK / 16; ++k)  // 16 fp16 = 32 bytes = 2 descriptor units per step
                tc_mma(tmem, da + 2u * k, db + 2u * k, (it | k) != 0u);
            tc_commit(&bar[s]);
        }
    }
    // the last commit covers every MMA issued before it
    if (steps > 0 && ok) ok = mbar_wait(&bar[(steps - 1) & 1u], ((steps - 1) >> 1) & 1u, a.err, ERR_WAIT_FULL);
    // a thread whose wait failed must not free TMEM the MMAs may still write
    // to: it waits (bounded) again with the others below before the release
    tc_fence_after();
    if (ok && steps > 0) {
        const uint32_t m = m0 + warp * 32 + lane;
#pragma unroll 1
        for (uint32_t c0 = 0; c0 < kTcN; c0 += 32) {
            float v[32];
            tc_ld32(tmem + ((warp * 32u) << 16) + c0, v);
            if (m < a.M) {
                float *yr = a.y + (size_t)m * a.ldy + n0 + c0;
#pragma unroll
                for (uint32_t i = 0; i < 32; ++i)
                    if (n0 + c0 + i < a.N) yr[i] = a.mode == TC_ADD ? __fadd_rn(yr[i], v[i]) : v[i];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (!ok && tid == 0 && steps > 0)  // drain: the final commit must have landed before the release
        mbar_wait(&bar[(steps - 1) & 1u], ((steps - 1) >> 1) & 1u, a.err, ERR_WAIT_DRAIN);
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcN) : "memory");
    }
}

}  // namespace fwb
