// common.cuh — device helpers shared by the forword-b200 kernels (sm_100a).
//
// Inline PTX for the Blackwell data-movement primitives the kernels use:
// mbarrier phases with transaction counts, 1-D bulk async copies
// (cp.async.bulk, global -> shared, no multicast), and programmatic
// dependent launch (griddepcontrol).  Every wait is bounded: on timeout it
// records an error code in the device error word and returns false, so a
// kernel can wind down instead of hanging the GPU.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace fwb {

// Error word bits (device status, read back by the host after a step).
enum : uint32_t {
    ERR_NONE = 0,
    ERR_WAIT_FULL = 1u << 0,    // consumer timed out waiting for a weight stage
    ERR_WAIT_EMPTY = 1u << 1,   // producer timed out waiting for a free stage
    ERR_WAIT_DRAIN = 1u << 2,   // producer timed out draining its copies on error
    ERR_BAD_POS = 1u << 3,      // step position outside the KV cache
    ERR_BAD_TOKEN = 1u << 4,    // token id outside the vocabulary
    ERR_ATTN_TIMEOUT = 1u << 5,
    ERR_GRID_SYNC = 1u << 6,     // a grid barrier of the persistent kernel timed out
    ERR_EXCHANGE = 1u << 7,      // a rank's tagged partial sums did not arrive (tensor parallelism)
};

// Tensor parallelism: ranks of one box.
constexpr uint32_t kMaxRanks = 8;

// Tagged 8-byte words of the cross-rank exchange: value bits in the low
// half, the exchange's tag in the high half, written and read as one
// single-copy-atomic 8-byte access, so a reader that sees the tag sees the
// value with it and no fence is needed between them.
__device__ __forceinline__ void st_tagged(unsigned long long *p, float v, uint32_t tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Upper bound on polls of one barrier phase.  With the back-off below this is
// several seconds, far beyond any legitimate wait inside one decode step.
constexpr uint32_t kMaxPolls = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
            smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for `parity` of an mbarrier phase.  Returns false (and sets
// `code` in *err) when the bound is exceeded or another thread already
// flagged an error.  The first poll is inline (the phase has normally
// completed already); the polling loop is out of line.
__device__ __noinline__ bool mbar_wait_slow(uint64_t *bar, uint32_t parity, uint32_t *err, uint32_t code) {
    for (uint32_t i = 0; i < kMaxPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (i > 64) __nanosleep(i < 4096 ? 32 : 256);
        if ((i & 1023) == 1023 && *(volatile uint32_t *)err) return false;
    }
    atomicOr(err, code);
    return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *err,
                                          uint32_t code) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, err, code);
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` of
// transaction count on `bar`.  src, dst 16-byte aligned; bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk prefetch of [src, src+bytes) into L2 (no shared memory, no
// completion tracking).  src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 16-byte asynchronous copy global -> shared (no register staging); both
// addresses 16-byte aligned.  Completed by cp_async_wait_all() in the issuing
// thread, visible to the CTA after a following barrier.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// gpu-scope release add / acquire load (grid barrier)
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void red_release_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Programmatic dependent launch.  wait: block until the preceding kernel in
// the stream has completed and its writes are visible.  launch: allow the
// next kernel to begin launching (its pre-wait prologue then overlaps us).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Named barrier over the first `nthreads` threads (multiple of 32).
__device__ __forceinline__ void bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xffffu)));
}

__device__ __forceinline__ int dp4a_us(uint32_t a, int32_t b, int c) {
    // a: 4 unsigned bytes, b: 4 signed bytes
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(int32_t a, int32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_su(int32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

}  // namespace fwb
