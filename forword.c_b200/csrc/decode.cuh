// decode.cuh — the persistent decode-step kernel.
//
// One launch runs a whole transformer_forward (transformer.c:149-326) for
// one token: embedding, then per layer QKV+RoPE+KV-append, attention,
// o-proj+residual, gate/up+SwiGLU, down+residual, and the LM head with the
// greedy argmax.  Grid = one CTA per SM (cooperative launch, so every CTA is
// resident); phases are separated by a grid barrier.
//
// The weight ring is shared by all GEMV phases.  Each CTA's weights for the
// whole step form one sequence of ring stages (global stage index j); when
// the last warp finishes stage j it immediately issues stage j + NS, even if
// that stage belongs to a later phase.  So weight streaming does not stop at
// phase boundaries: while the CTA waits at a barrier or runs the attention
// phase, the next GEMV's first NS stages are already landing in shared
// memory.
#pragma once
#include "attention.cuh"
#include "gemv.cuh"
#include "misc_kernels.cuh"

namespace fwb {

struct EmbedArgs {
    const uint8_t *table;
    uint32_t type, cols;
    uint64_t row_bytes;
    const uint32_t *step;
    float *x;
};

// Tensor parallelism: sum of the ranks' partial outputs (all-reduce), read
// straight from every rank's exchange buffer over NVLink (peer pointers; no
// multicast), added to the residual x.  Every rank sums in rank order, so all
// ranks hold bit-identical x afterwards.
struct ArArgs {
    float *x;                      // [n] residual stream of this rank (x += sum of parts)
    const unsigned long long *in;  // this rank's receive slot: [rank q][n] tagged partials
    const uint32_t *epoch;         // exchange epoch of the step (tags are epoch + k + 1)
    uint32_t k;                    // index of this exchange within the step
    uint32_t n, world;
    uint32_t *err, *abort;
};
// Tensor parallelism: the greedy token from the ranks' (value, index)
// candidates (lowest index among equal maxima, as sampler_argmax).
struct TpArgmaxArgs {
    const float *cand[kMaxRanks];  // every rank's candidate pair
    uint32_t world;
    uint32_t *out_token, *step_rw, *hist;
};

enum PhaseKind : uint32_t { PH_EMBED = 0, PH_GEMV = 1, PH_ATTN = 2, PH_ALLREDUCE = 3, PH_TPARGMAX = 4 };

struct __align__(16) Phase {
    uint32_t kind, qt, mode, a4;  // PH_GEMV: quant type, mode, 4-byte-aligned units
    uint32_t hd, gq;              // PH_ATTN: head_dim, GQA group
    uint32_t gsync;               // the barrier before this phase spans every rank
    uint32_t nobar;               // no grid barrier before this phase (it waits on tagged data)
    GemvArgs g;
    AttnArgs at;
    EmbedArgs e;
    ArArgs ar;
    TpArgmaxArgs am;
};

// This CTA's weight stream of one GEMV phase (host-computed).
struct StageSrc {
    uint64_t a, b;         // first source byte of the CTA's rows (gate / up for SWIGLU; b = 0 otherwise)
    uint32_t rows;         // rows of matrix a (= pairs for SWIGLU)
    uint32_t row_bytes;
    uint32_t R;            // local rows per stage (both halves for SWIGLU)
    uint32_t first;        // global index of the phase's first stage in this CTA's ring sequence
    uint32_t n_st;         // stages (0 for phases without weights)
    uint32_t paired;
};

constexpr uint32_t kDecodeThreads = 512;

struct DecodeArgs {
    const Phase *ph;
    const StageSrc *src;   // [gridDim.x][n_ph]
    uint32_t n_ph;
    uint32_t total_st;     // stages per CTA (max over CTAs is fine: CTAs read their own table)
    uint32_t NS, stage_bytes, scratch_bytes;
    const uint32_t *step;  // [0] token, [1] position of this step
    uint32_t *sync;        // [0] barrier arrivals, [1] abort, [2] cross-rank barriers passed (zeroed before each launch)
    uint32_t *err;
    uint32_t *n_st_cta;    // [gridDim.x] stages of each CTA
    // tensor parallelism (world > 1): cross-rank barrier counters (every rank's,
    // mapped; each CTA of each rank adds 1 to all of them per barrier), and the
    // number of such barriers completed before this step ([0], advanced by
    // n_gsync at the end of the step by CTA 0)
    unsigned long long *gcount[kMaxRanks];
    unsigned long long *gbase;
    uint32_t *xepoch;      // exchange epoch: advanced by n_exchange at the end of the step by CTA 0
    uint32_t world, n_gsync, n_exchange;
    unsigned long long *trace;  // optional: CTA 0's globaltimer at phase start [2p] and barrier arrival [2p+1]
    unsigned long long *trace_cta;  // optional: every CTA's barrier arrival [p * gridDim.x + cta]
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Issue stage k of one CTA stream into ring slot `slot` (one thread), or,
// with slot == kPrefetchOnly, only prefetch its bytes into L2.
constexpr uint32_t kPrefetchOnly = 0xffffffffu;

__device__ __forceinline__ void issue_src(const StageSrc &s, uint32_t k, uint8_t *ring, uint32_t stage_bytes,
                                          uint64_t *full, uint32_t slot) {
    const bool pf = slot == kPrefetchOnly;
    uint8_t *dst = pf ? nullptr : ring + (size_t)slot * stage_bytes;
    if (!s.paired) {
        const uint32_t r0 = k * s.R, nr = min(s.R, s.rows - r0);
        const uint64_t src = s.a + (uint64_t)r0 * s.row_bytes;
        const uint64_t s0 = src & ~15ull;
        const uint32_t bytes = (uint32_t)(((src + (uint64_t)nr * s.row_bytes + 15) & ~15ull) - s0);
        if (pf) { bulk_prefetch_l2(reinterpret_cast<const void *>(s0), bytes); return; }
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_g2s(dst, reinterpret_cast<const void *>(s0), bytes, &full[slot]);
    } else {
        const uint32_t p0 = k * (s.R / 2), np = min(s.R / 2, s.rows - p0);
        const uint64_t g = s.a + (uint64_t)p0 * s.row_bytes, u = s.b + (uint64_t)p0 * s.row_bytes;
        const uint64_t g0 = g & ~15ull, u0 = u & ~15ull;
        const uint32_t gb = (uint32_t)(((g + (uint64_t)np * s.row_bytes + 15) & ~15ull) - g0);
        const uint32_t ub = (uint32_t)(((u + (uint64_t)np * s.row_bytes + 15) & ~15ull) - u0);
        if (pf) {
            bulk_prefetch_l2(reinterpret_cast<const void *>(g0), gb);
            bulk_prefetch_l2(reinterpret_cast<const void *>(u0), ub);
            return;
        }
        mbar_arrive_expect_tx(&full[slot], gb + ub);
        bulk_g2s(dst, reinterpret_cast<const void *>(g0), gb, &full[slot]);
        bulk_g2s(dst + stage_bytes / 2, reinterpret_cast<const void *>(u0), ub, &full[slot]);
    }
}

// Issue global stage j of this CTA.  The phase holding j is found by
// scanning forward from a shared cursor: refills come in increasing j, so the
// scan is normally zero or one step.  Concurrent refills may race on the
// cursor; it then only lags behind, which keeps the scan correct.
__device__ __forceinline__ void issue_global(const StageSrc *tab, uint32_t n_ph, uint32_t j, uint8_t *ring,
                                             uint32_t stage_bytes, uint64_t *full, uint32_t slot,
                                             uint32_t *cursor) {
    uint32_t p = *(volatile uint32_t *)cursor;
    if (p >= n_ph || tab[p].first > j) p = 0;  // defensive restart
    while (p + 1 < n_ph && (tab[p].n_st == 0 || j >= tab[p].first + tab[p].n_st)) ++p;
    atomicMax(cursor, p);
    issue_src(tab[p], j - tab[p].first, ring, stage_bytes, full, slot);
}

struct PhaseResult {
    RingState rs;
    bool ok;
};

// L2 prefetch of the K and V rows [0, pos) of the layer whose QKV phase `g`
// is next: the rows the attention phase after it reads besides the new one.
// Issued a phase ahead, so HBM serves them while the QKV phase runs.  The
// rows of every KV head are split evenly over the CTAs.
__device__ __noinline__ void prefetch_kv_rows(const GemvArgs &g, uint32_t pos) {
    const uint32_t hd = g.head_dim, nkv = hd ? g.n_kv / hd : 0u;
    if (!pos || !nkv || pos > g.kv_ctx) return;
    const uint32_t parts = max(1u, gridDim.x / nkv);
    for (uint32_t it = blockIdx.x; it < nkv * parts; it += gridDim.x) {
        const uint32_t h = it / parts, pt = it % parts;
        const uint32_t r0 = (uint32_t)((uint64_t)pos * pt / parts), r1 = (uint32_t)((uint64_t)pos * (pt + 1) / parts);
        if (r1 <= r0) continue;
        const size_t off = ((size_t)h * g.kv_ctx + r0) * hd;
        bulk_prefetch_l2(g.kcache + off, (r1 - r0) * hd * 4u);
        bulk_prefetch_l2(g.vcache + off, (r1 - r0) * hd * 4u);
    }
}

// Grid-wide barrier number `epoch` (1, 2, ...).  Bounded: on timeout, or
// when another CTA already gave up (the abort flag sync[1]), it sets the
// abort flag and returns false.  While waiting, the CTAs start the next
// phase `nx`'s first reads that miss L2: a GEMV's RMSNorm weight (128 bytes
// per CTA) and, before a QKV phase, the K/V rows of the attention after it.
// pos: the step's position.
__device__ bool grid_sync(uint32_t *sync, uint32_t epoch, uint32_t *err, const Phase *nx, uint32_t pos) {
    __shared__ uint32_t ok_flag;
    __syncthreads();
    if (threadIdx.x == 0) {
        // release: this CTA's writes of the phase become visible with the add;
        // acquire: the other CTAs' writes are visible once the count is seen
        red_release_add(&sync[0], 1u);
        if (nx && nx->kind == PH_GEMV && nx->g.norm && blockIdx.x * 128u < nx->g.K * 4u)
            bulk_prefetch_l2(reinterpret_cast<const uint8_t *>(nx->g.norm_w) + blockIdx.x * 128u,
                             min(128u, nx->g.K * 4u - blockIdx.x * 128u));
        if (nx && nx->kind == PH_GEMV && nx->mode == GM_QKV) prefetch_kv_rows(nx->g, pos);
        const uint32_t target = epoch * gridDim.x;
        uint32_t ok = 0;
        for (uint32_t i = 0; i < (1u << 25); ++i) {
            if (ld_acquire(&sync[0]) >= target) { ok = 1; break; }
            if ((i & 255) == 255) {
                if (ld_acquire(&sync[1])) break;
                __nanosleep(32);
            }
        }
        if (!ok) {
            atomicOr(err, ERR_GRID_SYNC);
            atomicExch(&sync[1], 1u);
        }
        ok_flag = ok;
    }
    __syncthreads();
    return ok_flag != 0;
}

__device__ __forceinline__ void red_release_sys_add64(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Barrier across every CTA of every rank (tensor parallelism), after this
// rank's own grid barrier: CTA 0 alone adds one to every rank's counter
// (release, system scope: after the grid barrier before it, every local CTA's
// writes of the phase are covered and become visible to the peers) and waits
// (acquire) until its own counter shows all `world` arrivals of barrier
// number `nb` (counted across launches); it then publishes `gk` (this
// launch's count of such barriers) in sync[2], which the other CTAs wait for
// (acquire).  One system-scope atomic per rank and barrier instead of one per
// CTA.  Bounded like grid_sync; a timeout sets the local abort flag and the
// error.
__device__ bool global_sync(const DecodeArgs &d, unsigned long long nb, uint32_t gk) {
    __shared__ uint32_t ok_flag;
    if (threadIdx.x == 0) {
        uint32_t ok = 0;
        if (blockIdx.x == 0) {
            for (uint32_t q = 0; q < d.world; ++q) red_release_sys_add64(d.gcount[q], 1ull);
            const unsigned long long *mine = d.gcount[0];
            const unsigned long long target = nb * d.world;
            for (uint32_t i = 0; i < (1u << 25); ++i) {
                if (ld_acquire_sys64(mine) >= target) { ok = 1; break; }
                if ((i & 255) == 255) {
                    if (ld_acquire(&d.sync[1])) break;
                    __nanosleep(64);
                }
            }
            if (ok) st_release_gpu(&d.sync[2], gk);
        } else {
            for (uint32_t i = 0; i < (1u << 25); ++i) {
                if (ld_acquire(&d.sync[2]) >= gk) { ok = 1; break; }
                if ((i & 255) == 255) {
                    if (ld_acquire(&d.sync[1])) break;
                    __nanosleep(32);
                }
            }
        }
        if (!ok) {
            atomicOr(d.err, ERR_GRID_SYNC);
            atomicExch(&d.sync[1], 1u);
        }
        ok_flag = ok;
    }
    __syncthreads();
    return ok_flag != 0;
}

// x[i] += sum over ranks of part_q[i] for this CTA's rows.  Every rank's
// GEMV epilogue pushed its partial rows into this rank's receive slot as
// tagged words (GM_PUSH); here each row waits for the W tags of this
// exchange (bounded polling of local memory: no barrier and no fence), then
// the partials are added in rank order, so every rank computes bit-identical
// x.  Returns false if a tag did not arrive (error word and abort flag set).
__device__ bool allreduce_phase(const ArArgs &a) {
    const uint32_t b = (uint32_t)((uint64_t)blockIdx.x * a.n / gridDim.x);
    const uint32_t e = (uint32_t)((uint64_t)(blockIdx.x + 1) * a.n / gridDim.x);
    const uint32_t tag = __ldcg(a.epoch) + a.k + 1;
    bool ok = true;
    for (uint32_t i = b + threadIdx.x; i < e; i += blockDim.x) {
        float t = 0.f;
        for (uint32_t q = 0; q < a.world; ++q) {
            const unsigned long long *p = a.in + (size_t)q * a.n + i;
            unsigned long long w = ld_tagged(p);
            for (uint32_t it = 0; (uint32_t)(w >> 32) != tag; ++it) {
                if (it >= kMaxPolls || (it % 1024 == 1023 && *(volatile uint32_t *)a.abort)) {
                    atomicOr(a.err, ERR_EXCHANGE);
                    atomicExch(a.abort, 1u);
                    ok = false;
                    break;
                }
                if (it > 64) __nanosleep(64);
                w = ld_tagged(p);
            }
            if (!ok) break;
            const float v = __uint_as_float((uint32_t)w);
            t = q == 0 ? v : __fadd_rn(t, v);
        }
        if (!ok) break;
        a.x[i] = __fadd_rn(__ldcg(&a.x[i]), t);
    }
    return __syncthreads_and(ok) != 0;
}

__device__ void tp_argmax_phase(const TpArgmaxArgs &a) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (uint32_t q = 0; q < a.world; ++q) {
        const float cv = __ldcg(a.cand[q]);
        const uint32_t ci = __ldcg(reinterpret_cast<const uint32_t *>(a.cand[q]) + 1);
        if (ci != 0xffffffffu && (bi == 0xffffffffu || cv > bv || (cv == bv && ci < bi))) { bv = cv; bi = ci; }
    }
    const uint32_t nxt = bi == 0xffffffffu ? 0u : bi;  // every logit NaN: index 0, as the reference
    *a.out_token = nxt;
    if (a.hist) {
        const uint32_t p = __ldcg(&a.step_rw[1]);
        a.hist[p] = nxt;
        a.step_rw[0] = nxt;
        a.step_rw[1] = p + 1;
    }
}

template <int HD, int GQ>
__device__ __noinline__ void attn_phase_t(const AttnArgs &a, uint8_t *scratch, uint32_t pos) {
    auto &sh = *reinterpret_cast<AttnSmem<HD, GQ, kDecodeThreads / 32> *>(scratch);
    const uint32_t n_pos = pos + 1;
    const uint32_t n_use = attn_splits_in_use(a, n_pos);
    const uint32_t n_kv = a.n_kv;
    for (uint32_t it = blockIdx.x; it < n_kv * n_use; it += gridDim.x)
        attn_item<HD, GQ, kDecodeThreads / 32>(a, it / n_use, it % n_use, n_pos, n_use, sh);
}

__device__ void attn_phase(const Phase &P, uint8_t *scratch, uint32_t pos) {
#define FWB_ATTN(HDv, GQv) \
    if (P.hd == HDv && P.gq == GQv) { attn_phase_t<HDv, GQv>(P.at, scratch, pos); return; }
    FWB_ATTN(128, 4) FWB_ATTN(128, 8) FWB_ATTN(128, 2) FWB_ATTN(128, 1)
    FWB_ATTN(64, 1) FWB_ATTN(64, 2) FWB_ATTN(64, 4) FWB_ATTN(64, 8)
    FWB_ATTN(48, 1) FWB_ATTN(48, 2) FWB_ATTN(48, 4) FWB_ATTN(48, 8)
    FWB_ATTN(32, 1) FWB_ATTN(32, 2) FWB_ATTN(32, 4) FWB_ATTN(32, 8)
#undef FWB_ATTN
}

// One GEMV phase.  Everything the hot loop touches is passed by value so it
// stays in registers (a reference would force the struct into local memory).
// One instantiation per (quant type, 4-byte alignment): the mode only changes
// the prologue / epilogue and the pairing only per-thread offsets, so a model
// with one quant type runs one copy of the row loop for every GEMV phase
// (instruction-cache footprint).
template <int QT, bool A4, bool HALF = false>
__device__ __noinline__ PhaseResult gemv_phase_t(const GemvArgs *g, GemvSmem sm, RingState rs, const StageSrc *tab,
                                                 uint32_t n_ph, uint32_t total, uint32_t NS, uint32_t stage_bytes,
                                                 uint32_t pos) {
    uint8_t *ring = sm.ring;
    uint64_t *full = sm.full;
    uint32_t *cursor = sm.done + kMaxStages;  // phase cursor word, next to the counters
    auto refill = [=](uint32_t j, uint32_t slot) {
        if (j + NS < total) issue_global(tab, n_ph, j + NS, ring, stage_bytes, full, slot, cursor);
    };
    PhaseResult r;
    r.ok = gemv_consume<QT, A4, decltype(refill), HALF>(*g, sm, threadIdx.x, rs, refill, pos);
    r.rs = rs;
    return r;
}

template <int QT, bool HALF = false>
__device__ PhaseResult gemv_phase_q(const Phase &P, const GemvSmem &sm, const RingState &rs, const StageSrc *tab,
                                    uint32_t n_ph, uint32_t total, uint32_t NS, uint32_t stage_bytes, uint32_t pos) {
    return P.a4 ? gemv_phase_t<QT, true, HALF>(&P.g, sm, rs, tab, n_ph, total, NS, stage_bytes, pos)
                : gemv_phase_t<QT, false, HALF>(&P.g, sm, rs, tab, n_ph, total, NS, stage_bytes, pos);
}

// The persistent kernel.  Q4A4 != 0: every GEMV phase is Q4_0 with 4-byte
// aligned units; AHD != 0: every attention phase has head_dim AHD and group
// AGQ.  Such a specialisation holds one copy of the row loop and one of the
// attention instead of all of them: less code to fetch at every phase switch
// (measured 4 % per decode step on the 8B model).  decode_kernel_t<0, 0, 0>
// runs any model.  HALF: two GEMV rows per thread per round instead of four
// (one instead of two for Q8_0), for models whose ring of four-row stages
// does not fit next to the other shared memory (the 70B shapes).
template <int Q4A4, int AHD, int AGQ, bool HALF = false>
__global__ void __launch_bounds__(kDecodeThreads, 1) decode_kernel_t(const __grid_constant__ DecodeArgs d) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t tid = threadIdx.x;
    const uint32_t ring_off = kHeaderBytes + d.scratch_bytes;
    GemvSmem sm = gemv_smem(smem, 32, 0);
    sm.ring = smem + ring_off;
    StageSrc *tab = reinterpret_cast<StageSrc *>(smem + ring_off + d.NS * d.stage_bytes + 128);
    const uint32_t total = d.n_st_cta[blockIdx.x];

    // this CTA's stream table -> shared memory
    {
        const uint32_t words = d.n_ph * (uint32_t)(sizeof(StageSrc) / 4);
        const uint32_t *g = reinterpret_cast<const uint32_t *>(d.src + (size_t)blockIdx.x * d.n_ph);
        uint32_t *s = reinterpret_cast<uint32_t *>(tab);
        for (uint32_t i = tid; i < words; i += blockDim.x) s[i] = g[i];
    }
    if (tid == 0) {
        for (uint32_t i = 0; i < d.NS; ++i) {
            mbar_init(&sm.full[i], 1);
            sm.done[i] = 0;
        }
        sm.done[kMaxStages] = 0;  // phase cursor of the refills
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        for (uint32_t j = 0; j < min(d.NS, total); ++j)
            issue_global(tab, d.n_ph, j, sm.ring, d.stage_bytes, sm.full, j, sm.done + kMaxStages);
    }

    RingState rs{0, 0, 0};
    // the step's position (fixed during the launch: only the last phase of a
    // greedy step advances it, for the next launch)
    const uint32_t pos = __ldcg(&d.step[1]);
    // cross-rank barriers completed before this step, and during it
    const unsigned long long gbase = d.world > 1 ? __ldcg(d.gbase) : 0ull;
    uint32_t gk = 0, nbar = 0;
    bool ok = true;
    // phase descriptors are staged in shared memory one phase ahead
    __shared__ __align__(16) Phase ph_buf[2];
    constexpr uint32_t kPhWords = sizeof(Phase) / 4;
    for (uint32_t i = tid; i < kPhWords; i += blockDim.x)
        reinterpret_cast<uint32_t *>(&ph_buf[0])[i] = reinterpret_cast<const uint32_t *>(d.ph)[i];
    __syncthreads();
    constexpr uint32_t kPhChunks = sizeof(Phase) / 16;
    static_assert(sizeof(Phase) % 16 == 0 && kPhChunks <= kDecodeThreads, "phase descriptor copy");
    for (uint32_t p = 0; p < d.n_ph; ++p) {
        const Phase &P = ph_buf[p & 1];
        // the next descriptor streams into the other buffer while this phase runs
        const bool next = p + 1 < d.n_ph;
        if (next && tid < kPhChunks) {
            cp_async16(reinterpret_cast<uint8_t *>(&ph_buf[(p + 1) & 1]) + 16 * tid,
                       reinterpret_cast<const uint8_t *>(d.ph + p + 1) + 16 * tid);
            cp_async_commit();
        }
        if (d.trace && blockIdx.x == 0 && tid == 0) d.trace[2 * p] = global_ns();
        if (ok) {
            if (P.kind == PH_GEMV) {
                sm.planes = reinterpret_cast<uint32_t *>(smem + kHeaderBytes);
                sm.nbp = ((P.g.K / 32) + 1) & ~1u;
                sm.red = reinterpret_cast<float *>(smem + kHeaderBytes + plane_bytes(P.g.K));
                PhaseResult r{rs, false};
                if constexpr (Q4A4 != 0) {
                    r = gemv_phase_t<QT_Q4_0, true, HALF>(&P.g, sm, rs, tab, d.n_ph, total, d.NS, d.stage_bytes, pos);
                } else {
                    switch (P.qt) {
                    case QT_Q4_0: r = gemv_phase_q<QT_Q4_0, HALF>(P, sm, rs, tab, d.n_ph, total, d.NS, d.stage_bytes, pos); break;
                    case QT_Q5_0: r = gemv_phase_q<QT_Q5_0, HALF>(P, sm, rs, tab, d.n_ph, total, d.NS, d.stage_bytes, pos); break;
                    case QT_Q8_0: r = gemv_phase_q<QT_Q8_0, HALF>(P, sm, rs, tab, d.n_ph, total, d.NS, d.stage_bytes, pos); break;
                    case QT_Q5_1: r = gemv_phase_t<QT_Q5_1, true, HALF>(&P.g, sm, rs, tab, d.n_ph, total, d.NS, d.stage_bytes, pos); break;
                    case QT_Q4_K: r = gemv_phase_t<QT_Q4_K, true, HALF>(&P.g, sm, rs, tab, d.n_ph, total, d.NS, d.stage_bytes, pos); break;
                    case QT_Q6_K: r = gemv_phase_t<QT_Q6_K, true, HALF>(&P.g, sm, rs, tab, d.n_ph, total, d.NS, d.stage_bytes, pos); break;
                    default: break;
                    }
                }
                rs = r.rs;
                ok = ok && r.ok;
            } else if (P.kind == PH_ATTN) {
                if constexpr (AHD != 0) attn_phase_t<AHD, AGQ>(P.at, smem + kHeaderBytes, pos);
                else attn_phase(P, smem + kHeaderBytes, pos);
            } else if (P.kind == PH_ALLREDUCE) {
                if (!allreduce_phase(P.ar)) ok = false;
            } else if (P.kind == PH_TPARGMAX) {
                tp_argmax_phase(P.am);
            } else {  // PH_EMBED: x = row step[0] of the table (linear_get_row, linear.c:60-151)
                const EmbedArgs &e = P.e;
                const uint32_t tok = __ldcg(&e.step[0]);
                const uint8_t *row = e.table + (uint64_t)tok * e.row_bytes;
                for (uint32_t i = blockIdx.x * blockDim.x + tid; i < e.cols; i += gridDim.x * blockDim.x)
                    e.x[i] = e.type == 0 ? reinterpret_cast<const float *>(row)[i] : decode_elem(row, e.type, i);
            }
        } else if (P.kind == PH_GEMV) {
            // aborted: still walk the ring so that every issued stage is
            // accounted for, without computing
            ok = false;
        }
        if (d.trace) {
            __syncthreads();
            if (tid == 0) {
                const unsigned long long t = global_ns();
                if (blockIdx.x == 0) d.trace[2 * p + 1] = t;
                d.trace_cta[(size_t)p * gridDim.x + blockIdx.x] = t;
            }
        }
        if (next && tid < kPhChunks) cp_async_wait_all();
        // (the barriers' leading __syncthreads makes the copied descriptor visible)
        if (next) {
            const Phase &N = ph_buf[(p + 1) & 1];
            // a phase after a cross-rank barrier is preceded by this rank's grid
            // barrier and then the cross-rank one (grid_sync counts epochs by
            // phase index)
            __syncthreads();
            if (!N.nobar && !grid_sync(d.sync, ++nbar, d.err, &N, pos)) ok = false;
            if (N.gsync) {
                ++gk;
                if (!global_sync(d, gbase + gk, gk)) ok = false;
            }
        }
    }
    if (d.trace && blockIdx.x == 0 && tid == 0) d.trace[2 * d.n_ph] = global_ns();
    // every CTA read gbase and the exchange epoch before the step's last barrier
    if (d.world > 1 && blockIdx.x == 0 && tid == 0) {
        *d.gbase = gbase + d.n_gsync;
        *d.xepoch = __ldcg(d.xepoch) + d.n_exchange;
    }
    if (!ok && tid == 0) ring_drain(sm, min(total, rs.j + d.NS), d.NS, d.err);
}

}  // namespace fwb
