// runtime.cu — device model, per-token launch sequence, CUDA graph, C ABI.
//
// transformer_init / transformer_forward of forword.c (transformer.c:14-326)
// become: upload every tensor once to one HBM arena in its GGUF byte layout,
// resolve all tensors once (instead of the per-token tensor_find string scans
// of transformer.c:212-222, attention.c:98-107, ffn.c:59-74), and replay one
// CUDA graph per token.  The graph holds 5 kernels per layer plus the
// embedding and the LM head, chained with programmatic dependent launch so
// that each GEMV's weights stream in while its predecessor finishes.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "../../include/forword_b200.h"
#include "attention.cuh"
#include "gemv.cuh"
#include "gguf_reader.h"
#include "tp_shard.h"
#include "upload.h"
#include "decode.cuh"
#include "misc_kernels.cuh"
#include "gemm_tc.cuh"
#include "prefill.cuh"
#include "sampler.cuh"

namespace fwb {

static thread_local std::string g_err;
static void set_err(const std::string &e) { g_err = e; }

#define CK(x)                                                                            \
    do {                                                                                 \
        cudaError_t e_ = (x);                                                            \
        if (e_ != cudaSuccess) {                                                         \
            set_err(std::string(#x) + " failed: " + cudaGetErrorString(e_));             \
            return false;                                                                \
        }                                                                                \
    } while (0)

// --------------------------------------------------------------------------
// kernel selection
// --------------------------------------------------------------------------
template <int QT>
static const void *pick_gemv_mode(int, bool a4, bool) {
    return a4 ? (const void *)gemv_kernel<QT, true> : (const void *)gemv_kernel<QT, false>;
}

static const void *gemv_fn(int qt, int mode, bool a4, bool big) {
    switch (qt) {
    case QT_Q4_0: return pick_gemv_mode<QT_Q4_0>(mode, a4, big);
    case QT_Q5_0: return pick_gemv_mode<QT_Q5_0>(mode, a4, big);
    case QT_Q8_0: return pick_gemv_mode<QT_Q8_0>(mode, a4, big);
    // (their units are always 4-byte aligned, or loaded without that assumption)
    case QT_Q5_1: return (const void *)gemv_kernel<QT_Q5_1, true>;
    case QT_Q4_K: return (const void *)gemv_kernel<QT_Q4_K, true>;
    case QT_Q6_K: return (const void *)gemv_kernel<QT_Q6_K, true>;
    default: return nullptr;
    }
}

// Values per block of a GEMV-able type (the input width must be a multiple).
static uint32_t gemv_block_values(int qt) { return qt == QT_Q4_K || qt == QT_Q6_K ? 256u : 32u; }

template <int HD>
static const void *pick_attn_gq(uint32_t gq) {
    switch (gq) {
    case 1: return (const void *)attn_decode_kernel<HD, 1>;
    case 2: return (const void *)attn_decode_kernel<HD, 2>;
    case 4: return (const void *)attn_decode_kernel<HD, 4>;
    case 8: return (const void *)attn_decode_kernel<HD, 8>;
    default: return nullptr;
    }
}
static const void *attn_fn(uint32_t hd, uint32_t gq) {
    switch (hd) {
    case 32: return pick_attn_gq<32>(gq);
    case 48: return pick_attn_gq<48>(gq);
    case 64: return pick_attn_gq<64>(gq);
    case 128: return pick_attn_gq<128>(gq);
    default: return nullptr;
    }
}

static int num_sms(int dev) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 1;
}

static cudaError_t launch_ex(const void *fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void **args,
                             bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? at : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// --------------------------------------------------------------------------
// GEMV launch geometry
// --------------------------------------------------------------------------
struct GemvLaunch {
    const void *fn = nullptr;
    dim3 grid, block;
    size_t smem = 0;
    GemvArgs a{};
    uint64_t weight_bytes = 0;  // algorithmic bytes streamed per launch
};

static uint32_t pow2ceil(uint32_t v) {
    uint32_t p = 1;
    while (p < v) p <<= 1;
    return p;
}

constexpr uint32_t kRingBudget = 192 * 1024;
constexpr uint32_t kMaxSmem = 227 * 1024;  // per-block opt-in limit (static + dynamic)

// Fills geometry fields of L.a (w, n_out, K, row_bytes set by the caller).
static bool plan_gemv(int qt, int mode, int sms, GemvLaunch &L, bool half_rows = false) {
    GemvArgs &a = L.a;
    const uint32_t nb = a.K / 32;
    if (a.K % gemv_block_values(qt) || nb == 0 || a.n_out == 0) { set_err("gemv: bad shape"); return false; }
    const bool paired = mode == GM_SWIGLU;
    a.mode = (uint32_t)mode;
    a.norm = (mode == GM_QKV || mode == GM_SWIGLU || mode == GM_LOGITS) ? 1u : 0u;
    a.gran = (mode == GM_QKV || paired) ? (paired ? 1u : 2u) : 1u;
    if (mode == GM_QKV && a.n_out % 2) { set_err("gemv: odd qkv rows"); return false; }
    a.U = (nb + 1) / 2;
    a.Upad = a.U <= 32 ? std::max(8u, pow2ceil(a.U)) : (a.U + 31) / 32 * 32;
    if (a.Upad > kMaxConsumers) { set_err("gemv: input width above 32768 is not supported"); return false; }
    a.S = std::max(1u, kMaxConsumers / a.Upad);
    a.NC = a.S * a.Upad;
    const bool big = true;
    const uint32_t units = a.n_out / a.gran;
    const uint32_t grid = std::max(1u, std::min((uint32_t)sms, units));
    const uint32_t max_units = (units + grid - 1) / grid;
    const uint32_t max_loc = max_units * a.gran * (paired ? 2 : 1);
    if ((paired || mode == GM_QKV) && (rows_per_thread(qt, half_rows) * a.S) % 2) {  // whole pairs per stage
        if (a.S == 1) { set_err("gemv: odd stage rows for a pair mode"); return false; }
        a.S &= ~1u;
        a.NC = a.S * a.Upad;
    }
    const uint32_t R = rows_per_thread(qt, half_rows) * a.S;  // rows per round = per ring stage
    a.R = R;
    uint32_t stage;
    if (paired) {
        const uint32_t half = ((R / 2) * a.row_bytes + 32 + kStageSlack + 127) / 128 * 128;
        stage = 2 * half;
    } else {
        stage = (R * a.row_bytes + 32 + kStageSlack + 127) / 128 * 128;
    }
    a.stage_bytes = stage;
    const uint32_t n_st = (max_loc + R - 1) / R;
    a.red_bytes = red_bytes_for(a.Upad, max_loc);
    const uint32_t fixed = plane_bytes(a.K) + a.red_bytes;
    if (fixed + kHeaderBytes + 1024 + stage + 128 > kMaxSmem) {
        set_err("gemv: too many rows per CTA for the shared partial sums");
        return false;
    }
    uint32_t ns = std::max(2u, std::min((uint32_t)kMaxStages, kRingBudget > fixed ? (kRingBudget - fixed) / stage : 1u));
    ns = std::max(1u, std::min(ns, n_st));
    if (const char *e = getenv("FWB_MAX_NS")) ns = std::max(1u, std::min(ns, (uint32_t)atoi(e)));
    const uint32_t room = kMaxSmem - 1024 - fixed;  // static shared memory stays below 1 KB
    while (ns > 1 && kHeaderBytes + ns * stage + 128 > room) --ns;
    if (kHeaderBytes + ns * stage + 128 > room) { set_err("gemv: stage does not fit shared memory"); return false; }
    a.NS = ns;
    const bool a4 = (nb % 2 == 0) && ((uintptr_t)a.w % 4 == 0) && (!a.w2 || (uintptr_t)a.w2 % 4 == 0);
    L.fn = gemv_fn(qt, mode, a4, big);
    if (!L.fn) { set_err("gemv: unsupported quant type"); return false; }
    L.grid = dim3(grid);
    L.block = dim3(a.NC);
    L.smem = kHeaderBytes + fixed + (size_t)ns * stage + 128;
    L.weight_bytes = (uint64_t)a.n_out * a.row_bytes * (paired ? 2 : 1);
    return true;
}

static bool g_attr_done[64];
static bool set_smem_attrs(int dev) {
    if (dev < 0 || dev >= 64) return true;
    if (g_attr_done[dev]) return true;
    const int qts[6] = {QT_Q4_0, QT_Q5_0, QT_Q8_0, QT_Q5_1, QT_Q4_K, QT_Q6_K};
    for (int qt : qts)
        for (int mode = 0; mode <= GM_LOGITS; ++mode)
            for (int a4 = 0; a4 < 2; ++a4)
                for (int big = 0; big < 1; ++big) {
                    const void *fn = gemv_fn(qt, mode, a4, big);
                    cudaFuncAttributes fa;
                    CK(cudaFuncGetAttributes(&fa, fn));
                    const int dyn = (int)kMaxSmem - (int)fa.sharedSizeBytes;
                    CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn));
                }
    g_attr_done[dev] = true;
    return true;
}

// --------------------------------------------------------------------------
// standalone matvec (quant_matvec / quant_matvec_dev)
// --------------------------------------------------------------------------
static bool block_bytes_of(uint32_t type, uint32_t &bb) {
    switch (type) {
    case 2: bb = 18; return true;
    case 6: bb = 22; return true;
    case 7: bb = 24; return true;
    case 8: bb = 34; return true;
    case 12: bb = 144; return true;
    case 14: bb = 210; return true;
    default: return false;
    }
}

struct DevScratch {
    uint32_t *err = nullptr;
};
static DevScratch g_scratch[64];

static uint32_t *device_err_word(int dev) {
    if (dev < 0 || dev >= 64) return nullptr;
    if (!g_scratch[dev].err) {
        if (cudaMalloc(&g_scratch[dev].err, 16) != cudaSuccess) return nullptr;
        cudaMemset(g_scratch[dev].err, 0, 16);
    }
    return g_scratch[dev].err;
}

static bool matvec_args_ok(const void *w, size_t w_size, uint32_t type, const void *x, const void *y, size_t in,
                           size_t out, uint32_t &bb, uint32_t &row_bytes) {
    // quant_matvec.c:270-289
    if (!w || !x || !y || in == 0 || out == 0) { set_err("quant_matvec: null pointer or zero size"); return false; }
    if (!block_bytes_of(type, bb)) { set_err("quant_matvec: unsupported ggml type"); return false; }
    const uint32_t bv = gemv_block_values((int)type);
    if (in % bv) { set_err("quant_matvec: input_size not a multiple of the block size"); return false; }
    const uint64_t rb = (uint64_t)(in / bv) * bb;
    if (rb > UINT32_MAX || out > UINT32_MAX || out > SIZE_MAX / rb || w_size < out * rb) {
        set_err("quant_matvec: weights smaller than output_size rows");
        return false;
    }
    row_bytes = (uint32_t)rb;
    return true;
}

// Bytes from w to the 16-byte boundary at or after the end of `rows` bytes
// of rows: the GEMV's bulk copies move 16-byte aligned supersets of the
// rows, so that span must lie inside the caller's buffer.
static uint64_t span16(const void *w, uint64_t rows) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(w);
    return ((a + rows + 15) & ~uintptr_t(15)) - a;
}

static bool matvec_dev(const void *w, size_t w_size, uint32_t type, const float *x, float *y, size_t in, size_t out,
                       cudaStream_t st) {
    uint32_t bb, row_bytes;
    if (!matvec_args_ok(w, w_size, type, x, y, in, out, bb, row_bytes)) return false;
    if ((uintptr_t)w % 2) { set_err("quant_matvec_dev: weights must be 2-byte aligned"); return false; }
    if ((type == 7 && (uintptr_t)w % 4) || (type == 12 && (uintptr_t)w % 16)) {
        set_err("quant_matvec_dev: Q5_1 weights must be 4-byte and Q4_K weights 16-byte aligned");
        return false;
    }
    if ((uintptr_t)x % 16) { set_err("quant_matvec_dev: input must be 16-byte aligned"); return false; }
    if (span16(w, (uint64_t)out * row_bytes) > w_size) {
        set_err("quant_matvec_dev: weights_size must reach the 16-byte boundary after the last row (" +
                std::to_string(span16(w, (uint64_t)out * row_bytes)) + " bytes from d_weights)");
        return false;
    }
    int dev;
    CK(cudaGetDevice(&dev));
    if (!set_smem_attrs(dev)) return false;
    GemvLaunch L;
    L.a.w = static_cast<const uint8_t *>(w);
    L.a.n_out = (uint32_t)out;
    L.a.K = (uint32_t)in;
    L.a.row_bytes = row_bytes;
    L.a.x = x;
    L.a.y = y;
    L.a.err = device_err_word(dev);
    if (!L.a.err) { set_err("quant_matvec: device error word allocation failed"); return false; }
    if (!plan_gemv((int)type, GM_STORE, num_sms(dev), L)) return false;
    CK(cudaMemsetAsync(L.a.err, 0, 4, st));  // status of this launch only
    void *args[] = {&L.a};
    CK(launch_ex(L.fn, L.grid, L.block, L.smem, st, args, false));
    return true;
}

// The device error word of the current device after the work queued on `st`
// (quant_matvec_dev / quant_gemm_dev): 0 when no bounded wait ran out.
static bool device_status(cudaStream_t st, const char *who) {
    int dev;
    CK(cudaGetDevice(&dev));
    uint32_t *w = device_err_word(dev);
    if (!w) { set_err(std::string(who) + ": device error word allocation failed"); return false; }
    uint32_t e = 0;
    CK(cudaMemcpyAsync(&e, w, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (e) {
        char b[96];
        snprintf(b, sizeof b, "%s: device error word 0x%x (a bounded wait in the kernel ran out)", who, e);
        set_err(b);
        return false;
    }
    return true;
}

// --------------------------------------------------------------------------
// quant_matvec_static: quant_matvec staged through one fixed device array
// instead of per-call allocations
// --------------------------------------------------------------------------
// Layout of the array for one call (byte offsets):
//   [0, 256)       the GEMV kernel's error word (uint32 at 0).  The only part
//                  that must be zero when the kernel starts; zeroed before
//                  every launch.
//   kStaticX       input vector, fp32
//   off_w          weight rows, 256-aligned with 256 bytes of slack on both
//                  sides (the kernel's 16-byte bulk copies read up to 15
//                  bytes outside the rows)
//   off_y          output vector, fp32
constexpr size_t kStaticScratchBytes = size_t(32) << 20;
constexpr size_t kStaticX = 256;
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];
static uint8_t *g_static_base[64];  // device address of g_static_scratch, per device

static size_t round256(size_t v) { return (v + 255) & ~size_t(255); }

// Set-up on the first call per device: the array's device address.
static uint8_t *static_scratch_base(int dev) {
    if (dev < 0 || dev >= 64) { set_err("quant_matvec_static: device ordinal out of range"); return nullptr; }
    if (!g_static_base[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || !p) {
            set_err(std::string("quant_matvec_static: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
            return nullptr;
        }
        g_static_base[dev] = static_cast<uint8_t *>(p);
    }
    return g_static_base[dev];
}

static bool matvec_static(const void *weights, size_t weights_size, uint32_t type, const float *input, float *output,
                          size_t in, size_t out) {
    uint32_t bb, row_bytes;
    if (!matvec_args_ok(weights, weights_size, type, input, output, in, out, bb, row_bytes)) return false;
    const size_t wbytes = out * (size_t)row_bytes;
    const size_t off_w = round256(kStaticX + in * 4) + 256;
    const size_t off_y = round256(off_w + wbytes) + 256;
    const size_t need = off_y + round256(out * 4);
    if (need > kStaticScratchBytes) {
        set_err("quant_matvec_static: this call needs " + std::to_string(need) +
                " bytes of device scratch; the static scratch holds " + std::to_string(kStaticScratchBytes) +
                " (32 MiB): use quant_matvec for larger matrices");
        return false;
    }
    int dev;
    CK(cudaGetDevice(&dev));
    uint8_t *base = static_scratch_base(dev);
    if (!base) return false;
    if (!set_smem_attrs(dev)) return false;
    uint32_t *err = reinterpret_cast<uint32_t *>(base);
    float *dx = reinterpret_cast<float *>(base + kStaticX);
    uint8_t *dw = base + off_w;
    float *dy = reinterpret_cast<float *>(base + off_y);
    CK(cudaMemset(err, 0, 4));
    CK(cudaMemcpy(dw, weights, wbytes, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dx, input, in * 4, cudaMemcpyHostToDevice));
    GemvLaunch L;
    L.a.w = dw;
    L.a.n_out = (uint32_t)out;
    L.a.K = (uint32_t)in;
    L.a.row_bytes = row_bytes;
    L.a.x = dx;
    L.a.y = dy;
    L.a.err = err;
    if (!plan_gemv((int)type, GM_STORE, num_sms(dev), L)) return false;
    void *args[] = {&L.a};
    CK(launch_ex(L.fn, L.grid, L.block, L.smem, nullptr, args, false));
    CK(cudaMemcpy(output, dy, out * 4, cudaMemcpyDeviceToHost));
    uint32_t e = 0;
    CK(cudaMemcpy(&e, err, 4, cudaMemcpyDeviceToHost));
    if (e) {
        char b[80];
        snprintf(b, sizeof b, "quant_matvec_static: device error word 0x%x", e);
        set_err(b);
        return false;
    }
    return true;
}

// --------------------------------------------------------------------------
// model
// --------------------------------------------------------------------------
struct Mat {
    const uint8_t *p = nullptr;
    uint32_t type = 0, rows = 0, cols = 0, row_bytes = 0;
};

struct LayerW {
    Mat qkv, o, gate, up, down;
    Mat v;                // attn_v when its quant type differs from attn_q / attn_k (qkv then holds q|k)
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
};

// m->step words: [0] token, [1] position, [2] greedy token out, [kErrWord]
// the device error word
constexpr uint32_t kErrWord = 8;

struct Step {
    std::string name;
    std::function<cudaError_t(cudaStream_t, bool)> run;
    uint64_t bytes = 0;  // algorithmic HBM bytes of this launch
    Phase phase{};       // the same work as a phase of the persistent kernel
};

}  // namespace fwb

struct fwb_model {
    int dev = 0;
    int sms = 1;
    cudaStream_t st = nullptr;
    fwb::GgufFile gguf;
    fwb::ModelConfig cfg;
    uint32_t kv_ctx = 0;
    uint8_t *arena = nullptr;
    fwb::Mat embd, head;
    const float *out_norm = nullptr;
    std::vector<fwb::LayerW> layers;
    float *x = nullptr, *q = nullptr, *att = nullptr, *h = nullptr, *logits = nullptr;
    float *kc = nullptr, *vc = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    float *attn_part = nullptr, *am_val = nullptr;
    uint32_t *attn_ticket = nullptr, *am_idx = nullptr, *am_ticket = nullptr;
    uint32_t *step = nullptr, *err = nullptr, *hist = nullptr;
    uint32_t *h_io = nullptr;     // pinned [8]: step in / status out
    float *h_logits = nullptr;    // pinned [n_vocab]
    uint64_t weight_bytes = 0;
    double load_s = 0;          // time of the tensor upload at open
    uint64_t load_bytes = 0;    // bytes it moved to the device
    std::vector<fwb::Step> steps;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool use_graph = true, use_pdl = true;
    bool persistent = true;          // one persistent kernel per token (else one kernel per phase)
    unsigned long long *prof = nullptr;  // [n_phases][G][kProfSlots] GEMV profile (FWB_TRACE=1)
    fwb::DecodeArgs dargs{};
    size_t dsmem = 0;
    const void *decode_fn = nullptr;  // the persistent kernel's specialisation for this model
    bool half_rows = false;           // GEMV stages of two rows per thread (persistent ring too large otherwise)
    uint32_t *sync = nullptr;
    std::vector<void *> allocs;
    // tensor parallelism (world > 1): this rank's exchange buffer, every
    // rank's mapping of it (peer[rank] = xbuf), barrier epochs
    uint32_t rank = 0, world = 1;
    uint8_t *xbuf = nullptr;
    uint64_t xbytes = 0, x_part = 0, x_logits = 0;
    uint8_t *peer[fwb::kMaxRanks] = {};
    bool peer_mapped[fwb::kMaxRanks] = {};
    unsigned long long *gbase = nullptr;
    bool connected = false;
    unsigned long long *attn_trace = nullptr;  // FWB_TRACE: [layer][8] CTA 0's attention item timeline
    // prompt path (fwb_prefill): scratch for kPrefillChunk tokens, allocated
    // at the first call
    // fwb_sample: scratch of the device sampler, allocated at the first call
    float *smp_w = nullptr;
    uint32_t *smp_cnt = nullptr, *smp_hist = nullptr, *smp_out = nullptr, *smp_h_io = nullptr;
    size_t smp_hist_cap = 0;
    uint32_t pf_cap = 0;
    uint32_t *pf_tok = nullptr;
    float *pf_x = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_g = nullptr, *pf_u = nullptr;
    __half *pf_h16 = nullptr, *pf_a16 = nullptr;
    __half *pf_k16 = nullptr, *pf_vt16 = nullptr;  // a layer's K / transposed V in fp16 (tensor-core attention)
    // the prompt GEMMs' weights expanded to fp16 once (qkv, o, gate, up, down per layer), or empty
    std::vector<__half *> pf_w16;
    uint32_t pf_ctx_pad = 0;
};

namespace fwb {

static bool dalloc(fwb_model *m, void **p, size_t bytes) {
    CK(cudaMalloc(p, bytes));
    m->allocs.push_back(*p);
    CK(cudaMemset(*p, 0, bytes));
    return true;
}

static bool check_mat(const GgufTensor *t, uint32_t rows, uint32_t cols, const char *what, bool allow_f32 = false) {
    if (!t) { set_err(std::string("missing tensor ") + what); return false; }
    if (t->n_dims < 1 || t->dims[0] != cols || (t->n_dims >= 2 ? t->dims[1] : 1) != rows) {
        set_err(std::string("unexpected shape for ") + t->name);
        return false;
    }
    uint32_t v, b;
    if (!ggml_block(t->type, v, b) || (t->type == 0 && !allow_f32)) {
        set_err(std::string("unsupported ggml type for ") + t->name);
        return false;
    }
    return true;
}

static void free_model(fwb_model *m) {
    if (!m) return;
    if (m->st) cudaStreamSynchronize(m->st);
    for (uint32_t q = 0; q < kMaxRanks; ++q)
        if (m->peer_mapped[q]) cudaIpcCloseMemHandle(m->peer[q]);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    for (void *p : m->allocs) cudaFree(p);
    if (m->h_io) cudaFreeHost(m->h_io);
    if (m->smp_h_io) cudaFreeHost(m->smp_h_io);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    if (m->st) cudaStreamDestroy(m->st);
    delete m;
}

static bool build_steps(fwb_model *m);
static bool build_decode(fwb_model *m);

static bool load_model(fwb_model *m, const char *path, size_t max_ctx) {
    std::string err;
    if (!m->gguf.open(path, err)) { set_err("gguf_open: " + err); return false; }
    if (!m->gguf.config(m->cfg, err)) { set_err("model_config: " + err); return false; }
    const ModelConfig &c = m->cfg;
    // transformer.c:43-52
    if (!max_ctx) max_ctx = c.n_ctx < 4096 ? c.n_ctx : 4096;
    if (max_ctx > c.n_ctx) max_ctx = c.n_ctx;
    if (!max_ctx) { set_err("invalid context length"); return false; }
    m->kv_ctx = (uint32_t)max_ctx;
    if (c.n_head % c.n_head_kv) { set_err("attention: invalid head configuration"); return false; }
    const uint32_t E = c.n_embd, F = c.n_ff, hd = c.head_dim, H = c.n_head, KV = c.n_head_kv;
    if (!attn_fn(hd, H / KV)) { set_err("head_dim / GQA group outside this build"); return false; }
    if (E % 32 || F % 32 || (H * hd) != E) { set_err("model widths outside this build"); return false; }
    const uint32_t W = m->world, rk = m->rank;
    if (W > 1 && !tp_check(c, W, err)) { set_err(err); return false; }
    const uint32_t Hr = H / W, KVr = KV / W, Fr = F / W, Vr = c.n_vocab / W;

    // resolve tensors once
    const GgufTensor *te = m->gguf.find("token_embd.weight");
    if (!check_mat(te, c.n_vocab, E, "token_embd.weight", true)) return false;
    const GgufTensor *tn = m->gguf.find("output_norm.weight");
    const GgufTensor *th = m->gguf.find("output.weight");
    if (!th) th = m->gguf.find("lm_head.weight");
    if (!th) th = te;
    if (!check_mat(th, c.n_vocab, E, "output.weight")) return false;
    if (tn && (tn->type != 0 || tn->dims[0] != E)) { set_err("output_norm.weight must be F32 [n_embd]"); return false; }
    struct LT { const GgufTensor *an, *q, *k, *v, *o, *fn, *g, *u, *d; };
    std::vector<LT> lt(c.n_layer);
    for (uint32_t l = 0; l < c.n_layer; ++l) {
        auto f = [&](const char *s) { return m->gguf.find("blk." + std::to_string(l) + "." + s); };
        LT &t = lt[l];
        t = {f("attn_norm.weight"), f("attn_q.weight"), f("attn_k.weight"), f("attn_v.weight"),
             f("attn_output.weight"), f("ffn_norm.weight"), f("ffn_gate.weight"), f("ffn_up.weight"),
             f("ffn_down.weight")};
        if (!t.an || !t.fn || t.an->type != 0 || t.fn->type != 0 || t.an->dims[0] != E || t.fn->dims[0] != E) {
            set_err("missing or non-F32 norm weights at layer " + std::to_string(l));
            return false;
        }
        if (!check_mat(t.q, H * hd, E, "attn_q") || !check_mat(t.k, KV * hd, E, "attn_k") ||
            !check_mat(t.v, KV * hd, E, "attn_v") || !check_mat(t.o, E, H * hd, "attn_output") ||
            !check_mat(t.g, F, E, "ffn_gate") || !check_mat(t.u, F, E, "ffn_up") || !check_mat(t.d, E, F, "ffn_down"))
            return false;
        if (t.q->type != t.k->type || t.g->type != t.u->type) {
            set_err("q/k (and gate/up) must share a quant type");
            return false;
        }
    }

    // arena layout: every tensor 256-aligned with 256 bytes of slack; the q,
    // k, v rows of a layer are adjacent so they form one [q|k|v] matrix.
    uint64_t off = 256;
    auto place = [&](uint64_t bytes) {
        const uint64_t o = off;
        off = (off + bytes + 256 + 255) / 256 * 256;
        return o;
    };
    // (tensor parallelism: every tensor is this rank's slice, see tp_shard.h)
    struct Pl { const GgufTensor *t; uint64_t off; ShardSpec sp; uint64_t bytes; };
    std::vector<Pl> plan;
    auto spec = [&](const GgufTensor *t, bool as_head) {
        const uint32_t cols = (uint32_t)t->dims[0], rows = t->n_dims >= 2 ? (uint32_t)t->dims[1] : 1u;
        return tp_shard_spec(c, t->name, rows, cols, rk, W, as_head);
    };
    std::string shard_err;
    auto whole_blocks = [&](const GgufTensor *t, const ShardSpec &sp) {
        uint32_t v = 1, b = 4;
        ggml_block(t->type, v, b);
        if (sp.c0 % v || sp.c1 % v) shard_err = t->name + ": the rank's columns are not whole quant blocks";
    };
    auto add = [&](const GgufTensor *t, bool as_head) {
        Pl e{t, 0, spec(t, as_head), 0};
        whole_blocks(t, e.sp);
        e.bytes = tp_shard_bytes(*t, e.sp);
        e.off = place(e.bytes);
        plan.push_back(e);
        return plan.back();
    };
    const uint64_t o_embd = add(te, false).off;
    uint64_t o_head = o_embd;
    uint64_t head_bytes = te->bytes;
    if (th != te || W > 1) {
        const Pl &e = add(th, true);
        o_head = e.off;
        head_bytes = e.bytes;
    }
    uint64_t o_onorm = 0;
    if (tn) o_onorm = add(tn, false).off;
    std::vector<uint64_t> lo(c.n_layer * 8);
    for (uint32_t l = 0; l < c.n_layer; ++l) {
        LT &t = lt[l];
        Pl pq{t.q, 0, spec(t.q, false), 0}, pk{t.k, 0, spec(t.k, false), 0}, pv{t.v, 0, spec(t.v, false), 0};
        pq.bytes = tp_shard_bytes(*t.q, pq.sp);
        pk.bytes = tp_shard_bytes(*t.k, pk.sp);
        pv.bytes = tp_shard_bytes(*t.v, pv.sp);
        // q, k (and v of the same type) adjacent: one [q|k|v] matrix; a v of
        // another type (the Q4_K_M mixes) is a matrix of its own
        const bool v_split = t.v->type != t.q->type;
        const uint64_t oq = place(pq.bytes + pk.bytes + (v_split ? 0 : pv.bytes));
        pq.off = oq;
        pk.off = oq + pq.bytes;
        pv.off = v_split ? place(pv.bytes) : oq + pq.bytes + pk.bytes;
        plan.push_back(pq); plan.push_back(pk); plan.push_back(pv);
        uint64_t *L = &lo[l * 8];
        L[0] = oq;
        L[7] = v_split ? pv.off : 0;
        L[1] = add(t.o, false).off;
        L[2] = add(t.g, false).off;
        L[3] = add(t.u, false).off;
        L[4] = add(t.d, false).off;
        L[5] = add(t.an, false).off;
        L[6] = add(t.fn, false).off;
        for (size_t i = plan.size() - 9; i < plan.size(); ++i)
            if (plan[i].t != t.an && plan[i].t != t.fn) m->weight_bytes += plan[i].bytes;
        m->weight_bytes += t.an->bytes + t.fn->bytes;
    }
    if (!shard_err.empty()) { set_err("tensor parallel: " + shard_err); return false; }
    const uint64_t arena_bytes = off + 256;
    if (!dalloc(m, (void **)&m->arena, arena_bytes)) return false;

    // upload: every tensor (or this rank's slice of it) into the arena,
    // staged through pinned buffers by several host threads
    {
        Uploader up;
        bool ok = up.open(m->st);
        for (size_t i = 0; ok && i < plan.size(); ++i) {
            const Pl &e = plan[i];
            if (e.bytes == e.t->bytes) {
                const uint8_t *src = e.t->data;
                ok = up.add(m->arena + e.off, e.bytes,
                            [src](uint64_t off, uint64_t n, uint8_t *dst) { std::memcpy(dst, src + off, n); });
            } else {  // a slice: packed straight into the staging buffer
                const GgufTensor *t = e.t;
                const ShardSpec sp = e.sp;
                ok = up.add(m->arena + e.off, e.bytes, [t, sp](uint64_t off, uint64_t n, uint8_t *dst) {
                    tp_extract_range(*t, sp, off, n, dst);
                });
            }
        }
        if (ok) ok = up.finish();
        if (!ok) { set_err(up.error().empty() ? "upload failed" : up.error()); return false; }
        m->load_s = up.seconds();
        m->load_bytes = up.bytes();
    }

    auto mat = [&](const GgufTensor *t, uint64_t o, uint32_t rows, uint32_t cols) {
        Mat mm;
        mm.p = m->arena + o;
        mm.type = t->type;
        mm.rows = rows;
        mm.cols = cols;
        uint32_t v, b;
        ggml_block(t->type, v, b);
        mm.row_bytes = cols / v * b;
        return mm;
    };
    m->embd = mat(te, o_embd, c.n_vocab, E);
    m->head = mat(th, o_head, Vr, E);
    m->out_norm = tn ? reinterpret_cast<const float *>(m->arena + o_onorm) : nullptr;
    m->layers.resize(c.n_layer);
    for (uint32_t l = 0; l < c.n_layer; ++l) {
        LT &t = lt[l];
        uint64_t *L = &lo[l * 8];
        LayerW &w = m->layers[l];
        const bool v_split = t.v->type != t.q->type;
        w.qkv = mat(t.q, L[0], (Hr + (v_split ? 1 : 2) * KVr) * hd, E);
        if (v_split) w.v = mat(t.v, L[7], KVr * hd, E);
        w.o = mat(t.o, L[1], E, Hr * hd);
        w.gate = mat(t.g, L[2], Fr, E);
        w.up = mat(t.u, L[3], Fr, E);
        w.down = mat(t.d, L[4], E, Fr);
        w.attn_norm = reinterpret_cast<const float *>(m->arena + L[5]);
        w.ffn_norm = reinterpret_cast<const float *>(m->arena + L[6]);
    }
    m->weight_bytes += head_bytes + (tn ? tn->bytes : 0) + m->embd.row_bytes;

    // state
    const size_t kvn = (size_t)c.n_layer * KVr * m->kv_ctx * hd;
    if (W > 1) {
        // exchange buffer, mapped by every other rank: [0] cross-rank barrier
        // counter (u64), [256] (value, index) argmax candidate, [512] two
        // receive slots of world x n_embd tagged partial sums (8 bytes each;
        // exchanges alternate between the slots), then this rank's logits
        m->x_part = 512;
        m->x_logits = (512 + 2ull * W * E * 8 + 255) / 256 * 256;
        m->xbytes = m->x_logits + (uint64_t)Vr * 4 + 256;
        if (!dalloc(m, (void **)&m->xbuf, m->xbytes) || !dalloc(m, (void **)&m->gbase, 64)) return false;
        m->logits = reinterpret_cast<float *>(m->xbuf + m->x_logits);
    } else if (!dalloc(m, (void **)&m->logits, (size_t)c.n_vocab * 4)) {
        return false;
    }
    if (!dalloc(m, (void **)&m->x, E * 4) || !dalloc(m, (void **)&m->q, (size_t)Hr * hd * 4) ||
        !dalloc(m, (void **)&m->att, (size_t)Hr * hd * 4) || !dalloc(m, (void **)&m->h, (size_t)Fr * 4) ||
        !dalloc(m, (void **)&m->kc, kvn * 4) ||
        !dalloc(m, (void **)&m->vc, kvn * 4) ||
        !dalloc(m, (void **)&m->rope_cos, (size_t)m->kv_ctx * (hd / 2) * 4 + 4) ||
        !dalloc(m, (void **)&m->rope_sin, (size_t)m->kv_ctx * (hd / 2) * 4 + 4) ||
        !dalloc(m, (void **)&m->step, 64) || !dalloc(m, (void **)&m->sync, 64) ||
        !dalloc(m, (void **)&m->hist, (size_t)m->kv_ctx * 4 + 4) ||
        !dalloc(m, (void **)&m->am_val, 4096 * 4) || !dalloc(m, (void **)&m->am_idx, 4096 * 4) ||
        !dalloc(m, (void **)&m->am_ticket, 64) || !dalloc(m, (void **)&m->attn_ticket, 4 * KVr + 64))
        return false;
    // the device error word shares the step's allocation: set_step clears it
    // with the same copy that sets the token and position
    m->err = m->step + kErrWord;
    CK(cudaMallocHost(&m->h_io, 64));
    std::memset(m->h_io, 0, 64);
    CK(cudaMallocHost(&m->h_logits, (size_t)c.n_vocab * 4));

    // RoPE tables exactly as rope_precompute (rope.c:6-17), on the host
    {
        const size_t half = hd / 2;
        std::vector<float> cs(m->kv_ctx * half), sn(m->kv_ctx * half);
        for (size_t p = 0; p < m->kv_ctx; ++p)
            for (size_t i = 0; i < half; ++i) {
                const float theta = (float)p / powf(c.rope_freq_base, (float)(2 * i) / (float)hd);
                cs[p * half + i] = cosf(theta);
                sn[p * half + i] = sinf(theta);
            }
        CK(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    }
    return W > 1 ? true : build_steps(m);  // tensor parallel: after fwb_tp_connect
}

// Splits per KV head: one work item per CTA of the persistent kernel
// (n_kv * splits <= number of SMs), so the attention phase is one wave.
static uint32_t attn_splits(const fwb_model *m) {
    const uint32_t KV = m->cfg.n_head_kv / m->world;
    uint32_t s = std::min<uint32_t>(kMaxSplits, std::max(1u, (uint32_t)m->sms / KV));
    s = std::min(s, std::max(1u, m->kv_ctx / 16));
    return std::max(1u, s);
}

static bool build_steps(fwb_model *m) {
    const ModelConfig &c = m->cfg;
    const uint32_t E = c.n_embd, F = c.n_ff, hd = c.head_dim, H = c.n_head, KV = c.n_head_kv;
    // per rank under tensor parallelism (world 1: the whole model)
    const uint32_t W = m->world, Hr = H / W, KVr = KV / W, Fr = F / W, Vr = c.n_vocab / W;
    const size_t layer_kv = (size_t)KVr * m->kv_ctx * hd;
    uint32_t n_ar = 0;  // exchanges so far this step (their receive slots alternate)
    const uint64_t slot_bytes = (uint64_t)W * E * 8;
    // the sum of every rank's partial output into x: each row waits for the
    // ranks' tagged partials in this rank's receive slot (no barrier before it)
    auto allreduce_step = [&](const std::string &name) {
        Step s;
        s.name = name;
        s.phase.kind = PH_ALLREDUCE;
        s.phase.nobar = 1;
        s.phase.ar.x = m->x;
        s.phase.ar.n = E;
        s.phase.ar.world = W;
        s.phase.ar.in = reinterpret_cast<const unsigned long long *>(m->xbuf + m->x_part + (n_ar & 1) * slot_bytes);
        s.phase.ar.epoch = reinterpret_cast<const uint32_t *>(m->gbase + 1);
        s.phase.ar.k = n_ar;
        s.phase.ar.err = m->err;
        s.phase.ar.abort = m->sync + 1;
        s.run = [](cudaStream_t, bool) { return cudaErrorNotSupported; };
        m->steps.push_back(std::move(s));
        ++n_ar;
    };
    // GEMV arguments of a partial-output phase: rows pushed to every rank's
    // receive slot (this rank's block of it)
    auto push_args = [&]() {
        GemvArgs ex{};
        for (uint32_t q = 0; q < W; ++q)
            ex.ll_out[q] = reinterpret_cast<unsigned long long *>(m->peer[q] + m->x_part + (n_ar & 1) * slot_bytes +
                                                                  (uint64_t)m->rank * E * 8);
        ex.ll_epoch = reinterpret_cast<const uint32_t *>(m->gbase + 1);
        ex.ll_k = n_ar;
        ex.world = W;
        return ex;
    };
    m->steps.clear();
    if (const char *hr = getenv("FWB_HALF_ROWS"))  // (testing: the two-row stages on any model)
        if (*hr == '1' && m->persistent) m->half_rows = true;

    {  // embedding
        Step s;
        s.name = "embed";
        const Mat e = m->embd;
        const uint64_t rb = e.row_bytes;
        uint32_t *step = m->step;
        float *x = m->x;
        s.bytes = rb;
        s.phase.kind = PH_EMBED;
        s.phase.e = EmbedArgs{e.p, e.type, e.cols, rb, step, x};
        s.run = [=](cudaStream_t st, bool pdl) {
            const uint8_t *p = e.p;
            uint32_t t = e.type, cols = e.cols;
            uint64_t r = rb;
            const uint32_t *sp = step;
            float *xp = x;
            void *args[] = {&p, &t, &cols, &r, &sp, &xp};
            return launch_ex((const void *)embed_kernel, dim3(std::min(16u, (cols + 255) / 256)), dim3(256), 0,
                             st, args, pdl);
        };
        m->steps.push_back(std::move(s));
    }

    auto gemv_step = [&](const std::string &name, int mode, const Mat &w, const Mat *w2, uint32_t n_out,
                         const float *x, const float *norm_w, float *y, GemvArgs extra) -> bool {
        GemvLaunch L;
        L.a = extra;
        L.a.w = w.p;
        L.a.w2 = w2 ? w2->p : nullptr;
        L.a.n_out = n_out;
        L.a.K = w.cols;
        L.a.row_bytes = w.row_bytes;
        L.a.x = x;
        L.a.norm_w = norm_w;
        L.a.eps = c.norm_eps;
        L.a.y = y;
        L.a.step = m->step;
        L.a.err = m->err;
        if (!plan_gemv((int)w.type, mode, m->sms, L, m->half_rows)) return false;
        if (!norm_w) L.a.norm = 0u;  // LM head of a model without output_norm
        Step s;
        s.name = name;
        s.bytes = L.weight_bytes;
        s.phase.kind = PH_GEMV;
        s.phase.qt = w.type;
        s.phase.mode = (uint32_t)mode;
        s.phase.a4 = (w.cols / 32) % 2 == 0 && (uintptr_t)w.p % 4 == 0 && (!w2 || (uintptr_t)w2->p % 4 == 0);
        s.phase.g = L.a;
        s.run = [L](cudaStream_t st, bool pdl) {
            GemvArgs a = L.a;
            void *args[] = {&a};
            return launch_ex(L.fn, L.grid, L.block, L.smem, st, args, pdl);
        };
        m->steps.push_back(std::move(s));
        return true;
    };

    const char *trc = getenv("FWB_TRACE");
    if (trc && *trc == '1' && !m->attn_trace && !dalloc(m, (void **)&m->attn_trace, (size_t)c.n_layer * m->sms * 8 * 8))
        return false;
    const uint32_t nsplit = attn_splits(m);
    if (!dalloc(m, (void **)&m->attn_part, (size_t)KVr * nsplit * (H / KV) * (hd + 2) * 4)) return false;
    const void *afn = attn_fn(hd, H / KV);

    for (uint32_t l = 0; l < c.n_layer; ++l) {
        const LayerW &w = m->layers[l];
        float *kc = m->kc + l * layer_kv, *vc = m->vc + l * layer_kv;
        GemvArgs ex{};
        ex.n_q = Hr * hd;
        ex.n_kv = KVr * hd;
        ex.head_dim = hd;
        ex.kv_ctx = m->kv_ctx;
        ex.rope_cos = m->rope_cos;
        ex.rope_sin = m->rope_sin;
        ex.q_out = m->q;
        ex.kcache = kc;
        ex.vcache = vc;
        const std::string p = "L" + std::to_string(l) + ".";
        if (!gemv_step(p + "qkv_rope", GM_QKV, w.qkv, nullptr, w.qkv.rows, m->x, w.attn_norm, nullptr, ex))
            return false;
        if (w.v.p) {  // v rows of their own type: every row of this GEMV is a v row
            GemvArgs ev = ex;
            ev.n_q = 0;
            ev.n_kv = 0;
            if (!gemv_step(p + "v", GM_QKV, w.v, nullptr, w.v.rows, m->x, w.attn_norm, nullptr, ev)) return false;
            m->steps.back().phase.nobar = 1;  // independent of the q|k phase: no barrier between them
        }
        {
            Step s;
            s.name = p + "attention";
            AttnArgs a{};
            a.q = m->q;
            a.kc = kc;
            a.vc = vc;
            a.out = m->att;
            a.part = m->attn_part;
            a.ticket = m->attn_ticket;
            a.kv_ctx = m->kv_ctx;
            a.n_split = nsplit;
            a.scale = 1.0f / sqrtf((float)hd);
            a.step = m->step;
            if (m->attn_trace) a.trace = m->attn_trace + (size_t)l * m->sms * 8;
            a.err = m->err;
            s.bytes = 0;  // KV bytes depend on pos; accounted separately
            a.n_kv = KVr;
            s.phase.kind = PH_ATTN;
            s.phase.hd = hd;
            s.phase.gq = H / KV;
            s.phase.at = a;
            // the persistent kernel runs one (KV head, split) item per CTA
            s.phase.at.n_split = std::max(1u, std::min(nsplit, (uint32_t)m->sms / KVr));
            s.run = [a, afn, KVr, nsplit](cudaStream_t st, bool pdl) {
                AttnArgs aa = a;
                void *args[] = {&aa};
                return launch_ex(afn, dim3(KVr, nsplit), dim3(kAttnWarps * 32), 0, st, args, pdl);
            };
            m->steps.push_back(std::move(s));
        }
        if (W == 1) {
            if (!gemv_step(p + "o_proj_resid", GM_RESID, w.o, nullptr, E, m->att, nullptr, m->x, GemvArgs{}))
                return false;
        } else {  // this rank's heads' share of o-proj, then the all-reduce into x
            if (!gemv_step(p + "o_proj_part", GM_PUSH, w.o, nullptr, E, m->att, nullptr, nullptr, push_args()))
                return false;
            allreduce_step(p + "o_proj_allreduce");
        }
        if (!gemv_step(p + "gate_up_swiglu", GM_SWIGLU, w.gate, &w.up, Fr, m->x, w.ffn_norm, m->h, GemvArgs{}))
            return false;
        if (W == 1) {
            if (!gemv_step(p + "down_resid", GM_RESID, w.down, nullptr, E, m->h, nullptr, m->x, GemvArgs{}))
                return false;
        } else {
            if (!gemv_step(p + "down_part", GM_PUSH, w.down, nullptr, E, m->h, nullptr, nullptr, push_args()))
                return false;
            allreduce_step(p + "down_allreduce");
        }
    }
    {
        GemvArgs ex{};
        ex.am_val = m->am_val;
        ex.am_idx = m->am_idx;
        ex.ticket = m->am_ticket;
        ex.out_token = m->step + 2;
        ex.step_rw = m->step;
        ex.hist = m->hist;
        ex.idx_base = m->rank * Vr;
        if (W > 1) ex.tp_cand = reinterpret_cast<float *>(m->xbuf + 256);
        if (!gemv_step("lm_head_argmax", GM_LOGITS, m->head, nullptr, Vr, m->x, m->out_norm, m->logits, ex))
            return false;
    }
    if (W > 1) {  // the greedy token from every rank's candidate
        Step s;
        s.name = "tp_argmax";
        s.phase.kind = PH_TPARGMAX;
        s.phase.gsync = 1;
        s.phase.am.world = W;
        for (uint32_t q = 0; q < W; ++q) s.phase.am.cand[q] = reinterpret_cast<const float *>(m->peer[q] + 256);
        s.phase.am.out_token = m->step + 2;
        s.phase.am.step_rw = m->step;
        s.phase.am.hist = m->hist;
        s.run = [](cudaStream_t, bool) { return cudaErrorNotSupported; };
        m->steps.push_back(std::move(s));
    }
    // (a model without output_norm feeds x to the head unnormalised, as
    // transformer.c:304-306 copies it: the head GEMV then runs without the
    // RMSNorm prologue)
    if (!m->persistent) return true;
    if (build_decode(m)) return true;
    // a ring of four-row stages that does not fit next to the attention
    // scratch and the stream tables (the 70B shapes): plan the GEMVs again
    // with two rows per thread per round
    if (m->half_rows || g_err.find("shared memory too small") == std::string::npos) return false;
    m->half_rows = true;
    g_err.clear();
    return build_steps(m);
}

// Bytes of the attention scratch of the persistent kernel (16 warps).
template <int HD>
static uint32_t attn_smem_bytes_hd(uint32_t gq) {
    constexpr int NW = kDecodeThreads / 32;
    switch (gq) {
    case 1: return sizeof(AttnSmem<HD, 1, NW>);
    case 2: return sizeof(AttnSmem<HD, 2, NW>);
    case 4: return sizeof(AttnSmem<HD, 4, NW>);
    default: return sizeof(AttnSmem<HD, 8, NW>);
    }
}
static uint32_t attn_smem_bytes(uint32_t hd, uint32_t gq) {
    switch (hd) {
    case 32: return attn_smem_bytes_hd<32>(gq);
    case 48: return attn_smem_bytes_hd<48>(gq);
    case 64: return attn_smem_bytes_hd<64>(gq);
    default: return attn_smem_bytes_hd<128>(gq);
    }
}

// Phases of the persistent kernel: the Step list's work, with one ring
// geometry for all GEMV phases and per-CTA weight-stream tables.
static bool build_decode(fwb_model *m) {
    const uint32_t G = (uint32_t)m->sms;
    std::vector<Phase> ph;
    for (const Step &s : m->steps) ph.push_back(s.phase);
    const uint32_t n_ph = (uint32_t)ph.size();
    uint32_t stage = 0, scratch = 0;
    for (const Phase &p : ph) {
        if (p.kind == PH_GEMV) {
            stage = std::max(stage, p.g.stage_bytes);
            scratch = std::max(scratch, plane_bytes(p.g.K) + p.g.red_bytes);
        }
    }
    {  // attention scratch of the persistent kernel (16 warps)
        const uint32_t hd = m->cfg.head_dim, gq = m->cfg.n_head / m->cfg.n_head_kv;
        const uint32_t nw = kDecodeThreads / 32;
        // the layout itself, and a formula check that every member is covered
        const uint32_t att = std::max<uint32_t>(attn_smem_bytes(hd, gq),
                                                (nw * 32 + 3 * nw * gq + nw * gq * hd + gq + gq * kMaxSplits + gq + 1) * 4);
        scratch = std::max(scratch, (att + 127) / 128 * 128);
    }
    // the specialisation of the persistent kernel for this model's phases
    {
        bool q4a4 = true;
        for (const Phase &p : ph)
            if (p.kind == PH_GEMV && (p.qt != QT_Q4_0 || !p.a4)) q4a4 = false;
        const uint32_t hd = m->cfg.head_dim, gq = m->cfg.n_head / m->cfg.n_head_kv;
        const char *gen = getenv("FWB_GENERIC_KERNEL");
        const bool generic = gen && *gen == '1';
        if (!m->half_rows) {
            m->decode_fn = (const void *)decode_kernel_t<0, 0, 0, false>;
            if (!generic && q4a4 && hd == 128 && gq == 4) m->decode_fn = (const void *)decode_kernel_t<1, 128, 4, false>;
            if (!generic && q4a4 && hd == 128 && gq == 8) m->decode_fn = (const void *)decode_kernel_t<1, 128, 8, false>;
        } else {
            m->decode_fn = (const void *)decode_kernel_t<0, 0, 0, true>;
            if (!generic && q4a4 && hd == 128 && gq == 8) m->decode_fn = (const void *)decode_kernel_t<1, 128, 8, true>;
        }
    }
    cudaFuncAttributes fa;
    CK(cudaFuncGetAttributes(&fa, m->decode_fn));
    const size_t tab_bytes = (size_t)n_ph * sizeof(StageSrc);
    const size_t fixed = kHeaderBytes + scratch + 128 + tab_bytes + fa.sharedSizeBytes + 1024;
    if (fixed + 2 * (size_t)stage > kMaxSmem) { set_err("persistent kernel: shared memory too small"); return false; }
    uint32_t ns = (uint32_t)std::min<size_t>(kMaxStages, (kMaxSmem - fixed) / stage);
    if (const char *e = getenv("FWB_MAX_NS")) ns = std::max(2u, std::min(ns, (uint32_t)atoi(e)));
    const char *trc = getenv("FWB_TRACE");
    const bool tracing = trc && *trc == '1';
    if (tracing && !dalloc(m, (void **)&m->prof, (size_t)n_ph * G * kProfSlots * 8)) return false;
    for (uint32_t i = 0; i < n_ph; ++i) {
        Phase &p = ph[i];
        if (p.kind == PH_GEMV) {
            p.g.NS = ns;
            p.g.stage_bytes = stage;
            p.g.prof = tracing ? m->prof + (size_t)i * G * kProfSlots : nullptr;
        }
    }
    // per-CTA stream tables
    std::vector<StageSrc> tab((size_t)G * n_ph);
    std::vector<uint32_t> nst(G, 0);
    for (uint32_t c = 0; c < G; ++c) {
        uint32_t first = 0;
        for (uint32_t p = 0; p < n_ph; ++p) {
            StageSrc &t = tab[(size_t)c * n_ph + p];
            t = StageSrc{};
            t.first = first;
            if (ph[p].kind != PH_GEMV) continue;
            const GemvArgs &g = ph[p].g;
            const uint32_t n = g.n_out / g.gran;
            const uint32_t b = (uint32_t)((uint64_t)c * n / G) * g.gran, e = (uint32_t)((uint64_t)(c + 1) * n / G) * g.gran;
            const bool paired = ph[p].mode == GM_SWIGLU;
            t.a = (uint64_t)(uintptr_t)g.w + (uint64_t)b * g.row_bytes;
            t.b = paired ? (uint64_t)(uintptr_t)g.w2 + (uint64_t)b * g.row_bytes : 0;
            t.rows = e - b;
            t.row_bytes = g.row_bytes;
            t.R = g.R;
            t.paired = paired;
            const uint32_t n_loc = paired ? 2 * (e - b) : (e - b);
            t.n_st = (n_loc + g.R - 1) / g.R;
            first += t.n_st;
        }
        nst[c] = first;
    }
    Phase *d_ph;
    StageSrc *d_tab;
    uint32_t *d_nst;
    if (!dalloc(m, (void **)&d_ph, ph.size() * sizeof(Phase)) || !dalloc(m, (void **)&d_tab, tab.size() * sizeof(StageSrc)) ||
        !dalloc(m, (void **)&d_nst, G * 4))
        return false;
    CK(cudaMemcpy(d_ph, ph.data(), ph.size() * sizeof(Phase), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_tab, tab.data(), tab.size() * sizeof(StageSrc), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_nst, nst.data(), G * 4, cudaMemcpyHostToDevice));
    DecodeArgs &d = m->dargs;
    d.ph = d_ph;
    d.src = d_tab;
    d.n_ph = n_ph;
    d.total_st = *std::max_element(nst.begin(), nst.end());
    d.NS = ns;
    d.stage_bytes = stage;
    d.scratch_bytes = scratch;
    d.step = m->step;
    d.sync = m->sync;
    d.err = m->err;
    d.n_st_cta = d_nst;
    d.world = m->world;
    d.gbase = m->gbase;
    d.xepoch = m->gbase ? reinterpret_cast<uint32_t *>(m->gbase + 1) : nullptr;
    d.n_gsync = 0;
    d.n_exchange = 0;
    for (const Phase &p : ph) {
        d.n_gsync += p.gsync;
        d.n_exchange += p.kind == PH_ALLREDUCE ? 1u : 0u;
    }
    if (m->world > 1) {  // [0] is this rank's own counter
        d.gcount[0] = reinterpret_cast<unsigned long long *>(m->xbuf);
        for (uint32_t q = 0, k = 1; q < m->world; ++q)
            if (q != m->rank) d.gcount[k++] = reinterpret_cast<unsigned long long *>(m->peer[q]);
    }
    const char *tr = getenv("FWB_TRACE");
    if (tr && *tr == '1') {
        if (!dalloc(m, (void **)&d.trace, (2 * n_ph + 1) * 8) ||
            !dalloc(m, (void **)&d.trace_cta, (size_t)n_ph * G * 8))
            return false;
    }
    m->dsmem = kHeaderBytes + scratch + (size_t)ns * stage + 128 + tab_bytes;
    CK(cudaFuncSetAttribute(m->decode_fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->dsmem));
    int per_sm = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, m->decode_fn, kDecodeThreads, m->dsmem));
    if (per_sm < 1) { set_err("persistent kernel does not fit on an SM"); return false; }
    return true;
}

static cudaError_t launch_decode(fwb_model *m) {
    cudaError_t e = cudaMemsetAsync(m->sync, 0, 16, m->st);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m->sms);
    cfg.blockDim = dim3(kDecodeThreads);
    cfg.dynamicSmemBytes = m->dsmem;
    cfg.stream = m->st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    DecodeArgs d = m->dargs;
    void *args[] = {&d};
    return cudaLaunchKernelExC(&cfg, m->decode_fn, args);
}

static bool run_steps(fwb_model *m) {
    if (m->persistent) {
        cudaError_t e = launch_decode(m);
        if (e != cudaSuccess) { set_err(std::string("persistent decode launch: ") + cudaGetErrorString(e)); return false; }
        return true;
    }
    for (size_t i = 0; i < m->steps.size(); ++i) {
        cudaError_t e = m->steps[i].run(m->st, m->use_pdl && i > 0);
        if (e != cudaSuccess) {
            set_err("launch " + m->steps[i].name + ": " + cudaGetErrorString(e));
            return false;
        }
    }
    return true;
}

static bool capture_graph(fwb_model *m) {
    CK(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    bool ok = run_steps(m);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(m->st, &g);
    if (!ok || e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        if (ok) set_err(std::string("graph capture: ") + cudaGetErrorString(e));
        return false;
    }
    m->graph = g;
    CK(cudaGraphInstantiate(&m->exec, g, 0));
    return true;
}

static bool enqueue_step(fwb_model *m) {
    if (m->use_graph && m->exec) {
        CK(cudaGraphLaunch(m->exec, m->st));
        return true;
    }
    return run_steps(m);
}

static bool finish(fwb_model *m) {
    CK(cudaMemcpyAsync(m->h_io + 4, m->err, 4, cudaMemcpyDeviceToHost, m->st));
    CK(cudaMemcpyAsync(m->h_io + 5, m->step + 2, 4, cudaMemcpyDeviceToHost, m->st));
    CK(cudaStreamSynchronize(m->st));
    if (m->h_io[4]) {
        char b[96];
        snprintf(b, sizeof b, "device error word 0x%x", m->h_io[4]);
        set_err(b);
        return false;
    }
    return true;
}

// Token and position of the next step.  On one GPU the same copy zeroes
// the device error word (step[kErrWord]), so each call reports only its own
// launches; under tensor parallelism the word stays set once a wait ran out
// (the ranks' cross-rank barrier counts no longer agree: reopen the model).
static bool set_step(fwb_model *m, uint32_t tok, size_t pos) {
    if (m->world > 1 && !m->connected) { set_err("tensor parallel model: call fwb_tp_connect first"); return false; }
    if (pos >= m->kv_ctx) { set_err("transformer_forward: position exceeds KV cache"); return false; }
    if (tok >= m->cfg.n_vocab) { set_err("transformer_forward: token ID out of range"); return false; }
    for (uint32_t i = 2; i <= kErrWord; ++i) m->h_io[i] = 0;
    m->h_io[0] = tok;
    m->h_io[1] = (uint32_t)pos;
    const size_t n = m->world > 1 ? 8 : 4 * (kErrWord + 1);
    CK(cudaMemcpyAsync(m->step, m->h_io, n, cudaMemcpyHostToDevice, m->st));
    return true;
}

}  // namespace fwb

// ==========================================================================
// C ABI
// ==========================================================================
using namespace fwb;

extern "C" {

const char *fwb_last_error(void) { return g_err.c_str(); }

int fwb_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

int quant_matvec(const void *weights, size_t weights_size, uint32_t ggml_type, const float *input, float *output,
                 size_t input_size, size_t output_size) {
    uint32_t bb, row_bytes;
    if (!matvec_args_ok(weights, weights_size, ggml_type, input, output, input_size, output_size, bb, row_bytes))
        return -1;
    const size_t wbytes = (size_t)output_size * row_bytes;
    void *dw = nullptr;
    float *dx = nullptr, *dy = nullptr;
    int rc = -1;
    if (cudaMalloc(&dw, wbytes + 64) == cudaSuccess && cudaMalloc(&dx, input_size * 4) == cudaSuccess &&
        cudaMalloc(&dy, output_size * 4) == cudaSuccess &&
        cudaMemcpy(dw, weights, wbytes, cudaMemcpyHostToDevice) == cudaSuccess &&
        cudaMemcpy(dx, input, input_size * 4, cudaMemcpyHostToDevice) == cudaSuccess) {
        if (matvec_dev(dw, wbytes + 64, ggml_type, dx, dy, input_size, output_size, nullptr) &&
            cudaMemcpy(output, dy, output_size * 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
            device_status(nullptr, "quant_matvec"))
            rc = 0;
        else if (g_err.empty())
            set_err("quant_matvec: device execution failed");
    } else {
        set_err("quant_matvec: device allocation or copy failed");
    }
    if (dw) cudaFree(dw);
    if (dx) cudaFree(dx);
    if (dy) cudaFree(dy);
    return rc;
}

int quant_matvec_static(const void *weights, size_t weights_size, uint32_t ggml_type, const float *input,
                        float *output, size_t input_size, size_t output_size) {
    return matvec_static(weights, weights_size, ggml_type, input, output, input_size, output_size) ? 0 : -1;
}

int quant_matvec_dev(const void *d_weights, size_t weights_size, uint32_t ggml_type, const float *d_input,
                     float *d_output, size_t input_size, size_t output_size, void *stream) {
    return matvec_dev(d_weights, weights_size, ggml_type, d_input, d_output, input_size, output_size,
                      static_cast<cudaStream_t>(stream))
               ? 0
               : -1;
}

int quant_device_status(void *stream) {
    return device_status(static_cast<cudaStream_t>(stream), "quant_device_status") ? 0 : -1;
}

// cuTensorMapEncodeTiled from the driver (through the runtime's entry-point
// query, so the library does not link libcuda itself).
static decltype(&cuTensorMapEncodeTiled) tensor_map_encoder() {
    static decltype(&cuTensorMapEncodeTiled) fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<decltype(&cuTensorMapEncodeTiled)>(p);
    }
    return fn;
}

// Tensor-core dequant-GEMM launch (gemm_tc.cuh): Y[m][0..N) (row stride ldy)
// = W X[m] for m < M, or += with TC_ADD.  Q4_0 with K a multiple of 64,
// 4-byte-aligned weights and 16-byte-aligned fp16 activations only.
static bool launch_tc_gemm(const void *w, size_t w_bytes, uint32_t type, const void *x, float *y, size_t K, size_t N,
                           size_t M, size_t ldy, uint32_t mode, cudaStream_t st, uint32_t *err,
                           const __half *w16 = nullptr) {
    static bool attr_set[64] = {};
    if (!w || !x || !y || !K || !N || !M) { set_err("quant_gemm: null pointer or zero size"); return false; }
    if (type != 2) { set_err("quant_gemm: only Q4_0 (type 2) runs on the tensor cores"); return false; }
    if (K % kTcK) { set_err("quant_gemm: input size must be a multiple of 64"); return false; }
    const size_t row_bytes = K / 32 * 18;
    if (w_bytes < N * row_bytes) { set_err("quant_gemm: weights_size too small"); return false; }
    if ((uintptr_t)w % 4 || (uintptr_t)x % 16 || ldy < N) { set_err("quant_gemm: misaligned operands"); return false; }
    if (M > 65535u * kTcM || N > 0xffffffffu / 2) { set_err("quant_gemm: too many rows"); return false; }
    int dev = 0;
    CK(cudaGetDevice(&dev));
    if (dev < 64 && !attr_set[dev]) {
        CK(cudaFuncSetAttribute((const void *)gemm_q4_0_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kTcSmem));
        CK(cudaFuncSetAttribute((const void *)gemm_q4_0_tc_kernel<false>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem));
        CK(cudaFuncSetAttribute((const void *)gemm_q4_0_tc_kernel<false, true>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem));
        attr_set[dev] = true;
    }
    TcArgs a{};
    {  // the activations [M][K] fp16 as a 2-D map: 64 x 128 boxes, 128-byte swizzle, zeros past M
        const auto enc = tensor_map_encoder();
        if (!enc) { set_err("quant_gemm: cuTensorMapEncodeTiled unavailable"); return false; }
        const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
        const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
        const cuuint32_t box[2] = {kTcK, kTcM}, estr[2] = {1, 1};
        const CUresult r = enc(&a.xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(x), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) { set_err("quant_gemm: activation tensor map rejected"); return false; }
        if (w16) {  // the fp16 copy of the weights [N][K], the same boxes
            const cuuint64_t wdims[2] = {(cuuint64_t)K, (cuuint64_t)N};
            const CUresult rw = enc(&a.wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(w16), wdims,
                                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (rw != CUDA_SUCCESS) { set_err("quant_gemm: weight tensor map rejected"); return false; }
        }
    }
    a.w = static_cast<const uint8_t *>(w);
    a.row_bytes = (uint32_t)row_bytes;
    a.x = static_cast<const __half *>(x);
    a.y = y;
    a.M = (uint32_t)M;
    a.N = (uint32_t)N;
    a.K = (uint32_t)K;
    a.ldy = (uint32_t)ldy;
    a.mode = mode;
    a.err = err;
    const dim3 grid((unsigned)((N + kTcN - 1) / kTcN), (unsigned)((M + kTcM - 1) / kTcM));
    if (w16)
        gemm_q4_0_tc_kernel<false, true><<<grid, kTcThreads, kTcSmem, st>>>(a);
    else if (row_bytes % 16 == 0 && (uintptr_t)w % 16 == 0)  // 16-byte weight loads
        gemm_q4_0_tc_kernel<true><<<grid, kTcThreads, kTcSmem, st>>>(a);
    else
        gemm_q4_0_tc_kernel<false><<<grid, kTcThreads, kTcSmem, st>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_err(std::string("quant_gemm launch: ") + cudaGetErrorString(e)); return false; }
    return true;
}

int quant_gemm_dev(const void *d_weights, size_t weights_size, uint32_t ggml_type, const void *d_input_f16,
                   float *d_output, size_t input_size, size_t output_size, size_t n_tokens, int accumulate,
                   void *stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { set_err("quant_gemm_dev: no device"); return -1; }
    uint32_t *err = device_err_word(dev);
    if (!err) { set_err("quant_gemm_dev: device error word"); return -1; }
    if (cudaMemsetAsync(err, 0, 4, static_cast<cudaStream_t>(stream)) != cudaSuccess) {  // this launch only
        set_err("quant_gemm_dev: error word reset failed");
        return -1;
    }
    if (!launch_tc_gemm(d_weights, weights_size, ggml_type, d_input_f16, d_output, input_size, output_size, n_tokens,
                        output_size, accumulate ? TC_ADD : TC_STORE, static_cast<cudaStream_t>(stream), err))
        return -1;
    return 0;
}

int quant_dequant_dev(const void *d_weights, size_t weights_size, uint32_t ggml_type, float *d_out, size_t n_values,
                      void *stream) {
    uint32_t bb;
    if (!d_weights || !d_out || !n_values || !block_bytes_of(ggml_type, bb) ||
        n_values % gemv_block_values((int)ggml_type) ||
        weights_size < n_values / gemv_block_values((int)ggml_type) * bb) {
        set_err("quant_dequant_dev: bad arguments");
        return -1;
    }
    const uint64_t n = n_values;
    const uint32_t grid = (uint32_t)std::min<uint64_t>(4096, (n + 255) / 256);
    dequant_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint8_t *>(d_weights),
                                                                         ggml_type, bb, d_out, n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_err(std::string("dequant launch: ") + cudaGetErrorString(e)); return -1; }
    return 0;
}

static fwb_model *open_model(const char *path, size_t max_ctx, int device, int rank, int world) {
    g_err.clear();
    if (!path) { set_err("null path"); return nullptr; }
    if (world < 1 || world > (int)kMaxRanks || rank < 0 || rank >= world) {
        set_err("tensor parallel: rank / world out of range (1 to 8 ranks)");
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) { set_err("cudaSetDevice failed"); return nullptr; }
    fwb_model *m = new fwb_model();
    m->dev = device;
    m->sms = num_sms(device);
    m->rank = (uint32_t)rank;
    m->world = (uint32_t)world;
    const char *ng = getenv("FWB_NO_GRAPH");
    const char *np = getenv("FWB_NO_PDL");
    m->use_graph = !(ng && *ng == '1');
    m->use_pdl = !(np && *np == '1');
    const char *mk = getenv("FWB_KERNEL_PER_PHASE");
    m->persistent = !(mk && *mk == '1');
    bool ok = cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) == cudaSuccess && set_smem_attrs(device);
    if (ok && world > 1 && !m->persistent) {
        set_err("tensor parallelism runs in the persistent decode kernel only (unset FWB_KERNEL_PER_PHASE)");
        ok = false;
    }
    // tensor parallel: the step is built once the peers are mapped (fwb_tp_connect)
    ok = ok && load_model(m, path, max_ctx) && (world > 1 || !m->use_graph || capture_graph(m));
    if (!ok) {
        std::string e = g_err;
        free_model(m);
        set_err(e.empty() ? "model load failed" : e);
        return nullptr;
    }
    return m;
}

fwb_model_t *fwb_model_open(const char *path, size_t max_ctx, int device) {
    return open_model(path, max_ctx, device, 0, 1);
}

fwb_model_t *fwb_model_open_tp(const char *path, size_t max_ctx, int device, int rank, int world) {
    return open_model(path, max_ctx, device, rank, world);
}

int fwb_tp_handle(fwb_model_t *m, void *handle) {
    if (!m || !handle || m->world < 2) { set_err("fwb_tp_handle: not a tensor parallel model"); return -1; }
    cudaSetDevice(m->dev);
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, m->xbuf) != cudaSuccess) { set_err("cudaIpcGetMemHandle failed"); return -1; }
    static_assert(sizeof(h) == 64, "IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    return 0;
}

int fwb_tp_connect(fwb_model_t *m, const void *handles) {
    if (!m || !handles || m->world < 2) { set_err("fwb_tp_connect: not a tensor parallel model"); return -1; }
    if (m->connected) { set_err("fwb_tp_connect: already connected"); return -1; }
    cudaSetDevice(m->dev);
    const uint8_t *hb = static_cast<const uint8_t *>(handles);
    for (uint32_t q = 0; q < m->world; ++q) {
        if (q == m->rank) { m->peer[q] = m->xbuf; continue; }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + 64 * q, 64);
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            set_err(std::string("cudaIpcOpenMemHandle (rank ") + std::to_string(q) + "): " + cudaGetErrorString(e));
            return -1;
        }
        m->peer[q] = static_cast<uint8_t *>(p);
        m->peer_mapped[q] = true;
    }
    if (!build_steps(m) || (m->use_graph && !capture_graph(m))) return -1;
    m->connected = true;
    return 0;
}

int fwb_tp_shard(const char *path, const char *tensor, int as_head, int rank, int world, void *out, size_t cap,
                 size_t *out_bytes) {
    if (!path || !tensor || world < 1 || world > (int)kMaxRanks || rank < 0 || rank >= world) {
        set_err("fwb_tp_shard: bad arguments");
        return -1;
    }
    GgufFile f;
    ModelConfig c;
    std::string err;
    if (!f.open(path, err) || !f.config(c, err) || !tp_check(c, (uint32_t)world, err)) { set_err(err); return -1; }
    const GgufTensor *t = f.find(tensor);
    if (!t) { set_err(std::string("fwb_tp_shard: no tensor ") + tensor); return -1; }
    const uint32_t cols = (uint32_t)t->dims[0], rows = t->n_dims >= 2 ? (uint32_t)t->dims[1] : 1u;
    const ShardSpec sp = tp_shard_spec(c, t->name, rows, cols, (uint32_t)rank, (uint32_t)world, as_head != 0);
    const uint64_t n = tp_shard_bytes(*t, sp);
    if (out_bytes) *out_bytes = n;
    if (!out) return 0;
    if (cap < n) { set_err("fwb_tp_shard: buffer too small"); return -1; }
    tp_extract(*t, sp, static_cast<uint8_t *>(out));
    return 0;
}

void fwb_model_close(fwb_model_t *m) {
    if (!m) return;
    cudaSetDevice(m->dev);
    free_model(m);
}

int fwb_model_dims(const fwb_model_t *m, uint32_t *d) {
    if (!m || !d) return -1;
    const ModelConfig &c = m->cfg;
    d[0] = c.n_vocab; d[1] = m->kv_ctx; d[2] = c.n_embd; d[3] = c.n_layer;
    d[4] = c.n_head; d[5] = c.n_head_kv; d[6] = c.n_ff; d[7] = c.head_dim;
    return 0;
}

uint64_t fwb_model_weight_bytes(const fwb_model_t *m) { return m ? m->weight_bytes : 0; }

int fwb_model_load_stats(const fwb_model_t *m, double *seconds, uint64_t *bytes) {
    if (!m) return -1;
    if (seconds) *seconds = m->load_s;
    if (bytes) *bytes = m->load_bytes;
    return 0;
}

int fwb_model_kernels_per_step(const fwb_model_t *m) {
    if (!m) return -1;
    return m->persistent ? 1 : (int)m->steps.size();
}

// The tensor-core prompt path needs every linear weight of the layers in
// Q4_0 with a multiple of 64 inputs, head_dim <= 128 (a multiple of 4), one
// GPU.  Other models take the per-token decode path for the prompt.
static bool prefill_eligible(const fwb_model *m) {
    const ModelConfig &c = m->cfg;
    if (m->world != 1 || c.head_dim > 128 || c.head_dim % 4 || c.n_head % c.n_head_kv) return false;
    if (c.n_embd > (uint32_t)kPfNormVec * 4 * 256) return false;  // the RMSNorm kernel's register row
    for (const LayerW &w : m->layers)
        if (w.v.p) return false;  // a v matrix of another type than q / k
    for (const LayerW &w : m->layers)
        for (const Mat *t : {&w.qkv, &w.o, &w.gate, &w.up, &w.down})
            if (t->type != 2 || t->cols % kTcK || (uintptr_t)t->p % 4) return false;
    return true;
}

constexpr uint32_t kPrefillChunk = 512;  // prompt tokens per pass through the layers

static bool prefill_alloc(fwb_model *m) {
    if (m->pf_cap) return true;
    const ModelConfig &c = m->cfg;
    const size_t C = kPrefillChunk, E = c.n_embd, F = c.n_ff, NQ = (size_t)c.n_head * c.head_dim;
    const size_t NQKV = NQ + 2 * (size_t)c.n_head_kv * c.head_dim;
    const size_t W16 = std::max({E, F, NQ});
    if (!dalloc(m, (void **)&m->pf_tok, C * 4) || !dalloc(m, (void **)&m->pf_x, C * E * 4) ||
        !dalloc(m, (void **)&m->pf_qkv, C * NQKV * 4) || !dalloc(m, (void **)&m->pf_q, C * NQ * 4) ||
        !dalloc(m, (void **)&m->pf_g, C * F * 4) || !dalloc(m, (void **)&m->pf_u, C * F * 4) ||
        !dalloc(m, (void **)&m->pf_h16, C * W16 * 2) || !dalloc(m, (void **)&m->pf_a16, C * NQ * 2))
        return false;
    {  // fp16 copies of the layer weights for the prompt GEMMs, if they fit with room to spare
        size_t need = 0;
        for (const LayerW &w : m->layers)
            for (const Mat *t : {&w.qkv, &w.o, &w.gate, &w.up, &w.down}) need += (size_t)t->rows * t->cols * 2;
        size_t free_b = 0, total_b = 0;
        if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess && free_b > need + ((size_t)8 << 30)) {
            for (const LayerW &w : m->layers)
                for (const Mat *t : {&w.qkv, &w.o, &w.gate, &w.up, &w.down}) {
                    __half *p16 = nullptr;
                    if (!dalloc(m, (void **)&p16, (size_t)t->rows * t->cols * 2)) return false;
                    const uint64_t nb = (uint64_t)t->rows * t->cols / 32;
                    q4_0_to_f16_kernel<<<(unsigned)std::min<uint64_t>(4096, (nb + 255) / 256), 256, 0, m->st>>>(
                        t->p, nb, p16);
                    m->pf_w16.push_back(p16);
                }
            CK(cudaGetLastError());
        }
    }
    if (c.head_dim == kAtHd) {
        m->pf_ctx_pad = (m->kv_ctx + 63) / 64 * 64;
        const size_t n16 = (size_t)c.n_head_kv * m->pf_ctx_pad * kAtHd;
        if (!dalloc(m, (void **)&m->pf_k16, n16 * 2) || !dalloc(m, (void **)&m->pf_vt16, n16 * 2)) return false;
    }
    m->pf_cap = (uint32_t)C;
    return true;
}

// Prompt attention: the tiled flash kernel for head_dim 64 / 128 and groups
// of 1, 2, 4 or 8 query heads; otherwise all query heads of a KV head per
// block when their scores fit in shared memory, else one block per query head.
static bool launch_pf_flash(fwb_model *m, const void *fn, uint32_t smem, uint32_t gq, const float *kc,
                            const float *vc, uint32_t T, uint32_t p0, float scale, cudaStream_t st) {
    CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const uint32_t H = m->cfg.n_head, QT = kPfRows / gq, nqt = (T + QT - 1) / QT;
    void *args[] = {(void *)&m->pf_q, (void *)&kc, (void *)&vc, (void *)&T, (void *)&p0,
                    (void *)&H, (void *)&m->kv_ctx, (void *)&scale, (void *)&m->pf_a16};
    CK(cudaLaunchKernel(fn, dim3((nqt + 1) / 2, m->cfg.n_head_kv), dim3(kPfThreads), args, smem, st));
    return true;
}

static bool launch_pf_attn(fwb_model *m, const float *kc, const float *vc, uint32_t T, uint32_t p0,
                           size_t att_smem, cudaStream_t st) {
    const ModelConfig &c = m->cfg;
    const uint32_t H = c.n_head, KV = c.n_head_kv, hd = c.head_dim, gq = H / KV;
    const float scale = 1.0f / sqrtf((float)hd);
    if (hd == kAtHd && (gq == 1 || gq == 2 || gq == 4 || gq == 8) && m->pf_k16) {  // tensor cores
        const uint32_t n_pos = p0 + T;
        pf_kv16_kernel<<<dim3((n_pos + 63) / 64, KV), 256, 0, st>>>(kc, vc, n_pos, m->kv_ctx, m->pf_ctx_pad,
                                                                   m->pf_k16, m->pf_vt16);
        const void *fn = gq == 1 ? (const void *)pf_attn_tc_kernel<1>
                       : gq == 2 ? (const void *)pf_attn_tc_kernel<2>
                       : gq == 4 ? (const void *)pf_attn_tc_kernel<4> : (const void *)pf_attn_tc_kernel<8>;
        CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAtSmem));
        const uint32_t QT = kAtRows / gq, nqt = (T + QT - 1) / QT;
        const __half *k16 = m->pf_k16, *vt16 = m->pf_vt16;
        void *args[] = {(void *)&m->pf_q, (void *)&k16, (void *)&vt16, (void *)&T, (void *)&p0, (void *)&H,
                        (void *)&m->pf_ctx_pad, (void *)&scale, (void *)&m->pf_a16, (void *)&m->err};
        CK(cudaLaunchKernel(fn, dim3(nqt, KV), dim3(kAtThreads), args, kAtSmem, st));
        return true;
    }
    if (hd == 128 || hd == 64) {
        switch (gq * 1000 + hd) {
        case 1128: return launch_pf_flash(m, (const void *)pf_flash_kernel<128, 1>, pf_flash_smem<128>(), 1, kc, vc, T, p0, scale, st);
        case 2128: return launch_pf_flash(m, (const void *)pf_flash_kernel<128, 2>, pf_flash_smem<128>(), 2, kc, vc, T, p0, scale, st);
        case 4128: return launch_pf_flash(m, (const void *)pf_flash_kernel<128, 4>, pf_flash_smem<128>(), 4, kc, vc, T, p0, scale, st);
        case 8128: return launch_pf_flash(m, (const void *)pf_flash_kernel<128, 8>, pf_flash_smem<128>(), 8, kc, vc, T, p0, scale, st);
        case 1064: return launch_pf_flash(m, (const void *)pf_flash_kernel<64, 1>, pf_flash_smem<64>(), 1, kc, vc, T, p0, scale, st);
        case 2064: return launch_pf_flash(m, (const void *)pf_flash_kernel<64, 2>, pf_flash_smem<64>(), 2, kc, vc, T, p0, scale, st);
        case 4064: return launch_pf_flash(m, (const void *)pf_flash_kernel<64, 4>, pf_flash_smem<64>(), 4, kc, vc, T, p0, scale, st);
        case 8064: return launch_pf_flash(m, (const void *)pf_flash_kernel<64, 8>, pf_flash_smem<64>(), 8, kc, vc, T, p0, scale, st);
        default: break;
        }
    }
    const size_t smem_g = att_smem * gq;
    auto run = [&](const void *fn) -> bool {
        if (smem_g > 48 * 1024)
            CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_g));
        void *args[] = {(void *)&m->pf_q, (void *)&kc, (void *)&vc, (void *)&p0, (void *)&H,
                        (void *)&hd, (void *)&m->kv_ctx, (void *)&scale, (void *)&m->pf_a16};
        CK(cudaLaunchKernel(fn, dim3(T, KV), dim3(128), args, smem_g, st));
        return true;
    };
    if (smem_g <= 200 * 1024) {
        switch (gq) {
        case 1: return run((const void *)pf_attn_gqa_kernel<1>);
        case 2: return run((const void *)pf_attn_gqa_kernel<2>);
        case 4: return run((const void *)pf_attn_gqa_kernel<4>);
        case 8: return run((const void *)pf_attn_gqa_kernel<8>);
        default: break;
        }
    }
    pf_attn_kernel<<<dim3(T, H), 128, att_smem, st>>>(m->pf_q, kc, vc, p0, H, gq, hd, m->kv_ctx, scale, m->pf_a16);
    return true;
}

// T prompt tokens (host array) at positions p0..p0+T-1 through every layer:
// fills the KV cache; the residual stream after the last layer is not needed.
static bool prefill_chunk(fwb_model *m, const uint32_t *tokens, uint32_t T, uint32_t p0) {
    const ModelConfig &c = m->cfg;
    const uint32_t E = c.n_embd, F = c.n_ff, hd = c.head_dim, H = c.n_head, KV = c.n_head_kv;
    const uint32_t NQ = H * hd, NKV = KV * hd, NQKV = NQ + 2 * NKV;
    const size_t layer_kv = (size_t)KV * m->kv_ctx * hd;
    cudaStream_t st = m->st;
    CK(cudaMemcpyAsync(m->pf_tok, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, st));
    pf_embed_kernel<<<T, 256, 0, st>>>(m->embd.p, m->embd.type, E, m->embd.row_bytes, m->pf_tok, m->pf_x);
    const size_t att_smem = (size_t)(p0 + T) * 4;
    if (att_smem > 48 * 1024)
        CK(cudaFuncSetAttribute((const void *)pf_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)std::min<size_t>(att_smem, 200 * 1024)));
    if (att_smem > 200 * 1024) { set_err("prefill: context too long for the attention scratch"); return false; }
    for (uint32_t l = 0; l < c.n_layer; ++l) {
        const LayerW &w = m->layers[l];
        float *kc = m->kc + l * layer_kv, *vc = m->vc + l * layer_kv;
        // the layer's fp16 weight copies (qkv, o, gate, up, down), when the model has them
        auto w16 = [&](int i) -> const __half * { return m->pf_w16.empty() ? nullptr : m->pf_w16[5 * l + i]; };
        pf_rmsnorm_f16_kernel<<<T, 256, 0, st>>>(m->pf_x, w.attn_norm, c.norm_eps, E, m->pf_h16);
        if (!launch_tc_gemm(w.qkv.p, (size_t)w.qkv.rows * w.qkv.row_bytes, 2, m->pf_h16, m->pf_qkv, E, NQKV, T, NQKV,
                            TC_STORE, st, m->err, w16(0)))
            return false;
        pf_rope_kv_kernel<<<T, 256, 0, st>>>(m->pf_qkv, p0, NQ, NKV, hd, m->rope_cos, m->rope_sin, m->pf_q, kc, vc,
                                             m->kv_ctx);
        if (!launch_pf_attn(m, kc, vc, T, p0, att_smem, st)) return false;
        if (l + 1 == c.n_layer) break;  // the last layer's output feeds only the logits
        if (!launch_tc_gemm(w.o.p, (size_t)w.o.rows * w.o.row_bytes, 2, m->pf_a16, m->pf_x, NQ, E, T, E, TC_ADD, st,
                            m->err, w16(1)))
            return false;
        pf_rmsnorm_f16_kernel<<<T, 256, 0, st>>>(m->pf_x, w.ffn_norm, c.norm_eps, E, m->pf_h16);
        if (!launch_tc_gemm(w.gate.p, (size_t)w.gate.rows * w.gate.row_bytes, 2, m->pf_h16, m->pf_g, E, F, T, F,
                            TC_STORE, st, m->err, w16(2)) ||
            !launch_tc_gemm(w.up.p, (size_t)w.up.rows * w.up.row_bytes, 2, m->pf_h16, m->pf_u, E, F, T, F, TC_STORE,
                            st, m->err, w16(3)))
            return false;
        pf_swiglu_kernel<<<std::min<size_t>(4 * 148, ((size_t)T * F / 4 + 255) / 256), 256, 0, st>>>(
            m->pf_g, m->pf_u, (size_t)T * F, m->pf_h16);
        if (!launch_tc_gemm(w.down.p, (size_t)w.down.rows * w.down.row_bytes, 2, m->pf_h16, m->pf_x, F, E, T, E,
                            TC_ADD, st, m->err, w16(4)))
            return false;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_err(std::string("prefill launch: ") + cudaGetErrorString(e)); return false; }
    return true;
}

int fwb_forward(fwb_model_t *m, uint32_t token, size_t pos, float *logits_host);

int fwb_prefill(fwb_model_t *m, const uint32_t *tokens, size_t n, size_t pos0, float *logits_host) {
    if (!m || !tokens || n == 0) { set_err("fwb_prefill: null model or tokens, or no tokens"); return -1; }
    if (pos0 + n > m->kv_ctx) { set_err("fwb_prefill: positions exceed the KV cache"); return -1; }
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] >= m->cfg.n_vocab) { set_err("fwb_prefill: token ID out of range"); return -1; }
    cudaSetDevice(m->dev);
    const char *env = getenv("FWB_PREFILL_PER_TOKEN");
    const bool batched = n > 1 && prefill_eligible(m) && !(env && *env == '1');
    if (!batched) {  // the decode path, one token after the other (as main.c does)
        for (size_t i = 0; i + 1 < n; ++i)
            if (fwb_forward(m, tokens[i], pos0 + i, nullptr) != 0) return -1;
    } else {
        if (!prefill_alloc(m)) return -1;
        if (cudaMemsetAsync(m->err, 0, 4, m->st) != cudaSuccess) { set_err("prefill: error word reset"); return -1; }
        for (size_t i = 0; i + 1 < n; i += kPrefillChunk) {
            const uint32_t T = (uint32_t)std::min<size_t>(kPrefillChunk, n - 1 - i);
            if (!prefill_chunk(m, tokens + i, T, (uint32_t)(pos0 + i))) return -1;
        }
        if (!finish(m)) return -1;  // a GEMM's bounded wait that ran out
    }
    // the last token through the decode step gives the logits
    return fwb_forward(m, tokens[n - 1], pos0 + n - 1, logits_host);
}

int fwb_forward(fwb_model_t *m, uint32_t token, size_t pos, float *logits_host) {
    if (!m) return -1;
    cudaSetDevice(m->dev);
    if (!set_step(m, token, pos) || !enqueue_step(m)) return -1;
    float *dst = logits_host ? logits_host : nullptr;
    if (dst && m->world > 1) {
        // every rank's slice: this rank's own and the peers' (mapped), after the
        // step; the step's closing cross-rank barrier has seen every head phase
        if (!finish(m)) return -1;
        const size_t vr = m->cfg.n_vocab / m->world;
        for (uint32_t q = 0; q < m->world; ++q)
            if (cudaMemcpy(dst + q * vr, m->peer[q] + m->x_logits, vr * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
                set_err("logits gather failed");
                return -1;
            }
        return 0;
    }
    if (dst) {
        cudaPointerAttributes pa;
        const bool pinned = cudaPointerGetAttributes(&pa, dst) == cudaSuccess && pa.type == cudaMemoryTypeHost;
        float *target = pinned ? dst : m->h_logits;
        if (cudaMemcpyAsync(target, m->logits, (size_t)m->cfg.n_vocab * 4, cudaMemcpyDeviceToHost, m->st) !=
            cudaSuccess) {
            set_err("logits copy failed");
            return -1;
        }
        if (!finish(m)) return -1;
        if (!pinned) std::memcpy(dst, m->h_logits, (size_t)m->cfg.n_vocab * 4);
        return 0;
    }
    return finish(m) ? 0 : -1;
}

int fwb_forward_argmax(fwb_model_t *m, uint32_t token, size_t pos, uint32_t *next_token) {
    if (!m) return -1;
    cudaSetDevice(m->dev);
    if (!set_step(m, token, pos) || !enqueue_step(m) || !finish(m)) return -1;
    if (next_token) *next_token = m->h_io[5];
    return 0;
}

int fwb_generate_greedy(fwb_model_t *m, uint32_t first, size_t pos0, size_t n, uint32_t *out) {
    if (!m) return -1;
    cudaSetDevice(m->dev);
    if (n == 0) return 0;
    if (pos0 + n > m->kv_ctx) { set_err("generate: positions exceed KV cache"); return -1; }
    if (!set_step(m, first, pos0)) return -1;
    for (size_t i = 0; i < n; ++i)
        if (!enqueue_step(m)) return -1;
    if (out && cudaMemcpyAsync(out, m->hist + pos0, n * 4, cudaMemcpyDeviceToHost, m->st) != cudaSuccess) {
        set_err("token copy failed");
        return -1;
    }
    return finish(m) ? 0 : -1;
}

static int kv_copy(fwb_model_t *m, size_t layer, size_t pos0, size_t n, float *k, float *v, bool load) {
    if (!m || !k || !v) return -1;
    cudaSetDevice(m->dev);
    const ModelConfig &c = m->cfg;
    if (layer >= c.n_layer || pos0 > m->kv_ctx || n > m->kv_ctx - pos0) { set_err("kv: range"); return -1; }
    if (n == 0) return 0;
    // the host arrays hold every KV head; this rank's cache holds KV/world of them
    const size_t hd = c.head_dim, KV = c.n_head_kv, KVr = KV / m->world, h0 = (size_t)m->rank * KVr;
    const size_t base = layer * KVr * m->kv_ctx * hd;
    for (size_t h = 0; h < KVr; ++h) {
        float *dk = m->kc + base + (h * m->kv_ctx + pos0) * hd;
        float *dv = m->vc + base + (h * m->kv_ctx + pos0) * hd;
        const size_t hh = h0 + h;
        cudaError_t e1, e2;
        if (load) {
            e1 = cudaMemcpy2DAsync(dk, hd * 4, k + hh * hd, KV * hd * 4, hd * 4, n, cudaMemcpyHostToDevice, m->st);
            e2 = cudaMemcpy2DAsync(dv, hd * 4, v + hh * hd, KV * hd * 4, hd * 4, n, cudaMemcpyHostToDevice, m->st);
        } else {
            e1 = cudaMemcpy2DAsync(k + hh * hd, KV * hd * 4, dk, hd * 4, hd * 4, n, cudaMemcpyDeviceToHost, m->st);
            e2 = cudaMemcpy2DAsync(v + hh * hd, KV * hd * 4, dv, hd * 4, hd * 4, n, cudaMemcpyDeviceToHost, m->st);
        }
        if (e1 != cudaSuccess || e2 != cudaSuccess) { set_err("kv copy failed"); return -1; }
    }
    if (cudaStreamSynchronize(m->st) != cudaSuccess) { set_err("kv copy failed"); return -1; }
    return 0;
}

int fwb_kv_load(fwb_model_t *m, size_t layer, size_t pos0, size_t n, const float *k, const float *v) {
    return kv_copy(m, layer, pos0, n, const_cast<float *>(k), const_cast<float *>(v), true);
}

int fwb_kv_read(fwb_model_t *m, size_t layer, size_t pos0, size_t n, float *k, float *v) {
    return kv_copy(m, layer, pos0, n, k, v, false);
}

const float *fwb_logits_dev(fwb_model_t *m) { return m ? m->logits : nullptr; }

int fwb_prof_read(fwb_model_t *m, uint64_t *out, size_t n) {
    if (!m || !m->prof) { set_err("profiling is off (set FWB_TRACE=1 before opening)"); return -1; }
    const size_t cnt = (size_t)m->dargs.n_ph * m->sms * kProfSlots;
    if (n < cnt) { set_err("profile buffer too small"); return -1; }
    cudaSetDevice(m->dev);
    if (cudaMemcpy(out, m->prof, cnt * 8, cudaMemcpyDeviceToHost) != cudaSuccess) { set_err("profile copy"); return -1; }
    cudaMemset(m->prof, 0, cnt * 8);
    return (int)cnt;
}

int fwb_trace_read(fwb_model_t *m, uint64_t *out, size_t n, char *names, size_t name_stride) {
    if (!m || !m->persistent || !m->dargs.trace) { set_err("tracing is off (set FWB_TRACE=1 before opening)"); return -1; }
    const size_t np = 2 * (size_t)m->dargs.n_ph + 1;
    if (n < np) { set_err("trace buffer too small"); return -1; }
    cudaSetDevice(m->dev);
    if (cudaMemcpy(out, m->dargs.trace, np * 8, cudaMemcpyDeviceToHost) != cudaSuccess) { set_err("trace copy"); return -1; }
    if (names)
        for (size_t i = 0; i < m->steps.size(); ++i)
            snprintf(names + i * name_stride, name_stride, "%s", m->steps[i].name.c_str());
    return (int)np;
}
int fwb_trace_cta_read(fwb_model_t *m, uint64_t *out, size_t n) {
    if (!m || !m->persistent || !m->dargs.trace_cta) { set_err("tracing is off (set FWB_TRACE=1 before opening)"); return -1; }
    const size_t cnt = (size_t)m->dargs.n_ph * m->sms;
    if (n < cnt) { set_err("trace buffer too small"); return -1; }
    cudaSetDevice(m->dev);
    if (cudaMemcpy(out, m->dargs.trace_cta, cnt * 8, cudaMemcpyDeviceToHost) != cudaSuccess) { set_err("trace copy"); return -1; }
    return (int)cnt;
}

int fwb_trace_attn_read(fwb_model_t *m, uint64_t *out, size_t n) {
    if (!m || !m->attn_trace) { set_err("tracing is off (set FWB_TRACE=1 before opening)"); return -1; }
    const size_t cnt = (size_t)m->cfg.n_layer * m->sms * 8;
    if (n < cnt) { set_err("trace buffer too small"); return -1; }
    cudaSetDevice(m->dev);
    if (cudaMemcpy(out, m->attn_trace, cnt * 8, cudaMemcpyDeviceToHost) != cudaSuccess) { set_err("trace copy"); return -1; }
    // CTAs without an item in the next step stay 0
    if (cudaMemset(m->attn_trace, 0, cnt * 8) != cudaSuccess) { set_err("trace reset failed"); return -1; }
    return (int)cnt;
}

void *fwb_stream(fwb_model_t *m) { return m ? (void *)m->st : nullptr; }

// xorshift64 of sampler.c:8-10 and the uniform draw of sampler.c:93
static float sample_uniform(uint64_t *s) {
    uint64_t x = *s;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *s = x;
    return (float)(x >> 11) / (float)(UINT64_MAX >> 11);
}

int fwb_sample(fwb_model_t *m, const uint32_t *history, size_t n_history, float temperature, float top_p,
               float rep_penalty, uint64_t *rng_state, uint32_t *next_token) {
    if (!m || !next_token || (n_history && !history) || (temperature > 0.0f && !rng_state)) {
        set_err("fwb_sample: null argument");
        return -1;
    }
    if (m->world > 1 && !m->connected) { set_err("fwb_sample: tensor parallel model not connected"); return -1; }
    cudaSetDevice(m->dev);
    const uint32_t n = m->cfg.n_vocab;
    static bool attr_set[64] = {};
    if (m->dev < 64 && !attr_set[m->dev]) {
        if (cudaFuncSetAttribute((const void *)sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSampleDynSmem) != cudaSuccess) {
            set_err("fwb_sample: shared memory attribute");
            return -1;
        }
        attr_set[m->dev] = true;
    }
    if (!m->smp_w) {
        if (!dalloc(m, (void **)&m->smp_w, (size_t)n * 4) || !dalloc(m, (void **)&m->smp_cnt, (size_t)n * 4) ||
            !dalloc(m, (void **)&m->smp_out, 64))
            return -1;
        if (cudaMallocHost(&m->smp_h_io, 64) != cudaSuccess) { set_err("fwb_sample: pinned buffer"); return -1; }
    }
    if (n_history > m->smp_hist_cap) {
        const size_t cap = std::max<size_t>(n_history, 2 * (size_t)m->kv_ctx);
        if (!dalloc(m, (void **)&m->smp_hist, cap * 4)) return -1;
        m->smp_hist_cap = cap;
    }
    SampleArgs a{};
    a.n = n;
    a.world = m->world;
    a.slice = n / m->world;
    if (m->world == 1) a.lg[0] = m->logits;
    else
        for (uint32_t q = 0; q < m->world; ++q) a.lg[q] = reinterpret_cast<const float *>(m->peer[q] + m->x_logits);
    a.w = m->smp_w;
    a.cnt = m->smp_cnt;
    a.hist = m->smp_hist;
    a.n_hist = (uint32_t)n_history;
    a.temp = temperature;
    a.top_p = top_p;
    a.pen = rep_penalty;
    a.u = temperature > 0.0f ? sample_uniform(rng_state) : 0.0f;
    a.out = m->smp_out;
    if (n_history && cudaMemcpyAsync(m->smp_hist, history, n_history * 4, cudaMemcpyHostToDevice, m->st) != cudaSuccess) {
        set_err("fwb_sample: history copy failed");
        return -1;
    }
    sample_kernel<<<1, kSampleThreads, kSampleDynSmem, m->st>>>(a);
    if (cudaGetLastError() != cudaSuccess ||
        cudaMemcpyAsync(m->smp_h_io, m->smp_out, 4, cudaMemcpyDeviceToHost, m->st) != cudaSuccess ||
        cudaStreamSynchronize(m->st) != cudaSuccess) {
        set_err("fwb_sample: kernel failed");
        return -1;
    }
    *next_token = m->smp_h_io[0];
    return 0;
}

void *fwb_host_alloc(size_t bytes) {
    void *p = nullptr;
    if (!bytes || cudaMallocHost(&p, bytes) != cudaSuccess) {
        set_err("fwb_host_alloc: page-locked allocation failed");
        return nullptr;
    }
    return p;
}

void fwb_host_free(void *p) {
    if (p) cudaFreeHost(p);
}

}  // extern "C"
