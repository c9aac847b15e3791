/*
 * fwd_oracle.c — CPU restatement of forword.c's per-token decode forward.
 *
 * TEST INFRASTRUCTURE ONLY (see fwd_oracle.h).  Single-threaded, plain C11.
 *
 * Scope: the llama family as model_config.c:150-159 configures it (RMSNorm,
 * gated SiLU FFN, adjacent-pair RoPE, no biases, embedding scale 1), with
 * F32 / Q4_0 / Q5_0 / Q8_0 tensors.  GGML Q4_0 is an addition: the reference
 * has no decoder for it (quant_matvec.c:52-62, linear.c:127-147); it is
 * restated from GGML's published block definition and pinned against the
 * gguf-py implementation by tests/golden.
 */
#define _POSIX_C_SOURCE 200809L
#include "fwd_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

enum { T_F32 = 0, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8 };

/* ------------------------------------------------------------------------ */
/* numerics                                                                 */
/* ------------------------------------------------------------------------ */

/* fp16 -> fp32, subnormal-correct; quant.c:22-55 / quant_matvec.c:18-46. */
float orc_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = -14;
            while ((mant & 0x400u) == 0) { mant <<= 1; --e; }
            mant &= 0x3ffu;
            bits = sign | ((uint32_t)(e + 127) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Horizontal sum of one 8-lane register as simd.h:60-65 performs it. */
static float hsum8(const float *v)
{
    float s0 = v[0] + v[4], s1 = v[1] + v[5], s2 = v[2] + v[6], s3 = v[3] + v[7];
    return (s0 + s2) + (s1 + s3);
}

/* simd_dot_f32, AVX2+FMA build (simd.h:27-66): two 8-lane FMA accumulators
 * over 16-element steps, folded, then 8-element FMA steps, the horizontal
 * tree, and a scalar (uncontracted) tail. */
float orc_dot(const float *a, const float *b, size_t n)
{
    size_t i = 0;
    float sum = 0.0f;
    float acc0[8] = {0}, acc1[8] = {0};
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 8; l++) {
            acc0[l] = fmaf(a[i + l], b[i + l], acc0[l]);
            acc1[l] = fmaf(a[i + 8 + l], b[i + 8 + l], acc1[l]);
        }
    for (int l = 0; l < 8; l++) acc0[l] = acc0[l] + acc1[l];
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) acc0[l] = fmaf(a[i + l], b[i + l], acc0[l]);
    sum += hsum8(acc0);
    for (; i < n; i++) {
        float p = a[i] * b[i];
        sum += p;
    }
    return sum;
}

/* simd_axpy_f32, AVX2+FMA build (simd.h:262-307): out += a*s. */
static void orc_axpy(float *out, const float *a, float s, size_t n)
{
    size_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) out[i + l] = fmaf(a[i + l], s, out[i + l]);
    for (; i < n; i++) {
        float p = a[i] * s;
        out[i] += p;
    }
}

/* rms_norm, norm.c:7-16: ss = dot(x,x); scale = 1/sqrtf(ss/n + eps);
 * out = (x*w)*scale. */
void orc_rms_norm(const float *x, const float *w, float *out, size_t n, float eps)
{
    float ss = orc_dot(x, x, n);
    float scale = 1.0f / sqrtf((ss / (float)n) + eps);
    for (size_t i = 0; i < n; i++) {
        float t = w ? x[i] * w[i] : x[i];
        out[i] = t * scale;
    }
}

/* rope_precompute, rope.c:6-17 (theta in fp32 via powf, then cosf/sinf). */
void orc_rope_tables(float *cos_tab, float *sin_tab, size_t n_ctx,
                     size_t head_dim, float freq_base)
{
    size_t half = head_dim / 2;
    for (size_t pos = 0; pos < n_ctx; pos++)
        for (size_t i = 0; i < half; i++) {
            float theta = (float)pos / powf(freq_base, (float)(2 * i) / (float)head_dim);
            cos_tab[pos * half + i] = cosf(theta);
            sin_tab[pos * half + i] = sinf(theta);
        }
}

/* rope_apply, normal (adjacent-pair) variant, rope.c:28-45. */
void orc_rope_apply(float *qk, size_t pos, size_t n_heads, size_t head_dim,
                    const float *cos_tab, const float *sin_tab)
{
    size_t half = head_dim / 2;
    const float *c = cos_tab + pos * half;
    const float *s = sin_tab + pos * half;
    for (size_t h = 0; h < n_heads; h++) {
        float *v = qk + h * head_dim;
        for (size_t i = 0; i < half; i++) {
            float v0 = v[2 * i], v1 = v[2 * i + 1];
            float a = v0 * c[i], b = v1 * s[i];
            float e = v0 * s[i], f = v1 * c[i];
            v[2 * i] = a - b;
            v[2 * i + 1] = e + f;
        }
    }
}

/* sampler_argmax, sampler.c:28-32: strict '>' keeps the lowest index. */
uint32_t orc_argmax(const float *x, size_t n)
{
    size_t best = 0;
    for (size_t i = 1; i < n; i++)
        if (x[i] > x[best]) best = i;
    return (uint32_t)best;
}

/* softmax, attention.c:18-33. */
static void orc_softmax(float *x, size_t n)
{
    if (n == 0) return;
    float mx = x[0];
    for (size_t i = 1; i < n; i++)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    if (sum <= 0.0f || !isfinite(sum)) return;
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; i++) x[i] *= inv;
}

/* apply_silu, ffn.c:17-25 (two-sided stable sigmoid). */
static void orc_silu(float *x, size_t n)
{
    for (size_t i = 0; i < n; i++) {
        float v = x[i];
        float sig = v >= 0.0f ? 1.0f / (1.0f + expf(-v)) : expf(v) / (1.0f + expf(v));
        x[i] = v * sig;
    }
}

/* ------------------------------------------------------------------------ */
/* block quants                                                              */
/* ------------------------------------------------------------------------ */

static int block_layout(uint32_t type, size_t *bytes)
{
    switch (type) {
    case T_Q4_0: *bytes = 18; return 0;
    case T_Q5_0: *bytes = 22; return 0;
    case T_Q8_0: *bytes = 34; return 0;
    default: return -1;
    }
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* One 32-value block -> floats.
 * Q8_0: q8_0_decode, quant.c:232-263 (d * (float)q).
 * Q5_0: q5_0_decode, linear.c:40-56 (d * (float)(q - 16), q = nibble | hbit<<4).
 * Q4_0: GGML layout, d * (float)(nibble - 8); element j = low nibble of quant
 *       byte j, element j+16 = high nibble. */
static void decode_block(const uint8_t *p, uint32_t type, float *out)
{
    float d = orc_f16_to_f32(rd16(p));
    if (type == T_Q8_0) {
        const int8_t *qs = (const int8_t *)(p + 2);
        for (int j = 0; j < 32; j++) out[j] = d * (float)qs[j];
    } else if (type == T_Q5_0) {
        const uint8_t *qh = p + 2, *qs = p + 6;
        for (int j = 0; j < 16; j++) {
            int h0 = (qh[j / 8] >> (j % 8)) & 1;
            int h1 = (qh[(j + 16) / 8] >> ((j + 16) % 8)) & 1;
            int q0 = (qs[j] & 15) | (h0 << 4);
            int q1 = (qs[j] >> 4) | (h1 << 4);
            out[j] = d * (float)(q0 - 16);
            out[j + 16] = d * (float)(q1 - 16);
        }
    } else { /* Q4_0 */
        const uint8_t *qs = p + 2;
        for (int j = 0; j < 16; j++) {
            out[j] = d * (float)((qs[j] & 15) - 8);
            out[j + 16] = d * (float)((qs[j] >> 4) - 8);
        }
    }
}

/* dot_q8_0_block, AVX2+FMA build (quant_matvec.c:65-114): four 8-lane
 * products, ((a0+a1)+(a2+a3)), horizontal tree, times d. */
static float dot_q8_0_block(const uint8_t *p, const float *x)
{
    float d = orc_f16_to_f32(rd16(p));
    const int8_t *qs = (const int8_t *)(p + 2);
    float acc[8];
    for (int l = 0; l < 8; l++) {
        float a0 = fmaf((float)qs[l], x[l], 0.0f);
        float a1 = fmaf((float)qs[8 + l], x[8 + l], 0.0f);
        float a2 = fmaf((float)qs[16 + l], x[16 + l], 0.0f);
        float a3 = fmaf((float)qs[24 + l], x[24 + l], 0.0f);
        acc[l] = (a0 + a1) + (a2 + a3);
    }
    return d * hsum8(acc);
}

/* quant_matvec, quant_matvec.c:263-312: per row, sum the per-block partials in
 * block order.  Q8_0 uses the factored block dot; Q5_0 (and Q4_0, following
 * the same pattern) decode the block and call simd_dot_f32 (:243-247). */
int orc_quant_matvec(const void *w, size_t w_size, uint32_t type,
                     const float *x, float *y, size_t in, size_t out)
{
    size_t bb;
    if (!w || !x || !y || in == 0 || out == 0 || block_layout(type, &bb) != 0 ||
        in % 32 != 0)
        return -1;
    size_t bpr = in / 32;
    if (bpr > SIZE_MAX / bb) return -1;
    size_t row_bytes = bpr * bb;
    if (out > SIZE_MAX / row_bytes || w_size < out * row_bytes) return -1;
    const uint8_t *raw = (const uint8_t *)w;
    float dec[32];
    for (size_t r = 0; r < out; r++) {
        float sum = 0.0f;
        const uint8_t *row = raw + r * row_bytes;
        for (size_t b = 0; b < bpr; b++) {
            float partial;
            if (type == T_Q8_0) {
                partial = dot_q8_0_block(row + b * bb, x + b * 32);
            } else {
                decode_block(row + b * bb, type, dec);
                partial = orc_dot(dec, x + b * 32, 32);
            }
            sum += partial;
        }
        y[r] = sum;
    }
    return 0;
}

int orc_dequant(const void *w, size_t w_size, uint32_t type, float *out,
                size_t n_values)
{
    size_t bb;
    if (!w || !out || block_layout(type, &bb) != 0 || n_values % 32 != 0 ||
        w_size < (n_values / 32) * bb)
        return -1;
    const uint8_t *raw = (const uint8_t *)w;
    for (size_t b = 0; b < n_values / 32; b++) decode_block(raw + b * bb, type, out + b * 32);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* minimal GGUF v2/v3 reader (gguf.c:256-353 semantics for what we need)     */
/* ------------------------------------------------------------------------ */

typedef struct {
    char name[96];
    uint32_t n_dims, type;
    uint64_t dims[4], offset, bytes;
    const uint8_t *data;
} orc_tensor_t;

typedef struct {
    const uint8_t *p, *end;
    int err;
} rd_t;

static uint64_t rd_u(rd_t *r, size_t n)
{
    uint64_t v = 0;
    if ((size_t)(r->end - r->p) < n) { r->err = 1; return 0; }
    memcpy(&v, r->p, n);
    r->p += n;
    return v;
}

static const char *rd_str(rd_t *r, uint64_t *len)
{
    *len = rd_u(r, 8);
    if (r->err || *len > (uint64_t)(r->end - r->p)) { r->err = 1; return NULL; }
    const char *s = (const char *)r->p;
    r->p += *len;
    return s;
}

static size_t scalar_size(uint32_t t)
{
    switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
    }
}

static void skip_val(rd_t *r, uint32_t t, int depth)
{
    if (depth > 8) { r->err = 1; return; }
    if (t == 8) { uint64_t l; rd_str(r, &l); return; }
    if (t == 9) {
        uint32_t et = (uint32_t)rd_u(r, 4);
        uint64_t n = rd_u(r, 8);
        size_t es = scalar_size(et);
        if (es && !r->err) {
            if (n > (uint64_t)(r->end - r->p) / es) { r->err = 1; return; }
            r->p += n * es;
            return;
        }
        for (uint64_t i = 0; i < n && !r->err; i++) skip_val(r, et, depth + 1);
        return;
    }
    size_t s = scalar_size(t);
    if (!s) { r->err = 1; return; }
    rd_u(r, s);
}

struct orc_model {
    int fd;
    void *map;
    size_t map_size;
    orc_tensor_t *tensors;
    size_t n_tensors;
    /* config (model_config.c:61-146 for the llama family) */
    uint32_t n_vocab, n_ctx, n_embd, n_layer, n_head, n_head_kv, n_ff, head_dim;
    float eps, rope_base;
    size_t kv_ctx;
    /* resolved tensors */
    const orc_tensor_t *tok_embd, *out_norm, *out_w;
    const orc_tensor_t **blk; /* per layer: attn_norm q k v o ffn_norm gate up down */
    /* state */
    float *k_cache, *v_cache, *cos_tab, *sin_tab;
    float *x, *xn, *q, *k, *v, *att, *sc, *attn_out, *gate, *up, *ffn_out;
};

enum { B_ANORM, B_Q, B_K, B_V, B_O, B_FNORM, B_GATE, B_UP, B_DOWN, B_N };
static const char *blk_names[B_N] = {"attn_norm.weight", "attn_q.weight", "attn_k.weight",
                                     "attn_v.weight", "attn_output.weight", "ffn_norm.weight",
                                     "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};

static const orc_tensor_t *find_t(const orc_model_t *m, const char *name)
{
    for (size_t i = 0; i < m->n_tensors; i++)
        if (strcmp(m->tensors[i].name, name) == 0) return &m->tensors[i];
    return NULL;
}

static int tensor_bytes(uint32_t type, const uint64_t *dims, uint32_t nd, uint64_t *out)
{
    uint64_t n = 1;
    for (uint32_t i = 0; i < nd; i++) n *= dims[i];
    if (type == T_F32) { *out = n * 4; return 0; }
    size_t bb;
    if (block_layout(type, &bb) != 0) { *out = 0; return 1; }
    if (dims[0] % 32) return -1;
    *out = n / 32 * bb;
    return 0;
}

void orc_close(orc_model_t *m)
{
    if (!m) return;
    if (m->map) munmap(m->map, m->map_size);
    if (m->fd >= 0) close(m->fd);
    free(m->tensors);
    free(m->blk);
    free(m->k_cache); free(m->v_cache); free(m->cos_tab); free(m->sin_tab);
    free(m->x); free(m->xn); free(m->q); free(m->k); free(m->v); free(m->att);
    free(m->sc); free(m->attn_out); free(m->gate); free(m->up); free(m->ffn_out);
    free(m);
}

int orc_open(orc_model_t **out, const char *path, size_t max_ctx)
{
    *out = NULL;
    orc_model_t *m = (orc_model_t *)calloc(1, sizeof(*m));
    if (!m) return -1;
    m->fd = open(path, O_RDONLY);
    if (m->fd < 0) { orc_close(m); return -1; }
    struct stat st;
    if (fstat(m->fd, &st) || st.st_size < 24) { orc_close(m); return -1; }
    m->map_size = (size_t)st.st_size;
    m->map = mmap(NULL, m->map_size, PROT_READ, MAP_PRIVATE, m->fd, 0);
    if (m->map == MAP_FAILED) { m->map = NULL; orc_close(m); return -1; }

    rd_t r = {(const uint8_t *)m->map, (const uint8_t *)m->map + m->map_size, 0};
    uint32_t magic = (uint32_t)rd_u(&r, 4), ver = (uint32_t)rd_u(&r, 4);
    uint64_t n_t = rd_u(&r, 8), n_kv = rd_u(&r, 8);
    if (r.err || magic != 0x46554747u || ver < 2 || ver > 3 || n_t > 10000000u) {
        orc_close(m);
        return -1;
    }

    char arch[64] = "";
    uint32_t alignment = 32, ttc = 0;
    uint64_t n_tokens = 0;
    /* arch-prefixed keys are matched after the arch string is known; the
     * architecture key precedes them in every writer we read, but be safe and
     * remember raw positions. */
    struct { char key[80]; uint32_t type; const uint8_t *val; } kvs[128];
    size_t nk = 0;
    for (uint64_t i = 0; i < n_kv && !r.err; i++) {
        uint64_t kl;
        const char *k = rd_str(&r, &kl);
        uint32_t t = (uint32_t)rd_u(&r, 4);
        if (r.err) break;
        const uint8_t *vp = r.p;
        if (kl == 20 && !memcmp(k, "general.architecture", 20) && t == 8) {
            uint64_t al;
            const char *a = rd_str(&r, &al);
            if (a && al < sizeof(arch)) { memcpy(arch, a, al); arch[al] = 0; }
            continue;
        }
        if (kl == 21 && !memcmp(k, "tokenizer.ggml.tokens", 21) && t == 9) {
            rd_t r2 = r;
            rd_u(&r2, 4);
            n_tokens = rd_u(&r2, 8);
        }
        if (kl < sizeof(kvs[0].key) && nk < 128) {
            memcpy(kvs[nk].key, k, kl);
            kvs[nk].key[kl] = 0;
            kvs[nk].type = t;
            kvs[nk].val = vp;
            nk++;
        }
        skip_val(&r, t, 0);
    }
    if (r.err || strcmp(arch, "llama") != 0) { orc_close(m); return -1; }

#define FIND_U32(suffix, dst, def)                                              \
    do {                                                                        \
        char kk[128];                                                           \
        snprintf(kk, sizeof kk, "%s.%s", arch, suffix);                         \
        dst = def;                                                              \
        for (size_t j = 0; j < nk; j++)                                         \
            if (!strcmp(kvs[j].key, kk) && (kvs[j].type == 4 || kvs[j].type == 5)) \
                memcpy(&dst, kvs[j].val, 4);                                    \
    } while (0)
#define FIND_F32(suffix, dst, def)                                              \
    do {                                                                        \
        char kk[128];                                                           \
        snprintf(kk, sizeof kk, "%s.%s", arch, suffix);                         \
        dst = def;                                                              \
        for (size_t j = 0; j < nk; j++)                                         \
            if (!strcmp(kvs[j].key, kk) && kvs[j].type == 6) memcpy(&dst, kvs[j].val, 4); \
    } while (0)

    FIND_U32("embedding_length", m->n_embd, 0);
    FIND_U32("block_count", m->n_layer, 0);
    FIND_U32("attention.head_count", m->n_head, 0);
    FIND_U32("attention.head_count_kv", m->n_head_kv, m->n_head);
    FIND_U32("feed_forward_length", m->n_ff, 0);
    FIND_U32("context_length", m->n_ctx, 2048);
    FIND_F32("attention.layer_norm_rms_epsilon", m->eps, 1e-5f);
    if (m->eps == 1e-5f) FIND_F32("attention.layer_norm_epsilon", m->eps, 1e-5f);
    FIND_F32("rope.freq_base", m->rope_base, 10000.0f);
    for (size_t j = 0; j < nk; j++) {
        if (!strcmp(kvs[j].key, "general.alignment") && kvs[j].type == 4) {
            uint32_t a;
            memcpy(&a, kvs[j].val, 4);
            if (a > 0 && a <= 4096 && (a & (a - 1)) == 0) alignment = a;
        }
        if (!strcmp(kvs[j].key, "tokenizer.ggml.token_type_count") &&
            (kvs[j].type == 4 || kvs[j].type == 5))
            memcpy(&ttc, kvs[j].val, 4);
    }
    if (!m->n_embd || !m->n_layer || !m->n_head) { orc_close(m); return -1; }
    m->head_dim = m->n_embd / m->n_head;

    m->tensors = (orc_tensor_t *)calloc(n_t ? n_t : 1, sizeof(orc_tensor_t));
    if (!m->tensors) { orc_close(m); return -1; }
    for (uint64_t i = 0; i < n_t && !r.err; i++) {
        orc_tensor_t *t = &m->tensors[i];
        uint64_t nl;
        const char *nm = rd_str(&r, &nl);
        if (r.err || nl >= sizeof(t->name)) { r.err = 1; break; }
        memcpy(t->name, nm, nl);
        t->name[nl] = 0;
        t->n_dims = (uint32_t)rd_u(&r, 4);
        if (t->n_dims == 0 || t->n_dims > 4) { r.err = 1; break; }
        for (uint32_t d = 0; d < t->n_dims; d++) t->dims[d] = rd_u(&r, 8);
        t->type = (uint32_t)rd_u(&r, 4);
        t->offset = rd_u(&r, 8);
        if (tensor_bytes(t->type, t->dims, t->n_dims, &t->bytes) < 0) r.err = 1;
    }
    if (r.err) { orc_close(m); return -1; }
    m->n_tensors = n_t;
    uint64_t after = (uint64_t)(r.p - (const uint8_t *)m->map);
    uint64_t data_off = (after + alignment - 1) & ~((uint64_t)alignment - 1);
    for (size_t i = 0; i < m->n_tensors; i++) {
        orc_tensor_t *t = &m->tensors[i];
        if (data_off + t->offset + t->bytes > m->map_size) { orc_close(m); return -1; }
        t->data = (const uint8_t *)m->map + data_off + t->offset;
    }

    /* n_vocab: token_type_count, else output.weight / lm_head.weight dims[1]
     * (model_config.c:133-146), else the token list length
     * (transformer.c:112-113). */
    m->n_vocab = ttc;
    if (!m->n_vocab) {
        const orc_tensor_t *ow = find_t(m, "output.weight");
        if (!ow) ow = find_t(m, "lm_head.weight");
        if (ow) m->n_vocab = (uint32_t)(ow->n_dims >= 2 ? ow->dims[1] : ow->dims[0]);
    }
    if (!m->n_vocab) m->n_vocab = (uint32_t)n_tokens;
    if (!m->n_vocab) { orc_close(m); return -1; }

    /* max_ctx clamp, transformer.c:43-52 */
    if (!max_ctx) max_ctx = m->n_ctx < 4096 ? m->n_ctx : 4096;
    if (max_ctx > m->n_ctx) max_ctx = m->n_ctx;
    if (!max_ctx) { orc_close(m); return -1; }
    m->kv_ctx = max_ctx;

    m->tok_embd = find_t(m, "token_embd.weight");
    m->out_norm = find_t(m, "output_norm.weight");
    m->out_w = find_t(m, "output.weight");
    if (!m->out_w) m->out_w = find_t(m, "lm_head.weight");
    if (!m->out_w) m->out_w = m->tok_embd;
    m->blk = (const orc_tensor_t **)calloc((size_t)m->n_layer * B_N, sizeof(void *));
    if (!m->tok_embd || !m->out_w || !m->blk) { orc_close(m); return -1; }
    for (uint32_t l = 0; l < m->n_layer; l++)
        for (int b = 0; b < B_N; b++) {
            char nm[128];
            snprintf(nm, sizeof nm, "blk.%u.%s", l, blk_names[b]);
            m->blk[l * B_N + b] = find_t(m, nm);
            if (!m->blk[l * B_N + b]) { orc_close(m); return -1; }
        }

    size_t hd = m->head_dim, half = hd / 2;
    size_t kvrow = (size_t)m->n_head_kv * hd;
    size_t kvn = (size_t)m->n_layer * m->kv_ctx * kvrow;
    m->k_cache = (float *)calloc(kvn, 4);
    m->v_cache = (float *)calloc(kvn, 4);
    m->cos_tab = (float *)malloc((m->kv_ctx * half + 1) * 4);
    m->sin_tab = (float *)malloc((m->kv_ctx * half + 1) * 4);
    size_t E = m->n_embd;
    m->x = (float *)malloc(E * 4);
    m->xn = (float *)malloc(E * 4);
    m->q = (float *)malloc((size_t)m->n_head * hd * 4);
    m->k = (float *)malloc(kvrow * 4);
    m->v = (float *)malloc(kvrow * 4);
    m->att = (float *)malloc((size_t)m->n_head * hd * 4);
    m->sc = (float *)malloc((m->kv_ctx + 1) * 4);
    m->attn_out = (float *)malloc(E * 4);
    m->gate = (float *)malloc((size_t)m->n_ff * 4 + 4);
    m->up = (float *)malloc((size_t)m->n_ff * 4 + 4);
    m->ffn_out = (float *)malloc(E * 4);
    if (!m->k_cache || !m->v_cache || !m->cos_tab || !m->sin_tab || !m->x || !m->xn ||
        !m->q || !m->k || !m->v || !m->att || !m->sc || !m->attn_out || !m->gate ||
        !m->up || !m->ffn_out) {
        orc_close(m);
        return -1;
    }
    orc_rope_tables(m->cos_tab, m->sin_tab, m->kv_ctx, hd, m->rope_base);
    *out = m;
    return 0;
}

void orc_dims(const orc_model_t *m, uint32_t *d)
{
    d[0] = m->n_vocab; d[1] = (uint32_t)m->kv_ctx; d[2] = m->n_embd; d[3] = m->n_layer;
    d[4] = m->n_head; d[5] = m->n_head_kv; d[6] = m->n_ff; d[7] = m->head_dim;
}

static float *kv_row(float *base, const orc_model_t *m, size_t l, size_t p)
{
    return base + (l * m->kv_ctx + p) * (size_t)m->n_head_kv * m->head_dim;
}

int orc_kv_write(orc_model_t *m, size_t layer, size_t pos0, size_t n,
                 const float *k, const float *v)
{
    if (layer >= m->n_layer || pos0 > m->kv_ctx || n > m->kv_ctx - pos0) return -1;
    size_t row = (size_t)m->n_head_kv * m->head_dim;
    for (size_t i = 0; i < n; i++) {
        memcpy(kv_row(m->k_cache, m, layer, pos0 + i), k + i * row, row * 4);
        memcpy(kv_row(m->v_cache, m, layer, pos0 + i), v + i * row, row * 4);
    }
    return 0;
}

int orc_kv_read(const orc_model_t *m, size_t layer, size_t pos0, size_t n,
                float *k, float *v)
{
    if (layer >= m->n_layer || pos0 > m->kv_ctx || n > m->kv_ctx - pos0) return -1;
    size_t row = (size_t)m->n_head_kv * m->head_dim;
    for (size_t i = 0; i < n; i++) {
        memcpy(k + i * row, kv_row(m->k_cache, m, layer, pos0 + i), row * 4);
        memcpy(v + i * row, kv_row(m->v_cache, m, layer, pos0 + i), row * 4);
    }
    return 0;
}

/* linear_forward without bias, linear.c:155-223: F32 rows via simd_dot_f32,
 * block quants via quant_matvec.  dims[0] = in, dims[1] = out. */
static int linear(const orc_tensor_t *w, const float *x, float *y)
{
    size_t in = (size_t)w->dims[0], out = w->n_dims >= 2 ? (size_t)w->dims[1] : 1;
    if (w->type == T_F32) {
        const float *W = (const float *)w->data;
        for (size_t r = 0; r < out; r++) y[r] = orc_dot(W + r * in, x, in);
        return 0;
    }
    return orc_quant_matvec(w->data, (size_t)w->bytes, w->type, x, y, in, out);
}

/* linear_get_row, linear.c:60-151 (F32 copy, else block decode of one row). */
static int get_row(const orc_tensor_t *w, size_t row, float *out)
{
    size_t ncols = (size_t)w->dims[0];
    if (w->type == T_F32) {
        if ((row + 1) * ncols * 4 > w->bytes) return -1;
        memcpy(out, w->data + row * ncols * 4, ncols * 4);
        return 0;
    }
    size_t bb;
    if (block_layout(w->type, &bb) != 0 || ncols % 32) return -1;
    size_t rb = ncols / 32 * bb;
    if ((row + 1) * rb > w->bytes) return -1;
    return orc_dequant(w->data + row * rb, rb, w->type, out, ncols);
}

/* transformer_forward, transformer.c:149-326, sequential-residual llama path;
 * attention_forward (attention.c:35-170) and the gated ffn_forward
 * (ffn.c:44-107) inlined. */
int orc_forward(orc_model_t *m, uint32_t token, size_t pos, float *logits)
{
    if (pos >= m->kv_ctx || token >= m->n_vocab) return -1;
    const size_t E = m->n_embd, H = m->n_head, KV = m->n_head_kv, hd = m->head_dim;
    if (get_row(m->tok_embd, token, m->x) != 0) return -1;

    const size_t group = H / KV;
    const float scale = 1.0f / sqrtf((float)hd);
    for (size_t l = 0; l < m->n_layer; l++) {
        const orc_tensor_t **B = &m->blk[l * B_N];
        orc_rms_norm(m->x, (const float *)B[B_ANORM]->data, m->xn, E, m->eps);
        if (linear(B[B_Q], m->xn, m->q) || linear(B[B_K], m->xn, m->k) ||
            linear(B[B_V], m->xn, m->v))
            return -1;
        orc_rope_apply(m->q, pos, H, hd, m->cos_tab, m->sin_tab);
        orc_rope_apply(m->k, pos, KV, hd, m->cos_tab, m->sin_tab);
        memcpy(kv_row(m->k_cache, m, l, pos), m->k, KV * hd * 4);
        memcpy(kv_row(m->v_cache, m, l, pos), m->v, KV * hd * 4);
        memset(m->att, 0, H * hd * 4);
        for (size_t h = 0; h < H; h++) {
            size_t kvh = h / group;
            const float *qh = m->q + h * hd;
            float *oh = m->att + h * hd;
            for (size_t t = 0; t <= pos; t++)
                m->sc[t] = orc_dot(qh, kv_row(m->k_cache, m, l, t) + kvh * hd, hd) * scale;
            orc_softmax(m->sc, pos + 1);
            for (size_t t = 0; t <= pos; t++)
                orc_axpy(oh, kv_row(m->v_cache, m, l, t) + kvh * hd, m->sc[t], hd);
        }
        if (linear(B[B_O], m->att, m->attn_out)) return -1;
        for (size_t i = 0; i < E; i++) m->x[i] += m->attn_out[i];

        orc_rms_norm(m->x, (const float *)B[B_FNORM]->data, m->xn, E, m->eps);
        if (linear(B[B_GATE], m->xn, m->gate) || linear(B[B_UP], m->xn, m->up)) return -1;
        orc_silu(m->gate, m->n_ff);
        for (size_t i = 0; i < m->n_ff; i++) m->gate[i] *= m->up[i];
        if (linear(B[B_DOWN], m->gate, m->ffn_out)) return -1;
        for (size_t i = 0; i < E; i++) m->x[i] += m->ffn_out[i];
    }
    if (m->out_norm)
        orc_rms_norm(m->x, (const float *)m->out_norm->data, m->xn, E, m->eps);
    else
        memcpy(m->xn, m->x, E * 4);
    return linear(m->out_w, m->xn, logits);
}
