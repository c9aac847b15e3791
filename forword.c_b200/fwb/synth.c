/*
 * synth.c — seeded synthetic tensor generator for GGUF test and benchmark
 * models (the configurations of the benchmark spec use random-init weights;
 * no checkpoint is involved).  Built into libfwb_synth.so and driven by
 * fwb/gguf_synth.py, which writes the GGUF container around it.
 *
 * Values are a pure function of (seed, tensor key, element index), so any
 * thread count and any row range produce the same bytes.  Rows are split
 * over the host's cores with pthreads.
 *
 * Normal variates: Irwin-Hall sum of 8 uniform bytes of one splitmix64 hash,
 * standardised (mean 1020, sd sqrt(8*(256^2-1)/12)); a close, fast stand-in
 * for N(0,1) bounded at about +-4.9 sd.
 *
 * Quantisers restate GGML's published reference quantisers:
 *   Q8_0: d = amax/127, q = round(x/d)                      (34-byte blocks)
 *   Q4_0: d = max/-8 (max = the signed value of largest |x|),
 *         q = min(15, (int)(x/d + 8.5)), low nibbles hold elements 0-15,
 *         high nibbles 16-31                               (18-byte blocks)
 *   Q5_0: d = max/-16, q = min(31, (int)(x/d + 16.5)), low 4 bits as Q4_0,
 *         bit 4 of element j in bit j of a 32-bit plane    (22-byte blocks)
 *   Q5_1: d = (max - min)/31, m = min, q = round((x - m)/d) in [0, 31],
 *         nibbles and bit plane as Q5_0 after d and m  (24-byte blocks)
 * and, for the K-quants (256-value superblocks), simple quantisers of my own
 * (any valid encoding serves the tests; the byte formats are GGML's):
 *   Q4_K: 8 groups of 32, x ~ d*sc*q - dmin*m with 6-bit sc, m packed in 12
 *         bytes, q in [0, 15]; groups 2k and 2k+1 share 32 bytes (low and
 *         high nibbles)                                    (144-byte blocks)
 *   Q6_K: 16 groups of 16 with int8 scales, x ~ d*sc*(q - 32), q in
 *         [0, 63] as 4 low bits (ql) and 2 high bits (qh) (210-byte blocks)
 * d is stored as IEEE fp16 (round to nearest even, via _Float16).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static inline uint64_t splitmix64(uint64_t x)
{
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static inline float normal_at(uint64_t key, uint64_t i)
{
    uint64_t h = splitmix64(key ^ (i * 0xD1B54A32D192ED03ull));
    uint32_t s = 0;
    for (int b = 0; b < 8; b++) s += (uint32_t)((h >> (8 * b)) & 0xff);
    return ((float)s - 1020.0f) * (1.0f / 209.02392f);
}

static inline uint16_t to_f16(float f)
{
    _Float16 h = (_Float16)f;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

static void quant_q8_0(const float *x, uint8_t *o)
{
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
    float d = amax / 127.0f, id = d ? 1.0f / d : 0.0f;
    uint16_t dh = to_f16(d);
    memcpy(o, &dh, 2);
    for (int j = 0; j < 32; j++) o[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
}

static float signed_max(const float *x)
{
    float amax = 0.0f, mx = 0.0f;
    for (int j = 0; j < 32; j++)
        if (fabsf(x[j]) > amax) { amax = fabsf(x[j]); mx = x[j]; }
    return mx;
}

static void quant_q4_0(const float *x, uint8_t *o)
{
    float d = signed_max(x) / -8.0f, id = d ? 1.0f / d : 0.0f;
    uint16_t dh = to_f16(d);
    memcpy(o, &dh, 2);
    for (int j = 0; j < 16; j++) {
        int a = (int)(int8_t)(x[j] * id + 8.5f), b = (int)(int8_t)(x[j + 16] * id + 8.5f);
        a = a > 15 ? 15 : a;
        b = b > 15 ? 15 : b;
        o[2 + j] = (uint8_t)(a | (b << 4));
    }
}

static void quant_q5_0(const float *x, uint8_t *o)
{
    float d = signed_max(x) / -16.0f, id = d ? 1.0f / d : 0.0f;
    uint16_t dh = to_f16(d);
    memcpy(o, &dh, 2);
    uint32_t qh = 0;
    for (int j = 0; j < 16; j++) {
        int a = (int)(int8_t)(x[j] * id + 16.5f), b = (int)(int8_t)(x[j + 16] * id + 16.5f);
        a = a > 31 ? 31 : a;
        b = b > 31 ? 31 : b;
        o[6 + j] = (uint8_t)((a & 15) | ((b & 15) << 4));
        qh |= (uint32_t)((a >> 4) & 1) << j;
        qh |= (uint32_t)((b >> 4) & 1) << (j + 16);
    }
    memcpy(o + 2, &qh, 4);
}

static void quant_q5_1(const float *x, uint8_t *o)
{
    float mn = x[0], mx = x[0];
    for (int j = 1; j < 32; j++) { mn = fminf(mn, x[j]); mx = fmaxf(mx, x[j]); }
    float d = (mx - mn) / 31.0f, id = d ? 1.0f / d : 0.0f;
    uint16_t dh = to_f16(d), mh = to_f16(mn);
    memcpy(o, &dh, 2);
    memcpy(o + 2, &mh, 2);
    uint32_t qh = 0;
    for (int j = 0; j < 16; j++) {
        int a = (int)((x[j] - mn) * id + 0.5f), b = (int)((x[j + 16] - mn) * id + 0.5f);
        a = a < 0 ? 0 : a > 31 ? 31 : a;
        b = b < 0 ? 0 : b > 31 ? 31 : b;
        o[8 + j] = (uint8_t)((a & 15) | ((b & 15) << 4));
        qh |= (uint32_t)((a >> 4) & 1) << j;
        qh |= (uint32_t)((b >> 4) & 1) << (j + 16);
    }
    memcpy(o + 4, &qh, 4);
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

/* 6-bit scales and mins of the 8 groups into the 12 bytes read back by the
 * reference's get_scale_min_k4 (quant.c) */
static void pack_scale_min_k4(const int *sc, const int *mn, uint8_t *s)
{
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
}

static void quant_q4_k(const float *x, uint8_t *o)
{
    float gs[8], gm[8], smax = 0.0f, mmax = 0.0f;
    for (int g = 0; g < 8; g++) {
        float lo = 0.0f, hi = 0.0f;
        for (int i = 0; i < 32; i++) { lo = fminf(lo, x[32 * g + i]); hi = fmaxf(hi, x[32 * g + i]); }
        gs[g] = (hi - lo) / 15.0f;
        gm[g] = -lo;
        smax = fmaxf(smax, gs[g]);
        mmax = fmaxf(mmax, gm[g]);
    }
    const float d = smax / 63.0f, dmin = mmax / 63.0f;
    int sc[8], mn[8];
    for (int g = 0; g < 8; g++) {
        sc[g] = d > 0 ? clampi((int)lrintf(gs[g] / d), 0, 63) : 0;
        mn[g] = dmin > 0 ? clampi((int)lrintf(gm[g] / dmin), 0, 63) : 0;
    }
    uint16_t dh = to_f16(d), mh = to_f16(dmin);
    memcpy(o, &dh, 2);
    memcpy(o + 2, &mh, 2);
    pack_scale_min_k4(sc, mn, o + 4);
    for (int k = 0; k < 4; k++)
        for (int i = 0; i < 32; i++) {
            int q[2];
            for (int h = 0; h < 2; h++) {
                const int g = 2 * k + h;
                const float ds = d * (float)sc[g], dm = dmin * (float)mn[g];
                q[h] = ds > 0 ? clampi((int)lrintf((x[32 * g + i] + dm) / ds), 0, 15) : 0;
            }
            o[16 + 32 * k + i] = (uint8_t)(q[0] | (q[1] << 4));
        }
}

static void quant_q6_k(const float *x, uint8_t *o)
{
    float gs[16], smax = 0.0f;
    for (int g = 0; g < 16; g++) {
        float a = 0.0f;
        for (int i = 0; i < 16; i++) a = fmaxf(a, fabsf(x[16 * g + i]));
        gs[g] = a / 31.0f;
        smax = fmaxf(smax, gs[g]);
    }
    const float d = smax / 127.0f;
    int8_t sc[16];
    for (int g = 0; g < 16; g++) sc[g] = (int8_t)(d > 0 ? clampi((int)lrintf(gs[g] / d), 1, 127) : 0);
    int q[256];
    for (int e = 0; e < 256; e++) {
        const float s = d * (float)sc[e / 16];
        q[e] = s > 0 ? clampi((int)lrintf(x[e] / s) + 32, 0, 63) : 32;
    }
    uint8_t *ql = o, *qh = o + 128;
    for (int half = 0; half < 2; half++) {
        const int *qq = q + 128 * half;
        for (int l = 0; l < 32; l++) {
            const int q1 = qq[l], q2 = qq[l + 32], q3 = qq[l + 64], q4 = qq[l + 96];
            ql[64 * half + l] = (uint8_t)((q1 & 15) | ((q3 & 15) << 4));
            ql[64 * half + l + 32] = (uint8_t)((q2 & 15) | ((q4 & 15) << 4));
            qh[32 * half + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    }
    memcpy(o + 192, sc, 16);
    uint16_t dh = to_f16(d);
    memcpy(o + 208, &dh, 2);
}

static int block_bytes(uint32_t type)
{
    switch (type) {
    case 2: return 18;
    case 6: return 22;
    case 7: return 24;
    case 8: return 34;
    case 12: return 144;
    case 14: return 210;
    default: return 0;
    }
}

static int block_values(uint32_t type) { return type == 12 || type == 14 ? 256 : 32; }

typedef struct {
    void *dst;
    uint32_t type;
    uint64_t cols, row0, key, r_begin, r_end, row_bytes;
    float mean, sd;
    int mode, bb;
} fill_job_t;

static void fill_rows(const fill_job_t *j)
{
    const int bb = j->bb;
    for (uint64_t rr = j->r_begin; rr < j->r_end; rr++) {
        uint64_t r = j->row0 + rr;
        uint8_t *row = (uint8_t *)j->dst + rr * j->row_bytes;
        if (j->type == 0) {
            float *f = (float *)row;
            for (uint64_t c = 0; c < j->cols; c++) f[c] = j->mean + j->sd * normal_at(j->key, r * j->cols + c);
            continue;
        }
        float x[256];
        const int bv = block_values(j->type);
        for (uint64_t b = 0; b < j->cols / bv; b++) {
            uint8_t *o = row + b * bb;
            if (j->mode == 1) {
                uint64_t h = splitmix64(j->key ^ ((r * j->cols + b * bv) * 0xD1B54A32D192ED03ull));
                for (int k = 0; k < bb; k += 8) {
                    uint64_t q = splitmix64(h + (uint64_t)k);
                    int n = bb - k < 8 ? bb - k : 8;
                    memcpy(o + k, &q, (size_t)n);
                }
                /* fp16 scales ~ U(lo, hi) (lo = mean, hi = sd); min / dmin too */
                float u = (float)(h >> 40) * (1.0f / 16777216.0f);
                uint16_t dh = to_f16(j->mean + (j->sd - j->mean) * u);
                const int d_off = j->type == 14 ? 208 : 0;
                memcpy(o + d_off, &dh, 2);
                if (j->type == 7 || j->type == 12) {
                    float u2 = (float)(splitmix64(h ^ 0x5555ull) >> 40) * (1.0f / 16777216.0f);
                    uint16_t mh = to_f16((j->type == 7 ? -8.0f : 1.0f) * (j->mean + (j->sd - j->mean) * u2));
                    memcpy(o + 2, &mh, 2);
                }
                continue;
            }
            for (int e = 0; e < bv; e++) x[e] = j->mean + j->sd * normal_at(j->key, r * j->cols + b * bv + e);
            if (j->type == 8) quant_q8_0(x, o);
            else if (j->type == 2) quant_q4_0(x, o);
            else if (j->type == 6) quant_q5_0(x, o);
            else if (j->type == 7) quant_q5_1(x, o);
            else if (j->type == 12) quant_q4_k(x, o);
            else quant_q6_k(x, o);
        }
    }
}

static void *fill_worker(void *arg)
{
    fill_rows((const fill_job_t *)arg);
    return NULL;
}

static int n_workers(uint64_t work)
{
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 64) n = 64;
    if (work < (1u << 20)) n = 1;
    return (int)n;
}

/*
 * Fill rows [row0, row1) of a [rows x cols] tensor of ggml type `type`
 * (0 = F32, 2 = Q4_0, 6 = Q5_0, 7 = Q5_1, 8 = Q8_0, 12 = Q4_K, 14 = Q6_K) at dst
 * (dst points at row row0).
 * mode 0: values mean + sd * N(0,1), quantised as above.
 * mode 1: uniform random quants over their full range and d ~ U(lo, hi)
 *         (lo = mean, hi = sd) — the standalone matvec microbench inputs.
 * Returns 0, or -1 on a bad argument.
 */
int fwb_synth_fill(void *dst, uint32_t type, uint64_t cols, uint64_t row0,
                   uint64_t row1, uint64_t key, float mean, float sd, int mode)
{
    int bb = block_bytes(type);
    if (type != 0 && (!bb || cols % (uint64_t)block_values(type))) return -1;
    if (type == 0 && mode != 0) return -1;
    uint64_t rows = row1 - row0;
    fill_job_t base = {dst, type, cols, row0, key, 0, rows,
                       type == 0 ? cols * 4 : cols / (uint64_t)block_values(type) * (uint64_t)bb, mean, sd, mode,
                       bb};
    int nw = n_workers(rows * cols);
    if ((uint64_t)nw > rows) nw = rows ? (int)rows : 1;
    pthread_t th[64];
    fill_job_t jobs[64];
    int created[64] = {0};
    for (int w = 0; w < nw; w++) {
        jobs[w] = base;
        jobs[w].r_begin = rows * (uint64_t)w / (uint64_t)nw;
        jobs[w].r_end = rows * (uint64_t)(w + 1) / (uint64_t)nw;
        if (nw > 1 && pthread_create(&th[w], NULL, fill_worker, &jobs[w]) == 0)
            created[w] = 1;
        else
            fill_rows(&jobs[w]);
    }
    for (int w = 0; w < nw; w++)
        if (created[w]) pthread_join(th[w], NULL);
    return 0;
}

/* Fill n fp32 values with mean + sd * N(0,1) from (key, index) — prompts, KV
 * pre-fill and activation vectors for tests. */
void fwb_synth_normal(float *dst, uint64_t n, uint64_t key, float mean, float sd)
{
    for (uint64_t i = 0; i < n; i++) dst[i] = mean + sd * normal_at(key, i);
}
