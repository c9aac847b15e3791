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

static int block_bytes(uint32_t type)
{
    switch (type) {
    case 2: return 18;
    case 6: return 22;
    case 8: return 34;
    default: return 0;
    }
}

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
        float x[32];
        for (uint64_t b = 0; b < j->cols / 32; b++) {
            uint8_t *o = row + b * bb;
            if (j->mode == 1) {
                uint64_t h = splitmix64(j->key ^ ((r * j->cols + b * 32) * 0xD1B54A32D192ED03ull));
                float u = (float)(h >> 40) * (1.0f / 16777216.0f);
                uint16_t dh = to_f16(j->mean + (j->sd - j->mean) * u);
                memcpy(o, &dh, 2);
                for (int k = 2; k < bb; k += 8) {
                    uint64_t q = splitmix64(h + (uint64_t)k);
                    int n = bb - k < 8 ? bb - k : 8;
                    memcpy(o + k, &q, (size_t)n);
                }
                continue;
            }
            for (int e = 0; e < 32; e++) x[e] = j->mean + j->sd * normal_at(j->key, r * j->cols + b * 32 + e);
            if (j->type == 8) quant_q8_0(x, o);
            else if (j->type == 2) quant_q4_0(x, o);
            else quant_q5_0(x, o);
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
 * (0 = F32, 2 = Q4_0, 6 = Q5_0, 8 = Q8_0) at dst (dst points at row row0).
 * mode 0: values mean + sd * N(0,1), quantised as above.
 * mode 1: uniform random quants over their full range and d ~ U(lo, hi)
 *         (lo = mean, hi = sd) — the standalone matvec microbench inputs.
 * Returns 0, or -1 on a bad argument.
 */
int fwb_synth_fill(void *dst, uint32_t type, uint64_t cols, uint64_t row0,
                   uint64_t row1, uint64_t key, float mean, float sd, int mode)
{
    int bb = block_bytes(type);
    if (type != 0 && (!bb || cols % 32)) return -1;
    if (type == 0 && mode != 0) return -1;
    uint64_t rows = row1 - row0;
    fill_job_t base = {dst, type, cols, row0, key, 0, rows,
                       type == 0 ? cols * 4 : cols / 32 * (uint64_t)bb, mean, sd, mode, bb};
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
