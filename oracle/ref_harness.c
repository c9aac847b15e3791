/*
 * ref_harness.c — TEST INFRASTRUCTURE (oracle).  A ctypes-friendly wrapper
 * around the compiled reference so that tests (and bench.py's CPU-baseline
 * leg) can drive it without knowing sizeof(transformer_t).
 *
 * Everything here calls the reference's own public API:
 *   transformer_init / transformer_forward / transformer_free
 *     (transformer.h:39-48, transformer.c:14-326)
 *   kv_k / kv_v (kv_cache.h:45-51) for the KV pre-fill that config 4 needs,
 *   gguf_open + model_config_load (gguf.h:42, model_config.h:95) to read the
 *     config the reference derives from a GGUF file.
 */
#define _POSIX_C_SOURCE 200809L
#include "transformer.h"
#include "quant_matvec.h"
#include "sampler.h"

#include <stdlib.h>
#include <string.h>

void *refh_open(const char *path, size_t max_ctx)
{
    transformer_t *t = (transformer_t *)calloc(1, sizeof(*t));
    if (!t) return NULL;
    if (transformer_init(t, path, max_ctx) != 0) {
        free(t);
        return NULL;
    }
    return t;
}

void refh_close(void *h)
{
    if (!h) return;
    transformer_free((transformer_t *)h);
    free(h);
}

/* One decode step; copies n_vocab logits into out.  0 / -1. */
int refh_forward(void *h, uint32_t token, size_t pos, float *out)
{
    transformer_t *t = (transformer_t *)h;
    float *lg = transformer_forward(t, token, pos);
    if (!lg) return -1;
    memcpy(out, lg, (size_t)t->cfg.n_vocab * sizeof(float));
    return 0;
}

/* Greedy argmax of the last logits (sampler.c:28-32). */
uint32_t refh_argmax(void *h)
{
    transformer_t *t = (transformer_t *)h;
    return sampler_argmax(t->logits, t->cfg.n_vocab);
}

/* dims: n_vocab n_ctx(kv) n_embd n_layer n_head n_head_kv n_ff head_dim */
void refh_dims(void *h, uint32_t *d)
{
    transformer_t *t = (transformer_t *)h;
    d[0] = t->cfg.n_vocab;
    d[1] = (uint32_t)t->kv.n_ctx;
    d[2] = t->cfg.n_embd;
    d[3] = t->cfg.n_layer;
    d[4] = t->cfg.n_head;
    d[5] = t->cfg.n_head_kv;
    d[6] = t->cfg.n_ff;
    d[7] = t->cfg.head_dim;
}

/* Write K/V for n positions starting at pos0 of one layer; k and v are
 * [n][n_head_kv][head_dim] fp32 (the reference's own cache row order). */
int refh_kv_write(void *h, size_t layer, size_t pos0, size_t n,
                  const float *k, const float *v)
{
    transformer_t *t = (transformer_t *)h;
    kv_cache_t *kv = &t->kv;
    if (layer >= kv->n_layer || pos0 > kv->n_ctx || n > kv->n_ctx - pos0)
        return -1;
    size_t row = kv->n_head_kv * kv->head_dim;
    for (size_t i = 0; i < n; i++) {
        memcpy(kv_k(kv, layer, pos0 + i, 0), k + i * row, row * sizeof(float));
        memcpy(kv_v(kv, layer, pos0 + i, 0), v + i * row, row * sizeof(float));
    }
    return 0;
}

/* Read K/V rows back (same layout as refh_kv_write). */
int refh_kv_read(void *h, size_t layer, size_t pos0, size_t n, float *k, float *v)
{
    transformer_t *t = (transformer_t *)h;
    kv_cache_t *kv = &t->kv;
    if (layer >= kv->n_layer || pos0 > kv->n_ctx || n > kv->n_ctx - pos0)
        return -1;
    size_t row = kv->n_head_kv * kv->head_dim;
    for (size_t i = 0; i < n; i++) {
        memcpy(k + i * row, kv_k(kv, layer, pos0 + i, 0), row * sizeof(float));
        memcpy(v + i * row, kv_v(kv, layer, pos0 + i, 0), row * sizeof(float));
    }
    return 0;
}

/* The model_config_t the reference derives from a GGUF file, as numbers:
 * u[0..9] = arch n_vocab n_ctx n_embd n_layer n_head n_head_kv n_ff head_dim n_rot
 * f[0..2] = norm_eps rope_freq_base rope_freq_scale.  Returns 0 / -1. */
int refh_config(const char *path, uint32_t *u, float *f)
{
    gguf_file_t g;
    char err[256];
    if (gguf_open(&g, path, err, sizeof(err)) != 0) return -1;
    model_config_t c;
    int rc = model_config_load(&c, &g);
    if (rc == 0) {
        u[0] = (uint32_t)c.arch; u[1] = c.n_vocab; u[2] = c.n_ctx;
        u[3] = c.n_embd; u[4] = c.n_layer; u[5] = c.n_head;
        u[6] = c.n_head_kv; u[7] = c.n_ff; u[8] = c.head_dim; u[9] = c.n_rot;
        f[0] = c.norm_eps; f[1] = c.rope_freq_base; f[2] = c.rope_freq_scale;
    }
    gguf_close(&g);
    return rc;
}

/* Direct access to the (Q4_0-extended) quant_matvec for the microbench. */
int refh_quant_matvec(const void *w, size_t w_size, uint32_t type,
                      const float *x, float *y, size_t in, size_t out)
{
    return quant_matvec(w, w_size, type, x, y, in, out);
}
