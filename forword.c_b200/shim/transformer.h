/*
 * transformer.h — drop-in replacement for forword.c's transformer.h
 * (transformer.h:1-53) when the decode forward runs on a B200.
 *
 * Same three entry points with the same signatures, return values and
 * lifetime rules (transformer.h:35-48).  transformer_t keeps the members the
 * rest of forword.c reads (g, cfg, tok: main.c:125,136,154-155,191,194); the
 * reference's host-side KV cache, RoPE tables and work buffers are replaced by
 * one opaque handle to the device state (weights, KV cache and activations in
 * HBM, owned by libforword_b200.so).
 */
#ifndef TRANSFORMER_H
#define TRANSFORMER_H

#include "gguf.h"
#include "model_config.h"
#include "tokenizer.h"
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct fwb_model;

typedef struct {
    gguf_file_t       g;      /* memory-mapped model (host metadata, tokenizer) */
    model_config_t    cfg;
    tokenizer_t      *tok;
    struct fwb_model *dev;    /* device state on the selected GPU */
    size_t            n_ctx;  /* KV positions (the reference's kv.n_ctx) */
    float            *logits; /* [n_vocab] host copy returned by transformer_forward */
} transformer_t;

/*
 * Load a GGUF model file, upload every tensor once to HBM in its GGUF byte
 * layout and allocate the device KV cache.  max_ctx limits the KV cache
 * (0 -> min(cfg.n_ctx, 4096); larger than cfg.n_ctx -> cfg.n_ctx).  The GPU
 * is device 0, or the one named by the FORWORD_CUDA_DEVICE environment
 * variable.  Returns 0 on success, -1 on error (message on stderr).
 */
int transformer_init(transformer_t *t, const char *path, size_t max_ctx);

/* Free all resources (safe on a partially initialised or zeroed struct). */
void transformer_free(transformer_t *t);

/*
 * Run one forward step: feed token_id at sequence position pos.
 * Returns pointer to logits[n_vocab] (valid until next call), or NULL on error.
 */
float *transformer_forward(transformer_t *t, uint32_t token_id, size_t pos);

#ifdef __cplusplus
}
#endif
#endif /* TRANSFORMER_H */
