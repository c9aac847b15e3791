/*
 * transformer_b200.c — transformer_init / transformer_free /
 * transformer_forward (transformer.h:39-48) backed by libforword_b200.so.
 *
 * Compiled together with forword.c's unchanged host C (gguf.c, gguf_raw.c,
 * model_config.c, tokenizer.c, sampler.c, chat_template.c, main.c) in place
 * of transformer.c, attention.c, ffn.c, linear.c, norm.c, rope.c, quant*.c,
 * tensor_data.c and tensor_ops.c.  The host keeps parsing the GGUF for the
 * tokenizer and chat template; the decode step runs entirely on the GPU and
 * only the logits row comes back.
 *
 * Messages and failure cases follow transformer.c:14-147 (init) and
 * transformer.c:149-164 (forward argument checks).
 */
#define _POSIX_C_SOURCE 200809L
#include "transformer.h"
#include "forword_b200.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static int device_from_env(void) {
    const char *s = getenv("FORWORD_CUDA_DEVICE");
    return (s && *s) ? atoi(s) : 0;
}

int transformer_init(transformer_t *t, const char *path, size_t max_ctx) {
    memset(t, 0, sizeof(*t));

    char errbuf[256];
    if (gguf_open(&t->g, path, errbuf, sizeof(errbuf)) != 0) {
        fprintf(stderr, "gguf_open: %s\n", errbuf);
        return -1;
    }
    if (model_config_load(&t->cfg, &t->g) != 0) {
        fprintf(stderr, "transformer_init: failed to read model config\n");
        gguf_close(&t->g);
        return -1;
    }
    model_config_t *c = &t->cfg;
    const char *name = gguf_get_metadata(&t->g, "general.name");
    fprintf(stderr, "Model: %s arch=%s layers=%u embd=%u heads=%u/%u ff=%u vocab=%u\n",
            name ? name : "(unnamed)", c->arch_str, c->n_layer, c->n_embd, c->n_head,
            c->n_head_kv, c->n_ff, c->n_vocab);

    if (!c->n_embd || !c->n_head || !c->n_layer) {
        fprintf(stderr, "transformer_init: invalid model dimensions\n");
        goto fail;
    }
    if (tokenizer_init(&t->tok, &t->g, c) != 0) {
        fprintf(stderr, "transformer_init: tokenizer_init failed\n");
        goto fail;
    }
    if (!c->n_vocab) c->n_vocab = (uint32_t)tokenizer_vocab_size(t->tok);
    if (!c->n_vocab) {
        fprintf(stderr, "transformer_init: invalid vocabulary size\n");
        goto fail;
    }

    t->dev = fwb_model_open(path, max_ctx, device_from_env());
    if (!t->dev) {
        fprintf(stderr, "transformer_init: %s\n", fwb_last_error());
        goto fail;
    }
    uint32_t d[8];
    if (fwb_model_dims(t->dev, d) != 0 || d[0] != c->n_vocab) {
        fprintf(stderr, "transformer_init: device model disagrees with the host config\n");
        goto fail;
    }
    t->n_ctx = d[1];
    /* page-locked (library-side cudaMallocHost): the logits row then comes
     * back with one device-to-host copy and no staging memcpy */
    t->logits = fwb_host_alloc((size_t)c->n_vocab * sizeof(float));
    if (!t->logits) {
        fprintf(stderr, "transformer_init: working buffer allocation failed\n");
        goto fail;
    }
    return 0;

fail:
    transformer_free(t);
    return -1;
}

void transformer_free(transformer_t *t) {
    if (!t) return;
    fwb_model_close(t->dev);
    fwb_host_free(t->logits);
    tokenizer_free(t->tok);
    if (t->g.mapping) gguf_close(&t->g);  /* a zeroed struct holds no file (fd 0 is not ours) */
    memset(t, 0, sizeof(*t));
}

float *transformer_forward(transformer_t *t, uint32_t token_id, size_t pos) {
    if (!t->dev) return NULL;
    if (pos >= t->n_ctx) {
        fprintf(stderr, "transformer_forward: position exceeds KV cache\n");
        return NULL;
    }
    if (token_id >= t->cfg.n_vocab) {
        fprintf(stderr, "transformer_forward: token ID out of range\n");
        return NULL;
    }
    if (fwb_forward(t->dev, token_id, pos, t->logits) != 0) {
        fprintf(stderr, "transformer_forward: %s\n", fwb_last_error());
        return NULL;
    }
    return t->logits;
}
