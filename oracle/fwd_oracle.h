/*
 * fwd_oracle.h — CPU restatement of forword.c's per-token decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load oracle/_build/liboracle.so as the checker; the
 * product library (forword.c_b200) never links or calls it.
 *
 * Every function restates a reference function, cited at its definition in
 * fwd_oracle.c.  Floating-point order follows the reference's AVX2+FMA build
 * of simd.h, so on the same GGUF file the restatement agrees with the compiled
 * reference to the last bit in practice (checked by tests/test_oracle.py).
 */
#ifndef FWD_ORACLE_H
#define FWD_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_model orc_model_t;

/* transformer_init / transformer_free / transformer_forward (transformer.h:39-48) */
int  orc_open(orc_model_t **out, const char *path, size_t max_ctx);
void orc_close(orc_model_t *m);
int  orc_forward(orc_model_t *m, uint32_t token, size_t pos, float *logits_out);

/* n_vocab n_ctx(kv) n_embd n_layer n_head n_head_kv n_ff head_dim */
void orc_dims(const orc_model_t *m, uint32_t *d);
/* KV rows for n positions of one layer, [n][n_head_kv][head_dim] fp32 */
int  orc_kv_write(orc_model_t *m, size_t layer, size_t pos0, size_t n,
                  const float *k, const float *v);
int  orc_kv_read(const orc_model_t *m, size_t layer, size_t pos0, size_t n,
                 float *k, float *v);

/* quant_matvec (quant_matvec.h:7-15) for Q4_0 / Q5_0 / Q8_0 */
int orc_quant_matvec(const void *w, size_t w_size, uint32_t type,
                     const float *x, float *y, size_t in, size_t out);
/* dequantize n_values (a multiple of 32) from Q4_0 / Q5_0 / Q8_0 blocks */
int orc_dequant(const void *w, size_t w_size, uint32_t type, float *out,
                size_t n_values);

float    orc_f16_to_f32(uint16_t h);
float    orc_dot(const float *a, const float *b, size_t n);
void     orc_rms_norm(const float *x, const float *w, float *out, size_t n, float eps);
void     orc_rope_tables(float *cos_tab, float *sin_tab, size_t n_ctx,
                         size_t head_dim, float freq_base);
void     orc_rope_apply(float *qk, size_t pos, size_t n_heads, size_t head_dim,
                        const float *cos_tab, const float *sin_tab);
uint32_t orc_argmax(const float *x, size_t n);

#ifdef __cplusplus
}
#endif
#endif
