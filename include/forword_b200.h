/*
 * forword_b200.h — C ABI of libforword_b200.so, the B200 (sm_100a) decode
 * path of forword.c.
 *
 * Plain C types only (pointers, sizes, ints).  Every function returns 0 on
 * success and -1 on failure (NULL for constructors), matching the reference's
 * error convention (transformer.c:156-164, quant_matvec.c:270-289); the
 * failure text is available from fwb_last_error().
 *
 * Threading: like the reference (single-threaded, non-reentrant), one model
 * handle must be used from one thread at a time.  Each model owns one CUDA
 * stream on its device.
 *
 * The drop-in entry points with the reference's own names
 * (transformer_init / transformer_forward / transformer_free) are in
 * forword.c_b200/shim/transformer_b200.c, which a maintainer compiles
 * together with forword.c's unchanged host C (gguf.c, model_config.c,
 * tokenizer.c, ...); it calls the fwb_* functions below.
 */
#ifndef FORWORD_B200_H
#define FORWORD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Text of the last error on this thread ("" if none).  Never NULL. */
const char *fwb_last_error(void);

/* Number of visible CUDA devices (0 when none). */
int fwb_device_count(void);

/* ------------------------------------------------------------------------
 * Quantised matrix-vector product.
 * ------------------------------------------------------------------------ */

/*
 * Replaces quant_matvec (quant_matvec.h:7-15, quant_matvec.c:263-312) with
 * the same signature and argument meaning: `weights` holds output_size rows
 * of GGUF blocks (row r at r * (input_size/32) * block_bytes), input[in] and
 * output[out] are host fp32 arrays.  The call copies weights and input to the
 * current device, runs the GEMV there and copies output back.
 * Types: 2 (Q4_0), 6 (Q5_0), 7 (Q5_1), 8 (Q8_0), 12 (Q4_K), 14 (Q6_K): the
 * reference's set (quant_matvec.c:52-62) plus GGML's Q4_0, which the
 * reference lacks.
 * Returns -1 for NULL pointers, zero sizes, an unsupported type,
 * input_size not a multiple of the block (32 values; 256 for Q4_K / Q6_K)
 * or weights_size < output_size * row bytes, like the reference.
 */
int quant_matvec(const void *weights, size_t weights_size, uint32_t ggml_type,
                 const float *input, float *output, size_t input_size,
                 size_t output_size);

/*
 * quant_matvec without any device allocation.  No counterpart in forword.c:
 * the reference's quant_matvec (quant_matvec.h:7-15) runs on the CPU; the
 * quant_matvec above keeps its signature but cudaMallocs and cudaFrees
 * device copies of weights, input and output on every call.  This variant
 * stages them in one fixed 32 MiB device array that is part of the library
 * (one per device), so a call makes no cudaMalloc, cudaFree or other
 * allocation.
 *
 * It is for callers that cannot allocate device memory at call time: a
 * process whose own memory pool (a framework's caching allocator, a serving
 * engine's KV-cache reservation) already holds the device's free memory, so
 * cudaMalloc fails or fragments it; and latency-bound loops, where the
 * implicit device-wide synchronisation of cudaFree would stall every other
 * stream of the process.
 *
 * Same arguments, element types and -1 cases as quant_matvec, and also -1,
 * with fwb_last_error() naming the bytes needed, when the call does not fit:
 * 4*input_size + the weight rows + 4*output_size + about 1 KB of alignment
 * must stay within 32 MiB (Q4_0 4096x4096 and 14336x4096 and Q8_0 4096x4096
 * fit; Q8_0 14336x4096 does not).  Synchronous, on the legacy default stream
 * of the current device.
 *
 * Set-up: the first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) and sets kernel attributes; make that first call
 * before any stream capture on that device.  Only the kernel's error word
 * (the array's first 4 bytes) must be zero when the kernel starts; each call
 * zeroes it before its launch.  All calls on a device share the array: calls
 * that overlap in time on one device (from different host threads) race and
 * corrupt each other's results, so serialise them.
 */
int quant_matvec_static(const void *weights, size_t weights_size, uint32_t ggml_type,
                        const float *input, float *output, size_t input_size,
                        size_t output_size);

/*
 * Device-pointer form of quant_matvec for callers whose data already lives
 * in HBM; no reference counterpart (quant_matvec.h:7-15 is host-only).
 * d_weights must be 2-byte aligned (4-byte for Q5_1, 16-byte for Q4_K).
 * The kernel copies 16-byte aligned
 * supersets of the rows: it reads from d_weights rounded down to 16 bytes
 * (inside the same allocation unless d_weights is 16-byte aligned, as
 * cudaMalloc pointers are) up to the 16-byte boundary at or after the last
 * row, and weights_size must reach that boundary (-1 otherwise).  d_input /
 * d_output are fp32 device arrays (d_input 16-byte aligned).  `stream` is a
 * cudaStream_t (NULL = legacy default stream).  Asynchronous: returns after
 * enqueueing; quant_device_status reports a kernel-side failure.
 */
int quant_matvec_dev(const void *d_weights, size_t weights_size, uint32_t ggml_type,
                     const float *d_input, float *d_output, size_t input_size,
                     size_t output_size, void *stream);

/*
 * Status of the last quant_matvec_dev / quant_gemm_dev launch on the current
 * device after the work queued on `stream` (synchronises it): 0 if the
 * kernel completed, -1 (fwb_last_error() names the device error word) if one
 * of its bounded waits ran out and part of the output was not written.  Each
 * launch clears the word on its own stream first, so launches overlapping on
 * different streams of one device share it.  No reference counterpart: the
 * reference's quant_matvec is synchronous CPU code.
 */
int quant_device_status(void *stream);

/*
 * Batched (prompt) form of quant_matvec_dev on the tensor cores:
 * output[m * output_size + o] = sum_k W[o][k] * input[m * input_size + k] for
 * m < n_tokens (or += with accumulate != 0).  d_input_f16 holds fp16
 * activations (16-byte aligned); the products are accumulated in fp32.  This
 * is the dense contraction of a prompt's tokens sharing each weight tile, the
 * batched counterpart of linear_forward (linear.c:155-223), which the
 * reference only runs one token at a time.  Only Q4_0 (type 2) with
 * input_size a multiple of 64; other cases return -1.  Asynchronous.
 */
int quant_gemm_dev(const void *d_weights, size_t weights_size, uint32_t ggml_type, const void *d_input_f16,
                   float *d_output, size_t input_size, size_t output_size, size_t n_tokens, int accumulate,
                   void *stream);

/*
 * Dequantise n_values (a multiple of the block) from Q4_0 / Q5_0 / Q5_1 /
 * Q8_0 / Q4_K / Q6_K blocks into fp32 on the device, bit-identical to the
 * reference decoders (quant.c: q5_1_decode, q8_0_decode, q4_k_decode,
 * q6_k_decode; q5_0 as linear.c:40-56; GGML's Q4_0).
 */
int quant_dequant_dev(const void *d_weights, size_t weights_size, uint32_t ggml_type,
                      float *d_out, size_t n_values, void *stream);

/* ------------------------------------------------------------------------
 * Decode model (transformer.h:39-48 semantics).
 * ------------------------------------------------------------------------ */

typedef struct fwb_model fwb_model_t;

/*
 * transformer_init (transformer.c:14-147): open a GGUF file, derive the
 * model configuration, clamp the KV length (max_ctx 0 -> min(n_ctx, 4096);
 * max_ctx > n_ctx -> n_ctx) and upload every tensor once to HBM in its GGUF
 * byte layout.  `device` selects the CUDA device.  NULL on failure.
 */
fwb_model_t *fwb_model_open(const char *gguf_path, size_t max_ctx, int device);

/* transformer_free (transformer.c:149-165).  NULL is accepted. */
void fwb_model_close(fwb_model_t *m);

/* dims[8] = n_vocab, kv_ctx, n_embd, n_layer, n_head, n_head_kv, n_ff, head_dim */
int fwb_model_dims(const fwb_model_t *m, uint32_t *dims);

/* Quantised bytes one decode step streams (weights + norms + one embedding row). */
uint64_t fwb_model_weight_bytes(const fwb_model_t *m);

/* Time (seconds) and bytes of the tensor upload fwb_model_open did: every
 * tensor (this rank's slice under tensor parallelism) copied from the GGUF
 * mapping through pinned staging buffers by parallel host threads, with the
 * copies to the device overlapped.  No reference counterpart: the reference
 * reads its mmap on every step (tensor_data.c:25-62). */
int fwb_model_load_stats(const fwb_model_t *m, double *seconds, uint64_t *bytes);

/* Kernels one decode step launches: 1 for the persistent decode kernel
 * (default), one per phase with FWB_KERNEL_PER_PHASE=1.  -1 for NULL. */
int fwb_model_kernels_per_step(const fwb_model_t *m);

/*
 * transformer_forward (transformer.c:149-326): feed token_id at position pos
 * and write n_vocab fp32 logits to logits_host (host memory; may be NULL to
 * skip the copy).  Errors as the reference: pos >= kv_ctx or
 * token_id >= n_vocab -> -1.  A bounded wait that ran out inside the step
 * also returns -1; on one GPU the next call starts clean, under tensor
 * parallelism the model must be closed and reopened on every rank.
 */
int fwb_forward(fwb_model_t *m, uint32_t token_id, size_t pos, float *logits_host);

/*
 * Prompt processing: feed tokens[0..n) at positions pos0..pos0+n-1, as n
 * calls of fwb_forward would (main.c:145-151 feeds a prompt that way), and
 * write the logits of the last token to logits_host (may be NULL).  The first
 * n-1 tokens go through every layer together: their linear layers run as
 * dequant-GEMMs on the tensor cores (see quant_gemm_dev) with fp16
 * activations, and their K/V rows are appended to the cache; the last token
 * takes the decode step.  Models whose layer weights are not all Q4_0 (or
 * with an input width that is not a multiple of 64, or head_dim > 128, or
 * tensor parallelism) take the decode step for every token.  Set
 * FWB_PREFILL_PER_TOKEN=1 to force that path.  -1 (with fwb_last_error()) for
 * positions beyond the KV cache or token ids beyond the vocabulary.
 */
int fwb_prefill(fwb_model_t *m, const uint32_t *tokens, size_t n, size_t pos0, float *logits_host);

/* Same step, returning only the greedy next token (sampler_argmax,
 * sampler.c:28-32: the lowest index among equal maxima). */
int fwb_forward_argmax(fwb_model_t *m, uint32_t token_id, size_t pos, uint32_t *next_token);

/*
 * Greedy decode of n_steps tokens entirely on the device: step i feeds the
 * token chosen by step i-1 (first_token for i = 0) at position pos0 + i.
 * tokens_out[i] receives the token chosen by step i.
 */
int fwb_generate_greedy(fwb_model_t *m, uint32_t first_token, size_t pos0, size_t n_steps,
                        uint32_t *tokens_out);

/*
 * Sample the next token from the logits of the last step without copying
 * them to the host: main.c:176-188 with sampler.c, on the device.  The
 * repetition penalty (sampler_rep_penalty, sampler.c:86-100) is applied for
 * every entry of history[0..n_history) (prompt and generated tokens, as
 * main.c keeps them); then temperature <= 0 gives the greedy argmax
 * (sampler_argmax), otherwise temperature, softmax and top-p sampling
 * (sampler_top_p, sampler.c:46-84) with one draw of the reference's
 * xorshift64 generator, whose state *rng_state advances exactly as the
 * reference's does (only when temperature > 0).  The nucleus and the draw
 * are found by radix selection with exact fixed-point sums instead of a
 * sort of the vocabulary and the reference's fp32 running sum; the token can
 * differ from the reference's only where the draw or top_p falls within that
 * sum's rounding drift of a cumulative probability boundary (about 1e-6 of
 * the total for a nucleus of thousands of tokens, far less for peaked
 * distributions).  Under tensor parallelism every rank makes the same call (the
 * other ranks' logits are read over NVLink).  Synchronous.
 */
int fwb_sample(fwb_model_t *m, const uint32_t *history, size_t n_history, float temperature, float top_p,
               float rep_penalty, uint64_t *rng_state, uint32_t *next_token);

/*
 * Write (load) or read K/V of n positions [pos0, pos0+n) of one layer.
 * k and v are host fp32 arrays [n][n_head_kv][head_dim] — the reference's
 * kv_cache row order (kv_cache.h:13,45-51).
 */
int fwb_kv_load(fwb_model_t *m, size_t layer, size_t pos0, size_t n, const float *k,
                const float *v);
int fwb_kv_read(fwb_model_t *m, size_t layer, size_t pos0, size_t n, float *k, float *v);

/*
 * Phase timeline of the last decode step of the persistent kernel (tracing
 * aid; open the model with FWB_TRACE=1 in the environment).  GPU global timer
 * (ns) seen by CTA 0: out[2i] at the start of phase i, out[2i+1] when it
 * reaches the barrier after phase i, out[2*n_phases] at the end.  names
 * (optional) gets one NUL-terminated phase name per name_stride bytes.
 * Returns 2*n_phases + 1, or -1.
 */
int fwb_trace_read(fwb_model_t *m, uint64_t *out, size_t n, char *names, size_t name_stride);

/*
 * Barrier arrival time (GPU global timer, ns) of every CTA after every phase
 * of the last step (FWB_TRACE=1): out[phase * n_sm + cta].  Shows which CTAs
 * a barrier waits for.  Returns n_phases * n_sm, or -1.
 */
int fwb_trace_cta_read(fwb_model_t *m, uint64_t *out, size_t n);

/*
 * Timeline of every CTA's attention work item in every layer of the last
 * step (FWB_TRACE=1): out[(layer * n_sm + cta) * 8 + i], GPU global timer (ns)
 * at i = 0 start, 1 its warp 0 done with its positions, 2 partial written,
 * 3 CTA barrier passed, 4 split ticket taken, 5 item done; 0 for CTAs without
 * an item.  Clears the record.  Returns n_layer * n_sm * 8, or -1.
 */
int fwb_trace_attn_read(fwb_model_t *m, uint64_t *out, size_t n);

/*
 * Accumulated GEMV profile of the persistent kernel since the last read
 * (FWB_TRACE=1), as seen by thread 0 of each CTA:
 * out[(phase * n_sm + cta) * 8 + i] = ns spent in i = 0 input prologue,
 * 1 waiting for the first weight stage, 2 row loop, 3 tail (loop end to phase
 * end); from the phase start to 4 the first input loads landing, 5 the input
 * planes' CTA barrier; 6 from its loop end until every warp's; 7 unused.
 * Resets the counters.  Returns the number of values written, or -1.
 */
int fwb_prof_read(fwb_model_t *m, uint64_t *out, size_t n);

/* ------------------------------------------------------------------------
 * Tensor parallelism across the GPUs of one box (no reference counterpart:
 * forword.c runs on one CPU).  One process and one model handle per GPU;
 * rank r of `world` (1..8) keeps its query/KV heads, its slice of the FFN and
 * of the vocabulary, and the matching input columns of attn_output and
 * ffn_down.  After o-proj and after down-proj the ranks' partial sums are
 * added together inside the persistent decode kernel, each rank reading the
 * others' partials over NVLink from their exchange buffers; every rank ends
 * the step with the same residual stream and the same greedy token.
 * ------------------------------------------------------------------------ */

/*
 * Open rank `rank` of a `world`-rank model on CUDA device `device`: uploads
 * only this rank's slices.  n_head, n_head_kv and n_vocab must divide by
 * world, and n_ff / world and (n_head / world) * head_dim must be multiples of
 * 32.  The model can decode only after fwb_tp_connect.
 */
fwb_model_t *fwb_model_open_tp(const char *gguf_path, size_t max_ctx, int device, int rank, int world);

/* 64-byte CUDA IPC handle of this rank's exchange buffer (send it to every rank). */
int fwb_tp_handle(fwb_model_t *m, void *handle64);

/*
 * Map every rank's exchange buffer: handles = world consecutive 64-byte
 * handles in rank order (this rank's own entry is ignored).  Builds the step.
 * Every rank must then call the same forward functions with the same tokens
 * and positions; a rank that stops leaves the others waiting until their
 * bounded waits expire (an error, not a hang).  fwb_forward on any rank
 * returns all n_vocab logits (the other ranks' slices are read over NVLink);
 * fwb_logits_dev returns this rank's slice only.
 */
int fwb_tp_connect(fwb_model_t *m, const void *handles);

/*
 * Host only (no GPU): the bytes rank `rank` of `world` keeps of tensor
 * `tensor` of a GGUF file, packed row-major in GGUF block layout.  as_head:
 * the tensor is used as the LM head (vocabulary-row split).  With out NULL
 * only *out_bytes is set.
 */
int fwb_tp_shard(const char *gguf_path, const char *tensor, int as_head, int rank, int world,
                 void *out, size_t cap, size_t *out_bytes);

/* Device logits of the last step (n_vocab fp32) and the model's CUDA stream. */
const float *fwb_logits_dev(fwb_model_t *m);
void *fwb_stream(fwb_model_t *m);

/*
 * Page-locked host memory (cudaMallocHost) for logits_host buffers: fwb_forward
 * then copies the logits straight into it, without the staging copy a pageable
 * buffer needs.  transformer_b200.c allocates transformer_t.logits this way
 * (the reference mallocs it, transformer.c:103-115).  NULL on failure;
 * fwb_host_free accepts NULL.
 */
void *fwb_host_alloc(size_t bytes);
void fwb_host_free(void *p);

#ifdef __cplusplus
}
#endif
#endif /* FORWORD_B200_H */
