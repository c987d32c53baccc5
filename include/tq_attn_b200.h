/*
 * tq_attn_b200.h -- drop-in replacement for the reference's Q8 attention entry points.
 *
 * libtq_attn_b200.so exports, with the reference's exact C signatures, the
 * functions of the reference files model/attention_layer.c, model/attn_q8.c and
 * model/kv_cache.c.  A caller of the reference (model/context.c,
 * tools/test_model.c, tools/bench_forward.c) links this library instead of those
 * three files and keeps every other reference file.  Q8 caches then run on the
 * B200 through libtqk.so (include/tqk.h); there is no CPU fallback for them.
 *
 * Symbols this library needs from the rest of the reference (left undefined,
 * resolved when the caller links): quantize_row_q8, get_matmul,
 * get_matmul_batch (kernel/), rmsnorm, rope_table, rope_apply, attention_head
 * (model/).  The F32 cache type stays on the reference's own F32 code
 * (attention_head, model/attention.c:35-44); only Q8 is the accelerated path.
 *
 * The struct definitions below restate the reference's types with identical
 * layout (packer/packer.h:7-12, kernel/kernel.h:6-9, model/model_ops.h:12-48,
 * :146-154) and are skipped when the reference's own headers were included first.
 */
#ifndef TQ_ATTN_B200_H
#define TQ_ATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TQ_B200_API __attribute__((visibility("default")))
#else
#define TQ_B200_API
#endif

#ifndef PACKER_H
#define QK 32
typedef struct { float d; int8_t q[QK]; } block_q8;   /* packer/packer.h:8 */
#endif

#ifndef KERNEL_H
typedef enum { TQ_FORMAT_Q8, TQ_FORMAT_Q4 } tq_format;  /* kernel/kernel.h:6-9 */
typedef void (*MatmulFn)(const void *W, const block_q8 *xq, float *y, int rows, int cols);
typedef void (*MatmulBatchFn)(const void *W, const block_q8 *xq, float *y, int rows, int cols, int n_tok);
void quantize_row_q8(const float *x, block_q8 *out, int n);
MatmulFn get_matmul(tq_format format);
MatmulBatchFn get_matmul_batch(tq_format format);
#endif

#ifndef TAILORQUANT_MODEL_OPS_H
typedef struct {                       /* model/model_ops.h:12-19 */
    int n_q_heads;
    int n_kv_heads;
    int head_dim;
    int hidden_size;
    float rope_theta;
    float rms_eps;
} tq_attn_config;

typedef struct {                       /* model/model_ops.h:21-26 */
    const void *data;
    tq_format format;
    int rows;
    int cols;
} tq_matrix;

typedef struct {                       /* model/model_ops.h:33-37 */
    tq_matrix wq, wk, wv, wo;
    const float *q_norm;
    const float *k_norm;
} tq_attn_weights;

typedef enum { TQ_KV_F32, TQ_KV_Q8 } tq_kv_type;   /* model/model_ops.h:39 */

typedef struct {                       /* model/model_ops.h:41-48 */
    tq_kv_type type;
    float *k_f32;
    float *v_f32;
    block_q8 *k_q8;
    block_q8 *v_q8;
    int max_tokens;
} tq_kv_cache;

typedef struct {                       /* model/model_ops.h:146-154 */
    int cap;
    float *x, *xn, *sub;
    float *gate, *up;
    float *q, *attn;
    float *k, *v;
    block_q8 *xq;
    block_q8 *hq;
} tq_batch_ws;

void rmsnorm(const float *x, const float *weight, float *out, int n, float eps);
void rope_table(float *cos_t, float *sin_t, int head_dim, int pos, float theta);
void rope_apply(float *x, int head_dim, const float *cos_t, const float *sin_t);
void attention_head(const float *q, const float *k_cache, const float *v_cache, int n, int head_dim, int stride,
                    float *scores, float *out);
#endif

/* ---- exported: the reference's entry points (same signatures, same error codes) ---- */

/* model/kv_cache.c:17-47 (model_ops.h:95): host planes as the reference allocates
 * them, plus a device-resident mirror on the current CUDA device for Q8. */
TQ_B200_API int tq_kv_cache_init(tq_kv_cache *cache, tq_kv_type type, const tq_attn_config *cfg, int max_tokens);
/* model/kv_cache.c:5-15 (model_ops.h:97): frees both. */
TQ_B200_API void tq_kv_cache_free(tq_kv_cache *cache);

/* model/attention_layer.c:10-36 (model_ops.h:123-124): codes -1..-9 as the reference. */
TQ_B200_API int tq_attn_validate(const tq_attn_weights *w, const tq_attn_config *cfg);
TQ_B200_API int tq_attn_validate_cache(const tq_kv_cache *cache);

/* model/attention_layer.c:169-194 (model_ops.h:119-121).  Returns -1 for pos
 * outside [0, max_tokens) before touching anything; a GPU failure returns a
 * tqk status (< -1) instead of aborting.  Every Q8 call ends by reading the
 * device's sticky error word in stream order: a kernel wait that gave up
 * (TQK_ETIMEOUT, -25) or a clamped device length (TQK_EDEVLEN, -27) is
 * returned, the word is cleared, the host cache planes are left without the
 * new rows and the device mirror is marked stale, so that calling again at
 * the same position recomputes from the host planes.  The same holds for
 * attention_layer_batch; the void entry points below report it through
 * tq_b200_last_status and fill their outputs with NaN. */
TQ_B200_API int attention_layer(const tq_attn_weights *w, const tq_attn_config *cfg, tq_kv_cache *cache, int pos,
                                const float *xn, float *scores, float *out);

/* model/attention_layer.c:200-243 (model_ops.h:160-162): causal chunk prefill;
 * the Q8 append + attention of all n tokens runs as one device call. */
TQ_B200_API int attention_layer_batch(const tq_attn_weights *w, const tq_attn_config *cfg, tq_kv_cache *cache,
                                      int pos0, int n, const float *xn, float *scores, float *out, tq_batch_ws *ws);

/* model/attn_q8.c:78-90 (model_ops.h:114-117): q_q8 receives the quantised q and
 * scores the softmax weights, as in the reference. */
TQ_B200_API void attention_head_q8(const float *q, block_q8 *q_q8, const block_q8 *k_cache,
                                   const block_q8 *v_cache, int n, int head_dim, float *scores, float *out);

/* model/attn_q8.c:56-76 (model_ops.h:174-178): the dispatchers, routed to the GPU. */
TQ_B200_API void attn_scores_q8(const block_q8 *q, int g, const block_q8 *k, int n, int nb, float scale,
                                float *scores, size_t stride);
TQ_B200_API void attn_accum_q8(const float *w, size_t w_stride, int g, const block_q8 *v, int n, int nb, float *out,
                               size_t out_stride);

/* ---- exported: drop-in control (no reference counterpart) ---- */

/* Device-resident attention layers.  Copies one layer's packed wq/wk/wv/wo rows
 * and q/k norm weights to the device and registers them under the caller's
 * tq_attn_weights (and the data pointers it holds now).  From then on
 * attention_layer and attention_layer_batch with these weights and a Q8 cache
 * run the whole layer on the B200 -- projections with the activation
 * quantisation, norm + RoPE, the Q8 append and attention, the output
 * projection (tqk_attention_layer / tqk_project) -- and move only xn, the RoPE
 * tables, the output and the appended cache rows across PCIe.  The host
 * weights must stay unchanged while registered (register again after changing
 * them).  All four matrices must share one format.  Returns 0, the
 * tq_attn_validate code of invalid weights, -10 for mixed formats, or a
 * negative status for a GPU failure.  A runtime calls it once per layer after
 * loading its weights. */
TQ_B200_API int tq_b200_register_attn_weights(const tq_attn_weights *w, const tq_attn_config *cfg);
/* Releases the device copy made for w (no-op when none). */
TQ_B200_API void tq_b200_unregister_attn_weights(const tq_attn_weights *w);

/* Status of the last drop-in call on this thread (0 = ok); the void entry points
 * report GPU failures here and fill their outputs with NaN. */
TQ_B200_API int tq_b200_last_status(void);
/* Marks a Q8 cache's device mirror stale: the next call re-uploads the host
 * planes.  Needed only after writing cache->k_q8 / v_q8 directly between calls. */
TQ_B200_API void tq_b200_cache_invalidate(const tq_kv_cache *cache);
/* Copies positions [0, n) of a Q8 cache's device mirror into its host planes. */
TQ_B200_API int tq_b200_cache_download(tq_kv_cache *cache, const tq_attn_config *cfg, int n);

#ifdef __cplusplus
}
#endif
#endif /* TQ_ATTN_B200_H */
