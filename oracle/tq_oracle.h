/*
 * tq_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * Scalar CPU restatement of TailorQuantKernel's Q8 attention hot path, used as
 * the parity checker for the CUDA kernels in tailorquantkernel_b200/csrc.  Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load this
 * library; the product path never calls it.
 *
 * Every function cites the reference file:line whose arithmetic it restates.
 * Pinning: tests/test_oracle_pin.py compares this restatement bit-for-bit with
 * the reference's own scalar build (oracle/_ref/libtqref_scalar.so, compiled
 * from the reference sources by oracle/Makefile) and with the committed golden
 * fixtures under tests/golden/ that script generated from it.
 */
#ifndef TQ_ORACLE_H
#define TQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TQO_QK 32

/* Same 36-byte layout as the reference block_q8 (packer/packer.h:7-11). */
typedef struct { float d; int8_t q[TQO_QK]; } tqo_block_q8;
/* packer/packer.h:10 */
typedef struct { float d; uint8_t q[TQO_QK / 2]; } tqo_block_q4;

/* kernel/quant_x.c:5-34 */
void tqo_quantize_row_q8(const float *x, tqo_block_q8 *out, int n);
/* rows x n floats -> rows x (n/32) blocks */
void tqo_quantize_rows_q8(const float *x, tqo_block_q8 *out, int rows, int n);

/* model/softmax.c:4-23 */
void tqo_softmax(float *x, int n);

/* model/attn_q8.c:17-34 */
void tqo_attn_scores_q8(const tqo_block_q8 *q, int g, const tqo_block_q8 *k, int n, int nb,
                        float scale, float *scores, size_t stride);
/* model/attn_q8.c:36-54 */
void tqo_attn_accum_q8(const float *w, size_t w_stride, int g, const tqo_block_q8 *v, int n, int nb,
                       float *out, size_t out_stride);

/* model/attn_q8.c:78-90 */
void tqo_attention_head_q8(const float *q, tqo_block_q8 *q_q8, const tqo_block_q8 *k_cache,
                           const tqo_block_q8 *v_cache, int n, int head_dim, float *scores, float *out);

/* Q8 branch of store_kv, model/attention_layer.c:62-90.  Planes are
 * [n_kv][max_tokens][head_dim/32]; returns -1 when pos is out of range. */
int tqo_store_kv_q8(tqo_block_q8 *k_plane, tqo_block_q8 *v_plane, int n_kv, int head_dim,
                    int max_tokens, int pos, const float *k, const float *v);

/* attend_q8, model/attention_layer.c:125-150: GQA decode over n = pos+1 cached
 * tokens.  scores is an [n_q][max_tokens] workspace.  n_threads > 1 runs the
 * kv-head loop with OpenMP like the reference (only when n >= 256, :8,134). */
void tqo_attend_q8(const tqo_block_q8 *k_plane, const tqo_block_q8 *v_plane, int n_q, int n_kv,
                   int head_dim, int max_tokens, int pos, const float *q, float *scores, float *out,
                   int n_threads);

/* Chunked prefill semantics of attention_layer_batch, model/attention_layer.c:221-236:
 * for each of the n new tokens in order, store its k/v at pos0+i and attend with
 * its q over positions <= pos0+i.  q/out: [n][n_q*hd], k/v: [n][n_kv*hd]. */
int tqo_prefill_q8(tqo_block_q8 *k_plane, tqo_block_q8 *v_plane, int n_q, int n_kv, int head_dim,
                   int max_tokens, int pos0, int n, const float *q, const float *k, const float *v,
                   float *scores, float *out, int n_threads);

/* Float64 attention of one q head over dequantised data (the reference test's
 * attention_reference, tools/test_model.c:424-454), for tolerance checks. */
/* model/rmsnorm.c:4-19 */
void tqo_rmsnorm(const float *x, const float *weight, float *out, int n, float eps);
/* model/rope.c:4-12 */
void tqo_rope_table(float *cos_t, float *sin_t, int head_dim, int pos, float theta);
/* model/rope.c:14-22 */
void tqo_rope_apply(float *x, int head_dim, const float *cos_t, const float *sin_t);

/* packer/packer.c:4-88 (bit_type '8' or '4'); 0 or -1 like pack_matrix */
int tqo_pack_matrix(const float *W, int rows, int cols, void *out, char bit_type);
/* kernel/q8_scalar.c:3-22 */
void tqo_matmul_q8(const void *W, const tqo_block_q8 *xq, float *y, int rows, int cols);
/* kernel/q4_scalar.c:3-24 */
void tqo_matmul_q4(const void *W, const tqo_block_q8 *xq, float *y, int rows, int cols);

void tqo_attention_f64(const float *q, const float *k, const float *v, int n, int head_dim,
                       double *out);

#ifdef __cplusplus
}
#endif
#endif
