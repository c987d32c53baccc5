/*
 * ref_attend.c -- TEST/BASELINE INFRASTRUCTURE ONLY.
 *
 * A thin driver that runs the REFERENCE's own exported Q8 attention functions
 * (quantize_row_q8, attn_scores_q8, softmax, attn_accum_q8 from the reference
 * sources compiled by oracle/Makefile) in exactly the composition of the
 * reference's static attend_q8 (model/attention_layer.c:125-150) and store_kv
 * (model/attention_layer.c:62-90), which are not exported themselves.  It is
 * linked into oracle/_ref/libtqref_{scalar,avx2}.so and serves two purposes:
 *   - the bit-level pin of oracle/tq_oracle.c (scalar build), and
 *   - the timed CPU baseline of bench.py (AVX2 build, cpu_baseline.kind
 *     "reference"), with the reference's OpenMP parallelisation over kv heads.
 */
#include <math.h>
#include <stddef.h>
#include <string.h>

#include "kernel/kernel.h"
#include "model/model_ops.h"

#ifdef _OPENMP
#include <omp.h>
#endif

/* model/attention_layer.c:62-90 (Q8 branch), pos range checked like :68. */
int refdrv_store_kv_q8(block_q8 *k_plane, block_q8 *v_plane, int n_kv, int head_dim, int max_tokens,
                       int pos, const float *k, const float *v) {
    if (pos < 0 || pos >= max_tokens) return -1;
    const int nb = head_dim / QK;
    for (int h = 0; h < n_kv; h++) {
        const size_t slot = (size_t)h * (size_t)max_tokens + (size_t)pos;
        quantize_row_q8(k + (size_t)h * head_dim, k_plane + slot * nb, head_dim);
        quantize_row_q8(v + (size_t)h * head_dim, v_plane + slot * nb, head_dim);
    }
    return 0;
}

/* model/attention_layer.c:125-150, with the thread count made explicit. */
void refdrv_attend_q8(const block_q8 *k_plane, const block_q8 *v_plane, int n_q, int n_kv, int head_dim,
                      int max_tokens, int pos, const float *q, float *scores, float *out, int n_threads) {
    const int hd = head_dim;
    const int nb = hd / QK;
    const int n = pos + 1;
    const int group = n_q / n_kv;
    const float scale = 1.0f / sqrtf((float)hd);
    const size_t stride = (size_t)max_tokens;
    const int nt = n_threads > 0 ? n_threads : 1;
    (void)nt;

#pragma omp parallel for schedule(static) num_threads(nt) if (n >= 256 && nt > 1)
    for (int kvh = 0; kvh < n_kv; kvh++) {
        block_q8 qq[group * nb];
        const float *qg = q + (size_t)kvh * group * hd;
        float *og = out + (size_t)kvh * group * hd;
        float *sc = scores + (size_t)kvh * group * stride;
        const size_t slot0 = (size_t)kvh * (size_t)max_tokens;

        for (int g = 0; g < group; g++) quantize_row_q8(qg + (size_t)g * hd, qq + (size_t)g * nb, hd);
        attn_scores_q8(qq, group, k_plane + slot0 * nb, n, nb, scale, sc, stride);
        for (int g = 0; g < group; g++) softmax(sc + (size_t)g * stride, n);
        attn_accum_q8(sc, stride, group, v_plane + slot0 * nb, n, nb, og, (size_t)hd);
    }
}

/* Sequential per-token store + attend of attention_layer_batch
 * (model/attention_layer.c:221-236). */
int refdrv_prefill_q8(block_q8 *k_plane, block_q8 *v_plane, int n_q, int n_kv, int head_dim, int max_tokens,
                      int pos0, int n, const float *q, const float *k, const float *v, float *scores,
                      float *out, int n_threads) {
    if (n <= 0 || pos0 < 0 || pos0 + n > max_tokens) return -1;
    const size_t qd = (size_t)n_q * head_dim, kd = (size_t)n_kv * head_dim;
    for (int i = 0; i < n; i++) {
        refdrv_store_kv_q8(k_plane, v_plane, n_kv, head_dim, max_tokens, pos0 + i, k + i * kd, v + i * kd);
        refdrv_attend_q8(k_plane, v_plane, n_q, n_kv, head_dim, max_tokens, pos0 + i, q + i * qd, scores,
                         out + i * qd, n_threads);
    }
    return 0;
}

/* quantize_row_q8 (kernel/quant_x.c:12) over `rows` rows of n floats. */
void refdrv_quantize_rows(const float *x, block_q8 *out, int rows, int n) {
    for (int r = 0; r < rows; r++) quantize_row_q8(x + (size_t)r * n, out + (size_t)r * (n / QK), n);
}

int refdrv_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
