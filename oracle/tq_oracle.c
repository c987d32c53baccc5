/*
 * tq_oracle.c -- TEST INFRASTRUCTURE ONLY (see tq_oracle.h).
 *
 * Scalar restatement of the reference's Q8 attention arithmetic.  It must be
 * compiled exactly like the reference's scalar objects: no FMA contraction
 * (-ffp-contract=off, no -mfma / -march=native), IEEE division and sqrt, so
 * that the quantiser and the score arithmetic round like the reference does.
 */
#include "tq_oracle.h"

#include <math.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* kernel/quant_x.c:5-10: adding 1.5*2^23 puts the rounded integer into the low
 * mantissa bits (round-half-to-even for |v| < 2^22); the int8 is the low byte of
 * the difference of bit patterns, truncated like the reference's cast. */
static int8_t tqo_round_to_int8(float v) {
    float shifted = v + 12582912.0f;
    int32_t bits;
    memcpy(&bits, &shifted, sizeof bits);
    return (int8_t)(bits - 0x4B400000);
}

/* kernel/quant_x.c:12-34: per 32-element block, scale = max|x| / 127 (NaN never
 * wins the max because the comparison is false), inverse 0 for a zero scale. */
void tqo_quantize_row_q8(const float *x, tqo_block_q8 *out, int n) {
    const int nb = n / TQO_QK;
    for (int b = 0; b < nb; b++) {
        const float *xb = x + (size_t)b * TQO_QK;
        float amax = 0.0f;
        for (int j = 0; j < TQO_QK; j++) {
            float a = xb[j];
            if (a < 0) a = -a;
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float inv = (d != 0.0f) ? 1.0f / d : 0.0f;
        out[b].d = d;
        for (int j = 0; j < TQO_QK; j++) out[b].q[j] = tqo_round_to_int8(xb[j] * inv);
    }
}

void tqo_quantize_rows_q8(const float *x, tqo_block_q8 *out, int rows, int n) {
    const int nb = n / TQO_QK;
    for (int r = 0; r < rows; r++) tqo_quantize_row_q8(x + (size_t)r * n, out + (size_t)r * nb, n);
}

/* model/softmax.c:4-23: max, exp(x - max) with a running float sum, then a
 * multiply by the float reciprocal of the sum. */
void tqo_softmax(float *x, int n) {
    if (n <= 0) return;
    float m = x[0];
    for (int i = 1; i < n; i++) if (x[i] > m) m = x[i];
    float s = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - m);
        s += x[i];
    }
    const float r = 1.0f / s;
    for (int i = 0; i < n; i++) x[i] *= r;
}

/* model/attn_q8.c:17-34: exact int32 block dot, then acc += (float)dot * (qd*kd)
 * in block order, finally acc * scale. */
void tqo_attn_scores_q8(const tqo_block_q8 *q, int g, const tqo_block_q8 *k, int n, int nb,
                        float scale, float *scores, size_t stride) {
    for (int t = 0; t < n; t++) {
        const tqo_block_q8 *kr = k + (size_t)t * nb;
        for (int h = 0; h < g; h++) {
            const tqo_block_q8 *qr = q + (size_t)h * nb;
            float acc = 0.0f;
            for (int b = 0; b < nb; b++) {
                int32_t dot = 0;
                for (int j = 0; j < TQO_QK; j++) dot += (int32_t)qr[b].q[j] * (int32_t)kr[b].q[j];
                const float dd = qr[b].d * kr[b].d;
                acc += (float)dot * dd;
            }
            scores[(size_t)h * stride + t] = acc * scale;
        }
    }
}

/* model/attn_q8.c:36-54: out[h][b*32+j] = sum_t (w[h][t] * vd[t][b]) * vq[t][b][j],
 * accumulated in token order after zeroing the head_dim outputs. */
void tqo_attn_accum_q8(const float *w, size_t w_stride, int g, const tqo_block_q8 *v, int n, int nb,
                       float *out, size_t out_stride) {
    const int hd = nb * TQO_QK;
    for (int h = 0; h < g; h++) {
        float *o = out + (size_t)h * out_stride;
        for (int j = 0; j < hd; j++) o[j] = 0.0f;
        for (int t = 0; t < n; t++) {
            const float wt = w[(size_t)h * w_stride + t];
            const tqo_block_q8 *vr = v + (size_t)t * nb;
            for (int b = 0; b < nb; b++) {
                const float f = wt * vr[b].d;
                for (int j = 0; j < TQO_QK; j++) o[b * TQO_QK + j] += f * (float)vr[b].q[j];
            }
        }
    }
}

/* model/attn_q8.c:78-90 */
void tqo_attention_head_q8(const float *q, tqo_block_q8 *q_q8, const tqo_block_q8 *k_cache,
                           const tqo_block_q8 *v_cache, int n, int head_dim, float *scores, float *out) {
    const int nb = head_dim / TQO_QK;
    const float scale = 1.0f / sqrtf((float)head_dim);
    tqo_quantize_row_q8(q, q_q8, head_dim);
    tqo_attn_scores_q8(q_q8, 1, k_cache, n, nb, scale, scores, (size_t)n);
    tqo_softmax(scores, n);
    tqo_attn_accum_q8(scores, (size_t)n, 1, v_cache, n, nb, out, (size_t)head_dim);
}

/* model/attention_layer.c:62-90 (Q8 case): slot = h*max_tokens + pos. */
int tqo_store_kv_q8(tqo_block_q8 *k_plane, tqo_block_q8 *v_plane, int n_kv, int head_dim,
                    int max_tokens, int pos, const float *k, const float *v) {
    if (pos < 0 || pos >= max_tokens) return -1;
    const int nb = head_dim / TQO_QK;
    for (int h = 0; h < n_kv; h++) {
        const size_t slot = (size_t)h * (size_t)max_tokens + (size_t)pos;
        tqo_quantize_row_q8(k + (size_t)h * head_dim, k_plane + slot * nb, head_dim);
        tqo_quantize_row_q8(v + (size_t)h * head_dim, v_plane + slot * nb, head_dim);
    }
    return 0;
}

/* One kv head of attend_q8 (model/attention_layer.c:136-149). */
static void tqo_attend_kv_head(const tqo_block_q8 *k_plane, const tqo_block_q8 *v_plane, int kvh,
                               int group, int head_dim, int max_tokens, int n, float scale,
                               const float *q, float *scores, float *out) {
    const int nb = head_dim / TQO_QK;
    tqo_block_q8 qq[64 * 8]; /* group * nb blocks; group <= 64 and head_dim <= 256 */
    const float *qg = q + (size_t)kvh * group * head_dim;
    float *og = out + (size_t)kvh * group * head_dim;
    float *sc = scores + (size_t)kvh * group * max_tokens;
    const size_t slot0 = (size_t)kvh * (size_t)max_tokens;
    for (int g = 0; g < group; g++) tqo_quantize_row_q8(qg + (size_t)g * head_dim, qq + (size_t)g * nb, head_dim);
    tqo_attn_scores_q8(qq, group, k_plane + slot0 * nb, n, nb, scale, sc, (size_t)max_tokens);
    for (int g = 0; g < group; g++) tqo_softmax(sc + (size_t)g * max_tokens, n);
    tqo_attn_accum_q8(sc, (size_t)max_tokens, group, v_plane + slot0 * nb, n, nb, og, (size_t)head_dim);
}

/* model/attention_layer.c:125-150 */
void tqo_attend_q8(const tqo_block_q8 *k_plane, const tqo_block_q8 *v_plane, int n_q, int n_kv,
                   int head_dim, int max_tokens, int pos, const float *q, float *scores, float *out,
                   int n_threads) {
    const int n = pos + 1;
    const int group = n_q / n_kv;
    const float scale = 1.0f / sqrtf((float)head_dim);
#ifdef _OPENMP
    const int par = (n_threads > 1 && n >= 256);
#pragma omp parallel for schedule(static) num_threads(n_threads > 1 ? n_threads : 1) if (par)
#endif
    for (int kvh = 0; kvh < n_kv; kvh++)
        tqo_attend_kv_head(k_plane, v_plane, kvh, group, head_dim, max_tokens, n, scale, q, scores, out);
    (void)n_threads;
}

/* model/attention_layer.c:221-236: per new token, in order, store then attend. */
int tqo_prefill_q8(tqo_block_q8 *k_plane, tqo_block_q8 *v_plane, int n_q, int n_kv, int head_dim,
                   int max_tokens, int pos0, int n, const float *q, const float *k, const float *v,
                   float *scores, float *out, int n_threads) {
    if (n <= 0 || pos0 < 0 || pos0 + n > max_tokens) return -1;
    const size_t qd = (size_t)n_q * head_dim, kd = (size_t)n_kv * head_dim;
    for (int i = 0; i < n; i++) {
        tqo_store_kv_q8(k_plane, v_plane, n_kv, head_dim, max_tokens, pos0 + i, k + i * kd, v + i * kd);
        tqo_attend_q8(k_plane, v_plane, n_q, n_kv, head_dim, max_tokens, pos0 + i, q + i * qd, scores,
                      out + i * qd, n_threads);
    }
    return 0;
}

/* tools/test_model.c:424-454: float64 softmax attention over float inputs. */
void tqo_attention_f64(const float *q, const float *k, const float *v, int n, int head_dim,
                       double *out) {
    const double scale = 1.0 / sqrt((double)head_dim);
    double m = -INFINITY;
    for (int t = 0; t < n; t++) {
        double s = 0.0;
        for (int j = 0; j < head_dim; j++) s += (double)q[j] * (double)k[(size_t)t * head_dim + j];
        s *= scale;
        if (s > m) m = s;
    }
    double l = 0.0;
    for (int j = 0; j < head_dim; j++) out[j] = 0.0;
    for (int t = 0; t < n; t++) {
        double s = 0.0;
        for (int j = 0; j < head_dim; j++) s += (double)q[j] * (double)k[(size_t)t * head_dim + j];
        const double p = exp(s * scale - m);
        l += p;
        for (int j = 0; j < head_dim; j++) out[j] += p * (double)v[(size_t)t * head_dim + j];
    }
    for (int j = 0; j < head_dim; j++) out[j] /= l;
}

/* model/rmsnorm.c:4-19: sum of squares in index order, sqrtf(eps + sum/n),
 * out = x * (1/rms) * w. */
void tqo_rmsnorm(const float *x, const float *weight, float *out, int n, float eps) {
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum += x[i] * x[i];
    const float inv_rms = 1.0f / sqrtf(eps + sum / (float)n);
    for (int i = 0; i < n; i++) out[i] = x[i] * inv_rms * weight[i];
}

/* model/rope.c:4-12: freq = theta^(-2i/head_dim), angle = pos * freq. */
void tqo_rope_table(float *cos_t, float *sin_t, int head_dim, int pos, float theta) {
    const float inv_head_dim = 1.0f / (float)head_dim;
    for (int i = 0; i < head_dim / 2; i++) {
        const float freq = powf(theta, -2.0f * i * inv_head_dim);
        const float a = pos * freq;
        cos_t[i] = cosf(a);
        sin_t[i] = sinf(a);
    }
}

/* model/rope.c:14-22: rotate (x[i], x[i+half]) by the table. */
void tqo_rope_apply(float *x, int head_dim, const float *cos_t, const float *sin_t) {
    const int half = head_dim / 2;
    for (int i = 0; i < half; i++) {
        const float x0 = x[i], x1 = x[i + half];
        x[i] = x0 * cos_t[i] - x1 * sin_t[i];
        x[i + half] = x0 * sin_t[i] + x1 * cos_t[i];
    }
}

/* ---------------------------------------------------------------------------
 * Weight packing and the projections' matrix-vector products.
 * ------------------------------------------------------------------------- */

/* packer/packer.c:4-9: round half away from zero, clamp to +-qmax. */
static int tqo_pack_round(float x, float inv, int qmax) {
    int q = (int)lroundf(x * inv);
    return q > qmax ? qmax : q < -qmax ? -qmax : q;
}

/* packer/packer.c:11-19: max |w| / qmax over the block, 1.0 for an all-zero block. */
static float tqo_pack_scale(const float *w, float qmax) {
    float amax = 0.0f;
    for (int j = 0; j < TQO_QK; j++) {
        const float a = fabsf(w[j]);
        if (a > amax) amax = a;
    }
    const float d = amax / qmax;
    return d == 0.0f ? 1.0f : d;
}

/* packer/packer.c:22-33 (Q8), 40-53 (Q4: element j in the low nibble and j+16 in the
 * high nibble of byte j, both offset by 8), 63-88 (row bytes, whole matrix). */
int tqo_pack_matrix(const float *W, int rows, int cols, void *out, char bit_type) {
    if (cols <= 0 || cols % TQO_QK != 0 || rows <= 0 || (bit_type != '8' && bit_type != '4')) return -1;
    const int nb = cols / TQO_QK;
    uint8_t *dst = (uint8_t *)out;
    for (int r = 0; r < rows; r++) {
        for (int b = 0; b < nb; b++) {
            const float *w = W + (size_t)r * cols + (size_t)b * TQO_QK;
            if (bit_type == '8') {
                tqo_block_q8 *o = (tqo_block_q8 *)dst + (size_t)r * nb + b;
                const float d = tqo_pack_scale(w, 127.0f), inv = 1.0f / d;
                o->d = d;
                for (int j = 0; j < TQO_QK; j++) o->q[j] = (int8_t)tqo_pack_round(w[j], inv, 127);
            } else {
                tqo_block_q4 *o = (tqo_block_q4 *)dst + (size_t)r * nb + b;
                const float d = tqo_pack_scale(w, 7.0f), inv = 1.0f / d;
                o->d = d;
                for (int j = 0; j < TQO_QK / 2; j++) {
                    const int lo = tqo_pack_round(w[j], inv, 7) + 8;
                    const int hi = tqo_pack_round(w[j + TQO_QK / 2], inv, 7) + 8;
                    o->q[j] = (uint8_t)((hi << 4) | lo);
                }
            }
        }
    }
    return 0;
}

/* kernel/q8_scalar.c:3-22: y[r] = sum over blocks, in block order, of
 * (float)(int dot of the int8 values) * w.d * x.d, rounded left to right. */
void tqo_matmul_q8(const void *W, const tqo_block_q8 *xq, float *y, int rows, int cols) {
    const int nb = cols / TQO_QK;
    const tqo_block_q8 *w = (const tqo_block_q8 *)W;
    for (int r = 0; r < rows; r++) {
        const tqo_block_q8 *wr = w + (size_t)r * nb;
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            int32_t s = 0;
            for (int j = 0; j < TQO_QK; j++) s += (int32_t)wr[b].q[j] * xq[b].q[j];
            sum += (float)s * wr[b].d * xq[b].d;
        }
        y[r] = sum;
    }
}

/* kernel/q4_scalar.c:3-24: as tqo_matmul_q8 with the Q4 nibbles (value - 8) paired
 * with x[j] (low) and x[j + 16] (high). */
void tqo_matmul_q4(const void *W, const tqo_block_q8 *xq, float *y, int rows, int cols) {
    const int nb = cols / TQO_QK;
    const tqo_block_q4 *w = (const tqo_block_q4 *)W;
    for (int r = 0; r < rows; r++) {
        const tqo_block_q4 *wr = w + (size_t)r * nb;
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            int32_t s = 0;
            for (int j = 0; j < TQO_QK / 2; j++) {
                const int lo = (wr[b].q[j] & 0x0F) - 8, hi = (wr[b].q[j] >> 4) - 8;
                s += lo * xq[b].q[j] + hi * xq[b].q[j + TQO_QK / 2];
            }
            sum += (float)s * wr[b].d * xq[b].d;
        }
        y[r] = sum;
    }
}
