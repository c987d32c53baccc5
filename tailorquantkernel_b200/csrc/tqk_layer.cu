// tqk_layer.cu -- one attention layer for one token on the device
// (attention_layer, reference model/attention_layer.c:169-194):
//   project_qkv      tqk_project: quantise xn, q/k/v matmuls      (:38-46, :180)
//   norm + rope      fused into the decode's q load and K append  (:48-60, :182-188)
//   store_kv+attend  the fused decode                              (:66-90, :125-150, :190-191)
//   project_output   tqk_project: quantise the attention, wo      (:161-167, :192)
// Three launches, each with programmatic stream serialization: every kernel
// waits for its predecessors before it reads their results and lets its
// successor start right after, so the next matmul's weight prefetch overlaps
// the running kernel.
#include "tqk_internal.h"

using namespace tqk;

extern "C" int tqk_attention_layer(const tqk_attn_layer_args *a, void *workspace, size_t workspace_bytes,
                                   tqk_stream_t stream) {
    if (!a) return fail(TQK_EINVAL, "tqk_attention_layer: NULL args");
    if (a->n_q_heads <= 0 || a->n_kv_heads <= 0 || a->head_dim <= 0 || a->hidden_size <= 0 || a->max_tokens <= 0)
        return fail(TQK_EINVAL, "tqk_attention_layer: non-positive shape");
    if (a->pos < 0 || a->pos >= a->max_tokens) return fail(TQK_EPOS, "tqk_attention_layer: position out of range");
    if (!a->wq || !a->wk || !a->wv || !a->wo || !a->q_norm || !a->k_norm || !a->k || !a->v || !a->rope_cos ||
        !a->rope_sin || !a->xn || !a->out || !a->scratch)
        return fail(TQK_EINVAL, "tqk_attention_layer: NULL pointer");
    if (a->hidden_size % QK || a->head_dim % QK || a->n_q_heads % a->n_kv_heads)
        return fail(TQK_EINVAL, "tqk_attention_layer: shape (hidden and head_dim multiples of 32, GQA grouping)");
    const int q_dim = a->n_q_heads * a->head_dim, kv_dim = a->n_kv_heads * a->head_dim;
    float *q = a->scratch, *k = q + q_dim, *v = k + kv_dim, *attn = v + kv_dim;

    // project_qkv: the three matrices share one launch and one quantisation of xn
    const tqk_proj_job qkv[3] = {{a->wq, q, q_dim}, {a->wk, k, kv_dim}, {a->wv, v, kv_dim}};
    int rc = tqk_project(qkv, 3, a->format, a->xn, a->hidden_size, 1, stream);
    if (rc) return rc;

    // norm_heads + rope_heads + store_kv + attend_q8 in one decode launch
    tqk_decode_args d{};
    d.k = a->k;
    d.v = a->v;
    d.n_items = 1;
    d.n_q_heads = a->n_q_heads;
    d.n_kv_heads = a->n_kv_heads;
    d.head_dim = a->head_dim;
    d.max_tokens = a->max_tokens;
    if (a->len) {
        d.lens = a->len;
        d.max_len = a->pos + 1;
    } else {
        d.len0 = a->pos + 1;
    }
    d.q = q;
    d.out = attn;
    d.k_new = k;
    d.v_new = v;
    d.out_mode = TQK_OUT_NORMALIZED;
    d.q_norm = a->q_norm;
    d.k_norm = a->k_norm;
    d.norm_eps = a->rms_eps;
    d.rope_cos = a->rope_cos;
    d.rope_sin = a->rope_sin;
    rc = tqk_decode_q8(&d, workspace, workspace_bytes, stream);
    if (rc) return rc;

    // project_output
    const tqk_proj_job o = {a->wo, a->out, a->hidden_size};
    return tqk_project(&o, 1, a->format, attn, q_dim, 1, stream);
}
