/*
 * tq_attn_b200.c -- plain-C drop-in for the reference's attention entry points
 * (include/tq_attn_b200.h), built into libtq_attn_b200.so over libtqk.so.
 *
 * The reference keeps its KV cache in host memory that callers own and read
 * (model/kv_cache.c:33-39; tools/test_model.c:842-850,1118-1126).  This library
 * keeps a device-resident mirror of every Q8 cache in HBM, keyed by the host
 * planes, and runs the append and the attention there:
 *
 *   - a call at position pos when the mirror already holds [0, pos) sends only
 *     the new q/k/v vectors (pinned staging, one H2D copy), runs the fused
 *     append+attention kernel, and copies back the attention output plus the
 *     2*n_kv appended rows, which it writes into the host planes so the host
 *     cache stays byte-identical to the reference's;
 *   - any other position (a rewound or fresh context, or a cache the caller
 *     filled itself) first uploads the host rows [0, pos) of every kv head.
 *
 * The layer steps around the hot path -- projections, per-head RMS norm, RoPE,
 * output projection -- are the reference's own exported functions, called in
 * the order of model/attention_layer.c:169-194 and :200-243.  The F32 cache
 * type is not the accelerated path and stays on the reference's F32 kernel
 * (attention_head, model/attention.c:35-44).  There is no CPU path for Q8.
 */
#include "../../../include/tq_attn_b200.h"
#include "../../../include/tqk.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

_Static_assert(sizeof(block_q8) == 36, "block_q8 must match the reference's 36-byte layout");
_Static_assert(sizeof(block_q8) == sizeof(tqk_block_q8), "block_q8 and tqk_block_q8 differ");

#define TQB_ECUDA (-23)  /* = TQK_ECUDA */

typedef struct mirror {
    const void *key_k, *key_v;  /* the host planes this mirror shadows */
    int n_kv, head_dim, max_tokens, device;
    tqk_block_q8 *dk, *dv;      /* device planes [n_kv][max_tokens][nb] */
    int synced;                 /* positions [0, synced) identical on host and device; -1 = unknown */
    unsigned char *last_rows;   /* the K then V rows of every kv head this library last wrote to the
                                   host planes, at position synced - 1: a caller who rewrites them
                                   between calls is noticed (tq_b200_cache_invalidate covers the rest) */
    struct mirror *next;
} mirror;

/* One layer's attention weights copied to the device by
 * tq_b200_register_attn_weights, keyed by the caller's tq_attn_weights and the
 * host data pointers it held at registration. */
typedef struct wreg {
    const tq_attn_weights *key;
    const void *src[4];          /* wq, wk, wv, wo data at registration */
    const float *src_norm[2];    /* q_norm, k_norm at registration */
    int device, format, hd;
    void *dw[4];                 /* device packed rows */
    float *dnorm[2];             /* device q_norm, k_norm */
    struct wreg *next;
} wreg;

static struct {
    int ready;
    int device;
    cudaStream_t stream;
    void *dscratch;
    size_t dscratch_bytes;
    void *hstage;
    size_t hstage_bytes;
    mirror *mirrors;
    wreg *wregs;
    int *herr;   /* pinned host copy of the device error word */
} G;

static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static __thread int t_status = 0;

static int set_status(int s) {
    t_status = s;
    return s;
}

static int cuda_fail(cudaError_t e, const char *what) {
    fprintf(stderr, "tq_attn_b200: %s: %s\n", what, cudaGetErrorString(e));
    return set_status(TQB_ECUDA);
}

static int tqk_fail(int rc, const char *what) {
    fprintf(stderr, "tq_attn_b200: %s: %s (%s)\n", what, tqk_status_string(rc), tqk_last_error());
    return set_status(rc);
}

#define CU(call, what)                               \
    do {                                             \
        cudaError_t e_ = (call);                     \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

/* Lazily binds the process to one CUDA device (TQ_B200_DEVICE, default the
 * current one) and creates the stream all drop-in work runs on. */
static int ctx_ready(void) {
    if (G.ready) return 0;
    int dev = 0;
    const char *env = getenv("TQ_B200_DEVICE");
    if (env) {
        dev = atoi(env);
        CU(cudaSetDevice(dev), "cudaSetDevice");
    } else {
        CU(cudaGetDevice(&dev), "cudaGetDevice");
    }
    CU(cudaStreamCreateWithFlags(&G.stream, cudaStreamNonBlocking), "cudaStreamCreate");
    CU(cudaHostAlloc((void **)&G.herr, sizeof(int), cudaHostAllocDefault), "cudaHostAlloc");
    *G.herr = 0;
    G.device = dev;
    G.ready = 1;
    return 0;
}

/* Ends a call's queued work: enqueues the read of the device error word behind
 * it, synchronises the stream and maps a recorded device failure (a bounded
 * wait that gave up, a clamped length) to its negative status, clearing the
 * word so that the next call starts clean.  Returns 0 when the call's results
 * can be used.  The word is per device, so a failure that another stream's
 * kernel recorded before this call's work finished is reported here too. */
static int finish(const char *what) {
    int rc = tqk_device_status_async(G.herr, G.stream);
    if (rc) return tqk_fail(rc, what);
    CU(cudaStreamSynchronize(G.stream), what);
    const int word = *G.herr;
    if (word) {
        int dummy = 0;
        tqk_device_status(&dummy, 1);
        *G.herr = 0;
        return tqk_fail(tqk_device_error_status(word), what);
    }
    return 0;
}

static int use_device(void) {
    int rc = ctx_ready();
    if (rc) return rc;
    CU(cudaSetDevice(G.device), "cudaSetDevice");
    return 0;
}

static void *dev_scratch(size_t bytes) {
    if (bytes <= G.dscratch_bytes) return G.dscratch;
    if (G.dscratch) {
        cudaStreamSynchronize(G.stream);
        cudaFree(G.dscratch);
        G.dscratch = NULL;
        G.dscratch_bytes = 0;
    }
    size_t want = bytes < ((size_t)4 << 20) ? ((size_t)4 << 20) : bytes;
    if (cudaMalloc(&G.dscratch, want) != cudaSuccess) return NULL;
    G.dscratch_bytes = want;
    return G.dscratch;
}

static void *host_stage(size_t bytes) {
    if (bytes <= G.hstage_bytes) return G.hstage;
    if (G.hstage) {
        cudaStreamSynchronize(G.stream);
        cudaFreeHost(G.hstage);
        G.hstage = NULL;
        G.hstage_bytes = 0;
    }
    size_t want = bytes < ((size_t)4 << 20) ? ((size_t)4 << 20) : bytes;
    if (cudaHostAlloc(&G.hstage, want, cudaHostAllocDefault) != cudaSuccess) return NULL;
    G.hstage_bytes = want;
    return G.hstage;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

/* ---------------------------------------------------------------------------
 * device mirrors of Q8 caches
 * ------------------------------------------------------------------------- */
static void mirror_release(mirror *m) {
    if (!m) return;
    cudaFree(m->dk);
    cudaFree(m->dv);
    free(m->last_rows);
    free(m);
}

/* The host rows at position pos of every kv head, K then V, into dst (or compared with it). */
static int rows_at(const mirror *m, const tq_kv_cache *cache, int pos, unsigned char *dst, int compare) {
    const size_t row = (size_t)(m->head_dim / QK) * sizeof(block_q8);
    for (int plane = 0; plane < 2; plane++) {
        const unsigned char *base = (const unsigned char *)(plane ? cache->v_q8 : cache->k_q8);
        for (int h = 0; h < m->n_kv; h++) {
            const unsigned char *src = base + ((size_t)h * m->max_tokens + pos) * row;
            unsigned char *d = dst + ((size_t)plane * m->n_kv + h) * row;
            if (compare) {
                if (memcmp(d, src, row) != 0) return 1;
            } else {
                memcpy(d, src, row);
            }
        }
    }
    return 0;
}

/* After a call wrote rows [.., pos] into the host planes: remember row pos. */
static void mirror_note_written(mirror *m, const tq_kv_cache *cache, int pos) {
    if (m->last_rows) rows_at(m, cache, pos, m->last_rows, 0);
}

static mirror *mirror_find(const void *kk, const void *vv) {
    for (mirror *m = G.mirrors; m; m = m->next)
        if (m->key_k == kk && m->key_v == vv) return m;
    return NULL;
}

static void mirror_drop(const void *kk, const void *vv) {
    mirror **pp = &G.mirrors;
    while (*pp) {
        if ((*pp)->key_k == kk && (*pp)->key_v == vv) {
            mirror *dead = *pp;
            *pp = dead->next;
            if (G.ready) cudaStreamSynchronize(G.stream);
            mirror_release(dead);
            return;
        }
        pp = &(*pp)->next;
    }
}

static int mirror_get(const tq_kv_cache *cache, const tq_attn_config *cfg, mirror **out) {
    mirror *m = mirror_find(cache->k_q8, cache->v_q8);
    if (m && (m->n_kv != cfg->n_kv_heads || m->head_dim != cfg->head_dim || m->max_tokens != cache->max_tokens ||
              m->device != G.device)) {
        mirror_drop(cache->k_q8, cache->v_q8);
        m = NULL;
    }
    if (!m) {
        m = (mirror *)calloc(1, sizeof *m);
        if (!m) return set_status(-1);
        const size_t bytes = (size_t)cfg->n_kv_heads * cache->max_tokens * (cfg->head_dim / QK) * sizeof(block_q8);
        if (cudaMalloc((void **)&m->dk, bytes) != cudaSuccess || cudaMalloc((void **)&m->dv, bytes) != cudaSuccess) {
            mirror_release(m);
            return cuda_fail(cudaErrorMemoryAllocation, "mirror allocation");
        }
        m->key_k = cache->k_q8;
        m->key_v = cache->v_q8;
        m->n_kv = cfg->n_kv_heads;
        m->head_dim = cfg->head_dim;
        m->max_tokens = cache->max_tokens;
        m->device = G.device;
        m->synced = -1;
        m->last_rows = (unsigned char *)malloc((size_t)2 * cfg->n_kv_heads * (cfg->head_dim / QK) * sizeof(block_q8));
        m->next = G.mirrors;
        G.mirrors = m;
    }
    *out = m;
    return 0;
}

/* Makes device rows [0, pos) of every kv head equal to the host's.  A mirror that
 * holds [0, pos) already is trusted unless the host's row pos - 1 no longer holds
 * what this library wrote there. */
static int mirror_sync_prefix(mirror *m, const tq_kv_cache *cache, int pos) {
    if (m->synced == pos && (pos == 0 || !m->last_rows || !rows_at(m, cache, pos - 1, m->last_rows, 1))) return 0;
    const size_t row = (size_t)(m->head_dim / QK) * sizeof(block_q8);
    const size_t pitch = (size_t)m->max_tokens * row;
    if (pos > 0) {
        CU(cudaMemcpy2DAsync(m->dk, pitch, cache->k_q8, pitch, (size_t)pos * row, (size_t)m->n_kv,
                             cudaMemcpyHostToDevice, G.stream), "upload K prefix");
        CU(cudaMemcpy2DAsync(m->dv, pitch, cache->v_q8, pitch, (size_t)pos * row, (size_t)m->n_kv,
                             cudaMemcpyHostToDevice, G.stream), "upload V prefix");
    }
    m->synced = pos;
    return 0;
}

/* Q8 append of n tokens at pos0.. and their attention (n == 1: one decode
 * step; n > 1: a causal prefill chunk).  q/attn: [n][n_q*hd], k/v: [n][n_kv*hd]. */
static int q8_append_attend(tq_kv_cache *cache, const tq_attn_config *cfg, int pos0, int n, const float *q,
                            const float *k, const float *v, float *attn) {
    int rc = use_device();
    if (rc) return rc;
    mirror *m = NULL;
    rc = mirror_get(cache, cfg, &m);
    if (rc) return rc;
    rc = mirror_sync_prefix(m, cache, pos0);
    if (rc) {
        m->synced = -1;
        return rc;
    }
    const int hd = cfg->head_dim;
    const size_t q_floats = (size_t)n * cfg->n_q_heads * hd;
    const size_t kv_floats = (size_t)n * cfg->n_kv_heads * hd;
    const size_t row = (size_t)(hd / QK) * sizeof(block_q8);
    const size_t pitch = (size_t)cache->max_tokens * row;
    const size_t in_bytes = (q_floats + 2 * kv_floats) * sizeof(float);
    const size_t out_bytes = q_floats * sizeof(float);
    const size_t rows_bytes = (size_t)cfg->n_kv_heads * n * row;  /* appended rows of one plane */
    const size_t off_out = align256(in_bytes), off_rk = off_out + align256(out_bytes),
                 off_rv = off_rk + align256(rows_bytes), total = off_rv + align256(rows_bytes);

    unsigned char *h = (unsigned char *)host_stage(total);
    unsigned char *d = (unsigned char *)dev_scratch(align256(in_bytes) + align256(out_bytes));
    if (!h || !d) return cuda_fail(cudaErrorMemoryAllocation, "staging buffers");
    float *hq = (float *)h, *hk = hq + q_floats, *hv = hk + kv_floats;
    memcpy(hq, q, q_floats * sizeof(float));
    memcpy(hk, k, kv_floats * sizeof(float));
    memcpy(hv, v, kv_floats * sizeof(float));
    float *dq = (float *)d, *dkin = dq + q_floats, *dvin = dkin + kv_floats;
    float *dout = (float *)(d + align256(in_bytes));

    m->synced = -1;  /* until this call has fully completed */
    CU(cudaMemcpyAsync(d, h, in_bytes, cudaMemcpyHostToDevice, G.stream), "upload q/k/v");
    if (n == 1)
        rc = tqk_append_attend_q8(m->dk, m->dv, cfg->n_q_heads, cfg->n_kv_heads, hd, cache->max_tokens, pos0, dq, dkin,
                                  dvin, dout, G.stream);
    else
        rc = tqk_prefill_q8(m->dk, m->dv, cfg->n_q_heads, cfg->n_kv_heads, hd, cache->max_tokens, pos0, n, dq, dkin,
                            dvin, dout, G.stream);
    if (rc) return tqk_fail(rc, n == 1 ? "tqk_append_attend_q8" : "tqk_prefill_q8");
    CU(cudaMemcpyAsync(h + off_out, dout, out_bytes, cudaMemcpyDeviceToHost, G.stream), "download attention");
    CU(cudaMemcpy2DAsync(h + off_rk, (size_t)n * row, (const unsigned char *)m->dk + (size_t)pos0 * row, pitch,
                         (size_t)n * row, (size_t)cfg->n_kv_heads, cudaMemcpyDeviceToHost, G.stream),
       "download K rows");
    CU(cudaMemcpy2DAsync(h + off_rv, (size_t)n * row, (const unsigned char *)m->dv + (size_t)pos0 * row, pitch,
                         (size_t)n * row, (size_t)cfg->n_kv_heads, cudaMemcpyDeviceToHost, G.stream),
       "download V rows");
    if ((rc = finish("append + attention"))) return rc;  /* m->synced stays -1: the next call re-uploads */
    memcpy(attn, h + off_out, out_bytes);
    for (int kvh = 0; kvh < cfg->n_kv_heads; kvh++) {
        const size_t dst = ((size_t)kvh * cache->max_tokens + pos0) * row;
        memcpy((unsigned char *)cache->k_q8 + dst, h + off_rk + (size_t)kvh * n * row, (size_t)n * row);
        memcpy((unsigned char *)cache->v_q8 + dst, h + off_rv + (size_t)kvh * n * row, (size_t)n * row);
    }
    m->synced = pos0 + n;
    mirror_note_written(m, cache, pos0 + n - 1);
    return set_status(0);
}

/* ---------------------------------------------------------------------------
 * model/kv_cache.c
 * ------------------------------------------------------------------------- */
void tq_kv_cache_free(tq_kv_cache *cache) {
    pthread_mutex_lock(&g_mu);
    if (cache->k_q8 || cache->v_q8) mirror_drop(cache->k_q8, cache->v_q8);
    pthread_mutex_unlock(&g_mu);
    free(cache->k_f32);
    free(cache->v_f32);
    free(cache->k_q8);
    free(cache->v_q8);
    cache->k_f32 = NULL;
    cache->v_f32 = NULL;
    cache->k_q8 = NULL;
    cache->v_q8 = NULL;
    cache->max_tokens = 0;
}

int tq_kv_cache_init(tq_kv_cache *cache, tq_kv_type type, const tq_attn_config *cfg, int max_tokens) {
    cache->type = type;
    cache->max_tokens = max_tokens;
    cache->k_f32 = NULL;
    cache->v_f32 = NULL;
    cache->k_q8 = NULL;
    cache->v_q8 = NULL;
    if (max_tokens <= 0) return -1;
    if (type == TQ_KV_F32) {
        const size_t n = (size_t)cfg->n_kv_heads * max_tokens * cfg->head_dim;
        cache->k_f32 = (float *)malloc(n * sizeof(float));
        cache->v_f32 = (float *)malloc(n * sizeof(float));
        if (!cache->k_f32 || !cache->v_f32) {
            tq_kv_cache_free(cache);
            return -1;
        }
        return 0;
    }
    if (type != TQ_KV_Q8) return -1;
    const size_t n = (size_t)cfg->n_kv_heads * max_tokens * (cfg->head_dim / QK);
    cache->k_q8 = (block_q8 *)malloc(n * sizeof(block_q8));
    cache->v_q8 = (block_q8 *)malloc(n * sizeof(block_q8));
    if (!cache->k_q8 || !cache->v_q8) {
        tq_kv_cache_free(cache);
        return -1;
    }
    /* the device mirror is created now, so a machine without a usable GPU fails here */
    pthread_mutex_lock(&g_mu);
    mirror *m = NULL;
    int rc = use_device();
    if (!rc) rc = mirror_get(cache, cfg, &m);
    pthread_mutex_unlock(&g_mu);
    if (rc) {
        tq_kv_cache_free(cache);
        return -1;
    }
    return 0;
}

/* ---------------------------------------------------------------------------
 * device-resident attention layers (weights registered by the runtime)
 * ------------------------------------------------------------------------- */
static const tq_matrix *wmat(const tq_attn_weights *w, int i) {
    return i == 0 ? &w->wq : i == 1 ? &w->wk : i == 2 ? &w->wv : &w->wo;
}

static wreg *wreg_find(const tq_attn_weights *w) {
    for (wreg *r = G.wregs; r; r = r->next) {
        if (r->key != w || r->device != G.device) continue;
        int same = r->src_norm[0] == w->q_norm && r->src_norm[1] == w->k_norm;
        for (int i = 0; i < 4; i++) same = same && r->src[i] == wmat(w, i)->data;
        if (same) return r;
    }
    return NULL;
}

static void wreg_release(wreg *r) {
    for (int i = 0; i < 4; i++) cudaFree(r->dw[i]);
    cudaFree(r->dnorm[0]);
    cudaFree(r->dnorm[1]);
    free(r);
}

static void wreg_drop(const tq_attn_weights *w) {
    wreg **pp = &G.wregs;
    while (*pp) {
        if ((*pp)->key == w) {
            wreg *dead = *pp;
            *pp = dead->next;
            if (G.ready) cudaStreamSynchronize(G.stream);
            wreg_release(dead);
            continue;
        }
        pp = &(*pp)->next;
    }
}

int tq_b200_register_attn_weights(const tq_attn_weights *w, const tq_attn_config *cfg) {
    if (!w || !cfg) return set_status(-1);
    const int v = tq_attn_validate(w, cfg);
    if (v) return set_status(v);
    const tq_format f = w->wq.format;
    if (w->wk.format != f || w->wv.format != f || w->wo.format != f || (f != TQ_FORMAT_Q8 && f != TQ_FORMAT_Q4))
        return set_status(-10);
    for (int i = 0; i < 4; i++)
        if (!wmat(w, i)->data) return set_status(-10);
    pthread_mutex_lock(&g_mu);
    int rc = use_device();
    if (rc) {
        pthread_mutex_unlock(&g_mu);
        return rc;
    }
    wreg_drop(w);
    wreg *r = (wreg *)calloc(1, sizeof *r);
    if (!r) {
        pthread_mutex_unlock(&g_mu);
        return set_status(-1);
    }
    r->key = w;
    r->device = G.device;
    r->format = f == TQ_FORMAT_Q8 ? TQK_FMT_Q8 : TQK_FMT_Q4;
    r->hd = cfg->head_dim;
    const size_t block = f == TQ_FORMAT_Q8 ? 36 : 20;
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < 4 && e == cudaSuccess; i++) {
        const tq_matrix *m = wmat(w, i);
        const size_t bytes = (size_t)m->rows * (size_t)(m->cols / QK) * block;
        r->src[i] = m->data;
        e = cudaMalloc(&r->dw[i], bytes);
        if (e == cudaSuccess) e = cudaMemcpy(r->dw[i], m->data, bytes, cudaMemcpyHostToDevice);
    }
    const float *norms[2] = {w->q_norm, w->k_norm};
    for (int i = 0; i < 2 && e == cudaSuccess; i++) {
        r->src_norm[i] = norms[i];
        e = cudaMalloc((void **)&r->dnorm[i], (size_t)cfg->head_dim * sizeof(float));
        if (e == cudaSuccess)
            e = cudaMemcpy(r->dnorm[i], norms[i], (size_t)cfg->head_dim * sizeof(float), cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        wreg_release(r);
        pthread_mutex_unlock(&g_mu);
        return cuda_fail(e, "register attention weights");
    }
    r->next = G.wregs;
    G.wregs = r;
    pthread_mutex_unlock(&g_mu);
    return set_status(0);
}

void tq_b200_unregister_attn_weights(const tq_attn_weights *w) {
    pthread_mutex_lock(&g_mu);
    wreg_drop(w);
    pthread_mutex_unlock(&g_mu);
}

/* attention_layer (n == 1) or attention_layer_batch (n > 1) with registered
 * weights and a Q8 cache, all on the device: xn (and the RoPE tables, computed
 * here by the reference's rope_table) go up, out and the appended cache rows
 * come back.  Caller holds g_mu. */
static int device_layers(const wreg *r, tq_kv_cache *cache, const tq_attn_config *cfg, int pos0, int n,
                         const float *xn, float *out) {
    int rc = use_device();
    if (rc) return rc;
    mirror *m = NULL;
    rc = mirror_get(cache, cfg, &m);
    if (rc) return rc;
    rc = mirror_sync_prefix(m, cache, pos0);
    if (rc) {
        m->synced = -1;
        return rc;
    }
    const int hd = cfg->head_dim, hidden = cfg->hidden_size;
    const size_t q_dim = (size_t)cfg->n_q_heads * hd, kv_dim = (size_t)cfg->n_kv_heads * hd;
    const size_t row = (size_t)(hd / QK) * sizeof(block_q8);
    const size_t pitch = (size_t)cache->max_tokens * row;
    const size_t x_bytes = (size_t)n * hidden * sizeof(float);
    const size_t tab_bytes = (size_t)n * hd * sizeof(float);  /* cos [n][hd/2], then sin [n][hd/2] */
    const size_t rows_bytes = (size_t)cfg->n_kv_heads * n * row;
    /* host staging: [xn][tables] up, [out][K rows][V rows] down */
    const size_t h_tab = align256(x_bytes), h_out = h_tab + align256(tab_bytes),
                 h_rk = h_out + align256(x_bytes), h_rv = h_rk + align256(rows_bytes), h_total = h_rv + align256(rows_bytes);
    /* device scratch: [xn][tables][out][q][k][v][attention] */
    const size_t d_out = align256(x_bytes) + align256(tab_bytes), d_q = d_out + align256(x_bytes),
                 d_k = d_q + align256((size_t)n * q_dim * sizeof(float)),
                 d_v = d_k + align256((size_t)n * kv_dim * sizeof(float)),
                 d_a = d_v + align256((size_t)n * kv_dim * sizeof(float)),
                 d_total = d_a + align256((size_t)n * q_dim * sizeof(float));
    unsigned char *h = (unsigned char *)host_stage(h_total);
    unsigned char *d = (unsigned char *)dev_scratch(d_total);
    if (!h || !d) return cuda_fail(cudaErrorMemoryAllocation, "staging buffers");
    memcpy(h, xn, x_bytes);
    float *hcos = (float *)(h + h_tab), *hsin = hcos + (size_t)n * (hd / 2);
    for (int i = 0; i < n; i++) rope_table(hcos + (size_t)i * (hd / 2), hsin + (size_t)i * (hd / 2), hd, pos0 + i,
                                           cfg->rope_theta);
    float *dx = (float *)d, *dcos = (float *)(d + align256(x_bytes)), *dsin = dcos + (size_t)n * (hd / 2);
    float *dout = (float *)(d + d_out), *dq = (float *)(d + d_q), *dk = (float *)(d + d_k), *dvv = (float *)(d + d_v),
          *da = (float *)(d + d_a);

    m->synced = -1;  /* until this call has fully completed */
    CU(cudaMemcpyAsync(d, h, align256(x_bytes) + tab_bytes, cudaMemcpyHostToDevice, G.stream), "upload xn");
    if (n == 1) {
        tqk_attn_layer_args a;
        memset(&a, 0, sizeof a);
        a.wq = r->dw[0];
        a.wk = r->dw[1];
        a.wv = r->dw[2];
        a.wo = r->dw[3];
        a.format = r->format;
        a.q_norm = r->dnorm[0];
        a.k_norm = r->dnorm[1];
        a.n_q_heads = cfg->n_q_heads;
        a.n_kv_heads = cfg->n_kv_heads;
        a.head_dim = hd;
        a.hidden_size = hidden;
        a.rms_eps = cfg->rms_eps;
        a.k = m->dk;
        a.v = m->dv;
        a.max_tokens = cache->max_tokens;
        a.pos = pos0;
        a.rope_cos = dcos;
        a.rope_sin = dsin;
        a.xn = dx;
        a.out = dout;
        a.scratch = dq;  /* q, k, v, attention follow one another */
        rc = tqk_attention_layer(&a, NULL, 0, G.stream);
        if (rc) return tqk_fail(rc, "tqk_attention_layer");
    } else {
        const tqk_proj_job qkv[3] = {{r->dw[0], dq, (int)q_dim}, {r->dw[1], dk, (int)kv_dim}, {r->dw[2], dvv, (int)kv_dim}};
        rc = tqk_project(qkv, 3, r->format, dx, hidden, n, G.stream);
        if (!rc)
            rc = tqk_qk_norm_rope(dq, dk, n, (int64_t)q_dim, (int64_t)kv_dim, cfg->n_q_heads, cfg->n_kv_heads, hd,
                                  r->dnorm[0], r->dnorm[1], 0, cfg->rms_eps, dcos, dsin, hd / 2, G.stream);
        if (!rc)
            rc = tqk_prefill_q8(m->dk, m->dv, cfg->n_q_heads, cfg->n_kv_heads, hd, cache->max_tokens, pos0, n, dq, dk,
                                dvv, da, G.stream);
        if (!rc) {
            const tqk_proj_job o = {r->dw[3], dout, hidden};
            rc = tqk_project(&o, 1, r->format, da, (int)q_dim, n, G.stream);
        }
        if (rc) return tqk_fail(rc, "device attention_layer_batch");
    }
    CU(cudaMemcpyAsync(h + h_out, dout, x_bytes, cudaMemcpyDeviceToHost, G.stream), "download output");
    CU(cudaMemcpy2DAsync(h + h_rk, (size_t)n * row, (const unsigned char *)m->dk + (size_t)pos0 * row, pitch,
                         (size_t)n * row, (size_t)cfg->n_kv_heads, cudaMemcpyDeviceToHost, G.stream),
       "download K rows");
    CU(cudaMemcpy2DAsync(h + h_rv, (size_t)n * row, (const unsigned char *)m->dv + (size_t)pos0 * row, pitch,
                         (size_t)n * row, (size_t)cfg->n_kv_heads, cudaMemcpyDeviceToHost, G.stream),
       "download V rows");
    if ((rc = finish("device attention layer"))) return rc;  /* m->synced stays -1: the next call re-uploads */
    memcpy(out, h + h_out, x_bytes);
    for (int kvh = 0; kvh < cfg->n_kv_heads; kvh++) {
        const size_t dst = ((size_t)kvh * cache->max_tokens + pos0) * row;
        memcpy((unsigned char *)cache->k_q8 + dst, h + h_rk + (size_t)kvh * n * row, (size_t)n * row);
        memcpy((unsigned char *)cache->v_q8 + dst, h + h_rv + (size_t)kvh * n * row, (size_t)n * row);
    }
    m->synced = pos0 + n;
    mirror_note_written(m, cache, pos0 + n - 1);
    return set_status(0);
}

/* ---------------------------------------------------------------------------
 * model/attention_layer.c
 * ------------------------------------------------------------------------- */
int tq_attn_validate(const tq_attn_weights *w, const tq_attn_config *cfg) {
    if (cfg->n_q_heads <= 0 || cfg->n_kv_heads <= 0 || cfg->head_dim <= 0) return -8;
    if (cfg->hidden_size % QK != 0) return -1;
    if (w->wk.cols != cfg->hidden_size || w->wq.cols != cfg->hidden_size || w->wv.cols != cfg->hidden_size ||
        w->wo.rows != cfg->hidden_size)
        return -2;
    if (w->wq.rows != cfg->n_q_heads * cfg->head_dim) return -3;
    if (w->wk.rows != cfg->n_kv_heads * cfg->head_dim || w->wv.rows != cfg->n_kv_heads * cfg->head_dim) return -4;
    if (cfg->n_q_heads % cfg->n_kv_heads != 0) return -5;
    if (cfg->head_dim % QK != 0) return -6;
    if (w->wo.cols != cfg->n_q_heads * cfg->head_dim) return -7;
    if (w->q_norm == NULL || w->k_norm == NULL) return -9;
    return 0;
}

int tq_attn_validate_cache(const tq_kv_cache *cache) {
    if (cache->max_tokens <= 0) return -1;
    switch (cache->type) {
        case TQ_KV_F32:
            if (cache->k_f32 == NULL || cache->v_f32 == NULL) return -2;
            return 0;
        case TQ_KV_Q8:
            if (cache->k_q8 == NULL || cache->v_q8 == NULL) return -2;
            return 0;
        default:
            return -3;
    }
}

/* per-head RMS norm in place + RoPE at pos (model/attention_layer.c:48-60,183-188) */
static void prepare_heads(float *x, int n_heads, int hd, const float *norm_w, float eps, const float *cs,
                          const float *sn) {
    for (int h = 0; h < n_heads; h++) {
        float *xh = x + (size_t)h * hd;
        rmsnorm(xh, norm_w, xh, hd, eps);
        rope_apply(xh, hd, cs, sn);
    }
}

/* F32 cache (not the accelerated path): store, then the reference's own
 * attention_head per q head, equivalent to attend_f32 (attention_layer.c:93-123). */
static void f32_store_attend(tq_kv_cache *cache, const tq_attn_config *cfg, int pos, const float *q, const float *k,
                             const float *v, float *scores, float *attn) {
    const int hd = cfg->head_dim;
    for (int h = 0; h < cfg->n_kv_heads; h++) {
        const size_t off = ((size_t)h * cache->max_tokens + pos) * hd;
        memcpy(cache->k_f32 + off, k + (size_t)h * hd, hd * sizeof(float));
        memcpy(cache->v_f32 + off, v + (size_t)h * hd, hd * sizeof(float));
    }
    const int group = cfg->n_q_heads / cfg->n_kv_heads;
    for (int h = 0; h < cfg->n_q_heads; h++) {
        const size_t base = (size_t)(h / group) * cache->max_tokens * hd;
        attention_head(q + (size_t)h * hd, cache->k_f32 + base, cache->v_f32 + base, pos + 1, hd, hd,
                       scores + (size_t)h * cache->max_tokens, attn + (size_t)h * hd);
    }
}

int attention_layer(const tq_attn_weights *w, const tq_attn_config *cfg, tq_kv_cache *cache, int pos,
                    const float *xn, float *scores, float *out) {
    if (pos < 0 || pos >= cache->max_tokens) return -1;
    if (cache->type == TQ_KV_Q8) {  /* registered weights: the whole layer on the device */
        pthread_mutex_lock(&g_mu);
        const wreg *r = G.ready ? wreg_find(w) : NULL;
        const int rc = r ? device_layers(r, cache, cfg, pos, 1, xn, out) : 1;
        pthread_mutex_unlock(&g_mu);
        if (rc <= 0) return rc == 0 ? 0 : (rc < -1 ? rc : TQB_ECUDA);
    }

    const int hd = cfg->head_dim;
    const int q_dim = cfg->n_q_heads * hd;
    const int kv_dim = cfg->n_kv_heads * hd;
    float q[q_dim], k[kv_dim], v[kv_dim], attn[q_dim];
    float cs[hd / 2], sn[hd / 2];
    block_q8 xq[cfg->hidden_size / QK];

    quantize_row_q8(xn, xq, cfg->hidden_size);
    get_matmul(w->wq.format)(w->wq.data, xq, q, w->wq.rows, w->wq.cols);
    get_matmul(w->wk.format)(w->wk.data, xq, k, w->wk.rows, w->wk.cols);
    get_matmul(w->wv.format)(w->wv.data, xq, v, w->wv.rows, w->wv.cols);

    rope_table(cs, sn, hd, pos, cfg->rope_theta);
    prepare_heads(q, cfg->n_q_heads, hd, w->q_norm, cfg->rms_eps, cs, sn);
    prepare_heads(k, cfg->n_kv_heads, hd, w->k_norm, cfg->rms_eps, cs, sn);

    if (cache->type == TQ_KV_Q8) {
        pthread_mutex_lock(&g_mu);
        const int rc = q8_append_attend(cache, cfg, pos, 1, q, k, v, attn);
        pthread_mutex_unlock(&g_mu);
        if (rc) return rc < -1 ? rc : TQB_ECUDA;
    } else {
        f32_store_attend(cache, cfg, pos, q, k, v, scores, attn);
    }

    block_q8 aq[q_dim / QK];
    quantize_row_q8(attn, aq, q_dim);
    get_matmul(w->wo.format)(w->wo.data, aq, out, w->wo.rows, w->wo.cols);
    return 0;
}

int attention_layer_batch(const tq_attn_weights *w, const tq_attn_config *cfg, tq_kv_cache *cache, int pos0, int n,
                          const float *xn, float *scores, float *out, tq_batch_ws *ws) {
    if (n <= 0 || n > ws->cap) return -1;
    if (pos0 < 0 || pos0 + n > cache->max_tokens) return -1;
    if (cache->type == TQ_KV_Q8) {  /* registered weights: the whole chunk on the device */
        pthread_mutex_lock(&g_mu);
        const wreg *r = G.ready ? wreg_find(w) : NULL;
        const int rc = r ? device_layers(r, cache, cfg, pos0, n, xn, out) : 1;
        pthread_mutex_unlock(&g_mu);
        if (rc <= 0) return rc == 0 ? 0 : (rc < -1 ? rc : TQB_ECUDA);
    }

    const int hd = cfg->head_dim;
    const int q_dim = cfg->n_q_heads * hd;
    const int kv_dim = cfg->n_kv_heads * hd;
    const int hidden = cfg->hidden_size;
    const int nbh = hidden / QK;
    const int nbq = q_dim / QK;

    for (int i = 0; i < n; i++) quantize_row_q8(xn + (size_t)i * hidden, ws->xq + (size_t)i * nbh, hidden);
    get_matmul_batch(w->wq.format)(w->wq.data, ws->xq, ws->q, w->wq.rows, w->wq.cols, n);
    get_matmul_batch(w->wk.format)(w->wk.data, ws->xq, ws->k, w->wk.rows, w->wk.cols, n);
    get_matmul_batch(w->wv.format)(w->wv.data, ws->xq, ws->v, w->wv.rows, w->wv.cols, n);

    float cs[hd / 2], sn[hd / 2];
    for (int i = 0; i < n; i++) {
        rope_table(cs, sn, hd, pos0 + i, cfg->rope_theta);
        prepare_heads(ws->q + (size_t)i * q_dim, cfg->n_q_heads, hd, w->q_norm, cfg->rms_eps, cs, sn);
        prepare_heads(ws->k + (size_t)i * kv_dim, cfg->n_kv_heads, hd, w->k_norm, cfg->rms_eps, cs, sn);
    }

    if (cache->type == TQ_KV_Q8) {
        /* one device call: append all n rows, then causal attention (token i sees
         * positions <= pos0+i), identical to the reference's per-token loop */
        pthread_mutex_lock(&g_mu);
        const int rc = q8_append_attend(cache, cfg, pos0, n, ws->q, ws->k, ws->v, ws->attn);
        pthread_mutex_unlock(&g_mu);
        if (rc) return rc < -1 ? rc : TQB_ECUDA;
    } else {
        for (int i = 0; i < n; i++)
            f32_store_attend(cache, cfg, pos0 + i, ws->q + (size_t)i * q_dim, ws->k + (size_t)i * kv_dim,
                             ws->v + (size_t)i * kv_dim, scores, ws->attn + (size_t)i * q_dim);
    }

    for (int i = 0; i < n; i++) quantize_row_q8(ws->attn + (size_t)i * q_dim, ws->xq + (size_t)i * nbq, q_dim);
    get_matmul_batch(w->wo.format)(w->wo.data, ws->xq, out, w->wo.rows, w->wo.cols, n);
    return 0;
}

/* ---------------------------------------------------------------------------
 * model/attn_q8.c: single-head and per-op entry points (stateless host buffers)
 * ------------------------------------------------------------------------- */
static void fill_nan(float *x, size_t n, size_t stride, size_t rows) {
    for (size_t r = 0; r < rows; r++)
        for (size_t i = 0; i < n; i++) x[r * stride + i] = NAN;
}

static int head_q8_impl(const float *q, block_q8 *q_q8, const block_q8 *k_cache, const block_q8 *v_cache, int n,
                        int head_dim, float *scores, float *out) {
    int rc = use_device();
    if (rc) return rc;
    const int nb = head_dim / QK;
    const size_t blk = sizeof(block_q8);
    const size_t o_q = 0, o_qq = align256(head_dim * sizeof(float)), o_k = o_qq + align256(nb * blk),
                 o_v = o_k + align256((size_t)n * nb * blk), o_s = o_v + align256((size_t)n * nb * blk),
                 o_o = o_s + align256((size_t)n * sizeof(float)), total = o_o + align256(head_dim * sizeof(float));
    unsigned char *d = (unsigned char *)dev_scratch(total);
    if (!d) return cuda_fail(cudaErrorMemoryAllocation, "scratch");
    const float scale = 1.0f / sqrtf((float)head_dim);
    CU(cudaMemcpyAsync(d + o_q, q, head_dim * sizeof(float), cudaMemcpyHostToDevice, G.stream), "upload q");
    if (n > 0) {
        CU(cudaMemcpyAsync(d + o_k, k_cache, (size_t)n * nb * blk, cudaMemcpyHostToDevice, G.stream), "upload K");
        CU(cudaMemcpyAsync(d + o_v, v_cache, (size_t)n * nb * blk, cudaMemcpyHostToDevice, G.stream), "upload V");
    }
    if ((rc = tqk_quantize_rows_q8((const float *)(d + o_q), (tqk_block_q8 *)(d + o_qq), 1, head_dim, G.stream)))
        return tqk_fail(rc, "tqk_quantize_rows_q8");
    if ((rc = tqk_attn_scores_q8((const tqk_block_q8 *)(d + o_qq), 1, (const tqk_block_q8 *)(d + o_k), n, nb, scale,
                                 (float *)(d + o_s), (size_t)n, G.stream)))
        return tqk_fail(rc, "tqk_attn_scores_q8");
    if ((rc = tqk_softmax_rows((float *)(d + o_s), 1, n, (size_t)n, G.stream))) return tqk_fail(rc, "tqk_softmax_rows");
    if ((rc = tqk_attn_accum_q8((const float *)(d + o_s), (size_t)n, 1, (const tqk_block_q8 *)(d + o_v), n, nb,
                                (float *)(d + o_o), (size_t)head_dim, G.stream)))
        return tqk_fail(rc, "tqk_attn_accum_q8");
    CU(cudaMemcpyAsync(q_q8, d + o_qq, nb * blk, cudaMemcpyDeviceToHost, G.stream), "download q_q8");
    if (n > 0) CU(cudaMemcpyAsync(scores, d + o_s, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost, G.stream), "download scores");
    CU(cudaMemcpyAsync(out, d + o_o, head_dim * sizeof(float), cudaMemcpyDeviceToHost, G.stream), "download out");
    if ((rc = finish("attention_head_q8"))) return rc;
    return set_status(0);
}

void attention_head_q8(const float *q, block_q8 *q_q8, const block_q8 *k_cache, const block_q8 *v_cache, int n,
                       int head_dim, float *scores, float *out) {
    pthread_mutex_lock(&g_mu);
    const int rc = head_q8_impl(q, q_q8, k_cache, v_cache, n, head_dim, scores, out);
    pthread_mutex_unlock(&g_mu);
    if (rc) fill_nan(out, (size_t)head_dim, 0, 1);
}

static int scores_impl(const block_q8 *q, int g, const block_q8 *k, int n, int nb, float scale, float *scores,
                       size_t stride) {
    if (g <= 0 || n <= 0) return set_status(0);
    int rc = use_device();
    if (rc) return rc;
    const size_t blk = sizeof(block_q8);
    const size_t o_q = 0, o_k = align256((size_t)g * nb * blk), o_s = o_k + align256((size_t)n * nb * blk),
                 total = o_s + align256((size_t)g * n * sizeof(float));
    unsigned char *d = (unsigned char *)dev_scratch(total);
    if (!d) return cuda_fail(cudaErrorMemoryAllocation, "scratch");
    CU(cudaMemcpyAsync(d + o_q, q, (size_t)g * nb * blk, cudaMemcpyHostToDevice, G.stream), "upload q");
    CU(cudaMemcpyAsync(d + o_k, k, (size_t)n * nb * blk, cudaMemcpyHostToDevice, G.stream), "upload K");
    if ((rc = tqk_attn_scores_q8((const tqk_block_q8 *)(d + o_q), g, (const tqk_block_q8 *)(d + o_k), n, nb, scale,
                                 (float *)(d + o_s), (size_t)n, G.stream)))
        return tqk_fail(rc, "tqk_attn_scores_q8");
    CU(cudaMemcpy2DAsync(scores, stride * sizeof(float), d + o_s, (size_t)n * sizeof(float), (size_t)n * sizeof(float),
                         (size_t)g, cudaMemcpyDeviceToHost, G.stream), "download scores");
    if ((rc = finish("attn_scores_q8"))) return rc;
    return set_status(0);
}

void attn_scores_q8(const block_q8 *q, int g, const block_q8 *k, int n, int nb, float scale, float *scores,
                    size_t stride) {
    pthread_mutex_lock(&g_mu);
    const int rc = scores_impl(q, g, k, n, nb, scale, scores, stride);
    pthread_mutex_unlock(&g_mu);
    if (rc) fill_nan(scores, (size_t)n, stride, (size_t)g);
}

static int accum_impl(const float *w, size_t w_stride, int g, const block_q8 *v, int n, int nb, float *out,
                      size_t out_stride) {
    if (g <= 0) return set_status(0);
    int rc = use_device();
    if (rc) return rc;
    const int hd = nb * QK;
    const size_t blk = sizeof(block_q8);
    const size_t o_w = 0, o_v = align256((size_t)g * n * sizeof(float)), o_o = o_v + align256((size_t)n * nb * blk),
                 total = o_o + align256((size_t)g * hd * sizeof(float));
    unsigned char *d = (unsigned char *)dev_scratch(total);
    if (!d) return cuda_fail(cudaErrorMemoryAllocation, "scratch");
    if (n > 0) {
        CU(cudaMemcpy2DAsync(d + o_w, (size_t)n * sizeof(float), w, w_stride * sizeof(float), (size_t)n * sizeof(float),
                             (size_t)g, cudaMemcpyHostToDevice, G.stream), "upload weights");
        CU(cudaMemcpyAsync(d + o_v, v, (size_t)n * nb * blk, cudaMemcpyHostToDevice, G.stream), "upload V");
    }
    if ((rc = tqk_attn_accum_q8((const float *)(d + o_w), (size_t)n, g, (const tqk_block_q8 *)(d + o_v), n, nb,
                                (float *)(d + o_o), (size_t)hd, G.stream)))
        return tqk_fail(rc, "tqk_attn_accum_q8");
    CU(cudaMemcpy2DAsync(out, out_stride * sizeof(float), d + o_o, (size_t)hd * sizeof(float), (size_t)hd * sizeof(float),
                         (size_t)g, cudaMemcpyDeviceToHost, G.stream), "download out");
    if ((rc = finish("attn_accum_q8"))) return rc;
    return set_status(0);
}

void attn_accum_q8(const float *w, size_t w_stride, int g, const block_q8 *v, int n, int nb, float *out,
                   size_t out_stride) {
    pthread_mutex_lock(&g_mu);
    const int rc = accum_impl(w, w_stride, g, v, n, nb, out, out_stride);
    pthread_mutex_unlock(&g_mu);
    if (rc) fill_nan(out, (size_t)nb * QK, out_stride, (size_t)g);
}

/* ---------------------------------------------------------------------------
 * drop-in control
 * ------------------------------------------------------------------------- */
int tq_b200_last_status(void) { return t_status; }

void tq_b200_cache_invalidate(const tq_kv_cache *cache) {
    pthread_mutex_lock(&g_mu);
    mirror *m = mirror_find(cache->k_q8, cache->v_q8);
    if (m) m->synced = -1;
    pthread_mutex_unlock(&g_mu);
}

int tq_b200_cache_download(tq_kv_cache *cache, const tq_attn_config *cfg, int n) {
    if (cache->type != TQ_KV_Q8 || n < 0 || n > cache->max_tokens) return -1;
    pthread_mutex_lock(&g_mu);
    int rc = use_device();
    mirror *m = rc ? NULL : mirror_find(cache->k_q8, cache->v_q8);
    if (!rc && !m) rc = -1;
    if (!rc && m->n_kv == cfg->n_kv_heads && n > 0) {
        const size_t row = (size_t)(m->head_dim / QK) * sizeof(block_q8);
        const size_t pitch = (size_t)m->max_tokens * row;
        cudaError_t e = cudaMemcpy2DAsync(cache->k_q8, pitch, m->dk, pitch, (size_t)n * row, (size_t)m->n_kv,
                                          cudaMemcpyDeviceToHost, G.stream);
        if (e == cudaSuccess)
            e = cudaMemcpy2DAsync(cache->v_q8, pitch, m->dv, pitch, (size_t)n * row, (size_t)m->n_kv,
                                  cudaMemcpyDeviceToHost, G.stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(G.stream);
        rc = e == cudaSuccess ? 0 : cuda_fail(e, "download cache");
    }
    pthread_mutex_unlock(&g_mu);
    return rc;
}
