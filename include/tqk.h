/*
 * tqk.h -- C ABI of the B200 (sm_100a) Q8 GQA attention kernels.
 *
 * This is the boundary the reference's plain-C attention layer binds to.  All
 * entry points take plain device pointers and sizes, run asynchronously on the
 * given CUDA stream (NULL = the legacy default stream), and return an int
 * status: 0 on success, a negative TQK_E* code otherwise (never abort).  Device
 * pointers to Q8 planes must be 16-byte aligned (cudaMalloc memory is).
 *
 * Data format (identical bytes to the reference):
 *   block_q8 = { float d; int8_t q[32]; }, 36 bytes, no padding
 *       (reference packer/packer.h:7-11);
 *   a cache plane is [n_kv_heads][max_tokens][head_dim/32] blocks and the row
 *       of kv head h at position t is slot h*max_tokens + t
 *       (reference model/attention_layer.c:62-64, model/kv_cache.c:33-39);
 *   q / out are head-major fp32 [n_q_heads][head_dim]; query head h reads kv
 *       head h / (n_q_heads/n_kv_heads) (reference model/attention_layer.c:130-137).
 */
#ifndef TQK_H
#define TQK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Exported symbols; the library is built with hidden default visibility. */
#if defined(__GNUC__)
#define TQK_API __attribute__((visibility("default")))
#else
#define TQK_API
#endif

#define TQK_QK 32
typedef struct { float d; int8_t q[TQK_QK]; } tqk_block_q8;

typedef void *tqk_stream_t; /* a cudaStream_t */

/* Status codes.  -1 keeps the reference's meaning "position out of range"
 * (reference model/attention_layer.c:172 and :203-204). */
#define TQK_OK               0
#define TQK_EPOS            -1
#define TQK_EINVAL         -20  /* bad shape or NULL pointer */
#define TQK_EALIGN         -21  /* a device pointer is not 16-byte aligned */
#define TQK_EWORKSPACE     -22  /* caller workspace smaller than tqk_decode_workspace_size() */
#define TQK_ECUDA          -23  /* CUDA runtime error; tqk_last_error() has the text */
#define TQK_ENODEV         -24  /* no usable CUDA device */
#define TQK_ETIMEOUT       -25  /* a device-side bounded wait gave up (see tqk_device_status) */
#define TQK_EUNSUPPORTED   -26  /* head_dim > 256 or another shape outside the kernels' range */
#define TQK_EDEVLEN        -27  /* a length read from device memory was outside [0, max_tokens] (clamped) */

TQK_API const char *tqk_status_string(int status);
/* Text of the last failure on the calling host thread ("" if none). */
TQK_API const char *tqk_last_error(void);
/* Library version string, e.g. "tqk 0.1 sm_100a". */
TQK_API const char *tqk_version(void);

/* Reads (and with clear != 0 resets) the sticky device-side error word of the
 * current device: 0 when no kernel reported a timeout or bad input.  Synchronises
 * the device.  The kernels set it instead of trapping. */
TQK_API int tqk_device_status(int *device_error, int clear);
/* Enqueues on `stream` a copy of the current device's error word into
 * *host_dst (pinned host memory for a truly asynchronous copy); read it after
 * synchronising the stream.  It shows what every kernel that finished before
 * the copy in stream order recorded (and whatever other streams' kernels
 * recorded by then: the word is per device).  Clear it with
 * tqk_device_status(&v, 1). */
TQK_API int tqk_device_status_async(int *host_dst, tqk_stream_t stream);
/* The status code of a device error word value: TQK_OK for 0, TQK_ETIMEOUT for
 * a bounded wait that gave up, TQK_EDEVLEN for a clamped device length. */
TQK_API int tqk_device_error_status(int device_error);

/* ---------------------------------------------------------------------------
 * Quantiser.  Replaces quantize_row_q8 (reference kernel/quant_x.c:12-34) for
 * rows resident in device memory: rows x n floats -> rows x n/32 blocks, n a
 * multiple of 32.  Bit-exact with the reference (int8 values and fp32 scales),
 * including zero, denormal, Inf and NaN inputs.
 */
TQK_API int tqk_quantize_rows_q8(const float *x, tqk_block_q8 *out, int rows, int n, tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * KV append.  Replaces the Q8 branch of store_kv (reference
 * model/attention_layer.c:66-90): quantises the n_kv rows of k and v (fp32
 * [n_kv][head_dim], device) into slot h*max_tokens+pos of each plane.
 * Returns TQK_EPOS without touching the planes when pos is outside [0, max_tokens).
 */
TQK_API int tqk_store_kv_q8(tqk_block_q8 *k_plane, tqk_block_q8 *v_plane, int n_kv_heads, int head_dim,
                    int max_tokens, int pos, const float *k, const float *v, tqk_stream_t stream);

/* Batched append of n consecutive positions pos0..pos0+n-1 (the append half of
 * attention_layer_batch, reference model/attention_layer.c:221-236): k, v are
 * [n][n_kv][head_dim] fp32 (token-major, as the reference's ws->k / ws->v). */
TQK_API int tqk_store_kv_q8_batch(tqk_block_q8 *k_plane, tqk_block_q8 *v_plane, int n_kv_heads, int head_dim,
                          int max_tokens, int pos0, int n, const float *k, const float *v,
                          tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * The step before the attention: per-head RMSNorm of q and k and rotary
 * embedding, in place.  Replaces norm_heads + rope_heads as attention_layer
 * calls them (reference model/attention_layer.c:48-60, :183-189;
 * model/rmsnorm.c:4-19, model/rope.c:14-22), bit-exact with the reference's
 * fp32 arithmetic so the K rows appended afterwards give identical Q8 bytes.
 * For each of n_items items: q + i*q_item_stride holds n_q_heads rows and
 * k + i*k_item_stride n_kv_heads rows of head_dim floats (strides in floats;
 * 0 = packed).  q_norm / k_norm: [head_dim] weights (+ i*norm_item_stride;
 * both NULL = no norm).  rope_cos / rope_sin: the [head_dim/2] table of
 * rope_table (reference model/rope.c:4-12) computed on the host (+
 * i*rope_item_stride; both NULL = no rope).  head_dim must be even.
 */
TQK_API int tqk_qk_norm_rope(float *q, float *k, int n_items, int64_t q_item_stride, int64_t k_item_stride,
                             int n_q_heads, int n_kv_heads, int head_dim, const float *q_norm, const float *k_norm,
                             int64_t norm_item_stride, float eps, const float *rope_cos, const float *rope_sin,
                             int64_t rope_item_stride, tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * Reference-shaped single kernels (model/attn_q8.c:56-76 dispatchers and
 * model/softmax.c:4).  These keep the reference's per-op contract (strided score
 * rows, strided outputs, nothing written past n or head_dim) so the reference's
 * kernel tests can drive them; the fused decode below is the fast path.
 */
/* scores[h*stride + t] = scale * sum_b (float)dot_int(q[h][b], k[t][b]) * (qd*kd),
 * bit-exact with attn_scores_q8_scalar (model/attn_q8.c:17-34). */
TQK_API int tqk_attn_scores_q8(const tqk_block_q8 *q, int g, const tqk_block_q8 *k, int n, int nb, float scale,
                       float *scores, size_t stride, tqk_stream_t stream);
/* out[h*out_stride + j] = sum_t (w[h*w_stride+t] * vd) * vq, token order, bit-exact
 * with attn_accum_q8_scalar (model/attn_q8.c:36-54). */
TQK_API int tqk_attn_accum_q8(const float *w, size_t w_stride, int g, const tqk_block_q8 *v, int n, int nb,
                      float *out, size_t out_stride, tqk_stream_t stream);
/* In-place softmax of `rows` rows of n floats, row r at x + r*stride (model/softmax.c:4-23). */
TQK_API int tqk_softmax_rows(float *x, int rows, int n, size_t stride, tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * Fused decode attention (the hot path).  Replaces attend_q8 (reference
 * model/attention_layer.c:125-150) -- quantise the group's q heads, int8 scores,
 * softmax, Q8 V accumulation -- as one split-sequence (flash-decoding) kernel
 * with an online FP32 softmax and a log-sum-exp merge of the splits, and
 * optionally fuses the KV append of store_kv (model/attention_layer.c:66-90).
 *
 * One call covers n_items independent items (layers of one token, sequences of
 * a batch, or both), each with its own planes, q, out and length:
 *   item i reads planes k + i*item_stride, v + i*item_stride (in blocks),
 *   q + i*q_item_stride, writes out + i*out_item_stride (in floats), and attends
 *   to its first len_i positions, where
 *     len_i = lens[i]                       if lens != NULL (device int32 array)
 *     len_i = len0 + i*len_step             otherwise.
 * With k_new/v_new non-NULL, item i first appends k_new + i*kv_new_item_stride
 * (fp32 [n_kv][head_dim]) at position len_i - 1, bit-exact with store_kv, and
 * the attention includes it, exactly as store_kv followed by attend_q8.
 * len_i == 0 writes zeros (the reference's empty softmax leaves accum's zeros).
 *
 * out_mode TQK_OUT_NORMALIZED writes the attention output; TQK_OUT_PARTIAL
 * writes per (item, q head) the unnormalised partial {acc[head_dim], m, l}
 * (layout: out + i*out_item_stride + h*(head_dim+2)) for a cross-device
 * log-sum-exp merge with tqk_merge_partials().
 */
#define TQK_SPLIT_BALANCED  -1  /* tqk_decode_args.split_tokens: see there */
#define TQK_OUT_NORMALIZED 0
#define TQK_OUT_PARTIAL    1

typedef struct {
    tqk_block_q8 *k, *v;          /* planes of item 0 (device) */
    int64_t item_stride;          /* blocks between consecutive items' planes (0 = shared planes) */
    int n_items;
    int n_q_heads, n_kv_heads, head_dim, max_tokens;
    const int32_t *lens;          /* device [n_items], or NULL */
    int len0, len_step;           /* used when lens == NULL */
    int max_len;                  /* upper bound of len_i; sizes the grid */
    const float *q;  int64_t q_item_stride;
    float *out;      int64_t out_item_stride;
    const float *k_new, *v_new;   /* optional fused append (device), or NULL */
    int64_t kv_new_item_stride;
    int out_mode;                 /* TQK_OUT_NORMALIZED or TQK_OUT_PARTIAL */
    int split_tokens;             /* tokens per split (multiple of 64); 0 = choose automatically;
                                     TQK_SPLIT_BALANCED = the balanced schedule (equal runs of tiles
                                     per CTA across items) whenever the call qualifies for it, else
                                     as 0 (tqk_decode_q8_static always treats it as 0) */
    /* Optional fused prologue (attention_layer.c:183-189, norm_heads + rope_heads): each q head
     * of item i, and each appended k_new head, is first RMS-normalised with q_norm / k_norm +
     * i*norm_item_stride ([head_dim] floats, shared by the heads; both NULL = no norm) and then
     * rotated with rope_cos / rope_sin + i*rope_item_stride ([head_dim/2] floats, the table of
     * the appended token's position; both NULL = no rope).  Bit-exact with tqk_qk_norm_rope
     * followed by the plain call.  q and k_new are read only: the normed rows are not written
     * back.  Zero-initialise the struct so that callers which set none of these get none. */
    const float *q_norm, *k_norm;
    int64_t norm_item_stride;
    float norm_eps;
    const float *rope_cos, *rope_sin;
    int64_t rope_item_stride;
} tqk_decode_args;

/* Bytes of device workspace tqk_decode_q8 needs for these arguments. */
TQK_API int tqk_decode_workspace_size(const tqk_decode_args *a, size_t *bytes);
/* A caller workspace starts with the split-merge tickets (17 ints per item and
 * head unit, at least 16384 units' worth: 1088 KiB) followed by the partials.
 * It must be zeroed once before first use (tqk_workspace_init); every
 * completed call leaves the
 * tickets at zero again, so calls of up to 16384 units (n_items x kv-head
 * units) can reuse it without re-initialising.  Zero it again before a call
 * with more units than any earlier one, and after a call that reported
 * TQK_ETIMEOUT.  Calls that share a workspace must be ordered on one stream.
 * workspace == NULL uses a library-owned workspace per (device, stream),
 * allocated on first use, whose tickets live apart from the partials. */
TQK_API int tqk_workspace_init(void *workspace, size_t bytes, tqk_stream_t stream);
TQK_API int tqk_decode_q8(const tqk_decode_args *a, void *workspace, size_t workspace_bytes, tqk_stream_t stream);

/* tqk_decode_q8 without any device allocation (no counterpart in the
 * reference): for callers that cannot allocate device memory at run time, for
 * instance a runtime whose memory is fully reserved up front.  The split
 * tickets and partials live in fixed static device arrays of this library
 * (tickets for 16384 units, 4 MiB of partials, present from module load); nothing else
 * is allocated, not even the device error word.  Same arguments as
 * tqk_decode_q8, and the same automatic split for equal lengths.  For a ragged
 * batch it always takes the fixed split, never tqk_decode_q8's balanced
 * schedule: the split merge then combines in another order, so the output
 * agrees with tqk_decode_q8's within the decode tolerance rather than bit for
 * bit, and ragged batches may run slower.
 *   - Calls whose split needs more than 16384 (item, head unit) pairs or more
 *     than 4 MiB of partials fail with TQK_EWORKSPACE; use tqk_decode_q8 with
 *     a workspace, or a larger split_tokens.
 *   - Each call clears its tickets on the stream (one memset) before the
 *     kernel, so nothing needs initialising by the caller.
 *   - The first call on a device sets up that device (looks up the static
 *     arrays' addresses and the kernels' attributes); make it before any
 *     stream capture begins.
 *   - The arrays are shared by every call in the process: calls that may
 *     overlap (other streams, other host threads) race on them and give wrong
 *     results; order such calls on one stream.
 *   - Device-side checks (lengths from a device array outside [0, max_tokens],
 *     pipeline waits over 1 s) still clamp or stop safely, but there is no
 *     error word to report them: tqk_device_status does not see this entry. */
TQK_API int tqk_decode_q8_static(const tqk_decode_args *a, tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * The projections around the attention: Q8 / Q4 weight rows (the reference's
 * packed format, packer/packer.h:9-10) times Q8 activations.  Bit-exact with
 * the reference's scalar kernels: each output adds, in block order,
 * (float)(int dot) * w.d * x.d rounded left to right.
 */
typedef struct { float d; uint8_t q[16]; } tqk_block_q4;  /* low nibble: element j, high: j + 16; value - 8 */
#define TQK_FMT_Q8 0
#define TQK_FMT_Q4 1

/* pack_matrix / packed_matrix_bytes (packer/packer.c:63-88) on the device:
 * fp32 rows W [rows][cols] (cols % 32 == 0) to Q8 ('8') or Q4 ('4') blocks in
 * out, bit-exact (scale max|w|/qmax, 1.0 for an all-zero block, values
 * lroundf(w / scale) clamped to +-127 / +-7).  tqk_packed_matrix_bytes returns
 * 0 for invalid arguments, as the reference's returns 0. */
TQK_API size_t tqk_packed_matrix_bytes(int rows, int cols, char bit_type);
TQK_API int tqk_pack_matrix(const float *W, int rows, int cols, void *out, char bit_type, tqk_stream_t stream);

/* matmul_q8_scalar / matmul_q4_scalar (kernel/q8_scalar.c:15-22,
 * kernel/q4_scalar.c:17-24; MatmulFn of kernel/kernel.h:17): y[r] = W[r] . xq
 * for rows x cols (cols % 32 == 0), all pointers on the device. */
TQK_API int tqk_matmul_q8(const tqk_block_q8 *W, const tqk_block_q8 *xq, float *y, int rows, int cols,
                          tqk_stream_t stream);
TQK_API int tqk_matmul_q4(const tqk_block_q4 *W, const tqk_block_q8 *xq, float *y, int rows, int cols,
                          tqk_stream_t stream);
/* matmul_*_scalar_batch (q8_scalar.c:25-29, q4_scalar.c:27-31; MatmulBatchFn,
 * kernel/kernel.h:21): n_tok activation rows xq [n_tok][cols/32], outputs
 * y[t*rows + r].  Up to 8 tokens share one read of W; more are looped. */
TQK_API int tqk_matmul_q8_batch(const tqk_block_q8 *W, const tqk_block_q8 *xq, float *y, int rows, int cols,
                                int n_tok, tqk_stream_t stream);
TQK_API int tqk_matmul_q4_batch(const tqk_block_q4 *W, const tqk_block_q8 *xq, float *y, int rows, int cols,
                                int n_tok, tqk_stream_t stream);

/* One matrix of a projection call: `rows` weight rows w (Q8 or Q4 blocks,
 * device), outputs y[t*rows + r] (device). */
typedef struct {
    const void *w;
    float *y;
    int rows;
} tqk_proj_job;
/* quantize_row_q8 of n_tok fp32 rows x [n_tok][cols] (bit-exact with
 * kernel/quant_x.c:12-34) and every job's matmul, in one launch: project_qkv
 * (model/attention_layer.c:38-46: jobs wq, wk, wv), project_output (:161-167:
 * job wo) and their batched forms (:207-214, :239-242).  1 to 4 jobs, all of
 * `format` (TQK_FMT_Q8 / TQK_FMT_Q4) and `cols` columns; weights 4-byte aligned
 * (16-byte aligned rows of whole 16-byte units take the TMA path). */
TQK_API int tqk_project(const tqk_proj_job *jobs, int n_jobs, int format, const float *x, int cols, int n_tok,
                        tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * One attention layer for one token, on the device: attention_layer
 * (model/attention_layer.c:169-194) -- project_qkv, norm_heads + rope_heads,
 * store_kv + attend_q8, project_output -- as three launches (q/k/v
 * projection with the activation quantisation, decode with the fused norm,
 * RoPE and append, output projection) chained by programmatic dependent
 * launch, so each launch's weight prefetch overlaps the previous kernel.
 * The appended cache rows are bit-exact with the reference's; the output
 * follows the decode's tolerance through the output projection.
 */
typedef struct {
    const void *wq, *wk, *wv, *wo;     /* packed weight rows (device), all of `format` */
    int format;                        /* TQK_FMT_Q8 or TQK_FMT_Q4 */
    const float *q_norm, *k_norm;      /* [head_dim] each (device) */
    int n_q_heads, n_kv_heads, head_dim, hidden_size;
    float rms_eps;
    tqk_block_q8 *k, *v;               /* the layer's cache planes [n_kv][max_tokens][head_dim/32] (device) */
    int max_tokens;
    int pos;                           /* the token's position: appended at pos, attention over [0, pos] */
    const int32_t *len;                /* optional device int holding pos + 1, read when the kernels run
                                          (CUDA-graph replay across tokens); pos then only bounds it */
    const float *rope_cos, *rope_sin;  /* rope_table of the position, [head_dim/2] each (device) */
    const float *xn;                   /* [hidden_size] input (device) */
    float *out;                        /* [hidden_size] output (device) */
    float *scratch;                    /* device floats: 2*n_q*head_dim + 2*n_kv*head_dim (q, k, v, attention) */
} tqk_attn_layer_args;
/* workspace: as tqk_decode_q8's (NULL = library-owned); a call made under
 * stream capture needs a caller workspace, or one earlier call on the same
 * stream outside capture. */
TQK_API int tqk_attention_layer(const tqk_attn_layer_args *a, void *workspace, size_t workspace_bytes,
                                tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * One token through a whole decoder stack on the device: tq_forward_token
 * (reference model/context.c:104-122) -- embed_lookup, then per layer
 * rmsnorm + attention_layer + residual add, rmsnorm + mlp_layer + residual
 * add (model/context.c:83-102, model/mlp.c:3-17), the final rmsnorm and the
 * lm_head over the tied embedding (model/embedding.c:36-41) -- with weights,
 * norms and Q8 caches in HBM.  Every matrix shares one format (TQK_FMT_Q8 or
 * TQK_FMT_Q4; the reference's packed rows).  Every step is the reference's
 * arithmetic except two: the decode's tolerance (within 1e-3, as everywhere),
 * and the RMSNorms, which add their squares in a fixed tree rather than the
 * reference's serial chain of hidden_size terms (which would cost about 8 us
 * per norm at 4096).  Either can move an activation's Q8 rounding by one step
 * now and then, so the logits and the appended cache rows agree with the
 * reference's within tolerance rather than bit for bit.
 */
typedef struct {
    const float *input_norm, *post_norm;   /* [hidden] (device) */
    const void *wq, *wk, *wv, *wo;          /* attention projections (device) */
    const float *q_norm, *k_norm;          /* [head_dim] (device) */
    const void *wgate, *wup, *wdown;        /* MLP: [inter][hidden], [inter][hidden], [hidden][inter] */
    tqk_block_q8 *k_cache, *v_cache;       /* the layer's Q8 planes [n_kv][max_tokens][head_dim/32] */
} tqk_layer_weights;
typedef struct {
    int n_layers, n_q_heads, n_kv_heads, head_dim, hidden_size, intermediate_size, vocab_size, max_tokens;
    float rms_eps;
    int format;                            /* TQK_FMT_Q8 or TQK_FMT_Q4 */
    const void *embed;                     /* [vocab][hidden] packed rows (device); also the lm_head */
    const float *final_norm;               /* [hidden] (device) */
    const float *rope_cos, *rope_sin;      /* rope_table (model/rope.c:4-12) of every position,
                                              [max_tokens][head_dim/2] (device), as the host's libm gives it */
    const tqk_layer_weights *layers;       /* HOST array of n_layers, device pointers inside */
} tqk_model;
/* Bytes of device scratch tqk_forward_token needs (the residual stream, its
 * norm, the MLP's gate and up rows and one attention layer's scratch). */
TQK_API size_t tqk_forward_scratch_bytes(const tqk_model *m);
/* One token at position pos (the caches hold positions [0, pos)): logits
 * [vocab_size] (device); next_token (device int, or NULL) receives the greedy
 * choice of sample_greedy (model/sampler.c:3-13).  Returns -1 (TQK_EPOS), as
 * the reference does, for pos outside [0, max_tokens) or a token outside
 * [0, vocab_size), before touching anything.  workspace: as tqk_decode_q8's. */
TQK_API int tqk_forward_token(const tqk_model *m, int token, int pos, void *scratch, float *logits,
                              int32_t *next_token, void *workspace, size_t workspace_bytes, tqk_stream_t stream);

/* attend_q8 for one layer of one sequence: n = pos + 1 positions
 * (reference model/attention_layer.c:125-150); TQK_EPOS if pos is out of range. */
TQK_API int tqk_attend_q8(const tqk_block_q8 *k_plane, const tqk_block_q8 *v_plane, int n_q_heads, int n_kv_heads,
                  int head_dim, int max_tokens, int pos, const float *q, float *out, tqk_stream_t stream);

/* store_kv + attend_q8 of one decode step for one layer, fused in one launch. */
TQK_API int tqk_append_attend_q8(tqk_block_q8 *k_plane, tqk_block_q8 *v_plane, int n_q_heads, int n_kv_heads,
                         int head_dim, int max_tokens, int pos, const float *q, const float *k,
                         const float *v, float *out, tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * Chunked causal prefill (attention_layer_batch's append+attend loop, reference
 * model/attention_layer.c:221-236): appends n tokens at pos0..pos0+n-1, then
 * token i attends over positions <= pos0+i.  q/out [n][n_q][hd], k/v [n][n_kv][hd].
 * For head_dim 128 and 1, 2, 4 or 8 q heads per kv head the attention runs on
 * the tensor cores after the cache rows 0 .. pos0+n-1 are staged as MMA
 * operands in a library-owned buffer per (device, stream), allocated on the
 * first call and grown when a call needs more: n_kv * ceil((pos0+n)/32) *
 * 20992 bytes (21.5 MB for 8 kv heads and 4096 positions).  Other shapes use
 * the decode kernel, one item per new token.
 */
TQK_API int tqk_prefill_q8(tqk_block_q8 *k_plane, tqk_block_q8 *v_plane, int n_q_heads, int n_kv_heads,
                   int head_dim, int max_tokens, int pos0, int n, const float *q, const float *k,
                   const float *v, float *out, tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * Log-sum-exp merge of n_parts partials written with TQK_OUT_PARTIAL (e.g. one
 * per GPU of a sequence split, gathered into one buffer): parts is
 * [n_parts][n_heads][head_dim+2], part p at parts + p*part_stride floats.
 * out[h][j] = sum_p acc_p e^{m_p-M} / sum_p l_p e^{m_p-M}, M = max_p m_p.
 */
TQK_API int tqk_merge_partials(const float *parts, int n_parts, int64_t part_stride, int n_heads, int head_dim,
                       float *out, tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * The sequence split's exchange over peer memory (the reference runs on one
 * CPU and has no such step; it replaces the all-gather + tqk_merge_partials
 * pair for ranks on the GPUs of one box).  Each rank allocates a mailbox of
 * tqk_exchange_mailbox_bytes with tqk_peer_buffer_alloc, publishes its IPC
 * handle (tqk_ipc_get_handle), maps every peer's (tqk_ipc_open_handle) and
 * then, once per step with epoch = 1, 2, 3, ...:
 *   1. writes this rank's TQK_OUT_PARTIAL records [n_heads][head_dim+2] into
 *      its own mailbox at byte offset tqk_exchange_slot_offset(epoch) (for
 *      instance as the decode's out);
 *   2. tqk_exchange_merge(..., mailboxes, epoch, out, stream), where
 *      mailboxes[r] is rank r's mailbox as mapped in this process
 *      (mailboxes[rank] = the local one).
 * The kernel raises this rank's flag in every peer's mailbox, waits for every
 * peer's flag of this epoch, reads the peers' records over NVLink and writes the
 * merged output (tqk_merge_partials' arithmetic).  All ranks must make the
 * same calls with the same epoch sequence, each rank on one stream; world <= 8.
 * The wait has a 1 s limit per block of the kernel: when it runs out,
 * tqk_device_status reports TQK_ETIMEOUT and the output is undefined (blocks
 * whose flags arrived in time merged, the others did not).  The mailboxes'
 * flags are then out of step: free them and set up the exchange again (new
 * zeroed mailboxes, epochs from 1) before the next step.
 */
#define TQK_IPC_HANDLE_BYTES 64
TQK_API size_t tqk_exchange_mailbox_bytes(int world, int n_heads, int head_dim);
TQK_API size_t tqk_exchange_slot_offset(int n_heads, int head_dim, int epoch);
TQK_API int tqk_peer_buffer_alloc(size_t bytes, void **ptr);
TQK_API int tqk_peer_buffer_free(void *ptr);
TQK_API int tqk_ipc_get_handle(void *ptr, unsigned char *handle);
TQK_API int tqk_ipc_open_handle(const unsigned char *handle, void **ptr);
TQK_API int tqk_ipc_close_handle(void *ptr);
TQK_API int tqk_exchange_merge(int n_heads, int head_dim, int world, int rank, void *const *mailboxes, int epoch,
                       float *out, tqk_stream_t stream);

/* The kv-head-group split with its gather fused into the decode (the
 * multi-GPU form of attend_q8's loop over kv heads, reference
 * model/attention_layer.c:134-149; the reference's one CPU has no such step).
 * Rank `rank` of `world` decodes its share of the kv heads of every layer
 * (arguments as for tqk_decode_q8, normalised output only), and every unit's
 * finishing CTA writes the unit's output heads straight into every rank's
 * buffer -- over NVLink for the peers -- as {value bits, epoch} pairs of 8
 * bytes, each one store, so that a reader that sees a pair's epoch sees its
 * value: no fence and no flag is needed (a system-scope fence per unit, or
 * even per launch, costs several microseconds on this path).
 *   out[r]: rank r's pair buffer as mapped in this process (r == rank: the
 *     local one), 8-byte aligned, [n_groups][world][chunk_heads][head_dim]
 *     pairs, where the rank's local flat q head f = item * n_q_heads + h lands
 *     in group f / chunk_heads at position f % chunk_heads of the rank's chunk
 *     (for the split of a layer stack: a group is a layer, chunk_heads the
 *     rank's q heads per layer, and the buffer is [layers][n_q_total][hd]);
 *   epoch: the step's number, >= 1, written with every value.
 * tqk_gather_collect then turns the local pairs into the plain output once
 * every pair shows the epoch.  Buffers must be reachable from this device
 * (tqk_peer_buffer_alloc + tqk_ipc_open_handle).  Never uses the balanced
 * schedule (equal lengths use the fixed split anyway).  A caller that reuses
 * a buffer across steps must make sure no rank's next step writes it before
 * every rank has collected it: pair buffers double-buffered by step parity
 * are enough, since a rank's step e + 2 starts only after it has collected
 * step e + 1, which needs every rank's step e + 1 pairs, which each rank
 * writes only after it has collected step e (shard.py, PeerHeadSplit). */
typedef struct {
    int world, rank;                  /* world <= 8 */
    void *out[8];
    int chunk_heads;
    int epoch;
} tqk_gather_dst;
TQK_API int tqk_decode_q8_gather(const tqk_decode_args *a, const tqk_gather_dst *g, void *workspace,
                                 size_t workspace_bytes, tqk_stream_t stream);
/* Head units (the kernels' unit of work) of a tqk_decode_q8_gather call with
 * these arguments. */
TQK_API int tqk_decode_unit_count(const tqk_decode_args *a, int *units);
/* Waits on the stream until each of the n {value bits, epoch} pairs at `pairs`
 * (device memory, 8-byte aligned) shows `epoch`, and writes the values to
 * out[0..n).  Each thread waits at most 1 s in all, then records TQK_ETIMEOUT
 * in the device error word and leaves the value it has (out is then
 * undefined).  It first waits for the kernel launched before it on the
 * stream (the decode) to complete, so that it polls only for the peers' pairs
 * and the next launch may reuse that kernel's workspace. */
TQK_API int tqk_gather_collect(const void *pairs, size_t n, int epoch, float *out, tqk_stream_t stream);

/* The kv-head-group split's gather over peer memory (the multi-GPU form of
 * attend_q8's loop over kv heads, reference model/attention_layer.c:134-149,
 * whose one CPU needs no such step).  Each rank attends to its own kv heads
 * and their q heads for every layer, and every rank needs the whole output.
 * Same mailboxes, IPC set-up, epochs, flags and timeout as tqk_exchange_merge;
 * the mailbox is tqk_gather_mailbox_bytes(world, n_groups, chunk_floats) bytes
 * and per step with epoch e:
 *   1. the rank writes its [n_groups][chunk_floats] floats (for instance the
 *      decode's output, [layers][its q heads][head_dim]) at byte offset
 *      tqk_gather_slot_offset(n_groups, chunk_floats, e) of its own mailbox;
 *   2. tqk_exchange_gather(...) then writes out[g][r][:] = rank r's group g,
 *      out being [n_groups][world][chunk_floats] (16-byte aligned).
 * chunk_floats % 4 == 0 and world * chunk_floats <= 8192; n_groups <= 65535. */
TQK_API size_t tqk_gather_mailbox_bytes(int world, int n_groups, int chunk_floats);
TQK_API size_t tqk_gather_slot_offset(int n_groups, int chunk_floats, int epoch);
TQK_API int tqk_exchange_gather(int n_groups, int chunk_floats, int world, int rank, void *const *mailboxes,
                                int epoch, float *out, tqk_stream_t stream);

/* ---------------------------------------------------------------------------
 * Synthetic inputs (host).  The reference's benches draw every input from one
 * xorshift64 generator through uniform_open / normal_sample, seeded with
 * TQK_REF_SEED (tools/bench_forward.c:82,199-210; tools/bench.c:102,119-130).
 * These fill host memory with the same values, bit for bit on the same C
 * library, from any position of that stream, on `threads` host threads (<= 0:
 * all cores); the values do not depend on the thread count.
 *   tqk_fill_normal:  out[i] = normal_sample #(first + i) * scale
 *                     (normal sample k takes generator steps 2k+1 and 2k+2);
 *   tqk_fill_uniform: out[i] = uniform_open #(first + i), in (0, 1];
 *   tqk_xorshift_jump: the generator state `steps` steps after `state`.
 * The seed must be non-zero. */
#define TQK_REF_SEED 88172645463325252ull
TQK_API int tqk_fill_normal(uint64_t seed, uint64_t first, float *out, size_t n, float scale, int threads);
TQK_API int tqk_fill_uniform(uint64_t seed, uint64_t first, float *out, size_t n, int threads);
TQK_API uint64_t tqk_xorshift_jump(uint64_t state, uint64_t steps);

#ifdef __cplusplus
}
#endif
#endif /* TQK_H */
