// tqk_forward.cu -- one token through a whole decoder stack on the device:
// tq_forward_token (reference model/context.c:104-122) with every step in HBM.
//
//   embed_lookup                    embedding row dequantised       (model/embedding.c:4-34)
//   per layer:
//     rmsnorm(x, input_norm)         residual_rmsnorm_kernel         (model/rmsnorm.c:4-20)
//     attention_layer                tqk_attention_layer (3 launches: q/k/v projection, the decode
//                                    with the fused norm + RoPE + Q8 append, output projection)
//     x += attn; rmsnorm(x, post_norm)  residual_rmsnorm_kernel      (model/vec.c:3-7, context.c:96-98)
//     mlp_layer                      tqk_project (gate, up) -> silu_mul_q8_kernel -> tqk_matmul (down)
//                                    (model/mlp.c:3-17, model/silu.c:6-20)
//     x += mlp                       folded into the next layer's (or the final) rmsnorm launch
//   rmsnorm(x, final_norm) + lm_head  residual_rmsnorm_kernel + tqk_project over the tied embedding
//                                    (model/embedding.c:36-41)
//   greedy sampling (optional)       argmax_kernel                   (model/sampler.c:3-13)
//
// Every kernel is launched with programmatic stream serialization and waits
// for its predecessor before it reads anything, so the projections' weight
// prefetch overlaps the small kernels.  Arithmetic follows the reference's
// fp32 operation order (explicitly rounded intrinsics), except the RMSNorm's
// sum of squares, which the reference adds in one serial chain of
// hidden_size terms: here it is a fixed tree over the CTA (deterministic, but
// not the reference's rounding), which with 4096 terms would otherwise cost
// about 8 us per norm.
#include "tqk_internal.h"

#include <cmath>

namespace tqk {
namespace {

constexpr int FW_THREADS = 1024;

// out[b*32 + j] = d * q (Q8), or d * ((nibble) - 8) with element j in the low
// nibble and j + 16 in the high nibble of byte j (Q4): embed_lookup.
template <int FMT>
__global__ void __launch_bounds__(256) embed_kernel(const uint8_t *table, int token, int cols, float *out) {
    grid_dependency_wait();
    grid_dependents_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= cols) return;
    const int b = i / QK, j = i - b * QK;
    if constexpr (FMT == TQK_FMT_Q8) {
        const uint8_t *blk = table + ((long long)token * (cols / QK) + b) * BLOCK_BYTES;
        out[i] = __fmul_rn(*reinterpret_cast<const float *>(blk), (float)(int8_t)blk[4 + j]);
    } else {
        const uint8_t *blk = table + ((long long)token * (cols / QK) + b) * 20;
        const uint8_t byte = blk[4 + (j & 15)];
        const int nib = j < 16 ? (byte & 0x0F) : (byte >> 4);
        out[i] = __fmul_rn(*reinterpret_cast<const float *>(blk), (float)(nib - 8));
    }
}

// x += y (when y != NULL, the residual add of model/vec.c), then
// out = x * (1 / sqrt(eps + sum(x^2) / n)) * w, left to right as rmsnorm.
__global__ void __launch_bounds__(FW_THREADS) residual_rmsnorm_kernel(float *x, const float *y, const float *w,
                                                                      float *out, int n, float eps) {
    grid_dependency_wait();
    grid_dependents_launch();
    __shared__ float warp_sums[FW_THREADS / 32];
    float sq = 0.0f;
    for (int i = threadIdx.x; i < n; i += FW_THREADS) {
        float xi = x[i];
        if (y) {
            xi = __fadd_rn(xi, y[i]);
            x[i] = xi;
        }
        sq = __fadd_rn(sq, __fmul_rn(xi, xi));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
    if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x < 32) {
        float s = warp_sums[threadIdx.x];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (threadIdx.x == 0) warp_sums[0] = s;
    }
    __syncthreads();
    const float rms = __fsqrt_rn(__fadd_rn(eps, __fdiv_rn(warp_sums[0], (float)n)));
    const float inv = __fdiv_rn(1.0f, rms);
    for (int i = threadIdx.x; i < n; i += FW_THREADS)  // x[i] is this thread's own element
        out[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

// silu(gate) * up, silu(g) = g * (1 / (1 + expf(-g))) (model/silu.c:6-20), fused with the Q8
// quantisation of the result, which is the down projection's input (model/mlp.c:12-14 quantises
// the silu * up row before that matmul): one warp per 32-element block, every step rounded as the
// reference's separate silu_mul and quantize_row_q8, so the blocks are bit-identical to those two
// steps and one launch shorter.
__global__ void __launch_bounds__(256) silu_mul_q8_kernel(const float *gate, const float *up, uint8_t *xq, int n) {
    grid_dependency_wait();
    grid_dependents_launch();
    const int blk = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (blk >= n / QK) return;  // whole warps: blockDim is a multiple of 32
    const int i = blk * QK + lane;
    const float g = gate[i];
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    float d;
    const int8_t q = warp_quantize_block(__fmul_rn(__fmul_rn(g, sig), up[i]), &d);
    uint8_t *o = xq + (long long)blk * BLOCK_BYTES;
    o[4 + lane] = (uint8_t)q;
    if (lane == 0) *reinterpret_cast<float *>(o) = d;
}

// sample_greedy: the index of the first maximum of logits[0..n), scanning as the
// reference does (max starts at logits[0]; only a strictly greater value moves
// it, so NaNs past index 0 are never chosen and a NaN at index 0 keeps 0).
__global__ void __launch_bounds__(FW_THREADS) argmax_kernel(const float *logits, int n, int32_t *out) {
    grid_dependency_wait();
    grid_dependents_launch();
    __shared__ float sv[FW_THREADS / 32];
    __shared__ int si[FW_THREADS / 32];
    float best = -INFINITY;
    int bi = -1;
    for (int i = threadIdx.x; i < n; i += FW_THREADS) {
        const float v = logits[i];
        if (v > best) { best = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi < bi))) { best = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x < 32) {
        best = sv[threadIdx.x];
        bi = si[threadIdx.x];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi < bi))) { best = ov; bi = oi; }
        }
        if (threadIdx.x == 0) *out = (logits[0] != logits[0] || bi < 0) ? 0 : bi;
    }
}

struct ScratchLayout {
    float *x, *xn, *attn, *mlp, *gate, *up, *layer;
    uint8_t *xq;  // the down projection's Q8 input, [inter / 32] blocks
};

// Floats of the attention layer's scratch region.
size_t layer_floats(const tqk_model *m) {
    return 2 * (size_t)m->n_q_heads * m->head_dim + 2 * (size_t)m->n_kv_heads * m->head_dim;
}

ScratchLayout scratch_layout(const tqk_model *m, void *scratch) {
    ScratchLayout s{};
    const size_t hidden = (size_t)m->hidden_size, inter = (size_t)m->intermediate_size;
    float *p = static_cast<float *>(scratch);
    s.x = p;
    s.xn = s.x + hidden;
    s.attn = s.xn + hidden;
    s.mlp = s.attn + hidden;
    s.gate = s.mlp + hidden;
    s.up = s.gate + inter;
    s.layer = s.up + inter;
    s.xq = reinterpret_cast<uint8_t *>(s.layer + ((layer_floats(m) + 3) / 4) * 4);  // 16-byte aligned
    return s;
}

int residual_rmsnorm(float *x, const float *y, const float *w, float *out, int n, float eps, cudaStream_t st) {
    return launch_pdl(residual_rmsnorm_kernel, dim3(1), dim3(FW_THREADS), 0, st, x, y, w, out, n, eps);
}

}  // namespace
}  // namespace tqk

using namespace tqk;

extern "C" size_t tqk_forward_scratch_bytes(const tqk_model *m) {
    if (!m || m->hidden_size <= 0 || m->intermediate_size <= 0 || m->n_q_heads <= 0 || m->n_kv_heads <= 0 ||
        m->head_dim <= 0)
        return 0;
    const size_t floats =
        4 * (size_t)m->hidden_size + 2 * (size_t)m->intermediate_size + ((layer_floats(m) + 3) / 4) * 4;
    return floats * sizeof(float) + (size_t)(m->intermediate_size / QK) * BLOCK_BYTES;
}

extern "C" int tqk_forward_token(const tqk_model *m, int token, int pos, void *scratch, float *logits,
                                 int32_t *next_token, void *workspace, size_t workspace_bytes, tqk_stream_t stream) {
    if (!m || !m->layers || m->n_layers <= 0 || !m->embed || !m->final_norm || !m->rope_cos || !m->rope_sin ||
        !scratch || !logits)
        return fail(TQK_EINVAL, "tqk_forward_token: NULL model, scratch or logits");
    if (m->format != TQK_FMT_Q8 && m->format != TQK_FMT_Q4) return fail(TQK_EINVAL, "tqk_forward_token: format");
    if (m->hidden_size <= 0 || m->hidden_size % QK || m->intermediate_size <= 0 || m->intermediate_size % QK ||
        m->vocab_size <= 0 || m->max_tokens <= 0 || m->head_dim <= 0 || m->head_dim % 2)
        return fail(TQK_EINVAL, "tqk_forward_token: shape");
    // the reference's guards (model/context.c:105-111): -1 for a full cache or a bad token
    if (pos < 0 || pos >= m->max_tokens) return fail(TQK_EPOS, "tqk_forward_token: position out of range");
    if (token < 0 || token >= m->vocab_size) return fail(TQK_EPOS, "tqk_forward_token: token out of range");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    const ScratchLayout s = scratch_layout(m, scratch);
    const int hidden = m->hidden_size, inter = m->intermediate_size;

    if (m->format == TQK_FMT_Q8)
        rc = launch_pdl(embed_kernel<TQK_FMT_Q8>, dim3((hidden + 255) / 256), dim3(256), 0, st,
                        static_cast<const uint8_t *>(m->embed), token, hidden, s.x);
    else
        rc = launch_pdl(embed_kernel<TQK_FMT_Q4>, dim3((hidden + 255) / 256), dim3(256), 0, st,
                        static_cast<const uint8_t *>(m->embed), token, hidden, s.x);
    if (rc) return rc;
    rc = residual_rmsnorm(s.x, nullptr, m->layers[0].input_norm, s.xn, hidden, m->rms_eps, st);
    if (rc) return rc;
    const long long half = m->head_dim / 2;
    for (int l = 0; l < m->n_layers; l++) {
        const tqk_layer_weights &w = m->layers[l];
        if (!w.input_norm || !w.post_norm || !w.wgate || !w.wup || !w.wdown)
            return fail(TQK_EINVAL, "tqk_forward_token: NULL layer weights");
        tqk_attn_layer_args a{};
        a.wq = w.wq;
        a.wk = w.wk;
        a.wv = w.wv;
        a.wo = w.wo;
        a.format = m->format;
        a.q_norm = w.q_norm;
        a.k_norm = w.k_norm;
        a.n_q_heads = m->n_q_heads;
        a.n_kv_heads = m->n_kv_heads;
        a.head_dim = m->head_dim;
        a.hidden_size = hidden;
        a.rms_eps = m->rms_eps;
        a.k = w.k_cache;
        a.v = w.v_cache;
        a.max_tokens = m->max_tokens;
        a.pos = pos;
        a.rope_cos = m->rope_cos + (long long)pos * half;
        a.rope_sin = m->rope_sin + (long long)pos * half;
        a.xn = s.xn;
        a.out = s.attn;
        a.scratch = s.layer;
        rc = tqk_attention_layer(&a, workspace, workspace_bytes, stream);
        if (rc) return rc;
        rc = residual_rmsnorm(s.x, s.attn, w.post_norm, s.xn, hidden, m->rms_eps, st);
        if (rc) return rc;
        const tqk_proj_job gu[2] = {{w.wgate, s.gate, inter}, {w.wup, s.up, inter}};
        rc = tqk_project(gu, 2, m->format, s.xn, hidden, 1, stream);
        if (rc) return rc;
        const int blocks = inter / QK;
        rc = launch_pdl(silu_mul_q8_kernel, dim3((blocks + 7) / 8), dim3(256), 0, st, (const float *)s.gate,
                        (const float *)s.up, s.xq, inter);
        if (rc) return rc;
        const tqk_block_q8 *xq = reinterpret_cast<const tqk_block_q8 *>(s.xq);
        rc = m->format == TQK_FMT_Q8
                 ? tqk_matmul_q8(static_cast<const tqk_block_q8 *>(w.wdown), xq, s.mlp, hidden, inter, stream)
                 : tqk_matmul_q4(static_cast<const tqk_block_q4 *>(w.wdown), xq, s.mlp, hidden, inter, stream);
        if (rc) return rc;
        const float *next_norm = l + 1 < m->n_layers ? m->layers[l + 1].input_norm : m->final_norm;
        rc = residual_rmsnorm(s.x, s.mlp, next_norm, s.xn, hidden, m->rms_eps, st);
        if (rc) return rc;
    }
    const tqk_proj_job head = {m->embed, logits, m->vocab_size};  // lm_head: the tied embedding
    rc = tqk_project(&head, 1, m->format, s.xn, hidden, 1, stream);
    if (rc) return rc;
    if (next_token) rc = launch_pdl(argmax_kernel, dim3(1), dim3(FW_THREADS), 0, st, (const float *)logits,
                                    m->vocab_size, next_token);
    return rc;
}
