// tqk_prologue.cu -- the step right before the attention: per-head RMSNorm of q
// and k (norm_heads, reference model/attention_layer.c:48-53, model/rmsnorm.c:4-19)
// and rotary embedding (rope_heads / rope_apply, attention_layer.c:55-60,
// model/rope.c:14-22), as called by attention_layer (attention_layer.c:183-189).
//
// Bit-exact with the reference's fp32 arithmetic, so that the K rows appended
// afterwards quantise to the same Q8 bytes: the squares are added in index
// order with separately rounded products and sums, sqrtf(eps + sum/n) and
// 1/rms are IEEE operations, x*inv_rms*w is scaled left to right, and the
// rotation uses the caller's cos/sin table (rope_table's powf/cosf/sinf values
// are the host libm's, so the table comes from the host).  head_dim 32, 64,
// 128 and 256 take one warp per row (the decode kernels' fused-prologue
// helper); any other even head_dim one thread per row.
#include "tqk_internal.h"

namespace tqk {
namespace {

struct PrologueParams {
    float *q, *k;
    int n_items, n_q, n_kv, head_dim;
    long long q_item_stride, k_item_stride;  // floats
    const float *q_norm, *k_norm;            // [head_dim] per item, or NULL (no norm)
    long long norm_item_stride;              // floats; 0 = shared
    float eps;
    const float *rope_cos, *rope_sin;        // [head_dim/2] per item, or NULL (no rope)
    long long rope_item_stride;              // floats; 0 = shared
};

// Any even head_dim: one thread per head row.
__global__ void qk_norm_rope_kernel(const PrologueParams p) {
    const int item = blockIdx.y;
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= p.n_q + p.n_kv) return;
    const bool is_q = row < p.n_q;
    float *x = is_q ? p.q + item * p.q_item_stride + (long long)row * p.head_dim
                    : p.k + item * p.k_item_stride + (long long)(row - p.n_q) * p.head_dim;
    const float *w = is_q ? p.q_norm : p.k_norm;
    const int n = p.head_dim, half = n / 2;
    float inv_rms = 1.0f;
    if (w) {
        w += item * p.norm_item_stride;
        float sum = 0.0f;
        for (int i = 0; i < n; i++) sum = __fadd_rn(sum, __fmul_rn(x[i], x[i]));
        const float rms = __fsqrt_rn(__fadd_rn(p.eps, __fdiv_rn(sum, (float)n)));
        inv_rms = __fdiv_rn(1.0f, rms);
    }
    const float *ct = p.rope_cos ? p.rope_cos + item * p.rope_item_stride : nullptr;
    const float *st = p.rope_sin ? p.rope_sin + item * p.rope_item_stride : nullptr;
    for (int i = 0; i < half; i++) {
        float x0 = x[i], x1 = x[i + half];
        if (w) {
            x0 = __fmul_rn(__fmul_rn(x0, inv_rms), w[i]);
            x1 = __fmul_rn(__fmul_rn(x1, inv_rms), w[i + half]);
        }
        if (ct) {
            const float c = ct[i], s = st[i];
            x[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            x[i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        } else {
            x[i] = x0;
            x[i + half] = x1;
        }
    }
}

// head_dim = NB*32: one warp per head row, four rows per CTA, with the decode
// kernels' fused-prologue helper (squares staged in shared memory, one serial
// chain per row).
constexpr int PRO_WARPS = 4;

template <int NB>
__global__ void __launch_bounds__(PRO_WARPS * 32) qk_norm_rope_warp_kernel(const PrologueParams p) {
    __shared__ __align__(16) float scratch[PRO_WARPS][pro_stride<NB>()];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.y;
    const int row = blockIdx.x * PRO_WARPS + warp;
    if (row >= p.n_q + p.n_kv) return;  // whole warps
    const bool is_q = row < p.n_q;
    float *x = is_q ? p.q + item * p.q_item_stride + (long long)row * (NB * 32)
                    : p.k + item * p.k_item_stride + (long long)(row - p.n_q) * (NB * 32);
    const float *w = is_q ? p.q_norm : p.k_norm;
    if (w) w += item * p.norm_item_stride;
    const float *cs = p.rope_cos ? p.rope_cos + item * p.rope_item_stride : nullptr;
    const float *sn = p.rope_cos ? p.rope_sin + item * p.rope_item_stride : nullptr;
    float v[1][NB];
#pragma unroll
    for (int b = 0; b < NB; b++) v[0][b] = x[b * 32 + lane];
    warp_norm_rope<NB, 1>(v, w, cs, sn, p.eps, scratch[warp], lane);
#pragma unroll
    for (int b = 0; b < NB; b++) x[b * 32 + lane] = v[0][b];
}

template <int NB>
void launch_warp(const PrologueParams &p, int rows, cudaStream_t stream) {
    const dim3 grid((unsigned)((rows + PRO_WARPS - 1) / PRO_WARPS), (unsigned)p.n_items);
    qk_norm_rope_warp_kernel<NB><<<grid, PRO_WARPS * 32, 0, stream>>>(p);
}

}  // namespace
}  // namespace tqk

using namespace tqk;

extern "C" int tqk_qk_norm_rope(float *q, float *k, int n_items, int64_t q_item_stride, int64_t k_item_stride,
                                int n_q_heads, int n_kv_heads, int head_dim, const float *q_norm, const float *k_norm,
                                int64_t norm_item_stride, float eps, const float *rope_cos, const float *rope_sin,
                                int64_t rope_item_stride, tqk_stream_t stream) {
    if (n_items <= 0 || n_q_heads < 0 || n_kv_heads < 0 || head_dim <= 0 || (head_dim & 1))
        return fail(TQK_EINVAL, "tqk_qk_norm_rope: bad shape (head_dim must be even)");
    if ((n_q_heads && !q) || (n_kv_heads && !k)) return fail(TQK_EINVAL, "tqk_qk_norm_rope: NULL q or k");
    if ((q_norm == nullptr) != (k_norm == nullptr))
        return fail(TQK_EINVAL, "tqk_qk_norm_rope: q_norm and k_norm go together");
    if ((rope_cos == nullptr) != (rope_sin == nullptr))
        return fail(TQK_EINVAL, "tqk_qk_norm_rope: rope_cos and rope_sin go together");
    if (n_items > 65535) return fail(TQK_EINVAL, "tqk_qk_norm_rope: n_items > 65535");
    const int rows = n_q_heads + n_kv_heads;
    if (rows == 0) return TQK_OK;
    int rc = ensure_device();
    if (rc) return rc;
    PrologueParams p{};
    p.q = q;
    p.k = k;
    p.n_items = n_items;
    p.n_q = n_q_heads;
    p.n_kv = n_kv_heads;
    p.head_dim = head_dim;
    p.q_item_stride = q_item_stride ? q_item_stride : (long long)n_q_heads * head_dim;
    p.k_item_stride = k_item_stride ? k_item_stride : (long long)n_kv_heads * head_dim;
    p.q_norm = q_norm;
    p.k_norm = k_norm;
    p.norm_item_stride = norm_item_stride;
    p.eps = eps;
    p.rope_cos = rope_cos;
    p.rope_sin = rope_sin;
    p.rope_item_stride = rope_item_stride;
    const cudaStream_t st = (cudaStream_t)stream;
    switch (head_dim) {
        case 32: launch_warp<1>(p, rows, st); break;
        case 64: launch_warp<2>(p, rows, st); break;
        case 128: launch_warp<4>(p, rows, st); break;
        case 256: launch_warp<8>(p, rows, st); break;
        default: {
            const dim3 grid((unsigned)((rows + 63) / 64), (unsigned)n_items);
            qk_norm_rope_kernel<<<grid, 64, 0, st>>>(p);
        }
    }
    return check_launch("qk_norm_rope_kernel");
}
