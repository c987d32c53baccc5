// tqk_ref_ops.cu -- the reference's per-op Q8 attention kernels on the GPU.
//
// attn_scores_q8 / attn_accum_q8 (reference model/attn_q8.c:56-76) and softmax
// (model/softmax.c:4-23) keep their strided, materialised-score contracts so the
// reference's own kernel sweep (tools/test_model.c:1612-1697) can drive them
// through the drop-in library.  They are not the decode fast path (see
// tqk_decode.cu); scores and accum follow the scalar kernels' rounding sequence
// and token order exactly, so both are bit-exact with attn_*_q8_scalar.
#include "tqk_internal.h"

namespace tqk {

// One thread per (q head, token): attn_scores_q8_scalar, model/attn_q8.c:17-34.
__global__ void attn_scores_kernel(const uint8_t *__restrict__ q, int g, const uint8_t *__restrict__ k, int n, int nb,
                                   float scale, float *__restrict__ scores, long long stride) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)g * n) return;
    const int h = (int)(i / n), t = (int)(i % n);
    const uint32_t *kr = reinterpret_cast<const uint32_t *>(k + (long long)t * nb * BLOCK_BYTES);
    const uint32_t *qr = reinterpret_cast<const uint32_t *>(q + (long long)h * nb * BLOCK_BYTES);
    float acc = 0.0f;
    for (int b = 0; b < nb; b++) {
        int sum = 0;
#pragma unroll
        for (int w = 0; w < 8; w++) sum = __dp4a((int)__ldg(qr + b * 9 + 1 + w), (int)__ldg(kr + b * 9 + 1 + w), sum);
        const float dd = __fmul_rn(__uint_as_float(__ldg(qr + b * 9)), __uint_as_float(__ldg(kr + b * 9)));
        acc = __fadd_rn(acc, __fmul_rn(__int2float_rn(sum), dd));
    }
    scores[(long long)h * stride + t] = __fmul_rn(acc, scale);
}

// One thread per (q head, output column), tokens in order: attn_accum_q8_scalar,
// model/attn_q8.c:36-54 (out = 0; out += (w*vd) * q).
__global__ void attn_accum_kernel(const float *__restrict__ w, long long w_stride, int g, const uint8_t *__restrict__ v,
                                  int n, int nb, float *__restrict__ out, long long out_stride) {
    const int hd = nb * QK;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)g * hd) return;
    const int h = (int)(i / hd), j = (int)(i % hd);
    const int b = j / QK, jj = j % QK;
    float o = 0.0f;
    for (int t = 0; t < n; t++) {
        const uint8_t *blk = v + ((long long)t * nb + b) * BLOCK_BYTES;
        const float vd = *reinterpret_cast<const float *>(blk);
        const float q = (float)(int8_t)blk[4 + jj];
        o = __fadd_rn(o, __fmul_rn(__fmul_rn(__ldg(w + (long long)h * w_stride + t), vd), q));
    }
    out[(long long)h * out_stride + j] = o;
}

// One CTA per row: max, exp(x - max), sum, multiply by 1/sum (model/softmax.c:4-23).
__global__ void __launch_bounds__(256) softmax_rows_kernel(float *__restrict__ x, int n, long long stride) {
    float *row = x + (long long)blockIdx.x * stride;
    __shared__ float red[8];
    __shared__ float bcast;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, row[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = red[0];
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) mm = fmaxf(mm, red[i]);
        bcast = mm;
    }
    __syncthreads();
    m = bcast;
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(row[i] - m);
        row[i] = e;
        s += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float ss = 0.0f;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) ss += red[i];
        bcast = 1.0f / ss;
    }
    __syncthreads();
    const float r = bcast;
    for (int i = threadIdx.x; i < n; i += blockDim.x) row[i] *= r;
}

}  // namespace tqk

using namespace tqk;

extern "C" int tqk_attn_scores_q8(const tqk_block_q8 *q, int g, const tqk_block_q8 *k, int n, int nb, float scale,
                                  float *scores, size_t stride, tqk_stream_t stream) {
    if (g < 0 || n < 0 || nb <= 0 || (n > 0 && stride < (size_t)n)) return fail(TQK_EINVAL, "tqk_attn_scores_q8: bad shape");
    if (g == 0 || n == 0) return TQK_OK;
    if (!q || !k || !scores) return fail(TQK_EINVAL, "tqk_attn_scores_q8: NULL pointer");
    int rc = ensure_device();
    if (rc) return rc;
    const long long total = (long long)g * n;
    attn_scores_kernel<<<(unsigned)((total + 127) / 128), 128, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint8_t *>(q), g, reinterpret_cast<const uint8_t *>(k), n, nb, scale, scores,
        (long long)stride);
    return check_launch("attn_scores_kernel");
}

extern "C" int tqk_attn_accum_q8(const float *w, size_t w_stride, int g, const tqk_block_q8 *v, int n, int nb,
                                 float *out, size_t out_stride, tqk_stream_t stream) {
    if (g < 0 || n < 0 || nb <= 0 || out_stride < (size_t)nb * QK) return fail(TQK_EINVAL, "tqk_attn_accum_q8: bad shape");
    if (g == 0) return TQK_OK;
    if (!out || (n > 0 && (!w || !v))) return fail(TQK_EINVAL, "tqk_attn_accum_q8: NULL pointer");
    int rc = ensure_device();
    if (rc) return rc;
    const long long total = (long long)g * nb * QK;
    attn_accum_kernel<<<(unsigned)((total + 127) / 128), 128, 0, (cudaStream_t)stream>>>(
        w, (long long)w_stride, g, reinterpret_cast<const uint8_t *>(v), n, nb, out, (long long)out_stride);
    return check_launch("attn_accum_kernel");
}

extern "C" int tqk_softmax_rows(float *x, int rows, int n, size_t stride, tqk_stream_t stream) {
    if (rows < 0 || n < 0 || (rows > 1 && stride < (size_t)n)) return fail(TQK_EINVAL, "tqk_softmax_rows: bad shape");
    if (rows == 0 || n == 0) return TQK_OK;
    if (!x) return fail(TQK_EINVAL, "tqk_softmax_rows: NULL pointer");
    int rc = ensure_device();
    if (rc) return rc;
    softmax_rows_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(x, n, (long long)stride);
    return check_launch("softmax_rows_kernel");
}
