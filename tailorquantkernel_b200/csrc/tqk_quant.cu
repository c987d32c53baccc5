// tqk_quant.cu -- bit-exact Q8 quantiser and KV append kernels (sm_100a).
//
// Replaces quantize_row_q8 (reference kernel/quant_x.c:12-34) for device rows
// and the Q8 branch of store_kv (reference model/attention_layer.c:66-90).
// Work unit: one 32-float block per group of 8 lanes; each lane loads 4 floats
// (one float4 when aligned), the group reduces max|x| with 3 shuffles and each
// lane writes one 4-byte word of int8s (lane 0 also the scale), so a warp moves
// 4 blocks = 512 B in and 144 B out per step, fully coalesced.
#include "tqk_internal.h"

namespace tqk {

// Quantise one block: `src` 32 floats, `dst` one block; `sub` = lane % 8.
__device__ __forceinline__ void quantize_block_8lanes(const float *__restrict__ src, uint8_t *__restrict__ dst,
                                                      int sub) {
    float x0, x1, x2, x3;
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        const float4 f = __ldg(reinterpret_cast<const float4 *>(src) + sub);
        x0 = f.x; x1 = f.y; x2 = f.z; x3 = f.w;
    } else {
        x0 = __ldg(src + 4 * sub + 0);
        x1 = __ldg(src + 4 * sub + 1);
        x2 = __ldg(src + 4 * sub + 2);
        x3 = __ldg(src + 4 * sub + 3);
    }
    float m = q8_absmax(q8_absmax(q8_absmax(q8_absmax(0.0f, x0), x1), x2), x3);
    // only this 8-lane group takes part: a warp's other groups may have retired
    const unsigned group_mask = 0xFFu << (threadIdx.x & 24u);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
        const float other = __shfl_xor_sync(group_mask, m, o);
        m = other > m ? other : m;
    }
    const float d = q8_scale(m);
    const float inv = q8_inverse(d);
    const uint32_t w = (uint32_t)(uint8_t)q8_round(x0, inv) | ((uint32_t)(uint8_t)q8_round(x1, inv) << 8) |
                       ((uint32_t)(uint8_t)q8_round(x2, inv) << 16) | ((uint32_t)(uint8_t)q8_round(x3, inv) << 24);
    reinterpret_cast<uint32_t *>(dst + 4)[sub] = w;
    if (sub == 0) *reinterpret_cast<float *>(dst) = d;
}

__global__ void __launch_bounds__(256) quantize_rows_kernel(const float *__restrict__ x, uint8_t *__restrict__ out,
                                                            long long n_blocks) {
    const long long gt = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long blk = gt >> 3;
    // all 8 lanes of a group share blk, so whole groups retire together
    if (blk >= n_blocks) return;
    quantize_block_8lanes(x + blk * QK, out + blk * BLOCK_BYTES, (int)(threadIdx.x & 7));
}

// Append n tokens at pos0..pos0+n-1.  Block index decomposition (fastest first):
// b (block within the row), h (kv head), kv (0 = K, 1 = V), i (token).  Idx is
// the index type: 32-bit whenever the block count fits, so the decomposition
// needs no 64-bit divisions.
template <typename Idx>
__global__ void __launch_bounds__(256) store_kv_kernel(const float *__restrict__ k, const float *__restrict__ v,
                                                       uint8_t *__restrict__ kp, uint8_t *__restrict__ vp, int n_kv,
                                                       int nb, int max_tokens, int pos0, Idx n_blocks) {
    const Idx blk = (Idx)(((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 3);
    if (blk >= n_blocks) return;
    const int b = (int)(blk % (Idx)nb);
    Idx r = blk / (Idx)nb;
    const int h = (int)(r % (Idx)n_kv);
    r /= (Idx)n_kv;
    const int kv = (int)(r & 1);
    const long long i = (long long)(r >> 1);
    const int hd = nb * QK;
    const float *src = (kv ? v : k) + (i * n_kv + h) * (long long)hd + b * QK;
    uint8_t *plane = kv ? vp : kp;
    const long long slot = (long long)h * max_tokens + pos0 + i;
    quantize_block_8lanes(src, plane + (slot * nb + b) * BLOCK_BYTES, (int)(threadIdx.x & 7));
}

}  // namespace tqk

using namespace tqk;

extern "C" int tqk_quantize_rows_q8(const float *x, tqk_block_q8 *out, int rows, int n, tqk_stream_t stream) {
    if (rows < 0 || n < 0 || n % QK != 0) return fail(TQK_EINVAL, "tqk_quantize_rows_q8: n must be a multiple of 32");
    if (rows == 0 || n == 0) return TQK_OK;
    if (!x || !out) return fail(TQK_EINVAL, "tqk_quantize_rows_q8: NULL pointer");
    int rc = ensure_device();
    if (rc) return rc;
    const long long n_blocks = (long long)rows * (n / QK);
    const long long threads = n_blocks * 8;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    quantize_rows_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, reinterpret_cast<uint8_t *>(out), n_blocks);
    return check_launch("quantize_rows_kernel");
}

extern "C" int tqk_store_kv_q8_batch(tqk_block_q8 *k_plane, tqk_block_q8 *v_plane, int n_kv_heads, int head_dim,
                                     int max_tokens, int pos0, int n, const float *k, const float *v,
                                     tqk_stream_t stream) {
    if (n_kv_heads <= 0 || head_dim <= 0 || head_dim % QK != 0 || max_tokens <= 0 || n < 0)
        return fail(TQK_EINVAL, "tqk_store_kv_q8: bad shape");
    if (pos0 < 0 || (long long)pos0 + n > max_tokens) return fail(TQK_EPOS, "tqk_store_kv_q8: position out of range");
    if (n == 0) return TQK_OK;
    if (!k_plane || !v_plane || !k || !v) return fail(TQK_EINVAL, "tqk_store_kv_q8: NULL pointer");
    int rc = ensure_device();
    if (rc) return rc;
    const int nb = head_dim / QK;
    const long long n_blocks = (long long)n * 2 * n_kv_heads * nb;
    const unsigned grid = (unsigned)((n_blocks * 8 + 255) / 256);
    if (n_blocks * 8 <= 0x7fffffffLL)
        store_kv_kernel<unsigned><<<grid, 256, 0, (cudaStream_t)stream>>>(
            k, v, reinterpret_cast<uint8_t *>(k_plane), reinterpret_cast<uint8_t *>(v_plane), n_kv_heads, nb,
            max_tokens, pos0, (unsigned)n_blocks);
    else
        store_kv_kernel<long long><<<grid, 256, 0, (cudaStream_t)stream>>>(
            k, v, reinterpret_cast<uint8_t *>(k_plane), reinterpret_cast<uint8_t *>(v_plane), n_kv_heads, nb,
            max_tokens, pos0, n_blocks);
    return check_launch("store_kv_kernel");
}

extern "C" int tqk_store_kv_q8(tqk_block_q8 *k_plane, tqk_block_q8 *v_plane, int n_kv_heads, int head_dim,
                               int max_tokens, int pos, const float *k, const float *v, tqk_stream_t stream) {
    if (pos < 0 || pos >= max_tokens) return fail(TQK_EPOS, "tqk_store_kv_q8: position out of range");
    return tqk_store_kv_q8_batch(k_plane, v_plane, n_kv_heads, head_dim, max_tokens, pos, 1, k, v, stream);
}
