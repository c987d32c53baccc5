// tqk_pack.cu -- the reference's weight packer on the device: pack_matrix
// (packer/packer.c:4-88) from fp32 rows to Q8 blocks {float d; int8 q[32]} or
// Q4 blocks {float d; uint8 q[16]} (element j in the low nibble and j + 16 in
// the high nibble of byte j, each value + 8), bit-exact.
//
// One thread per 32-element block:
//   d  = max|w| / qmax (IEEE division; NaN never wins the max), 1.0 for an
//        all-zero block (packer.c:11-19)
//   id = 1.0f / d (IEEE division)
//   q  = lroundf(w * id) clamped to +-qmax (packer.c:4-9): the product rounded
//        to fp32, then rounded half away from zero.  A NaN or infinite product
//        gives 0: x86's lroundf returns LONG_MIN there, whose int conversion in
//        the reference keeps the low 32 bits, 0.
#include "tqk_internal.h"

namespace tqk {
namespace {

__device__ __forceinline__ int pack_round(float x, float id, int qmax) {
    const float v = __fmul_rn(x, id);
    if (!isfinite(v)) return 0;
    int q = (int)roundf(v);  // |v| <= qmax * (1 + 2^-23) here: no overflow
    return q > qmax ? qmax : q < -qmax ? -qmax : q;
}

template <bool Q4>
__global__ void pack_rows_kernel(const float *W, uint8_t *out, long long n_blocks, int aligned) {
    constexpr int BB = Q4 ? 20 : 36;
    const float qmax = Q4 ? 7.0f : 127.0f;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_blocks;
         i += (long long)gridDim.x * blockDim.x) {
        const float *src = W + i * QK;
        float v[QK];
        if (aligned) {
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const float4 f = __ldg(reinterpret_cast<const float4 *>(src) + k);
                v[4 * k] = f.x;
                v[4 * k + 1] = f.y;
                v[4 * k + 2] = f.z;
                v[4 * k + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int k = 0; k < QK; k++) v[k] = __ldg(src + k);
        }
        float amax = 0.0f;
#pragma unroll
        for (int k = 0; k < QK; k++) amax = q8_absmax(amax, v[k]);
        float d = __fdiv_rn(amax, qmax);
        if (d == 0.0f) d = 1.0f;
        const float id = __fdiv_rn(1.0f, d);
        uint32_t w[(BB - 4) / 4];
        if constexpr (Q4) {
#pragma unroll
            for (int m = 0; m < 4; m++) {
                uint32_t word = 0;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int j = 4 * m + k;
                    const uint32_t lo = (uint32_t)(pack_round(v[j], id, 7) + 8);
                    const uint32_t hi = (uint32_t)(pack_round(v[j + QK / 2], id, 7) + 8);
                    word |= ((hi << 4) | lo) << (8 * k);
                }
                w[m] = word;
            }
        } else {
#pragma unroll
            for (int m = 0; m < 8; m++) {
                uint32_t word = 0;
#pragma unroll
                for (int k = 0; k < 4; k++) word |= (uint32_t)(uint8_t)pack_round(v[4 * m + k], id, 127) << (8 * k);
                w[m] = word;
            }
        }
        uint32_t *dst = reinterpret_cast<uint32_t *>(out + i * BB);
        dst[0] = __float_as_uint(d);
#pragma unroll
        for (int m = 0; m < (BB - 4) / 4; m++) dst[1 + m] = w[m];
    }
}

}  // namespace
}  // namespace tqk

using namespace tqk;

extern "C" size_t tqk_packed_matrix_bytes(int rows, int cols, char bit_type) {
    if (rows <= 0 || cols <= 0 || cols % QK) return 0;
    const size_t nb = (size_t)(cols / QK);
    if (bit_type == '8') return (size_t)rows * nb * 36;
    if (bit_type == '4') return (size_t)rows * nb * 20;
    return 0;
}

extern "C" int tqk_pack_matrix(const float *W, int rows, int cols, void *out, char bit_type, tqk_stream_t stream) {
    if (tqk_packed_matrix_bytes(rows, cols, bit_type) == 0)
        return fail(TQK_EINVAL, "tqk_pack_matrix: rows, cols (multiple of 32) or bit type ('8' / '4')");
    if (!W || !out) return fail(TQK_EINVAL, "tqk_pack_matrix: NULL pointer");
    if (reinterpret_cast<uintptr_t>(W) % 4 || reinterpret_cast<uintptr_t>(out) % 4)
        return fail(TQK_EINVAL, "tqk_pack_matrix: W and out must be 4-byte aligned");
    int rc = ensure_device();
    if (rc) return rc;
    const long long n_blocks = (long long)rows * (cols / QK);
    const DeviceInfo *d = device_info();
    const long long want = (n_blocks + 255) / 256;
    const long long cap = (long long)(d ? d->sm_count : 148) * 16;
    const unsigned grid = (unsigned)(want < cap ? want : cap);
    const int aligned = reinterpret_cast<uintptr_t>(W) % 16 == 0;
    if (bit_type == '8')
        pack_rows_kernel<false><<<grid, 256, 0, (cudaStream_t)stream>>>(W, static_cast<uint8_t *>(out), n_blocks,
                                                                           aligned);
    else
        pack_rows_kernel<true><<<grid, 256, 0, (cudaStream_t)stream>>>(W, static_cast<uint8_t *>(out), n_blocks,
                                                                          aligned);
    return check_launch("pack_rows_kernel");
}
