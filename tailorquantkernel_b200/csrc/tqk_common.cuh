// tqk_common.cuh -- device helpers shared by the sm_100a Q8 attention kernels.
//
// * The Q8 block format (36 bytes: fp32 scale + 32 int8) and the bit-exact
//   device quantiser of reference kernel/quant_x.c:5-34.
// * Thin inline-PTX wrappers for the 1-D TMA bulk copy (cp.async.bulk, never the
//   .multicast form) and mbarriers, with time-bounded waits that record an error
//   instead of hanging.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/tqk.h"

namespace tqk {

constexpr int QK = 32;
constexpr int BLOCK_BYTES = 36;
static_assert(sizeof(tqk_block_q8) == BLOCK_BYTES, "tqk_block_q8 must be 36 bytes");

// Device error codes written to the sticky error word (tqk_device_status).
enum : int { DEVERR_NONE = 0, DEVERR_TIMEOUT = 1, DEVERR_BADLEN = 2 };

// Kernels report failures into a sticky per-device error word that the runtime
// allocates (tqk_device_status reads it) and passes to every launch.
__device__ __forceinline__ void record_error(int *err, int code) {
    if (err != nullptr) atomicCAS(err, 0, code);
}

// ----------------------------------------------------------------------------
// Quantiser (reference kernel/quant_x.c:5-34).  Every float operation is an
// explicitly rounded intrinsic so nvcc cannot contract or reorder it:
//   d   = amax / 127.0f           (IEEE division)
//   inv = d != 0 ? 1.0f / d : 0   (IEEE division)
//   q   = low byte of bits(x*inv + 1.5*2^23) - 0x4B400000
// which reproduces the reference's magic-number rounding for every input,
// including Inf/NaN (where a cvt.rni would differ).
// ----------------------------------------------------------------------------
__device__ __forceinline__ float q8_scale(float amax) { return __fdiv_rn(amax, 127.0f); }
__device__ __forceinline__ float q8_inverse(float d) { return d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f; }
// NaN: the reference runs on x86, where x*inv returns x itself (quieted) when
// x is NaN and the "default NaN" 0xFFC00000 for Inf*0 or 0*Inf, and the add
// passes that NaN through; its int8 is the low byte of those bits (0x4B400000
// has a zero low byte).  The GPU would return its canonical 0x7FFFFFFF instead,
// so NaN products are mapped explicitly.
__device__ __forceinline__ int8_t q8_round(float x, float inv) {
    const float v = __fmul_rn(x, inv);
    if (isnan(v)) return isnan(x) ? (int8_t)(__float_as_uint(x) & 0xFFu) : (int8_t)0;
    const float shifted = __fadd_rn(v, 12582912.0f);
    return (int8_t)(__float_as_int(shifted) - 0x4B400000);
}
// |x| as the reference's max loop sees it: NaN never exceeds the running max.
__device__ __forceinline__ float q8_absmax(float a, float x) {
    const float ax = fabsf(x);
    return ax > a ? ax : a;
}

// Quantise one 32-float block held one element per lane of a full warp.
// Returns this lane's int8; *d receives the block scale (all lanes).
__device__ __forceinline__ int8_t warp_quantize_block(float x, float *d) {
    float m = q8_absmax(0.0f, x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float other = __shfl_xor_sync(0xffffffffu, m, o);
        m = other > m ? other : m;
    }
    const float s = q8_scale(m);
    *d = s;
    return q8_round(x, q8_inverse(s));
}

// warp_quantize_block for N blocks at once (block k's element on this lane in
// x[k]), phase by phase across the blocks -- the N max reductions, then the N
// scales, the N inverses and the N roundings -- so the N independent
// shuffle / division chains overlap instead of running one after another.
// Same arithmetic, same results.
template <int N>
__device__ __forceinline__ void warp_quantize_blocks(const float (&x)[N], int8_t (&q)[N], float (&d)[N]) {
    float m[N];
#pragma unroll
    for (int k = 0; k < N; k++) m[k] = q8_absmax(0.0f, x[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int k = 0; k < N; k++) {
            const float other = __shfl_xor_sync(0xffffffffu, m[k], o);
            m[k] = other > m[k] ? other : m[k];
        }
    float inv[N];
#pragma unroll
    for (int k = 0; k < N; k++) d[k] = q8_scale(m[k]);
#pragma unroll
    for (int k = 0; k < N; k++) inv[k] = q8_inverse(d[k]);
#pragma unroll
    for (int k = 0; k < N; k++) q[k] = q8_round(x[k], inv[k]);
}

// The attention prologue on head rows of head_dim = NB*32 floats held by a
// full warp, element b*32 + lane of a row in x[b]: RMSNorm with a weight
// (model/rmsnorm.c:4-19) and then the half-split RoPE rotation with a cos/sin
// table of head_dim/2 floats (model/rope.c:14-22).  Rounds exactly as the
// reference's scalar C: each row's squares are added in index order as one
// chain, sqrt and both divisions are IEEE, products and sums are never
// contracted.
constexpr int PRO_PAD = 4;  // floats of padding per staged row: the R lanes' loads hit distinct banks
template <int NB>
__host__ __device__ constexpr int pro_stride() { return NB * 32 + PRO_PAD; }

// This lane's elements of a norm weight ([head_dim] floats, element b*32 + lane).
template <int NB>
__device__ __forceinline__ void load_row(float (&w)[NB], const float *src, int lane) {
#pragma unroll
    for (int b = 0; b < NB; b++) w[b] = __ldg(src + b * 32 + lane);
}

// This lane's entries of a RoPE table pair ([head_dim/2] floats each): the
// pair (i, i + head_dim/2) sits in one lane for NB >= 2 (element b*32 + lane
// with b + NB/2), and in lanes i and i + 16 for head_dim 32.
template <int NB>
struct RopeTab {
    static constexpr int N = NB >= 2 ? NB / 2 : 1;
    float c[N], s[N];
    __device__ __forceinline__ void load(const float *cs, const float *sn, int lane) {
#pragma unroll
        for (int b = 0; b < N; b++) {
            const int i = NB >= 2 ? b * 32 + lane : (lane & 15);
            c[b] = __ldg(cs + i);
            s[b] = __ldg(sn + i);
        }
    }
};

// Sum of squares of each of R rows, added in index order as one chain per row:
// the squares are staged in `scratch` (R rows of pro_stride<NB>() floats,
// 16-byte aligned, private to the warp) and lane r walks row r with 16-byte
// loads, so the R chains run side by side and only the adds are serial.
template <int NB, int R>
__device__ __forceinline__ void warp_row_sumsq(const float (&x)[R][NB], float *scratch, int lane, float (&sums)[R]) {
    static_assert(R <= 32, "one lane per row");
    constexpr int HD = NB * 32, STRIDE = pro_stride<NB>();
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int b = 0; b < NB; b++) scratch[r * STRIDE + b * 32 + lane] = __fmul_rn(x[r][b], x[r][b]);
    __syncwarp();
    float sum = 0.0f;
    if (lane < R) {
        const float4 *row = reinterpret_cast<const float4 *>(scratch + lane * STRIDE);
#pragma unroll
        for (int i = 0; i < HD / 4; i++) {
            const float4 v = row[i];
            sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, v.x), v.y), v.z), v.w);
        }
    }
    __syncwarp();  // the scratch is free again
#pragma unroll
    for (int r = 0; r < R; r++) sums[r] = __shfl_sync(0xffffffffu, sum, r);
}

// x * (1 / sqrtf(eps + sum/n)) * w, left to right, as model/rmsnorm.c:4-19.
template <int NB>
__device__ __forceinline__ void apply_norm(float (&x)[NB], float sum, const float (&w)[NB], float eps) {
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(eps, __fdiv_rn(sum, (float)(NB * 32)))));
#pragma unroll
    for (int b = 0; b < NB; b++) x[b] = __fmul_rn(__fmul_rn(x[b], inv), w[b]);
}

// (x0, x1) -> (x0*c - x1*s, x0*s + x1*c) per pair, as model/rope.c:14-22.
template <int NB>
__device__ __forceinline__ void apply_rope(float (&x)[NB], const RopeTab<NB> &t, int lane) {
    if constexpr (NB == 1) {
        const float other = __shfl_xor_sync(0xffffffffu, x[0], 16);
        x[0] = lane < 16 ? __fsub_rn(__fmul_rn(x[0], t.c[0]), __fmul_rn(other, t.s[0]))
                         : __fadd_rn(__fmul_rn(other, t.s[0]), __fmul_rn(x[0], t.c[0]));
    } else {
#pragma unroll
        for (int b = 0; b < NB / 2; b++) {
            const float x0 = x[b], x1 = x[b + NB / 2];
            x[b] = __fsub_rn(__fmul_rn(x0, t.c[b]), __fmul_rn(x1, t.s[b]));
            x[b + NB / 2] = __fadd_rn(__fmul_rn(x0, t.s[b]), __fmul_rn(x1, t.c[b]));
        }
    }
}

// The whole prologue on R rows sharing one weight and one table (either
// pointer NULL skips that part).
template <int NB, int R>
__device__ __forceinline__ void warp_norm_rope(float (&x)[R][NB], const float *w, const float *cs, const float *sn,
                                               float eps, float *scratch, int lane) {
    if (w) {
        float wv[NB], sums[R];
        load_row<NB>(wv, w, lane);
        warp_row_sumsq<NB, R>(x, scratch, lane, sums);
#pragma unroll
        for (int r = 0; r < R; r++) apply_norm<NB>(x[r], sums[r], wv, eps);
    }
    if (cs) {
        RopeTab<NB> t;
        t.load(cs, sn, lane);
#pragma unroll
        for (int r = 0; r < R; r++) apply_rope<NB>(x[r], t, lane);
    }
}

// ----------------------------------------------------------------------------
// PTX wrappers: mbarrier + 1-D bulk async copy global -> shared.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Programmatic dependent launch (sm_90+).  grid_dependents_launch lets the
// next kernel on the stream, when it was launched with programmatic stream
// serialization, begin before this grid ends; grid_dependency_wait blocks
// until every prerequisite grid has completed and its memory is visible (a
// no-op when there is none).  Code before the wait may only read data that no
// earlier kernel of the stream writes.
__device__ __forceinline__ void grid_dependents_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Orders this thread's earlier shared-memory accesses (generic proxy) before
// later async-proxy (TMA) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// Plain arrive (count 1) with release semantics: the arriving warp's reads of
// the slot happen before the producer's next copy into it.
__device__ __forceinline__ void mbar_arrive_release(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// try_wait that suspends the thread until the phase completes or about
// `hint_ns` pass, so a waiting warp does not spin on the issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait: sleeps in try_wait until the phase completes or `limit_ns` of
// wall time pass.  Returns false on timeout and records DEVERR_TIMEOUT; never
// waits forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t limit_ns, int *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if (globaltimer_ns() - t0 > limit_ns) {
            record_error(err, DEVERR_TIMEOUT);
            return false;
        }
    }
}

// ----------------------------------------------------------------------------
// Thread-block cluster helpers (sm_90+): distributed shared memory and
// mbarriers that other CTAs of the cluster arrive on.
// ----------------------------------------------------------------------------
// Cluster-wide barrier of every thread of every CTA.  Only for code that every
// thread reaches unconditionally (kernel entry): it has no time bound.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of this CTA's shared-memory location `p` in the CTA of rank `rank`.
__device__ __forceinline__ uint32_t cluster_map(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
// Arrive (count 1, release at cluster scope) on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Bounded wait with acquire at cluster scope (arrivals from other CTAs of the cluster).
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t *bar, uint32_t parity, uint64_t limit_ns,
                                                          int *err) {
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
            : "memory");
        if (ok) return true;
        if (globaltimer_ns() - t0 > limit_ns) {
            record_error(err, DEVERR_TIMEOUT);
            return false;
        }
    }
}

// 1-D TMA bulk copy (non-multicast).  dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_copy_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Barrier over the first NT threads of the CTA (named barrier BAR; 0 = all).
template <int BAR, int NT>
__device__ __forceinline__ void cta_sync() {
    if constexpr (BAR == 0) {
        __syncthreads();
    } else {
        asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
    }
}

// 2^x as the MUFU computes it (ex2.approx, denormal results flushed to zero):
// exact at x = 0 and 0 at x = -inf.  Softmax weights need ~11 bits; the
// running-max correction is written as 1 exactly when the max is unchanged.
__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ----------------------------------------------------------------------------
// int8 helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Four signed bytes of w -> four exact floats, via the 2^23 exponent trick:
// bias each byte to unsigned (xor 0x80), place it in the low mantissa byte of
// 2^23 (0x4B000000) and subtract 2^23 + 128.  All integer ALU + one FADD each.
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float &f0, float &f1, float &f2, float &f3) {
    const uint32_t u = w ^ 0x80808080u;
    const float bias = 8388736.0f;  // 2^23 + 128
    f0 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)), bias);
    f1 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)), bias);
    f2 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)), bias);
    f3 = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)), bias);
}

}  // namespace tqk
