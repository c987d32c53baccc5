// tqk_prefill.cu -- chunked causal prefill attention over a Q8 KV cache on the
// sm_100a tensor cores (tcgen05), the attend half of attention_layer_batch
// (reference model/attention_layer.c:221-236: every new token i attends to
// positions 0..pos0+i after the chunk's K/V rows are appended).
//
// One CTA = 128 query rows (T = 128/G tokens x the G q heads of one kv head)
// against that kv head's keys 0 .. pos0 + last token, in 64-key tiles:
//   * a producer warp streams each tile's K and V rows (144-byte Q8 rows) into
//     a 2-stage ring with 1-D TMA bulk copies;
//   * PF_WG warpgroups of consumer threads, PF_WG threads per query row (each
//     takes an equal share of every tile's keys and of O's columns), repack
//     the tile once for all rows:
//     K's int8 block values into the canonical no-swizzle K-major layout of
//     the int8 MMA, V dequantised (v * vd) to an fp16 hi + lo pair in the
//     MN-major layout of the f16 MMA;
//   * QK: four kind::i8 MMAs (M=128, N=64, K=32), one per Q8 block, give the
//     exact int32 block dots in TMEM; each thread combines its row's dots as
//     score = sum_b (float)dot_b * (qd_b*kd_b) * scale (model/attn_q8.c:24-31)
//     with packed fp32 fused multiply-adds (scale and log2(e) folded into qd),
//     within a few ulps of attn_scores_q8_scalar's rounding sequence;
//   * softmax: base-2 online softmax per row with a lazily raised running max
//     (the accumulator is rescaled only when the max grows by more than 2^8,
//     which keeps P <= 256 in fp16); P is written as fp16 in the canonical
//     K-major layout;
//   * PV: kind::f16 MMAs (M=128, N=128, K=16) of P against V_hi and V_lo
//     accumulate O in TMEM (fp32); the epilogue divides by the row sum.
// Every wait is bounded (sticky device error word, no trap); TMEM is always
// released.
#include "tqk_internal.h"
#include "tqk_tcgen05.cuh"

#include <cmath>
#include <mutex>

namespace tqk {

namespace {

#ifndef TQK_PF_KT
#define TQK_PF_KT 64
#endif
#ifndef TQK_PF_WG
#define TQK_PF_WG 2
#endif
constexpr int PF_M = 128;          // query rows per CTA
constexpr int PF_KT = TQK_PF_KT;   // keys per tile (32 or 64)
constexpr int PF_WG = TQK_PF_WG;   // consumer warpgroups: row r is held by threads r, 128 + r, ...,
                                   // each taking an equal share of every tile's keys and of O's columns
constexpr int PF_NT = PF_WG * PF_M;            // consumer threads
constexpr int PF_WARPS = PF_NT / 32;
constexpr int PF_THREADS = PF_NT + 32;         // + the producer warp
constexpr int PF_STAGES = 2;
constexpr int PF_HD = 128;
constexpr int PF_NB = PF_HD / QK;
constexpr int PF_ROW = PF_NB * BLOCK_BYTES;  // 144
constexpr int PF_KH = PF_KT / PF_WG;         // keys of a tile per thread
constexpr int PF_TMEM_O = PF_NB * PF_KT;     // S: 4 blocks x PF_KT int32 columns, then O: 128 fp32 columns
constexpr int PF_TMEM_COLS = PF_TMEM_O + PF_HD <= 256 ? 256 : 512;
constexpr int PF_CTAS_PER_SM = 512 / PF_TMEM_COLS;  // TMEM bound; shared memory is sized to match
constexpr uint64_t PF_WAIT_NS = 1000000000ull;
constexpr uint64_t PF_DRAIN_NS = 20000000ull;

constexpr int RAW_TILE = PF_KT * PF_ROW;         // 9216
constexpr int OFF_RING = 0;                      // [stage][K raw, V raw]
constexpr int OFF_QC = OFF_RING + PF_STAGES * 2 * RAW_TILE;  // int8 Q, 4 blocks x [128 rows x 32 B]
constexpr int OFF_KC = OFF_QC + PF_NB * PF_M * 32;            // int8 K, 4 blocks x [64 keys x 32 B]
constexpr int OFF_VH = OFF_KC + PF_NB * PF_KT * 32;           // fp16 V hi [64 keys x 128 cols], MN-major
constexpr int OFF_VL = OFF_VH + PF_KT * PF_HD * 2;            // fp16 V lo
constexpr int OFF_PC = OFF_VL + PF_KT * PF_HD * 2;            // fp16 P [128 rows x 64 keys], K-major
constexpr int OFF_KD = OFF_PC + PF_M * PF_KT * 2;             // float kd [4 blocks][64 keys]
constexpr int OFF_QD = OFF_KD + PF_KT * PF_NB * 4;            // float qd [128 rows][4 blocks]
constexpr int OFF_MX = OFF_QD + PF_M * PF_NB * 4;             // float [2][128]: half-tile maxima, then sums
constexpr int OFF_BAR = OFF_MX + PF_WG * PF_M * 4;            // full[2], empty[2], s_done, pv_done
constexpr int OFF_TMEM = OFF_BAR + 6 * 8;
constexpr int PF_USED = OFF_TMEM + 16;
// more than 1/(n+1) of an SM's shared memory: at most PF_CTAS_PER_SM CTAs per SM, so a TMEM
// allocation never waits
constexpr int PF_SMEM_FLOOR = 228 * 1024 / (PF_CTAS_PER_SM + 1) + 1024;
constexpr int PF_SMEM = PF_USED > PF_SMEM_FLOOR ? PF_USED : PF_SMEM_FLOOR;
static_assert(PF_USED + 1024 <= 228 * 1024 / PF_CTAS_PER_SM, "shared memory must allow PF_CTAS_PER_SM CTAs");
static_assert(PF_KH % 16 == 0 && PF_KT % 16 == 0, "tile shape");
static_assert(OFF_QC % 1024 == 0 && OFF_KC % 16 == 0 && OFF_VH % 16 == 0 && OFF_PC % 16 == 0, "operand alignment");

// Core-matrix offsets of the canonical no-swizzle layouts (bytes).
//   Q / K blocks: K-major, 32 B of K per row: LBO 128 (K chunk), SBO 256 (8-row group).
__device__ __forceinline__ int qk_off(int row, int kc) { return (row >> 3) * 256 + kc * 128 + (row & 7) * 16; }
//   P: K-major, PF_KT keys = PF_KT/8 chunks per row: LBO 128, SBO PF_SBO.
//   V: MN-major, 8-column chunks: chunk (key, cg) at cg*PF_SBO + (key/8)*128 + (key%8)*16 (LBO 128).
constexpr int PF_SBO = PF_KT / 8 * 128;
__device__ __forceinline__ int p_off(int row, int kc) { return (row >> 3) * PF_SBO + kc * 128 + (row & 7) * 16; }
__device__ __forceinline__ int v_off(int key, int cg) { return cg * PF_SBO + (key >> 3) * 128 + (key & 7) * 16; }

struct PrefillParams {
    const uint8_t *k, *v;  // planes [n_kv][max_tokens][144 B]
    int n_kv, max_tokens, pos0, n;
    const float *q;        // [n][n_q][128]
    float *out;            // [n][n_q][128]
    float scale;
    int *err;
};

__device__ __forceinline__ uint32_t pack2_f16(float a, float b) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}
__device__ __forceinline__ float f16_lo_to_f32(uint32_t h) {
    float f;
    asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tcvt.f32.f16 %0, lo;\n\t}" : "=f"(f) : "r"(h));
    return f;
}
__device__ __forceinline__ float f16_hi_to_f32(uint32_t h) {
    float f;
    asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tcvt.f32.f16 %0, hi;\n\t}" : "=f"(f) : "r"(h));
    return f;
}
typedef unsigned long long pf2;  // packed fp32 pair
__device__ __forceinline__ pf2 pk(float x, float y) {
    pf2 r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(x), "f"(y));
    return r;
}
__device__ __forceinline__ void upk(pf2 v, float &x, float &y) { asm("mov.b64 {%0,%1}, %2;" : "=f"(x), "=f"(y) : "l"(v)); }
__device__ __forceinline__ pf2 mul2p(pf2 a, pf2 b) {
    pf2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ pf2 fma2p(pf2 a, pf2 b, pf2 c) {
    pf2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// 2^x (MUFU approximation, flushes denormal results to zero): P needs ~11 bits.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int G>
__global__ void __launch_bounds__(PF_THREADS, PF_CTAS_PER_SM) prefill_q8_tc_kernel(const PrefillParams p) {
    constexpr int T = PF_M / G;  // tokens per CTA
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tb = gridDim.x - 1 - blockIdx.x;  // longest key ranges first
    const int kvh = blockIdx.y;
    const int tok0 = tb * T;
    const int tok_last = min(tok0 + T, p.n) - 1;
    const int n_keys = p.pos0 + tok_last + 1;
    const int n_tiles = (n_keys + PF_KT - 1) / PF_KT;
    const long long head_bytes = (long long)p.max_tokens * PF_ROW;

    uint64_t *full = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *empty = full + PF_STAGES;
    uint64_t *s_done = empty + PF_STAGES;
    uint64_t *pv_done = s_done + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_TMEM);

    if (tid == 0) {
        for (int s = 0; s < PF_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], PF_WARPS);
        }
        mbar_init(s_done, 1);
        mbar_init(pv_done, 1);
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, PF_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // ---- producer warp: K and V rows of each 64-key tile
    if (warp == PF_WARPS) {
        if (lane == 0) {
            const uint8_t *kh = p.k + kvh * head_bytes, *vh = p.v + kvh * head_bytes;
            for (int j = 0; j < n_tiles; j++) {
                const int slot = j % PF_STAGES;
                if (j >= PF_STAGES &&
                    !mbar_wait_bounded(&empty[slot], (uint32_t)(((j / PF_STAGES) - 1) & 1), PF_WAIT_NS, p.err))
                    break;
                const uint32_t bytes = (uint32_t)(min(PF_KT, n_keys - j * PF_KT) * PF_ROW);
                uint8_t *dst = smem + OFF_RING + slot * 2 * RAW_TILE;
                mbar_arrive_expect_tx(&full[slot], 2 * bytes);
                bulk_copy_g2s(dst, kh + (long long)j * PF_KT * PF_ROW, bytes, &full[slot]);
                bulk_copy_g2s(dst + RAW_TILE, vh + (long long)j * PF_KT * PF_ROW, bytes, &full[slot]);
            }
        }
        return;
    }

    // ---- consumers: thread (wg, r) = half wg of query row r
    const int wg = tid >> 7, r = tid & (PF_M - 1);
    const int token = tok0 + r / G;
    const bool valid_row = token <= tok_last;
    const int head = kvh * G + r % G;
    const int limit = p.pos0 + token;  // last key the row may see (causal)
    uint8_t *qc = smem + OFF_QC, *kc = smem + OFF_KC, *vhi = smem + OFF_VH, *vlo = smem + OFF_VL, *pc = smem + OFF_PC;
    float *kdT = reinterpret_cast<float *>(smem + OFF_KD);
    float *qd_s = reinterpret_cast<float *>(smem + OFF_QD);
    float *mx_s = reinterpret_cast<float *>(smem + OFF_MX);
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;

    // quantise the row's q (quant_x.c:12-34) into the int8 A operand: this thread's share of the blocks
    {
        const float4 *src = reinterpret_cast<const float4 *>(
            p.q + ((long long)(valid_row ? token : tok0) * (p.n_kv * G) + head) * PF_HD);
#pragma unroll
        for (int bb = 0; bb < PF_NB / PF_WG; bb++) {
            const int b = (PF_NB / PF_WG) * wg + bb;
            float x[QK];
#pragma unroll
            for (int i = 0; i < QK / 4; i++) {
                const float4 v4 = __ldg(src + b * (QK / 4) + i);
                x[4 * i] = v4.x, x[4 * i + 1] = v4.y, x[4 * i + 2] = v4.z, x[4 * i + 3] = v4.w;
            }
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < QK; i++) amax = q8_absmax(amax, x[i]);
            const float d = q8_scale(amax), inv = q8_inverse(d);
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; i++)
                w[i] = (uint32_t)(uint8_t)q8_round(x[4 * i], inv) | ((uint32_t)(uint8_t)q8_round(x[4 * i + 1], inv) << 8) |
                       ((uint32_t)(uint8_t)q8_round(x[4 * i + 2], inv) << 16) |
                       ((uint32_t)(uint8_t)q8_round(x[4 * i + 3], inv) << 24);
            if (!valid_row) {
#pragma unroll
                for (int i = 0; i < 8; i++) w[i] = 0u;
            }
            qd_s[r * PF_NB + b] = valid_row ? d : 0.0f;
            *reinterpret_cast<uint4 *>(qc + b * PF_M * 32 + qk_off(r, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4 *>(qc + b * PF_M * 32 + qk_off(r, 1)) = make_uint4(w[4], w[5], w[6], w[7]);
        }
    }
    cta_sync<1, PF_NT>();
    pf2 qd2[PF_NB];  // qd * scale * log2(e): scores come out in log2 units
    const float qs = __fmul_rn(p.scale, 1.4426950408889634f);
#pragma unroll
    for (int b = 0; b < PF_NB; b++) qd2[b] = pk(qd_s[r * PF_NB + b] * qs, qd_s[r * PF_NB + b] * qs);

    const uint32_t id_qk = idesc_i8(PF_M, PF_KT);
    const uint32_t id_pv = idesc_f16(PF_M, PF_HD, true);
    const int k_lo = wg * PF_KH;    // this thread's keys of a tile: [k_lo, k_lo + PF_KH)
    const int o_lo = wg * PF_HD / PF_WG;  // this thread's O columns: [o_lo, o_lo + 128 / PF_WG)
    float m = -INFINITY, l = 0.0f;  // running max (log2 units, shared by the row's two threads) and partial sum
    bool bad = false;               // a bounded wait gave up: drain quickly, issue nothing more

    for (int j = 0; j < n_tiles; j++) {
        const int slot = j % PF_STAGES;
        if (!mbar_wait_bounded(&full[slot], (uint32_t)((j / PF_STAGES) & 1), bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err))
            bad = true;
        const uint8_t *rk = smem + OFF_RING + slot * 2 * RAW_TILE, *rv = rk + RAW_TILE;
        const int rows = min(PF_KT, n_keys - j * PF_KT);

        // K: int8 block values -> canonical K-major operand, scales -> kdT
        //    (16-byte pieces (key, block, half), PF_KT*8 of them over PF_NT threads).  A warp takes
        //    8 consecutive keys x 4 blocks: each 8-lane store phase fills one 128-byte row of core
        //    matrices, and the 32 loads of a warp fall in 32 different banks.
#pragma unroll
        for (int id = tid; id < PF_KT * PF_NB * 2; id += PF_NT) {
            const int ln = id & 31, grp = id >> 5;
            const int key = (ln & 7) + 8 * (grp % (PF_KT / 8)), b = ln >> 3, half = grp / (PF_KT / 8);
            const uint32_t *src = reinterpret_cast<const uint32_t *>(rk + key * PF_ROW + b * BLOCK_BYTES + 4 + 16 * half);
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; i++) w[i] = key < rows ? src[i] : 0u;
            *reinterpret_cast<uint4 *>(kc + b * PF_KT * 32 + qk_off(key, half)) = make_uint4(w[0], w[1], w[2], w[3]);
            if (half == 0)
                kdT[b * PF_KT + key] = key < rows ? *reinterpret_cast<const float *>(rk + key * PF_ROW + b * BLOCK_BYTES) : 0.0f;
        }
        // the previous tile's PV MMAs read V and P: wait before overwriting them
        if (j > 0 && !mbar_wait_bounded(pv_done, (uint32_t)((j - 1) & 1), bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err))
            bad = true;
        // V: dequantise v * vd to fp16 hi + lo (8 columns per chunk)
#pragma unroll 2
        for (int i = 0; i < PF_KT * PF_HD / 8 / PF_NT; i++) {
            // a warp takes 8 consecutive keys x 4 blocks at one 8-column offset: conflict-free
            // 16-byte stores (one 128-byte core-matrix row per phase) and 32 banks for the loads
            const int id = tid + PF_NT * i, ln = id & 31, grp = id >> 5;
            const int key = (ln & 7) + 8 * (grp % (PF_KT / 8)), b = ln >> 3, cg = 4 * b + grp / (PF_KT / 8);
            const uint8_t *row = rv + key * PF_ROW + b * BLOCK_BYTES;
            const float vd = key < rows ? *reinterpret_cast<const float *>(row) : 0.0f;
            uint32_t w0 = 0u, w1 = 0u;
            if (key < rows) {
                w0 = *reinterpret_cast<const uint32_t *>(row + 4 + (cg & 3) * 8);
                w1 = *reinterpret_cast<const uint32_t *>(row + 8 + (cg & 3) * 8);
            }
            float x[8];
            s8x4_to_f32(w0, x[0], x[1], x[2], x[3]);
            s8x4_to_f32(w1, x[4], x[5], x[6], x[7]);
            uint32_t h[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float a = __fmul_rn(x[2 * e], vd), c = __fmul_rn(x[2 * e + 1], vd);
                h[e] = pack2_f16(a, c);
                lo[e] = pack2_f16(__fsub_rn(a, f16_lo_to_f32(h[e])), __fsub_rn(c, f16_hi_to_f32(h[e])));
            }
            *reinterpret_cast<uint4 *>(vhi + v_off(key, cg)) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4 *>(vlo + v_off(key, cg)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_release(&empty[slot]);  // the raw stage is consumed

        // ---- S_b = Q_b K_b^T (int32) for the four Q8 blocks
        fence_proxy_async();
        cta_sync<1, PF_NT>();
        if (tid == 0 && !bad) {
            tc_fence_after();
#pragma unroll
            for (int b = 0; b < PF_NB; b++)
                umma_i8(tmem + b * PF_KT, umma_desc(smem_u32(qc + b * PF_M * 32), 128, 256),
                        umma_desc(smem_u32(kc + b * PF_KT * 32), 128, 256), id_qk, false);
            umma_commit(s_done);
        }
        if (!mbar_wait_bounded(s_done, (uint32_t)(j & 1), bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err)) bad = true;
        tc_fence_after();

        // ---- scores of the row's 32 keys (exact reference rounding), log2 units, causal mask
        float s[PF_KH];
        const bool diag = j * PF_KT + PF_KT - 1 > p.pos0 + tok0;  // the tile reaches past some row's last key
#pragma unroll
        for (int c = 0; c < PF_KH / 16; c++) {
            uint32_t dv[PF_NB][16];
#pragma unroll
            for (int b = 0; b < PF_NB; b++) tmem_ld16(tmem + lane_base + b * PF_KT + k_lo + c * 16, dv[b]);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int kk = k_lo + c * 16 + 2 * i;  // key pair kk, kk+1 of the tile
                pf2 acc = pk(0.0f, 0.0f);
#pragma unroll
                for (int b = 0; b < PF_NB; b++) {
                    const pf2 kd2 = *reinterpret_cast<const pf2 *>(kdT + b * PF_KT + kk);
                    acc = fma2p(pk(__int2float_rn((int)dv[b][2 * i]), __int2float_rn((int)dv[b][2 * i + 1])),
                                mul2p(qd2[b], kd2), acc);
                }
                float x0, x1;
                upk(acc, x0, x1);
                if (diag) {
                    if (j * PF_KT + kk > limit) x0 = -INFINITY;
                    if (j * PF_KT + kk + 1 > limit) x1 = -INFINITY;
                }
                s[c * 16 + 2 * i] = valid_row ? x0 : 0.0f;
                s[c * 16 + 2 * i + 1] = valid_row ? x1 : 0.0f;
            }
        }
        float mt = -INFINITY;
#pragma unroll
        for (int kk = 0; kk < PF_KH; kk++) mt = fmaxf(mt, s[kk]);
        if constexpr (PF_WG > 1) {
            mx_s[wg * PF_M + r] = mt;
            tc_fence_before();
            cta_sync<1, PF_NT>();  // every share's maximum is in; every thread is done reading S
#pragma unroll
            for (int w2 = 0; w2 < PF_WG; w2++) mt = fmaxf(mt, mx_s[w2 * PF_M + r]);
        }
        // raise the running max lazily: only when it grows by more than 8 (P stays <= 2^8)
        const bool raise = mt > m + 8.0f;
        const float m_new = raise ? mt : m;
        const float factor = raise ? ex2(m - m_new) : 1.0f;
        if (j > 0 && __any_sync(0xffffffffu, raise && factor != 1.0f)) {
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < PF_HD / PF_WG / 16; c++) {
                uint32_t ov[16];
                tmem_ld16(tmem + lane_base + PF_TMEM_O + o_lo + c * 16, ov);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; i++) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * factor);
                tmem_st16(tmem + lane_base + PF_TMEM_O + o_lo + c * 16, ov);
            }
            tmem_wait_st();
        }
        l *= factor;
        m = m_new;
        float sum = 0.0f;
#pragma unroll
        for (int c8 = 0; c8 < PF_KH / 8; c8++) {
            float pv[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                pv[e] = ex2(s[c8 * 8 + e] - m);
                sum += pv[e];
            }
            *reinterpret_cast<uint4 *>(pc + p_off(r, k_lo / 8 + c8)) =
                make_uint4(pack2_f16(pv[0], pv[1]), pack2_f16(pv[2], pv[3]), pack2_f16(pv[4], pv[5]), pack2_f16(pv[6], pv[7]));
        }
        l += sum;

        // ---- O += P V_hi + P V_lo
        tc_fence_before();
        fence_proxy_async();
        cta_sync<1, PF_NT>();
        if (tid == 0 && !bad) {
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < PF_KT / 16; ks++)
                umma_f16(tmem + PF_TMEM_O, umma_desc(smem_u32(pc + ks * 256), 128, PF_SBO),
                         umma_desc(smem_u32(vhi + ks * 256), 128, PF_SBO), id_pv, j > 0 || ks > 0);
#pragma unroll
            for (int ks = 0; ks < PF_KT / 16; ks++)
                umma_f16(tmem + PF_TMEM_O, umma_desc(smem_u32(pc + ks * 256), 128, PF_SBO),
                         umma_desc(smem_u32(vlo + ks * 256), 128, PF_SBO), id_pv, true);
            umma_commit(pv_done);
        }
    }
    if (n_tiles > 0 &&
        !mbar_wait_bounded(pv_done, (uint32_t)((n_tiles - 1) & 1), bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err))
        bad = true;
    tc_fence_after();

    // ---- epilogue: O / (sum of the shares' partial sums)
    float l_row = l;
    if constexpr (PF_WG > 1) {
        mx_s[wg * PF_M + r] = l;
        cta_sync<1, PF_NT>();
        l_row = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < PF_WG; w2++) l_row += mx_s[w2 * PF_M + r];
    }
    const float inv_l = 1.0f / l_row;
    float *dst = p.out + ((long long)token * (p.n_kv * G) + head) * PF_HD + o_lo;
#pragma unroll
    for (int c = 0; c < PF_HD / PF_WG / 16; c++) {
        uint32_t ov[16];
        tmem_ld16(tmem + lane_base + PF_TMEM_O + o_lo + c * 16, ov);
        tmem_wait_ld();
        if (valid_row && !bad) {
#pragma unroll
            for (int i = 0; i < 4; i++)
                reinterpret_cast<float4 *>(dst + c * 16)[i] =
                    make_float4(__uint_as_float(ov[4 * i]) * inv_l, __uint_as_float(ov[4 * i + 1]) * inv_l,
                                __uint_as_float(ov[4 * i + 2]) * inv_l, __uint_as_float(ov[4 * i + 3]) * inv_l);
        }
    }
    tc_fence_before();
    cta_sync<1, PF_NT>();
    if (warp == 0) tmem_dealloc(tmem, PF_TMEM_COLS);
}

template <int G>
int launch_prefill(const PrefillParams &p, cudaStream_t stream) {
    static std::mutex mu;
    static bool ready[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return fail_cuda(e, "prefill: cudaGetDevice");
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!ready[dev]) {
            e = cudaFuncSetAttribute(prefill_q8_tc_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
            if (e != cudaSuccess) return fail_cuda(e, "prefill_q8_tc_kernel attributes");
            ready[dev] = true;
        }
    }
    constexpr int T = PF_M / G;
    const dim3 grid((unsigned)((p.n + T - 1) / T), (unsigned)p.n_kv);
    prefill_q8_tc_kernel<G><<<grid, PF_THREADS, PF_SMEM, stream>>>(p);
    return check_launch("prefill_q8_tc_kernel");
}

}  // namespace

// Tensor-core prefill attention (after the chunk's K/V rows were appended).
// Returns TQK_EUNSUPPORTED for shapes it does not cover, so the caller can
// use the decode kernel instead.
int prefill_attend_tc(const tqk_block_q8 *k_plane, const tqk_block_q8 *v_plane, int n_q_heads, int n_kv_heads,
                      int head_dim, int max_tokens, int pos0, int n, const float *q, float *out, cudaStream_t stream) {
    if (head_dim != PF_HD || n_kv_heads <= 0 || n_q_heads % n_kv_heads) return TQK_EUNSUPPORTED;
    const int g = n_q_heads / n_kv_heads;
    if (g != 1 && g != 2 && g != 4 && g != 8) return TQK_EUNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(k_plane) & 15) || (reinterpret_cast<uintptr_t>(v_plane) & 15) ||
        (reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
        return TQK_EUNSUPPORTED;
    PrefillParams p{};
    p.k = reinterpret_cast<const uint8_t *>(k_plane);
    p.v = reinterpret_cast<const uint8_t *>(v_plane);
    p.n_kv = n_kv_heads;
    p.max_tokens = max_tokens;
    p.pos0 = pos0;
    p.n = n;
    p.q = q;
    p.out = out;
    p.scale = 1.0f / sqrtf((float)head_dim);  // as attend_q8 computes it (attention_layer.c:131)
    p.err = device_info()->err_word;
    switch (g) {
        case 1: return launch_prefill<1>(p, stream);
        case 2: return launch_prefill<2>(p, stream);
        case 4: return launch_prefill<4>(p, stream);
        default: return launch_prefill<8>(p, stream);
    }
}

}  // namespace tqk
