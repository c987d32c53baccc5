// tqk_prefill.cu -- chunked causal prefill attention over a Q8 KV cache on the
// sm_100a tensor cores (tcgen05), the attend half of attention_layer_batch
// (reference model/attention_layer.c:221-236: every new token i attends to
// positions 0..pos0+i after the chunk's K/V rows are appended).
//
// Two kernels per call:
//   * stage_kv_tiles_kernel turns each 32-key tile of a kv head's cache rows
//     into an MMA-ready image once: K's int8 block values in the canonical
//     no-swizzle K-major layout of the int8 MMA, the four K scales per key,
//     and V dequantised (v * vd) to an fp16 hi + lo pair in the MN-major
//     layout of the f16 MMA.  Every CTA that reads the tile copies it as it is.
//   * prefill_q8_tc_kernel: one CTA holds two Q tiles of 128 query rows each
//     (128/G tokens x the G q heads of one kv head per tile) and walks that kv
//     head's keys 0 .. pos0 + its last token in 32-key steps.  Warps are
//     specialised:
//       - a TMA warp streams the staged tile images into a 4-stage ring;
//       - an MMA warp issues, per step and Q tile, four kind::i8 MMAs
//         (M=128, N=32, K=32; one per Q8 block, exact int32 block dots into
//         TMEM) and four kind::f16 MMAs (M=128, N=128, K=16) of P against
//         V_hi and V_lo accumulating O in TMEM.  Its shared-memory
//         descriptors are built once; each MMA adds a constant offset;
//       - eight softmax warps per Q tile, two threads per query row (each
//         takes 16 keys of a step and 64 columns of O; the pair shares its
//         row maximum through shared memory), copy the row's block dots out
//         of TMEM and release S at once, so the MMA warp computes the next
//         step's S while they work.  They combine the dots
//         with the Q8 scales as
//         score = sum_b (float)dot_b * (qd_b*kd_b) * scale (model/attn_q8.c:24-31)
//         with packed fp32 fused multiply-adds (scale and log2(e) folded into
//         qd), run a base-2 online softmax with a lazily raised running max
//         (O is rescaled only when the max grows by more than 2^8, which keeps
//         P <= 256 in fp16) and write P as fp16 in the canonical K-major
//         layout, double-buffered.
//     TMEM: per Q tile S (4 x 32 int32 columns) and O (128 fp32 columns) =
//     all 512 columns; one CTA per SM.  CTAs are ordered longest key range
//     first across all kv heads.
// Every wait is bounded (sticky device error word, no trap); TMEM is always
// released and every copy and MMA in flight is waited for before the CTA exits.
#include "tqk_internal.h"
#include "tqk_tcgen05.cuh"

#include <cmath>
#include <mutex>

namespace tqk {

namespace {

constexpr int PF_M = 128;     // query rows per Q tile (TMEM lanes)
constexpr int PF_QT = 2;      // Q tiles per CTA
constexpr int PF_KT = 32;     // keys per step (one staged tile)
constexpr int PF_HD = 128;
constexpr int PF_NB = PF_HD / QK;            // 4 Q8 blocks per row
constexpr int PF_ROW = PF_NB * BLOCK_BYTES;  // 144-byte cache row
// V as an fp16 hi + lo pair (default) or in one fp16 plane (v*vd rounded to
// nearest).  One plane saves half of the P*V MMAs and a third of their
// shared-memory operand reads, but was measured at only 5% faster (254.7 vs
// 268.4 us on config 5) while V's rounding alone then reaches 1e-3 absolute
// error on ordinary chunks and 2.4e-3 with x8 outlier blocks: over the bar.
#ifndef TQK_PF_VLO
#define TQK_PF_VLO 1
#endif
constexpr bool PF_VLO = TQK_PF_VLO != 0;
// P as an fp16 hi + lo pair: with fp16 P alone (about 11 bits) the output's
// absolute error grows with |V| and passed 2e-3 on chunks with x8 outlier
// blocks; P_hi * (V_hi + V_lo) + P_lo * V_hi carries about 21 bits.
#ifndef TQK_PF_PLO
#define TQK_PF_PLO 1
#endif
constexpr bool PF_PLO = TQK_PF_PLO != 0;
constexpr int PF_PPLANES = PF_PLO ? 2 : 1;
constexpr int PF_STAGES = PF_VLO ? 4 : 6;
constexpr int PF_TPR = 2;                      // softmax threads per query row
constexpr int PF_KH = PF_KT / PF_TPR;          // keys of a step per thread
constexpr int PF_OH = PF_HD / PF_TPR;          // O columns per thread
constexpr int PF_SM_WARPS = 4 * PF_TPR * PF_QT;  // softmax warps
constexpr int PF_TMA_WARP = PF_SM_WARPS;
constexpr int PF_MMA_WARP = PF_SM_WARPS + 1;
constexpr int PF_THREADS = 32 * (PF_SM_WARPS + 2);
constexpr uint32_t PF_TMEM_COLS = 512;
constexpr uint32_t S_COLS = PF_NB * PF_KT;                 // S_t: 4 blocks x 32 keys at t*128
constexpr uint32_t TM_O = PF_QT * S_COLS;                  // O_t at 256 + t*128
static_assert(TM_O + PF_QT * PF_HD == PF_TMEM_COLS, "TMEM budget");
constexpr uint64_t PF_WAIT_NS = 1000000000ull;
constexpr uint64_t PF_DRAIN_NS = 20000000ull;

// Staged tile image: one per 32 keys of one kv head.
constexpr int ST_K = 0;                               // int8 K, 4 blocks x [32 keys x 32 B], K-major
constexpr int ST_KD = ST_K + PF_NB * PF_KT * 32;      // float kd [4 blocks][32 keys]
constexpr int ST_VH = ST_KD + PF_NB * PF_KT * 4;      // fp16 (v*vd) hi [32 keys x 128 cols], MN-major
constexpr int ST_VL = ST_VH + PF_KT * PF_HD * 2;      // fp16 lo (with PF_VLO)
constexpr int ST_BYTES = ST_VL + (PF_VLO ? PF_KT * PF_HD * 2 : 0);  // 20992 with the lo plane, 12800 without
static_assert(ST_BYTES % 16 == 0 && ST_VH % 16 == 0 && ST_KD % 16 == 0, "bulk copy / operand alignment");

// CTA shared memory.
constexpr int OFF_RING = 0;                                   // [stage][tile image]
constexpr int OFF_QC = OFF_RING + PF_STAGES * ST_BYTES;       // int8 Q: [tile][block][128 rows x 32 B]
constexpr int QC_TILE = PF_NB * PF_M * 32;                    // 16 KB
constexpr int OFF_PC = OFF_QC + PF_QT * QC_TILE;              // fp16 P: [tile][buf][hi, lo][128 rows x 32 keys], K-major
constexpr int PC_BUF = PF_M * PF_KT * 2;                      // 8 KB per plane
constexpr int OFF_QD = OFF_PC + PF_QT * 2 * PF_PPLANES * PC_BUF;  // float qd [tile][row][block]
constexpr int OFF_MX = OFF_QD + PF_QT * PF_M * PF_NB * 4;     // float [step parity][tile][half][row]: row maxima
constexpr int OFF_SL = OFF_MX + 2 * PF_QT * PF_TPR * PF_M * 4;  // float [tile][half][row]: row sums
constexpr int OFF_BAR = OFF_SL + PF_QT * PF_TPR * PF_M * 4;
// full[4] empty[4] s_full[tile] s_free[tile] p_full[tile][buf] pv_done[tile] o_done.  P has a barrier
// per buffer: the softmax can finish step j+1 before the MMA warp looks at step j, and two completed
// phases on one barrier would be indistinguishable to a parity wait.
constexpr int N_BARS = 2 * PF_STAGES + PF_QT + PF_QT + 2 * PF_QT + PF_QT + 1;
constexpr int OFF_TMEM = OFF_BAR + 8 * N_BARS;
constexpr int PF_SMEM = OFF_TMEM + 16;
// more than half an SM's shared memory: one CTA per SM, so the 512-column TMEM allocation never waits
static_assert(PF_SMEM > 228 * 1024 / 2 && PF_SMEM + 1024 <= 227 * 1024, "one CTA per SM");
static_assert(OFF_QC % 16 == 0 && OFF_PC % 16 == 0 && OFF_BAR % 8 == 0, "operand alignment");

// Core-matrix offsets of the canonical no-swizzle layouts (bytes; a core matrix is 8 rows x 16 B).
//   Q / K blocks: K-major, 32 B of K per row: LBO 128 (K chunk), SBO 256 (8-row group).
//   P: K-major, 32 keys = 64 B per row: LBO 128, SBO 512.
//   V: MN-major, 8-column chunks: chunk (key, cg) at cg*512 + (key/8)*128 + (key%8)*16 (LBO 128, SBO 512).
__host__ __device__ constexpr int qk_off(int row, int kc) { return (row >> 3) * 256 + kc * 128 + (row & 7) * 16; }
constexpr int PV_SBO = PF_KT / 8 * 128;
__host__ __device__ constexpr int p_off(int row, int kc) { return (row >> 3) * PV_SBO + kc * 128 + (row & 7) * 16; }
__host__ __device__ constexpr int v_off(int key, int cg) { return cg * PV_SBO + (key >> 3) * 128 + (key & 7) * 16; }

struct PrefillParams {
    const uint8_t *stage;  // [n_kv][tiles][ST_BYTES]
    long long tiles;       // staged tiles per kv head
    int n_kv, pos0, n;
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
__device__ __forceinline__ pf2 add2p(pf2 a, pf2 b) {
    pf2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// ---- staging: tile j of kv head h -> its MMA-ready image (256 threads)
__global__ void __launch_bounds__(256) stage_kv_tiles_kernel(const uint8_t *k, const uint8_t *v, int max_tokens,
                                                             int n_keys, long long tiles, uint8_t *stage) {
    const int j = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
    // the attention kernel may start its prologue now; it reads the images only after this grid ends
    grid_dependents_launch();
    const long long head = (long long)h * max_tokens * PF_ROW;
    uint8_t *dst = stage + ((long long)h * tiles + j) * ST_BYTES;
    const int key0 = j * PF_KT;
    {
        // K: one 16-byte piece (key, block, half) per thread; 8 consecutive keys fill one core-matrix row
        const int key = t & 31, b = (t >> 5) & 3, half = t >> 7;
        const bool in = key0 + key < n_keys;
        const uint8_t *row = k + head + (long long)(key0 + key) * PF_ROW + b * BLOCK_BYTES;
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (in) {
            const uint32_t *src = reinterpret_cast<const uint32_t *>(row + 4 + 16 * half);
            w = make_uint4(src[0], src[1], src[2], src[3]);
        }
        *reinterpret_cast<uint4 *>(dst + ST_K + b * PF_KT * 32 + qk_off(key, half)) = w;
        if (half == 0) reinterpret_cast<float *>(dst + ST_KD)[b * PF_KT + key] = in ? *reinterpret_cast<const float *>(row) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < PF_KT * PF_HD / 8 / 256; i++) {
        // V: 8 columns (key, cg) of v * vd per step, as an fp16 hi + lo pair
        const int id = t + 256 * i, key = id & 31, cg = id >> 5, b = cg >> 2;
        const bool in = key0 + key < n_keys;
        const uint8_t *row = v + head + (long long)(key0 + key) * PF_ROW + b * BLOCK_BYTES;
        uint32_t w0 = 0u, w1 = 0u;
        float vd = 0.0f;
        if (in) {
            vd = *reinterpret_cast<const float *>(row);
            w0 = *reinterpret_cast<const uint32_t *>(row + 4 + (cg & 3) * 8);
            w1 = *reinterpret_cast<const uint32_t *>(row + 8 + (cg & 3) * 8);
        }
        float x[8];
        s8x4_to_f32(w0, x[0], x[1], x[2], x[3]);
        s8x4_to_f32(w1, x[4], x[5], x[6], x[7]);
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float a = __fmul_rn(x[2 * e], vd), c = __fmul_rn(x[2 * e + 1], vd);
            hi[e] = pack2_f16(a, c);
            lo[e] = pack2_f16(__fsub_rn(a, f16_lo_to_f32(hi[e])), __fsub_rn(c, f16_hi_to_f32(hi[e])));
        }
        *reinterpret_cast<uint4 *>(dst + ST_VH + v_off(key, cg)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        if constexpr (PF_VLO)
            *reinterpret_cast<uint4 *>(dst + ST_VL + v_off(key, cg)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

template <int G>
__global__ void __launch_bounds__(PF_THREADS, 1) prefill_q8_tc_kernel(const PrefillParams p) {
    constexpr int T = PF_M / G;  // tokens per Q tile
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kvh = blockIdx.x;
    const int cb = gridDim.y - 1 - blockIdx.y;  // longest key ranges first, across all kv heads
    const int tok0 = cb * PF_QT * T;
    const int tok_last = min(tok0 + PF_QT * T, p.n) - 1;
    const int n_keys = p.pos0 + tok_last + 1;
    const int n_tiles = (n_keys + PF_KT - 1) / PF_KT;

    uint64_t *full = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *empty = full + PF_STAGES;
    uint64_t *s_full = empty + PF_STAGES;
    uint64_t *s_free = s_full + PF_QT;
    uint64_t *p_full = s_free + PF_QT;  // [tile][buf]
    uint64_t *pv_done = p_full + 2 * PF_QT;
    uint64_t *o_done = pv_done + PF_QT;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_TMEM);
    uint8_t *const qc = smem + OFF_QC, *const pc = smem + OFF_PC;

    if (tid == 0) {
        for (int s = 0; s < PF_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int t = 0; t < PF_QT; t++) {
            mbar_init(&s_full[t], 1);
            mbar_init(&s_free[t], 4 * PF_TPR);  // one arrival per softmax warp of the tile
            mbar_init(&p_full[2 * t], 4 * PF_TPR);
            mbar_init(&p_full[2 * t + 1], 4 * PF_TPR);
            mbar_init(&pv_done[t], 1);
        }
        mbar_init(o_done, 1);
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, PF_TMEM_COLS);

    // softmax thread (qt, hf, r): row r of Q tile qt, half hf of every step's keys and of O's columns
    const int qt = warp / (4 * PF_TPR), hf = (warp >> 2) % PF_TPR, r = (warp & 3) * 32 + lane;
    const int tq0 = tok0 + qt * T;
    const int token = tq0 + r / G;
    const bool valid_row = warp < PF_SM_WARPS && token <= tok_last;
    const int head = kvh * G + r % G;
    float *const sqd = reinterpret_cast<float *>(smem + OFF_QD);
    if (warp < PF_SM_WARPS) {
        // quantise the row's q (quant_x.c:12-34) into the int8 A operand; rows past the chunk get
        // zeros (their scores are 0 and they are never written)
        const float4 *src = reinterpret_cast<const float4 *>(
            p.q + ((long long)(valid_row ? token : tok0) * (p.n_kv * G) + head) * PF_HD);
        const float qs = __fmul_rn(p.scale, 1.4426950408889634f);
#pragma unroll
        for (int bb = 0; bb < PF_NB / PF_TPR; bb++) {
            const int b = hf * (PF_NB / PF_TPR) + bb;  // this thread's share of the row's blocks
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
            sqd[(qt * PF_M + r) * PF_NB + b] = valid_row ? d * qs : 0.0f;
            uint8_t *dst = qc + qt * QC_TILE + b * PF_M * 32;
            *reinterpret_cast<uint4 *>(dst + qk_off(r, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4 *>(dst + qk_off(r, 1)) = make_uint4(w[4], w[5], w[6], w[7]);
        }
        fence_proxy_async();  // Q -> the tensor core's (async) view of shared memory
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool bad = false;  // a bounded wait gave up: drain quickly, issue nothing more

    if (warp == PF_TMA_WARP) {
        // ---- producer: staged tile images into the ring
        if (lane == 0) {
            // launched with programmatic stream serialization behind the staging kernel: the
            // images are complete once it has finished (q, read in the prologue, was complete
            // before the staging kernel started)
            grid_dependency_wait();
            const uint8_t *src = p.stage + (long long)kvh * p.tiles * ST_BYTES;
            int issued = 0;
            for (int j = 0; j < n_tiles; j++) {
                const int slot = j % PF_STAGES;
                if (j >= PF_STAGES &&
                    !mbar_wait_bounded(&empty[slot], (uint32_t)(((j / PF_STAGES) - 1) & 1), PF_WAIT_NS, p.err))
                    break;
                mbar_arrive_expect_tx(&full[slot], ST_BYTES);
                bulk_copy_g2s(smem + OFF_RING + slot * ST_BYTES, src + (long long)j * ST_BYTES, ST_BYTES, &full[slot]);
                issued = j + 1;
            }
            // the CTA must not exit with a copy in flight
            for (int j = issued > PF_STAGES ? issued - PF_STAGES : 0; j < issued; j++)
                mbar_wait_bounded(&full[j % PF_STAGES], (uint32_t)((j / PF_STAGES) & 1), PF_DRAIN_NS, p.err);
        }
        __syncwarp();
    } else if (warp == PF_MMA_WARP) {
        // ---- MMA issue.  Per step j and tile t: QK_t(j+1) as soon as the softmax has copied S_t(j)
        //      out of TMEM, then PV_t(j) once it has written P_(t, j%2).
        if (lane == 0) {
            const uint32_t id_qk = idesc_i8(PF_M, PF_KT);
            const uint32_t id_pv = idesc_f16(PF_M, PF_HD, true);
            // descriptors of the first operand of each kind; the others differ only in the start address
            const uint64_t d_q = umma_desc(smem_u32(qc), 128, 256);
            const uint64_t d_k = umma_desc(smem_u32(smem + OFF_RING + ST_K), 128, 256);
            const uint64_t d_p = umma_desc(smem_u32(pc), 128, PV_SBO);
            const uint64_t d_vh = umma_desc(smem_u32(smem + OFF_RING + ST_VH), 128, PV_SBO);
            const uint64_t d_vl = umma_desc(smem_u32(smem + OFF_RING + ST_VL), 128, PV_SBO);
            auto qk = [&](int t, int j) {
                const uint64_t so = (uint64_t)(((j % PF_STAGES) * ST_BYTES) >> 4);
#pragma unroll
                for (int b = 0; b < PF_NB; b++)
                    umma_i8(tmem + t * S_COLS + b * PF_KT, d_q + ((t * QC_TILE + b * PF_M * 32) >> 4),
                            d_k + so + ((b * PF_KT * 32) >> 4), id_qk, false);
            };
            auto pv = [&](int t, int j) {
                const uint64_t so = (uint64_t)(((j % PF_STAGES) * ST_BYTES) >> 4);
                const uint64_t pa = d_p + (((2 * t + (j & 1)) * PF_PPLANES * PC_BUF) >> 4);
                const uint32_t o = tmem + TM_O + t * PF_HD;
                umma_f16(o, pa, d_vh + so, id_pv, j > 0);
                umma_f16(o, pa + (256 >> 4), d_vh + so + (256 >> 4), id_pv, true);
                if constexpr (PF_VLO) {
                    umma_f16(o, pa, d_vl + so, id_pv, true);
                    umma_f16(o, pa + (256 >> 4), d_vl + so + (256 >> 4), id_pv, true);
                }
                if constexpr (PF_PLO) {
                    const uint64_t pl = pa + (PC_BUF >> 4);
                    umma_f16(o, pl, d_vh + so, id_pv, true);
                    umma_f16(o, pl + (256 >> 4), d_vh + so + (256 >> 4), id_pv, true);
                }
            };
            auto stage_ready = [&](int j) {  // staged tile j is in shared memory
                if (!mbar_wait_bounded(&full[j % PF_STAGES], (uint32_t)((j / PF_STAGES) & 1),
                                       bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err))
                    bad = true;
                tc_fence_after();
            };
            stage_ready(0);
            for (int t = 0; t < PF_QT; t++) {
                if (!bad) qk(t, 0);
                umma_commit(&s_full[t]);
            }
            for (int j = 0; j < n_tiles; j++) {
                for (int t = 0; t < PF_QT; t++) {
                    if (j + 1 < n_tiles) {
                        if (!mbar_wait_bounded(&s_free[t], (uint32_t)(j & 1), bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err))
                            bad = true;
                        if (t == 0) stage_ready(j + 1);
                        tc_fence_after();
                        if (!bad) qk(t, j + 1);
                        umma_commit(&s_full[t]);
                    }
                    if (!mbar_wait_bounded(&p_full[2 * t + (j & 1)], (uint32_t)((j >> 1) & 1),
                                           bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err))
                        bad = true;
                    tc_fence_after();
                    if (!bad) pv(t, j);
                    umma_commit(&pv_done[t]);
                    // both tiles' MMAs on staged tile j are issued: its slot may be refilled once they finish
                    if (t == PF_QT - 1) umma_commit(&empty[j % PF_STAGES]);
                }
            }
            umma_commit(o_done);
            mbar_wait_bounded(o_done, 0u, bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err);  // no MMA outlives the CTA
        }
        __syncwarp();
    } else {
        // ---- softmax: threads (hf = 0, 1) of row r of tile qt share TMEM lane r of S_qt and O_qt
        const int limit = p.pos0 + token;  // last key the row may see (causal)
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        const uint32_t t_s = tmem + lane_base + qt * S_COLS + hf * PF_KH;
        const uint32_t t_o = tmem + lane_base + TM_O + qt * PF_HD + hf * PF_OH;
        const int pair_bar = 1 + qt * 4 + (warp & 3);  // named barrier of the row's two warps
        float *const smx = reinterpret_cast<float *>(smem + OFF_MX);
        float *const ssl = reinterpret_cast<float *>(smem + OFF_SL);
        pf2 qd2[PF_NB];  // qd * scale * log2(e): scores come out in log2 units
#pragma unroll
        for (int b = 0; b < PF_NB; b++) {
            const float dq = sqd[(qt * PF_M + r) * PF_NB + b];
            qd2[b] = pk(dq, dq);
        }
        float m = -INFINITY, l = 0.0f;  // running max (log2 units, the same in both threads) and partial sum

        for (int j = 0; j < n_tiles; j++) {
            if (!mbar_wait_bounded(&s_full[qt], (uint32_t)(j & 1), bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err)) bad = true;
            tc_fence_after();
            const float *kd = reinterpret_cast<const float *>(smem + OFF_RING + (j % PF_STAGES) * ST_BYTES + ST_KD) +
                              hf * PF_KH;
            const int key0 = j * PF_KT + hf * PF_KH;  // this thread's first key of the step
            const bool diag = j * PF_KT + PF_KT - 1 > p.pos0 + tq0;  // the step reaches past some row's last key

            // this thread's 16 scores (the reference's per-block combine), log2 units; S is released
            // to the MMA warp as soon as it is in registers
            uint32_t dv[PF_NB][16];
#pragma unroll
            for (int b = 0; b < PF_NB; b++) tmem_ld16(t_s + b * PF_KT, dv[b]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_release(&s_free[qt]);
            float s[PF_KH];
#pragma unroll
            for (int i2 = 0; i2 < PF_KH / 2; i2++) {
                pf2 acc = mul2p(pk(__int2float_rn((int)dv[0][2 * i2]), __int2float_rn((int)dv[0][2 * i2 + 1])),
                                mul2p(qd2[0], *reinterpret_cast<const pf2 *>(kd + 2 * i2)));
#pragma unroll
                for (int b = 1; b < PF_NB; b++)
                    acc = fma2p(pk(__int2float_rn((int)dv[b][2 * i2]), __int2float_rn((int)dv[b][2 * i2 + 1])),
                                mul2p(qd2[b], *reinterpret_cast<const pf2 *>(kd + b * PF_KT + 2 * i2)), acc);
                upk(acc, s[2 * i2], s[2 * i2 + 1]);
            }
            if (diag) {
#pragma unroll
                for (int kk = 0; kk < PF_KH; kk++)
                    if (key0 + kk > limit) s[kk] = -INFINITY;
            }
            // tree maximum of the 16 scores, then the row's maximum with the partner thread's
            float mx[PF_KH / 2];
#pragma unroll
            for (int kk = 0; kk < PF_KH / 2; kk++) mx[kk] = fmaxf(s[2 * kk], s[2 * kk + 1]);
#pragma unroll
            for (int w2 = PF_KH / 4; w2 >= 1; w2 >>= 1)
#pragma unroll
                for (int kk = 0; kk < w2; kk++) mx[kk] = fmaxf(mx[kk], mx[kk + w2]);
            float *mxs = smx + ((j & 1) * PF_QT + qt) * PF_TPR * PF_M;  // by step parity: no overwrite before read
            mxs[hf * PF_M + r] = mx[0];
            asm volatile("bar.sync %0, %1;" ::"r"(pair_bar), "n"(64) : "memory");
            const float mt = fmaxf(mx[0], mxs[(1 - hf) * PF_M + r]);
            // raise the running max lazily: only when it grows by more than 8 (P stays <= 2^8)
            const bool raise = mt > m + 8.0f;
            const float m_new = raise ? mt : m;
            const float factor = raise ? ex2f(m - m_new) : 1.0f;
            if (j > 0 && __any_sync(0xffffffffu, raise && factor != 1.0f)) {
                // PV_qt(j-1) may still run: wait for it before rescaling this thread's half of O
                if (!mbar_wait_bounded(&pv_done[qt], (uint32_t)((j - 1) & 1), bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err))
                    bad = true;
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < PF_OH / 16; c++) {
                    uint32_t ov[16];
                    tmem_ld16(t_o + c * 16, ov);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; e++) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * factor);
                    tmem_st16(t_o + c * 16, ov);
                }
                tmem_wait_st();
            }
            l *= factor;
            m = m_new;
            const pf2 neg_m = pk(-m, -m), one2 = pk(1.0f, 1.0f);
            uint32_t ph[PF_KH / 2], pl[PF_KH / 2];
            pf2 sum2 = pk(0.0f, 0.0f);
#pragma unroll
            for (int i2 = 0; i2 < PF_KH / 2; i2++) {
                float a, c;
                upk(fma2p(pk(s[2 * i2], s[2 * i2 + 1]), one2, neg_m), a, c);
                const pf2 e2 = pk(ex2f(a), ex2f(c));
                sum2 = add2p(sum2, e2);
                float ea, ec;
                upk(e2, ea, ec);
                ph[i2] = pack2_f16(ea, ec);
                if constexpr (PF_PLO)
                    pl[i2] = pack2_f16(__fsub_rn(ea, f16_lo_to_f32(ph[i2])), __fsub_rn(ec, f16_hi_to_f32(ph[i2])));
            }
            float sa, sb;
            upk(sum2, sa, sb);
            l += sa + sb;
            uint8_t *pb = pc + (2 * qt + (j & 1)) * PF_PPLANES * PC_BUF;
#pragma unroll
            for (int kc = 0; kc < PF_KH / 8; kc++) {
                *reinterpret_cast<uint4 *>(pb + p_off(r, hf * (PF_KH / 8) + kc)) =
                    make_uint4(ph[4 * kc], ph[4 * kc + 1], ph[4 * kc + 2], ph[4 * kc + 3]);
                if constexpr (PF_PLO)
                    *reinterpret_cast<uint4 *>(pb + PC_BUF + p_off(r, hf * (PF_KH / 8) + kc)) =
                        make_uint4(pl[4 * kc], pl[4 * kc + 1], pl[4 * kc + 2], pl[4 * kc + 3]);
            }
            fence_proxy_async();  // P -> the tensor core
            tc_fence_before();    // the O rescale is done
            __syncwarp();
            if (lane == 0) mbar_arrive_release(&p_full[2 * qt + (j & 1)]);
        }

        // ---- epilogue: O / (the two threads' partial sums)
        ssl[(qt * PF_TPR + hf) * PF_M + r] = l;
        if (!mbar_wait_bounded(o_done, 0u, bad ? PF_DRAIN_NS : PF_WAIT_NS, p.err)) bad = true;
        tc_fence_after();
        asm volatile("bar.sync %0, %1;" ::"r"(pair_bar), "n"(64) : "memory");
        const float inv_l = 1.0f / (ssl[(qt * PF_TPR) * PF_M + r] + ssl[(qt * PF_TPR + 1) * PF_M + r]);
        float *dst = p.out + ((long long)token * (p.n_kv * G) + head) * PF_HD + hf * PF_OH;
#pragma unroll
        for (int c = 0; c < PF_OH / 16; c++) {
            uint32_t ov[16];
            tmem_ld16(t_o + c * 16, ov);
            tmem_wait_ld();
            if (valid_row && !bad) {
#pragma unroll
                for (int e = 0; e < 4; e++)
                    reinterpret_cast<float4 *>(dst + c * 16)[e] =
                        make_float4(__uint_as_float(ov[4 * e]) * inv_l, __uint_as_float(ov[4 * e + 1]) * inv_l,
                                    __uint_as_float(ov[4 * e + 2]) * inv_l, __uint_as_float(ov[4 * e + 3]) * inv_l);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, PF_TMEM_COLS);
    }
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
    const dim3 grid((unsigned)p.n_kv, (unsigned)((p.n + PF_QT * T - 1) / (PF_QT * T)));
    return launch_pdl(prefill_q8_tc_kernel<G>, grid, dim3(PF_THREADS), PF_SMEM, stream, p);
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
    if ((reinterpret_cast<uintptr_t>(k_plane) & 3) || (reinterpret_cast<uintptr_t>(v_plane) & 3) ||
        (reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
        return TQK_EUNSUPPORTED;
    const int n_keys = pos0 + n;
    const long long tiles = (n_keys + PF_KT - 1) / PF_KT;
    if (tiles > 65535 || n_kv_heads > 65535) return TQK_EUNSUPPORTED;  // grid limits of the staging launch
    uint8_t *stage = static_cast<uint8_t *>(library_prefill_stage(stream, (size_t)n_kv_heads * tiles * ST_BYTES));
    if (!stage) return fail(TQK_ECUDA, "tqk_prefill_q8: cannot allocate the staging buffer");
    stage_kv_tiles_kernel<<<dim3((unsigned)tiles, (unsigned)n_kv_heads), 256, 0, stream>>>(
        reinterpret_cast<const uint8_t *>(k_plane), reinterpret_cast<const uint8_t *>(v_plane), max_tokens, n_keys,
        tiles, stage);
    int rc = check_launch("stage_kv_tiles_kernel");
    if (rc) return rc;
    PrefillParams p{};
    p.stage = stage;
    p.tiles = tiles;
    p.n_kv = n_kv_heads;
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
