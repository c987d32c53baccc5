// tqk_decode_pack.cuh -- tensor-core Q8 decode with two kv heads packed into
// one MMA row block, for the 4-q-heads-per-kv-head grouping (Llama-3-8B:
// 32 q / 8 kv heads).  Included by tqk_decode.cu after tqk_decode_mma.cuh.
//
// With 4 q heads per kv head, the m16n8 fragments of tqk_decode_mma.cuh leave
// q rows 4-7 empty, so half of every lane's scalar work (score combine,
// softmax, P*vd) is spent on padding.  Here a CTA serves kv heads A = 2h and
// B = 2h+1 and a warp step covers 16 tokens of each, as two 8-token n-tiles:
//   QK  rows 0-3 = A's q heads, rows 4-7 = B's.  Per n-tile and Q8 block two
//       accumulating m16n8k32 MMAs: A operand {A's q rows, zeros} against A's
//       K rows, then {zeros, B's q rows} against B's, so every lane's D
//       fragment holds the exact int32 dots of its own row and head;
//   PV  the k = 16 dimension of m16n8k16 is A's 8 tokens then B's 8 tokens:
//       rows 0-3 carry P_A*vd in k 0-7 and zeros in k 8-15, rows 4-7 the
//       opposite, and the B operand stacks V_A over V_B, so one MMA (hi + lo)
//       accumulates both heads without wasted products.
// The online softmax updates once per 16 tokens, and the power-of-two PV scale
// K is kept per q-head row (a quad of lanes), so neither needs a warp-wide
// reduction.  Everything else -- TMA ring, exact scores, base-2 softmax, hi/lo
// fp16 split, split merge -- is as in tqk_decode_mma.cuh.
#pragma once

namespace tqk {

#ifndef TQK_PK_WARPS
#define TQK_PK_WARPS 4
#endif
#ifndef TQK_PK_STAGES
#define TQK_PK_STAGES 2
#endif
#ifndef TQK_PK_MINB
#define TQK_PK_MINB 2  // CTAs per SM the register budget is sized for
#endif
constexpr int PK_WARPS = TQK_PK_WARPS;         // consumer warps
constexpr int PK_THREADS = (PK_WARPS + 1) * 32; // + the producer warp
constexpr int PK_ROWS = 16;                    // tokens of each kv head per warp step
constexpr int PK_T = PK_ROWS * PK_WARPS;       // tokens per tile, per kv head
constexpr int PK_QR = (8 + PK_WARPS - 1) / PK_WARPS;  // q rows per consumer warp (8 q heads per CTA)
constexpr int PK_NJ = (4 + PK_WARPS - 1) / PK_WARPS;  // appended rows per consumer warp (K, V of 2 heads)

template <int NB>
struct PackLayout {
    static constexpr int HD = NB * QK;
    static constexpr int ROW = NB * BLOCK_BYTES;
    static constexpr int TILE = PK_T * ROW;       // one plane of one kv head
    // planes K_A, K_B, V_A, V_B of a stage, 16 bytes apart beyond the tile: TILE is a
    // multiple of 128 bytes, so without the pad head A and head B rows would share banks
    static constexpr int PLANE = TILE + 16;
    static constexpr int STAGES = TQK_PK_STAGES;
    static constexpr int STAGE_BYTES = 4 * PLANE;
    static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
    static constexpr int OFF_QQ = OFF_BAR + ((2 * STAGES * 8 + 15) / 16) * 16;  // int8 [8][HD]
    static constexpr int OFF_QD = OFF_QQ + 8 * HD;                              // float [8][NB]
    static constexpr int OFF_NEW = OFF_QD + ((8 * NB * 4 + 15) / 16) * 16;     // appended rows [head][K,V][ROW]
    static constexpr int OFF_PRO = OFF_NEW + ((4 * ROW + 15) / 16) * 16;       // prologue rows [warp][PK_QR + PK_NJ]
    static constexpr int OFF_FLAG = OFF_PRO + PK_WARPS * (PK_QR + PK_NJ) * pro_stride<NB>() * 4;
    // cluster merge (p.cluster > 1): two mbarriers; this CTA's partial, acc [8][HD] then m [8], l [8];
    // every cluster CTA's m and l [2][CL_MAX][8]; the final M and L [2][8] and a flag
    static constexpr int OFF_CBAR = OFF_FLAG + 16;
    static constexpr int OFF_CPART = OFF_CBAR + 16;
    static constexpr int OFF_CML = OFF_CPART + (8 * HD + 16) * 4;
    static constexpr int BYTES = OFF_CML + (2 * CL_MAX * 8 + 16 + 4) * 4;
    static constexpr int RED_STRIDE = HD + 1;  // reduction rows padded: the 32 lanes' stores hit 32 banks
    static constexpr int RED_FLOATS = PK_WARPS * 8 * RED_STRIDE;
    static constexpr int SCRATCH_FLOATS = RED_FLOATS + 3 * PK_WARPS * 8 + 2 * 8 + 2 * MAX_SPLITS * 8;
    static_assert(SCRATCH_FLOATS * 4 <= OFF_BAR, "stage ring too small for the epilogue scratch");
    static_assert(OFF_CBAR % 8 == 0 && OFF_CPART % 16 == 0, "cluster merge alignment");
    // the cluster merge gathers every rank's values of this CTA's share into the reduction rows
    static_assert(8 * HD + CL_MAX <= RED_FLOATS, "reduction rows too small for the cluster merge");
};

// D(rows 0-7) += A(16x32 s8, rows 8-15 zero) * B(32x8 s8), int32.
__device__ __forceinline__ void mma_s8_k32_lo(int &d0, int &d1, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    int x2, x3;
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%5}, {%7,%8}, {%0,%1,%9,%9};"
        : "+r"(d0), "+r"(d1), "=r"(x2), "=r"(x3)
        : "r"(a0), "r"(0u), "r"(a2), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// Per-warp state of the packed decode: q operands, running row max / sum
// (base 2), the row's PV scale exponent and the P*V accumulators.  Lane
// (g, t) owns q-head row g (head A for g < 4, head B otherwise).
template <int NB>
struct PackState {
    uint32_t qa[NB][2], qb[NB][2];  // score A operands {k 4t.., k 16+4t..}: own row in qa (head A) or qb (head B)
    f32x2 qd2[NB];
    float m, l;
    int kscale;  // exponent of the row's PV operand scale, in [-125, 126]
    float acc[NB][4][2];

    __device__ __forceinline__ void begin(const int8_t *qq, const float *qd, int g, int t, bool hb) {
        constexpr int HD = NB * QK;
#pragma unroll
        for (int b = 0; b < NB; b++) {
            const uint32_t x0 = *reinterpret_cast<const uint32_t *>(qq + g * HD + b * QK + 4 * t);
            const uint32_t x2 = *reinterpret_cast<const uint32_t *>(qq + g * HD + b * QK + 16 + 4 * t);
            qa[b][0] = hb ? 0u : x0;
            qa[b][1] = hb ? 0u : x2;
            qb[b][0] = hb ? x0 : 0u;
            qb[b][1] = hb ? x2 : 0u;
            const float d = qd[g * NB + b];
            qd2[b] = pk2(d, d);
        }
        m = -INFINITY;
        l = 0.0f;
        kscale = -125;
#pragma unroll
        for (int b = 0; b < NB; b++)
#pragma unroll
            for (int jj = 0; jj < 4; jj++) acc[b][jj][0] = acc[b][jj][1] = 0.0f;
    }
};

// Scores of lane (g, t)'s row for tokens 2t, 2t+1 (n-tile 0) and 8+2t, 9+2t
// (n-tile 1) of its head, in log2 units; masked tokens are -inf.  Rounded as
// the reference: acc += (float)dot * (qd*kd) per block, then * scale.
template <int NB, bool FULL>
__device__ __forceinline__ void pack_scores(const uint32_t (&qa)[NB][2], const uint32_t (&qb)[NB][2],
                                            const f32x2 (&qd2)[NB], const uint8_t *k_a, const uint8_t *k_b,
                                            const uint8_t *kmine, int nvalid, float scale, int g, int t, float &s0,
                                            float &s1, float &s2, float &s3) {
    constexpr int ROW = NB * BLOCK_BYTES;
    // ---- scores of row g for tokens 2t, 2t+1 (n-tile 0) and 8+2t, 9+2t (n-tile 1),
    //      rounded exactly as the reference: acc += (float)dot * (qd*kd) per block
    f32x2 sc0 = pk2(0.0f, 0.0f), sc1 = pk2(0.0f, 0.0f);
#pragma unroll
    for (int b = 0; b < NB; b++) {
        const int kb = b * BLOCK_BYTES + 4 + 4 * t;
        int c00 = 0, c01 = 0, c10 = 0, c11 = 0;
        mma_s8_k32_lo(c00, c01, qa[b][0], qa[b][1], *reinterpret_cast<const uint32_t *>(k_a + g * ROW + kb),
                      *reinterpret_cast<const uint32_t *>(k_a + g * ROW + kb + 16));
        mma_s8_k32_lo(c10, c11, qa[b][0], qa[b][1],
                      *reinterpret_cast<const uint32_t *>(k_a + (8 + g) * ROW + kb),
                      *reinterpret_cast<const uint32_t *>(k_a + (8 + g) * ROW + kb + 16));
        mma_s8_k32_lo(c00, c01, qb[b][0], qb[b][1], *reinterpret_cast<const uint32_t *>(k_b + g * ROW + kb),
                      *reinterpret_cast<const uint32_t *>(k_b + g * ROW + kb + 16));
        mma_s8_k32_lo(c10, c11, qb[b][0], qb[b][1],
                      *reinterpret_cast<const uint32_t *>(k_b + (8 + g) * ROW + kb),
                      *reinterpret_cast<const uint32_t *>(k_b + (8 + g) * ROW + kb + 16));
        const uint8_t *kd = kmine + (2 * t) * ROW + b * BLOCK_BYTES;
        const f32x2 kd0 = pk2(*reinterpret_cast<const float *>(kd), *reinterpret_cast<const float *>(kd + ROW));
        const f32x2 kd1 =
            pk2(*reinterpret_cast<const float *>(kd + 8 * ROW), *reinterpret_cast<const float *>(kd + 9 * ROW));
        sc0 = add2(sc0, mul2(pk2(__int2float_rn(c00), __int2float_rn(c01)), mul2(qd2[b], kd0)));
        sc1 = add2(sc1, mul2(pk2(__int2float_rn(c10), __int2float_rn(c11)), mul2(qd2[b], kd1)));
    }
    const f32x2 sl2 = pk2(scale, scale), l2e = pk2(1.4426950408889634f, 1.4426950408889634f);
    // the reference's scores (acc * scale), then in log2 units
    upk2(mul2(mul2(sc0, sl2), l2e), s0, s1);
    upk2(mul2(mul2(sc1, sl2), l2e), s2, s3);
    if constexpr (!FULL) {
        if (2 * t >= nvalid) s0 = -INFINITY;
        if (2 * t + 1 >= nvalid) s1 = -INFINITY;
        if (8 + 2 * t >= nvalid) s2 = -INFINITY;
        if (9 + 2 * t >= nvalid) s3 = -INFINITY;
    }

}

// One warp step: tokens 0-15 of kv head A (k_a, v_a) and of kv head B (k_b,
// v_b), 144*NB/4-byte rows; FULL steps skip the masking of tokens >= nvalid.
// g = lane/4, t = lane%4, hb = g >= 4; mask_a / mask_b = f16x2 1.0 for the
// lane's own head's k half of the PV operand, 0 for the other.
template <int NB, bool FULL>
__device__ __forceinline__ void pack_step(PackState<NB> &st, const uint8_t *k_a, const uint8_t *k_b,
                                          const uint8_t *v_a, const uint8_t *v_b, int nvalid, float scale, int g,
                                          int t, bool hb, uint32_t mask_a, uint32_t mask_b) {
    constexpr int ROW = NB * BLOCK_BYTES;
    const uint8_t *kmine = hb ? k_b : k_a;  // the lane's own head for scales
    const uint8_t *vmine = hb ? v_b : v_a;

    float s0, s1, s2, s3;
    pack_scores<NB, FULL>(st.qa, st.qb, st.qd2, k_a, k_b, kmine, nvalid, scale, g, t, s0, s1, s2, s3);

    // ---- online softmax of the row over its 16 tokens (the quad)
    float mx = fmaxf(fmaxf(s0, s1), fmaxf(s2, s3));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(st.m, mx);
    const float corr = mn == st.m ? 1.0f : ex2f(st.m - mn);
    const float p0 = ex2f(s0 - mn), p1 = ex2f(s1 - mn), p2 = ex2f(s2 - mn), p3 = ex2f(s3 - mn);
    float sum = (p0 + p1) + (p2 + p3);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    st.l = st.l * corr + sum;
    st.m = mn;

    // ---- V scales of the lane's tokens (own head); the row's largest picks K
    float vd[4][NB];
    float vmax = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int tk = (i >> 1) * 8 + 2 * t + (i & 1);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float d = *reinterpret_cast<const float *>(vmine + tk * ROW + b * BLOCK_BYTES);
            if constexpr (!FULL) d = tk < nvalid ? d : 0.0f;
            vd[i][b] = d;
            vmax = fmaxf(vmax, d);
        }
    }
    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
    const int kt = vmax >= 1.17549435e-38f ? ((__float_as_int(vmax) >> 23) & 0xFF) - 127 + 1 : -125;
    const int knew = max(st.kscale, min(kt, 126));
    if (__any_sync(0xffffffffu, corr != 1.0f || knew != st.kscale)) {
        const int df = st.kscale - knew;  // <= 0
        const float f = (df < -126 ? 0.0f : exp2_int(df)) * corr;
#pragma unroll
        for (int b = 0; b < NB; b++)
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                st.acc[b][jj][0] *= f;
                st.acc[b][jj][1] *= f;
            }
        st.kscale = knew;
    }
    const float inv_k = exp2_int(-st.kscale);
    const f32x2 ik2 = pk2(inv_k, inv_k);
    const f32x2 pp0 = mul2(pk2(p0, p1), ik2), pp1 = mul2(pk2(p2, p3), ik2);

    // ---- P*V: per n-tile, k 0-7 = head A's tokens, k 8-15 = head B's
#pragma unroll
    for (int b = 0; b < NB; b++) {
        uint32_t h0, l0, h1, l1;
        split_f16x2(mul2(pp0, pk2(vd[0][b], vd[1][b])), h0, l0);
        split_f16x2(mul2(pp1, pk2(vd[2][b], vd[3][b])), h1, l1);
        const uint32_t h0a = hmul2(h0, mask_a), h0b = hmul2(h0, mask_b);
        const uint32_t l0a = hmul2(l0, mask_a), l0b = hmul2(l0, mask_b);
        const uint32_t h1a = hmul2(h1, mask_a), h1b = hmul2(h1, mask_b);
        const uint32_t l1a = hmul2(l1, mask_a), l1b = hmul2(l1, mask_b);
        const int wo = b * BLOCK_BYTES + 4 + 4 * g;
        const uint32_t wa0 = *reinterpret_cast<const uint32_t *>(v_a + (2 * t) * ROW + wo);
        const uint32_t wa1 = *reinterpret_cast<const uint32_t *>(v_a + (2 * t + 1) * ROW + wo);
        const uint32_t wa8 = *reinterpret_cast<const uint32_t *>(v_a + (2 * t + 8) * ROW + wo);
        const uint32_t wa9 = *reinterpret_cast<const uint32_t *>(v_a + (2 * t + 9) * ROW + wo);
        const uint32_t wb0 = *reinterpret_cast<const uint32_t *>(v_b + (2 * t) * ROW + wo);
        const uint32_t wb1 = *reinterpret_cast<const uint32_t *>(v_b + (2 * t + 1) * ROW + wo);
        const uint32_t wb8 = *reinterpret_cast<const uint32_t *>(v_b + (2 * t + 8) * ROW + wo);
        const uint32_t wb9 = *reinterpret_cast<const uint32_t *>(v_b + (2 * t + 9) * ROW + wo);
#define TQK_PK_NTILE(JJ)                                                                        \
    {                                                                                           \
        float *a = st.acc[b][JJ];                                                               \
        const uint32_t x0 = s8pair_to_f16x2<JJ>(wa0, wa1), y0 = s8pair_to_f16x2<JJ>(wb0, wb1);  \
        mma_f16_k16_hl(a[0], a[1], h0a, l0a, h0b, l0b, x0, y0);                                 \
        const uint32_t x1 = s8pair_to_f16x2<JJ>(wa8, wa9), y1 = s8pair_to_f16x2<JJ>(wb8, wb9);  \
        mma_f16_k16_hl(a[0], a[1], h1a, l1a, h1b, l1b, x1, y1);                                 \
    }
        TQK_PK_NTILE(0)
        TQK_PK_NTILE(1)
        TQK_PK_NTILE(2)
        TQK_PK_NTILE(3)
#undef TQK_PK_NTILE
    }
}

// The CTA's preamble, per consumer warp `warp`:
//  * quantises q heads qh0 + warp, qh0 + warp + PK_WARPS, ... of `item`
//    (quant_x.c:12-34) into qq [8][HD] / qd [8][NB];
//  * with do_append, the fused append (store_kv, attention_layer.c:66-90):
//    quantises new-row jobs warp, warp + PK_WARPS, ... (job 0/1 = K/V of head
//    A, 2/3 = K/V of head B), writes them to the cache at position pos and to
//    newrow [head][K,V][ROW] for patching the staged tile;
//  * with a fused prologue (norm_heads + rope_heads), normalises and rotates
//    the q rows and the K rows first.  Every global load (q, new rows, norm
//    weights, RoPE table) is issued up front, and the rows' sum-of-squares
//    chains run side by side, so the prologue adds one short serial chain.
template <int NB>
__device__ __forceinline__ void pack_preamble(const DecodeParams &p, int item, int qh0, int kvh_a, int pos,
                                              bool do_append, int warp, int lane, int8_t *qq, float *qd,
                                              uint8_t *newrow, float *scratch) {
    constexpr int HD = NB * QK, ROW = NB * BLOCK_BYTES, QR = PK_QR, NJ = PK_NJ, R = QR + NJ;
    const float *qsrc = p.q + (long long)item * p.q_item_stride + (long long)qh0 * HD;
    float x[R][NB];  // q rows, then this warp's new rows
#pragma unroll
    for (int r = 0; r < QR; r++)
#pragma unroll
        for (int b = 0; b < NB; b++)
            x[r][b] = warp + PK_WARPS * r < 8 ? __ldg(qsrc + (warp + PK_WARPS * r) * HD + b * QK + lane) : 0.0f;
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int job = warp + PK_WARPS * j, kvh = kvh_a + (job >> 1);
        const float *src = ((job & 1) == 0 ? p.k_new : p.v_new) + (long long)item * p.kv_new_item_stride +
                           (long long)kvh * HD;
#pragma unroll
        for (int b = 0; b < NB; b++) x[QR + j][b] = do_append && job < 4 ? __ldg(src + b * QK + lane) : 0.0f;
    }
    const bool norm = p.q_norm != nullptr, rope = p.rope_cos != nullptr;
    if (norm || rope) {
        float wq[NB], wk[NB];
        RopeTab<NB> tab;
        if (norm) {
            load_row<NB>(wq, p.q_norm + (long long)item * p.norm_item_stride, lane);
            load_row<NB>(wk, p.k_norm + (long long)item * p.norm_item_stride, lane);
        }
        if (rope) tab.load(p.rope_cos + (long long)item * p.rope_item_stride,
                           p.rope_sin + (long long)item * p.rope_item_stride, lane);
        if (norm) {
            float sums[R];
            warp_row_sumsq<NB, R>(x, scratch, lane, sums);
#pragma unroll
            for (int r = 0; r < QR; r++) apply_norm<NB>(x[r], sums[r], wq, p.norm_eps);
#pragma unroll
            for (int j = 0; j < NJ; j++)
                if ((warp + PK_WARPS * j) % 2 == 0) apply_norm<NB>(x[QR + j], sums[QR + j], wk, p.norm_eps);
        }
        if (rope) {
#pragma unroll
            for (int r = 0; r < QR; r++) apply_rope<NB>(x[r], tab, lane);
#pragma unroll
            for (int j = 0; j < NJ; j++)
                if ((warp + PK_WARPS * j) % 2 == 0) apply_rope<NB>(x[QR + j], tab, lane);
        }
    }
    // every block of the q rows and the new rows quantised together (their
    // shuffle and division chains overlap)
    float xf[R * NB], dq[R * NB];
    int8_t q8[R * NB];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int b = 0; b < NB; b++) xf[r * NB + b] = x[r][b];
    warp_quantize_blocks<R * NB>(xf, q8, dq);
#pragma unroll
    for (int r = 0; r < QR; r++) {
        const int g = warp + PK_WARPS * r;
        if (g >= 8) break;
#pragma unroll
        for (int b = 0; b < NB; b++) {
            qq[g * HD + b * QK + lane] = q8[r * NB + b];
            if (lane == 0) qd[g * NB + b] = dq[r * NB + b];
        }
    }
    if (!do_append) return;
    const long long head_bytes = (long long)p.max_tokens * ROW;
#pragma unroll
    for (int j = 0; j < NJ; j++) {
        const int job = warp + PK_WARPS * j;
        if (job >= 4) break;
        const int hsel = job >> 1, plane = job & 1;
        uint8_t *nrow = newrow + (hsel * 2 + plane) * ROW;
        uint8_t *grow = (plane == 0 ? p.kw : p.vw) + (long long)item * p.item_stride +
                        (long long)(kvh_a + hsel) * head_bytes + (long long)pos * ROW;
#pragma unroll
        for (int b = 0; b < NB; b++) {
            const uint8_t v8 = (uint8_t)q8[(QR + j) * NB + b];
            const float d = dq[(QR + j) * NB + b];
            nrow[b * BLOCK_BYTES + 4 + lane] = v8;
            grow[b * BLOCK_BYTES + 4 + lane] = v8;
            if (lane == 0) {
                *reinterpret_cast<float *>(nrow + b * BLOCK_BYTES) = d;
                *reinterpret_cast<float *>(grow + b * BLOCK_BYTES) = d;
            }
        }
    }
}

// Copies the appended rows into the staged tile when position pos falls in the
// warp's rows [row0, row0 + PK_ROWS) of tile rows starting at token t0.
template <int NB>
__device__ __forceinline__ void pack_patch(int pos, int t0, int r0, int lane, uint8_t *k_a, uint8_t *k_b, uint8_t *v_a,
                                           uint8_t *v_b, const uint8_t *newrow) {
    constexpr int ROW = NB * BLOCK_BYTES;
    if (pos < t0 + r0 || pos >= t0 + r0 + PK_ROWS) return;
    const int r = pos - t0 - r0;
    uint8_t *dsts[4] = {k_a + r * ROW, v_a + r * ROW, k_b + r * ROW, v_b + r * ROW};
#pragma unroll
    for (int q = 0; q < 4; q++)
        for (int i = lane; i < ROW / 4; i += 32)
            reinterpret_cast<uint32_t *>(dsts[q])[i] = reinterpret_cast<const uint32_t *>(newrow + q * ROW)[i];
    __syncwarp();
}

// Cross-warp reduction of a CTA's span: every consumer warp's unnormalised
// P*V rows (red, [W][8][RED_STRIDE]) and its (m, l) go to shared memory; the
// per-row maximum fm (natural log units), sum fl and per-warp weights wsc
// follow.  acc(g, c) is then the CTA's sum for q row g, column c, relative to
// fm[g].
struct PackRed {
    float *red, *small;  // small: wm [W][8], wl [W][8], wsc [W][8], fm [8], fl [8]
    __device__ __forceinline__ float *wm() const { return small; }
    __device__ __forceinline__ float *wl() const { return small + PK_WARPS * 8; }
    __device__ __forceinline__ float *wsc() const { return small + 2 * PK_WARPS * 8; }
    __device__ __forceinline__ float *fm() const { return small + 3 * PK_WARPS * 8; }
    __device__ __forceinline__ float *fl() const { return small + 3 * PK_WARPS * 8 + 8; }
    template <int RS>
    __device__ __forceinline__ float acc(int g, int c) const {
        float a = 0.0f;
#pragma unroll
        for (int w = 0; w < PK_WARPS; w++) a = fmaf(red[(w * 8 + g) * RS + c], wsc()[w * 8 + g], a);
        return a;
    }
};
constexpr int PK_RED_SMALL = 3 * PK_WARPS * 8 + 16;  // floats of PackRed::small

template <int NB, int RS>
__device__ __forceinline__ void pack_reduce(const PackState<NB> &st, const PackRed &r, int warp, int g, int t,
                                            int tid) {
    float *wm = r.wm(), *wl = r.wl(), *wsc = r.wsc(), *fm = r.fm(), *fl = r.fl();
    if (t == 0) {
        wm[warp * 8 + g] = st.m;
        wl[warp * 8 + g] = st.l;
    }
    const float unscale = exp2_int(st.kscale);
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            const int c = b * QK + 8 * t + jj;  // permuted n-tile column n = 2t, 2t+1 -> 4n + jj
            r.red[(warp * 8 + g) * RS + c] = st.acc[b][jj][0] * unscale;
            r.red[(warp * 8 + g) * RS + c + 4] = st.acc[b][jj][1] * unscale;
        }
    cta_sync<1, PK_WARPS * 32>();
    if (tid < 8) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < PK_WARPS; w++) M = fmaxf(M, wm[w * 8 + tid]);
        float Lsum = 0.0f;
#pragma unroll
        for (int w = 0; w < PK_WARPS; w++) {
            const float mw = wm[w * 8 + tid];
            const float e = mw == -INFINITY ? 0.0f : exp2f(mw - M);
            wsc[w * 8 + tid] = e;
            Lsum += wl[w * 8 + tid] * e;
        }
        fm[tid] = M * 0.6931471805599453f;
        fl[tid] = Lsum;
    }
    cta_sync<1, PK_WARPS * 32>();
}

// The split merge through the thread-block cluster of a unit's splits
// (p.cluster > 1, cluster dims (p.cluster, 1, 1) over the split axis), in
// place of the tickets and the partials in global memory.  Every CTA puts its
// partial (acc [8][HD], m, l) into its own shared memory and arrives on every
// other CTA's cbar[0]; once its own cbar[0] completes, it merges its share of
// the 8 x HD output elements from every CTA's partial by log-sum-exp -- the
// values read over distributed shared memory, all in flight at once, folded in
// rank order -- and writes them; then it arrives on every other CTA's cbar[1]
// and leaves only when its own cbar[1] completes, i.e. when no CTA reads its
// shared memory any more.  Every wait is bounded (the error word records a
// timeout).  empty: this CTA holds no keys, or gave up on a wait.  Run by the
// consumer threads only.
constexpr uint64_t CL_WAIT_NS = 2000000000ull;  // above the 1 s bound of every wait before the merge
template <int NB>
__device__ __forceinline__ void pack_cluster_merge(const DecodeParams &p, uint8_t *smem, const PackRed &r, bool empty,
                                                   int tid, int item, int qh0, float *out_item) {
    using L = PackLayout<NB>;
    constexpr int HD = L::HD, NT = PK_WARPS * 32, E = 8 * HD;
    constexpr int KV = (E + CL_MAX + NT - 1) / NT;  // (element, rank) values per thread
    uint64_t *cbar = reinterpret_cast<uint64_t *>(smem + L::OFF_CBAR);
    float *cp = reinterpret_cast<float *>(smem + L::OFF_CPART);
    float *cm = reinterpret_cast<float *>(smem + L::OFF_CML);  // m, then the weights, [CL_MAX][8]
    float *cl = cm + CL_MAX * 8;                                // l [CL_MAX][8]
    float *fin = cl + CL_MAX * 8;                               // M [8], L [8]
    int *okf = reinterpret_cast<int *>(fin + 16);
    float *vals = r.red;                                        // [share][rank], free after the partial is out
    const int C = p.cluster;
    const int rank = (int)cluster_ctarank();
    for (int i = tid; i < E; i += NT) cp[i] = empty ? 0.0f : r.acc<L::RED_STRIDE>(i / HD, i % HD);
    if (tid < 8) {
        cp[E + tid] = empty ? -INFINITY : r.fm()[tid];
        cp[E + 8 + tid] = empty ? 0.0f : r.fl()[tid];
    }
    if (tid == 0) *okf = 1;
    cta_sync<1, NT>();  // the partial is complete (and the reduction rows are free)
    if (tid < C && tid != rank) mbar_arrive_remote(cluster_map(&cbar[0], (uint32_t)tid));
    if (!mbar_wait_cluster_bounded(&cbar[0], 0, CL_WAIT_NS, p.err)) *okf = 0;
    cta_sync<1, NT>();
    const int S = (E + C - 1) / C, i0 = rank * S, n_share = max(0, min(E, i0 + S) - i0);
    if (*okf) {
        // every load first (the (m, l) pairs and this thread's values), then the folds
        float mv = 0.0f, lv = 0.0f, v[KV];
        if (tid < C * 8) {
            mv = ld_cluster_f32(cluster_map(cp + E + (tid & 7), (uint32_t)(tid >> 3)));
            lv = ld_cluster_f32(cluster_map(cp + E + 8 + (tid & 7), (uint32_t)(tid >> 3)));
        }
#pragma unroll
        for (int k = 0; k < KV; k++) {
            const int q = tid + k * NT, e = q / C, rr = q - e * C;
            v[k] = e < n_share ? ld_cluster_f32(cluster_map(cp + i0 + e, (uint32_t)rr)) : 0.0f;
        }
        if (tid < C * 8) {
            cm[tid] = mv;
            cl[tid] = lv;
        }
#pragma unroll
        for (int k = 0; k < KV; k++) {
            const int q = tid + k * NT;
            if (q / C < n_share) vals[q] = v[k];
        }
        cta_sync<1, NT>();
        if (tid < 8) {
            float M = -INFINITY;
            for (int rr = 0; rr < C; rr++) M = fmaxf(M, cm[rr * 8 + tid]);
            float Ls = 0.0f;
            for (int rr = 0; rr < C; rr++) {
                const float m = cm[rr * 8 + tid];
                const float w = m == -INFINITY ? 0.0f : expf(m - M);
                cm[rr * 8 + tid] = w;
                Ls += cl[rr * 8 + tid] * w;
            }
            fin[tid] = M;
            fin[8 + tid] = Ls;
        }
        cta_sync<1, NT>();
        for (int e = tid; e < n_share; e += NT) {
            const int i = i0 + e, g = i / HD, c = i - g * HD;
            float a = 0.0f;
            for (int rr = 0; rr < C; rr++) {
                const float w = cm[rr * 8 + g];
                if (w != 0.0f) a = fmaf(w, vals[e * C + rr], a);
            }
            if (p.out_mode == TQK_OUT_NORMALIZED) {
                store_out<HD>(p, out_item, item, qh0 + g, c, a / fin[8 + g]);
            } else {
                float *o = out_item + (long long)(qh0 + g) * (HD + 2);
                o[c] = a;
                if (c == 0) { o[HD] = fin[g]; o[HD + 1] = fin[8 + g]; }
            }
        }
    }
    cta_sync<1, NT>();  // this CTA's reads of the other CTAs' shared memory are done
    if (tid < C && tid != rank) mbar_arrive_remote(cluster_map(&cbar[1], (uint32_t)tid));
    if (tid == 0) mbar_wait_cluster_bounded(&cbar[1], 0, CL_WAIT_NS, p.err);
}

template <int NB>
__global__ void __launch_bounds__(PK_THREADS, TQK_PK_MINB) decode_q8_pack_kernel(const DecodeParams p) {
    using L = PackLayout<NB>;
    constexpr int HD = L::HD, ROW = L::ROW, STAGES = L::STAGES;

    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool clustered = p.cluster > 1;
    if (clustered) {
        // the cluster merge's barriers, initialised and made visible to the whole cluster before
        // any CTA can arrive on them; every thread passes here unconditionally
        uint64_t *cbar = reinterpret_cast<uint64_t *>(smem + PackLayout<NB>::OFF_CBAR);
        if (tid == 0) {
            mbar_init(&cbar[0], (uint32_t)(p.cluster - 1));
            mbar_init(&cbar[1], (uint32_t)(p.cluster - 1));
            fence_barrier_init();
        }
        __syncwarp();
        cluster_sync_all();
    }
    // programmatic dependent launch: everything this kernel reads (q, new rows,
    // lengths, cache rows) may come from earlier kernels of the stream, so wait
    // for them first; then the next kernel may start its own prefetch
    grid_dependency_wait();
    grid_dependents_launch();

    const int item = blockIdx.z;
    const int pair = blockIdx.y;  // kv heads 2*pair and 2*pair+1
    const int kvh_a = 2 * pair;
    const int G = 8;              // q heads served: 4 of each kv head
    int len = p.lens ? p.lens[item] : p.len0 + item * p.len_step;
    if (len < 0 || len > p.max_tokens) {
        if (tid == 0) record_error(p.err, DEVERR_BADLEN);
        len = len < 0 ? 0 : p.max_tokens;
    }
    int n_splits = n_splits_of(len, p.split_tokens);
    if (n_splits > p.max_splits) {  // a device length above the max_len the grid was sized for
        if (tid == 0) record_error(p.err, DEVERR_BADLEN);
        n_splits = p.max_splits;    // the last split then runs to len (<= max_tokens)
    }
    const int s = blockIdx.x;
    const int qh0 = kvh_a * p.group;  // q heads qh0..qh0+7 are contiguous (group == 4)
    float *out_item = p.out + (long long)item * p.out_item_stride;
    if (s >= (n_splits > 0 ? n_splits : 1)) {
        // a split past this item's length: in a cluster it still takes part in the merge (an empty
        // partial); with len == 0 every CTA of the cluster (one item) leaves here or just below
        if (clustered && len > 0 && warp < PK_WARPS) {
            float *red = reinterpret_cast<float *>(smem);
            pack_cluster_merge<NB>(p, smem, PackRed{red, red + L::RED_FLOATS}, true, tid, item, qh0, out_item);
        }
        return;
    }

    if (len == 0) {
        for (int i = tid; i < G * HD; i += PK_THREADS) {
            const int g = i / HD, c = i - g * HD;
            if (p.out_mode == TQK_OUT_NORMALIZED) {
                store_out<HD>(p, out_item, item, qh0 + g, c, 0.0f);
            } else {
                float *o = out_item + (long long)(qh0 + g) * (HD + 2);
                o[c] = 0.0f;
                if (c == 0) { o[HD] = -INFINITY; o[HD + 1] = 0.0f; }
            }
        }
        return;
    }

    const int t_begin = s * p.split_tokens;
    const int t_end = split_end(s, n_splits, p.split_tokens, len);
    const int n_tiles = (t_end - t_begin + PK_T - 1) / PK_T;
    const long long head_bytes = (long long)p.max_tokens * ROW;
    const long long off_a = (long long)item * p.item_stride + (long long)kvh_a * head_bytes;
    const uint8_t *ka = p.k + off_a, *va = p.v + off_a;  // head B follows at + head_bytes

    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t *empty = full + STAGES;
    int8_t *qq = reinterpret_cast<int8_t *>(smem + L::OFF_QQ);
    float *qd = reinterpret_cast<float *>(smem + L::OFF_QD);
    uint8_t *newrow = smem + L::OFF_NEW;
    int *flag = reinterpret_cast<int *>(smem + L::OFF_FLAG);
    int *timeout = flag + 1;

    auto issue = [&](int j) {
        const int slot = j % STAGES;
        const int t0 = t_begin + j * PK_T;
        const int rows = min(PK_T, t_end - t0);
        const uint32_t bytes = (uint32_t)(rows * ROW);
        uint8_t *st = smem + slot * L::STAGE_BYTES;
        const long long o = (long long)t0 * ROW;
        mbar_arrive_expect_tx(&full[slot], 4 * bytes);
        bulk_copy_g2s(st, ka + o, bytes, &full[slot]);
        bulk_copy_g2s(st + L::PLANE, ka + head_bytes + o, bytes, &full[slot]);
        bulk_copy_g2s(st + 2 * L::PLANE, va + o, bytes, &full[slot]);
        bulk_copy_g2s(st + 3 * L::PLANE, va + head_bytes + o, bytes, &full[slot]);
    };

    const int producer = PK_WARPS * 32;
    if (tid == producer) {
#pragma unroll
        for (int st = 0; st < STAGES; st++) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], PK_WARPS);
        }
        fence_barrier_init();
        for (int j = 0; j < min(STAGES, n_tiles); j++) issue(j);
        *timeout = 0;
    }

    const bool do_append = p.k_new != nullptr && s == n_splits - 1;
    const int pos = len - 1;
    if (warp < PK_WARPS) {
        float *pro = reinterpret_cast<float *>(smem + L::OFF_PRO) + warp * (PK_QR + PK_NJ) * pro_stride<NB>();
        pack_preamble<NB>(p, item, qh0, kvh_a, pos, do_append, warp, lane, qq, qd, newrow, pro);
    }
    __syncthreads();

    if (warp == PK_WARPS) {
        if (lane == 0) {
            for (int j = STAGES; j < n_tiles; j++) {
                const int slot = j % STAGES;
                if (!mbar_wait_bounded(&empty[slot], (uint32_t)(((j / STAGES) - 1) & 1), WAIT_NS, p.err)) {
                    *timeout = 1;
                    break;
                }
                issue(j);
            }
        }
        return;
    }

    // ------------------------------------------------------------------ consumers
    const int g = lane >> 2, t = lane & 3;
    const bool hb = g >= 4;  // this lane's row belongs to kv head B
    PackState<NB> st;
    st.begin(qq, qd, g, t, hb);
    const uint32_t mask_a = hb ? 0u : 0x3C003C00u, mask_b = hb ? 0x3C003C00u : 0u;  // f16x2 {1, 1} or 0

    const int r0 = warp * PK_ROWS;  // this warp's tokens of each head in a tile
    bool timed_out = false;
    for (int j = 0; j < n_tiles; j++) {
        const int slot = j % STAGES;
        const int t0 = t_begin + j * PK_T;
        const int rows = min(PK_T, t_end - t0);
        const bool ok = mbar_wait_bounded(&full[slot], (uint32_t)((j / STAGES) & 1), WAIT_NS, p.err);
        if (!__all_sync(0xffffffffu, ok)) {
            timed_out = true;
            break;
        }
        const int nvalid = rows - r0;
        if (nvalid > 0) {
            uint8_t *stg = smem + slot * L::STAGE_BYTES;
            uint8_t *k_a = stg + r0 * ROW, *k_b = stg + L::PLANE + r0 * ROW;
            uint8_t *v_a = stg + 2 * L::PLANE + r0 * ROW, *v_b = stg + 3 * L::PLANE + r0 * ROW;
            if (do_append) pack_patch<NB>(pos, t0, r0, lane, k_a, k_b, v_a, v_b, newrow);
            if (nvalid >= PK_ROWS)
                pack_step<NB, true>(st, k_a, k_b, v_a, v_b, nvalid, p.scale, g, t, hb, mask_a, mask_b);
            else
                pack_step<NB, false>(st, k_a, k_b, v_a, v_b, nvalid, p.scale, g, t, hb, mask_a, mask_b);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_release(&empty[slot]);
    }

    // ------------------------------------------------------------------ epilogue
    if (timed_out) *timeout = 1;
    cta_sync<1, PK_WARPS * 32>();
    float *red = reinterpret_cast<float *>(smem);  // [W][8][RED_STRIDE]
    PackRed r{red, red + L::RED_FLOATS};
    if (*timeout) {
        if (clustered) pack_cluster_merge<NB>(p, smem, r, true, tid, item, qh0, out_item);
        return;
    }

    pack_reduce<NB, L::RED_STRIDE>(st, r, warp, g, t, tid);
    if (clustered) {
        pack_cluster_merge<NB>(p, smem, r, false, tid, item, qh0, out_item);
        return;
    }
    float *wts = r.fl() + 8;                       // [2][MAX_SPLITS][8]
    auto acc_of = [&](int gg, int c) { return r.acc<L::RED_STRIDE>(gg, c); };
    finish_split<HD, 8, PK_WARPS * 32, 1>(p, tid, item, pair, s, n_splits, qh0, G, out_item, acc_of, r.fm(), r.fl(),
                                          wts, flag);
}


// ---------------------------------------------------------------------------
// Balanced schedule (split_tokens = 0): the tiles of every (item, kv-head
// pair) unit, laid end to end in unit order, are cut into gridDim.x equal
// runs, one per CTA (stream-K).  A CTA's run crosses unit boundaries, so it
// walks one or more segments (unit, tiles [lt0, lt1)), each finished like a
// split: its partial goes to slot c + unit of the workspace and the CTAs that
// share a unit merge through that unit's tickets.  Every SM then streams the
// same number of tiles whatever the number of units or their lengths; a
// fixed split leaves the SMs that hold fewer CTAs idle for the tail.
// ---------------------------------------------------------------------------
constexpr int BAL_MAX_ITEMS = 256;  // items whose lengths and tile prefix fit in shared memory
constexpr int BAL_MAX_CTAS = 1024;
// The automatic choice takes the balanced schedule for ragged batches only from
// this many tiles per resident CTA slot on (every unit counted at max_len).
// Measured on B200, ragged batches of 64 / 32 / 16 / 8 config-3 sequences
// (about 110 / 55 / 27 / 14 such tiles per slot): balanced 124.1 / 70.8 / 47.1 /
// 43.7 us against the best fixed split tried 130.5 / 70.0 / 40.5 / 24.6 us.
constexpr int BAL_MIN_TILES = 40;

template <int NB>
struct PackBalLayout {
    using P = PackLayout<NB>;
    static constexpr int HD = P::HD, ROW = P::ROW, PLANE = P::PLANE, STAGES = P::STAGES;
    static constexpr int STAGE_BYTES = P::STAGE_BYTES;
    static constexpr int OFF_BAR = P::OFF_BAR;
    static constexpr int OFF_QQ = P::OFF_QQ, OFF_QD = P::OFF_QD, OFF_NEW = P::OFF_NEW, OFF_PRO = P::OFF_PRO;
    static constexpr int RED_STRIDE = P::RED_STRIDE;
    static constexpr int RED_FLOATS = P::RED_FLOATS;
    // the reduction lives beside the ring, which keeps streaming the next segment;
    // the merge weights [2][MAX_SPLITS][8] reuse the reduction rows once read
    static constexpr int OFF_RED = P::OFF_FLAG;
    static constexpr int OFF_SMALL = OFF_RED + RED_FLOATS * 4;
    static constexpr int OFF_LENS = OFF_SMALL + ((PK_RED_SMALL * 4 + 15) / 16) * 16;  // int [BAL_MAX_ITEMS]
    static constexpr int OFF_PRE = OFF_LENS + BAL_MAX_ITEMS * 4;                      // int [BAL_MAX_ITEMS + 1]
    static constexpr int OFF_FLAG = OFF_PRE + ((BAL_MAX_ITEMS + 1) * 4 + 15) / 16 * 16;
    static constexpr int BYTES = OFF_FLAG + 16;
    static_assert(2 * MAX_SPLITS * 8 <= RED_FLOATS, "merge weights must fit in the reduction rows");
};

// One segment of a CTA's run: tiles [lt0, lt1) of unit (item, pair), whose
// first tile is global tile ubase.
struct BalSeg {
    int item, pair, lt0, lt1, tiles, len, ubase;
};

// The segment holding global tile g, cut at g1 (the run's end).  pre[i] is the
// global index of item i's first tile (pre[n_items] = total); items without
// tiles have pre[i] == pre[i + 1] and are never chosen.
__device__ __forceinline__ BalSeg bal_segment(const int *pre, const int *lens, int n_items, int pairs, int g, int g1) {
    int lo = 0, hi = n_items - 1;  // the last item with pre[item] <= g
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= g) lo = mid;
        else hi = mid - 1;
    }
    BalSeg s;
    s.item = lo;
    s.len = lens[lo];
    s.tiles = (s.len + PK_T - 1) / PK_T;
    const int off = g - pre[lo];
    s.pair = off / s.tiles;
    s.lt0 = off - s.pair * s.tiles;
    s.ubase = pre[lo] + s.pair * s.tiles;
    s.lt1 = min(s.tiles, s.lt0 + (g1 - g));
    return s;
}

template <int NB>
__global__ void __launch_bounds__(PK_THREADS, TQK_PK_MINB) decode_q8_pack_bal_kernel(const DecodeParams p) {
    using L = PackBalLayout<NB>;
    constexpr int HD = L::HD, ROW = L::ROW, STAGES = L::STAGES;
    constexpr int G = 8;

    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    grid_dependency_wait();  // lengths, q, new rows and cache rows may come from earlier kernels
    grid_dependents_launch();

    const int n_items = p.n_items, pairs = p.pairs;
    int *lens = reinterpret_cast<int *>(smem + L::OFF_LENS);
    int *pre = reinterpret_cast<int *>(smem + L::OFF_PRE);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t *empty = full + STAGES;
    int *flag = reinterpret_cast<int *>(smem + L::OFF_FLAG);
    int *timeout = flag + 1;
    const int producer = PK_WARPS * 32;

    if (warp == 0) {
        // lengths (clamped like the fixed-split kernel) and the exclusive prefix of tiles
        constexpr int PER = BAL_MAX_ITEMS / 32;
        int tl[PER];
        int sum = 0;
#pragma unroll
        for (int k = 0; k < PER; k++) {
            const int i = lane * PER + k;
            int len = 0;
            if (i < n_items) {
                len = p.lens ? p.lens[i] : p.len0 + i * p.len_step;
                if (len < 0 || len > p.max_tokens) {
                    record_error(p.err, DEVERR_BADLEN);
                    len = len < 0 ? 0 : p.max_tokens;
                }
                lens[i] = len;
            }
            tl[k] = (len + PK_T - 1) / PK_T * pairs;
            sum += tl[k];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - sum;
#pragma unroll
        for (int k = 0; k < PER; k++) {
            const int i = lane * PER + k;
            if (i < n_items) pre[i] = run;
            run += tl[k];
        }
        if (lane == 31) pre[n_items] = incl;
    } else if (tid == producer) {
#pragma unroll
        for (int st = 0; st < STAGES; st++) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], PK_WARPS);
        }
        fence_barrier_init();
        *timeout = 0;
    }
    __syncthreads();

    // items of length 0 attend nothing: zero outputs, written by a share of the CTAs
    for (int i = blockIdx.x; i < n_items; i += gridDim.x) {
        if (lens[i] != 0) continue;
        float *out_item = p.out + (long long)i * p.out_item_stride;
        const int heads = pairs * G;
        for (int e = tid; e < heads * HD; e += PK_THREADS) {
            const int h = e / HD, c = e - h * HD;
            if (p.out_mode == TQK_OUT_NORMALIZED) {
                out_item[(long long)h * HD + c] = 0.0f;
            } else {
                float *o = out_item + (long long)h * (HD + 2);
                o[c] = 0.0f;
                if (c == 0) { o[HD] = -INFINITY; o[HD + 1] = 0.0f; }
            }
        }
    }

    const int T = pre[n_items];
    const int C = min((int)gridDim.x, T);  // every CTA below C gets at least one tile
    const int c = blockIdx.x;
    if (c >= C) return;
    const int g0 = (int)((long long)c * T / C), g1 = (int)((long long)(c + 1) * T / C);
    const long long head_bytes = (long long)p.max_tokens * ROW;

    if (warp == PK_WARPS) {
        if (lane != 0) return;
        int j = 0;
        for (int g = g0; g < g1;) {
            const BalSeg sg = bal_segment(pre, lens, n_items, pairs, g, g1);
            const long long off_a = (long long)sg.item * p.item_stride + (long long)(2 * sg.pair) * head_bytes;
            const uint8_t *ka = p.k + off_a, *va = p.v + off_a;
            for (int lt = sg.lt0; lt < sg.lt1; lt++, j++) {
                const int slot = j % STAGES;
                if (j >= STAGES &&
                    !mbar_wait_bounded(&empty[slot], (uint32_t)(((j / STAGES) - 1) & 1), WAIT_NS, p.err)) {
                    *timeout = 1;
                    return;
                }
                const int t0 = lt * PK_T;
                const uint32_t bytes = (uint32_t)(min(PK_T, sg.len - t0) * ROW);
                uint8_t *stg = smem + slot * L::STAGE_BYTES;
                const long long o = (long long)t0 * ROW;
                mbar_arrive_expect_tx(&full[slot], 4 * bytes);
                bulk_copy_g2s(stg, ka + o, bytes, &full[slot]);
                bulk_copy_g2s(stg + L::PLANE, ka + head_bytes + o, bytes, &full[slot]);
                bulk_copy_g2s(stg + 2 * L::PLANE, va + o, bytes, &full[slot]);
                bulk_copy_g2s(stg + 3 * L::PLANE, va + head_bytes + o, bytes, &full[slot]);
            }
            g = sg.ubase + sg.lt1;
        }
        return;
    }

    // ------------------------------------------------------------------ consumers
    int8_t *qq = reinterpret_cast<int8_t *>(smem + L::OFF_QQ);
    float *qd = reinterpret_cast<float *>(smem + L::OFF_QD);
    uint8_t *newrow = smem + L::OFF_NEW;
    float *pro = reinterpret_cast<float *>(smem + L::OFF_PRO) + warp * (PK_QR + PK_NJ) * pro_stride<NB>();
    const PackRed red{reinterpret_cast<float *>(smem + L::OFF_RED), reinterpret_cast<float *>(smem + L::OFF_SMALL)};
    const int g = lane >> 2, t = lane & 3;
    const bool hb = g >= 4;
    const uint32_t mask_a = hb ? 0u : 0x3C003C00u, mask_b = hb ? 0x3C003C00u : 0u;
    const int r0 = warp * PK_ROWS;

    // The segment is looked up again from shared memory where it is needed
    // rather than kept in registers across the tile loop (which holds the
    // P*V accumulators and the q operands).
    // the run's end, recomputed from shared memory
    auto run_end = [&]() {
        const int Tn = pre[n_items], Cn = min((int)gridDim.x, Tn);
        return (int)((long long)(blockIdx.x + 1) * Tn / Cn);
    };
    int j = 0;  // ring position of the next tile
    for (int gt = g0;;) {
        {
            const BalSeg sg = bal_segment(pre, lens, n_items, pairs, gt, run_end());
            const bool do_append = p.k_new != nullptr && sg.lt1 == sg.tiles;  // the segment holding the last tile
            pack_preamble<NB>(p, sg.item, 2 * sg.pair * p.group, 2 * sg.pair, sg.len - 1, do_append, warp, lane, qq,
                              qd, newrow, pro);
        }
        cta_sync<1, PK_WARPS * 32>();  // q operands visible; the previous segment's scratch is free
        PackState<NB> st;
        st.begin(qq, qd, g, t, hb);

        bool timed_out = false;
        {
            const BalSeg sg = bal_segment(pre, lens, n_items, pairs, gt, run_end());
            const bool do_append = p.k_new != nullptr && sg.lt1 == sg.tiles;
            const int pos = sg.len - 1;
            for (int lt = sg.lt0; lt < sg.lt1; lt++, j++) {
                const int slot = j % STAGES;
                const int t0 = lt * PK_T;
                const int rows = min(PK_T, sg.len - t0);
                const bool ok = mbar_wait_bounded(&full[slot], (uint32_t)((j / STAGES) & 1), WAIT_NS, p.err);
                if (!__all_sync(0xffffffffu, ok)) {
                    timed_out = true;
                    break;
                }
                const int nvalid = rows - r0;
                if (nvalid > 0) {
                    uint8_t *stg = smem + slot * L::STAGE_BYTES;
                    uint8_t *k_a = stg + r0 * ROW, *k_b = stg + L::PLANE + r0 * ROW;
                    uint8_t *v_a = stg + 2 * L::PLANE + r0 * ROW, *v_b = stg + 3 * L::PLANE + r0 * ROW;
                    if (do_append) pack_patch<NB>(pos, t0, r0, lane, k_a, k_b, v_a, v_b, newrow);
                    if (nvalid >= PK_ROWS)
                        pack_step<NB, true>(st, k_a, k_b, v_a, v_b, nvalid, p.scale, g, t, hb, mask_a, mask_b);
                    else
                        pack_step<NB, false>(st, k_a, k_b, v_a, v_b, nvalid, p.scale, g, t, hb, mask_a, mask_b);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive_release(&empty[slot]);
            }
        }
        if (timed_out) *timeout = 1;
        cta_sync<1, PK_WARPS * 32>();
        if (*timeout) return;

        pack_reduce<NB, L::RED_STRIDE>(st, red, warp, g, t, tid);
        const int Tn = pre[n_items];
        const int Cn = min((int)gridDim.x, Tn);
        const int cn = blockIdx.x;
        const int g1n = (int)((long long)(cn + 1) * Tn / Cn);
        const BalSeg sg = bal_segment(pre, lens, n_items, pairs, gt, g1n);
        // the CTAs covering this unit: c0 .. c1 (the owners of its first and last tiles)
        const int c0 = (int)((((long long)sg.ubase + 1) * Cn - 1) / Tn);
        const int c1 = (int)((((long long)sg.ubase + sg.tiles) * Cn - 1) / Tn);
        const long long unit = (long long)sg.item * pairs + sg.pair;
        float *pb = p.part + ((long long)c0 + unit) * G * (HD + 2);
        int *tickets = p.counters + unit * p.tickets_per_unit;
        float *out_item = p.out + (long long)sg.item * p.out_item_stride;
        auto acc_of = [&](int gg, int cc) { return red.acc<L::RED_STRIDE>(gg, cc); };
        finish_split_at<HD, G, PK_WARPS * 32, 1>(p, tid, pb, tickets, cn - c0, c1 - c0 + 1, sg.item,
                                                 2 * sg.pair * p.group, G,
                                                 out_item, acc_of, red.fm(), red.fl(), red.red, flag);
        gt = sg.ubase + sg.lt1;
        if (gt >= g1n) break;
    }
}

}  // namespace tqk
