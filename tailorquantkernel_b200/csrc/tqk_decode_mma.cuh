// tqk_decode_mma.cuh -- tensor-core Q8 decode attention for head_dim 128/256
// (included by tqk_decode.cu, which defines DecodeParams, finish_split and the
// warp helpers).
//
// One CTA = one token range of one kv head of one item, serving up to 16 q
// heads.  Warp roles:
//   * warp 4 (producer): one thread streams 64-token K/V tiles (144-byte rows,
//     contiguous per plane) into a STAGES-deep ring with 1-D TMA bulk copies,
//     paced by "empty" mbarriers the consumers release;
//   * warps 0-3 (consumers): warp w owns rows 16w..16w+15 of every tile and runs
//     its own online softmax, so there is no CTA-wide barrier per tile.
// Per 16-token slice a consumer warp does:
//   QK  mma.m16n8k32 s8*s8->s32, one per Q8 block (q heads = M rows, tokens =
//       N columns): exact int32 block dots, combined with the reference's
//       rounding sequence acc += (float)dot * (qd*kd) (model/attn_q8.c:24-31),
//       so every score equals attn_scores_q8_scalar's bit for bit;
//   softmax: per q-head row, max/sum over the quad of lanes holding the row;
//   PV  mma.m16n8k16 f16->f32 per (block, 8-column n-tile): A = p*vd*2^-K
//       split into fp16 hi + lo (two MMAs, ~22-bit precision), B = the int8 V
//       values converted exactly to fp16.  V columns are taken in a permuted
//       order inside each 32-column block (n-tile jj, column n -> 4n + jj) so
//       each lane's B fragment is one aligned word per token row (bank
//       conflict free); the output store undoes the permutation.
// K (a power-of-two scale that keeps p*vd inside fp16 range) only grows, and
// the accumulators are rescaled exactly when it or a row max changes.
#pragma once

#include <type_traits>

namespace tqk {

#ifndef TQK_MMA_WARPS
#define TQK_MMA_WARPS 4
#endif
#ifndef TQK_MMA_STAGES
#define TQK_MMA_STAGES 3
#endif
constexpr int MMA_WARPS = TQK_MMA_WARPS;        // consumer warps (16 tokens of each tile apiece)
constexpr int MMA_THREADS = (MMA_WARPS + 1) * 32;
constexpr int MMA_T = 16 * MMA_WARPS;           // tokens per tile
template <int NB>
constexpr int mma_stages() { return TQK_MMA_STAGES; }  // default 3 x 18 KB ring: 3 CTAs/SM at head_dim 128

template <int NB, int GPAD>
struct MmaLayout {
    static constexpr int HD = NB * QK;
    static constexpr int ROW = NB * BLOCK_BYTES;
    static constexpr int TILE = MMA_T * ROW;
    static constexpr int STAGES = mma_stages<NB>();
    static constexpr int STAGE_BYTES = 2 * TILE;
    static constexpr int OFF_BAR = STAGES * STAGE_BYTES;           // full[STAGES], empty[STAGES]
    static constexpr int OFF_QQ = OFF_BAR + ((2 * STAGES * 8 + 15) / 16) * 16;  // int8 [16][HD]
    static constexpr int OFF_QD = OFF_QQ + 16 * HD;                // float [16][NB]
    static constexpr int OFF_NEW = OFF_QD + ((16 * NB * 4 + 15) / 16) * 16;   // appended K, V rows
    static constexpr int OFF_PRO = OFF_NEW + ((2 * ROW + 15) / 16) * 16;      // prologue row per warp
    static constexpr int OFF_FLAG = OFF_PRO + MMA_WARPS * pro_stride<NB>() * 4;  // int flag, int timeout
    static constexpr int BYTES = OFF_FLAG + 16;
    // epilogue scratch, in the idle stage ring
    static constexpr int RED_FLOATS = MMA_WARPS * GPAD * HD;
    static constexpr int SCRATCH_FLOATS = RED_FLOATS + 3 * MMA_WARPS * GPAD + 2 * GPAD + 2 * MAX_SPLITS * GPAD;
    static_assert(SCRATCH_FLOATS * 4 <= OFF_BAR, "stage ring too small for the epilogue scratch");
    static_assert(TILE % 16 == 0, "tiles must be whole 16-byte units");
};

// D = A(16x32 s8, row) * B(32x8 s8, col), int32, C = 0.
__device__ __forceinline__ void mma_s8_k32(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32.
__device__ __forceinline__ void mma_f16_k16(float &d0, float &d1, float &d2, float &d3, uint32_t a0, uint32_t a1,
                                            uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Same, for at most 8 q heads: rows 8-15 of A are zero, so only d0/d1 are kept
// (the other two outputs are dead temporaries).
__device__ __forceinline__ void mma_f16_k16_lo(float &d0, float &d1, uint32_t a0, uint32_t a2, uint32_t b0,
                                               uint32_t b1) {
    float x2, x3;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%5}, {%7,%8}, {%0,%1,%9,%9};"
        : "+f"(d0), "+f"(d1), "=f"(x2), "=f"(x3)
        : "r"(a0), "r"(0u), "r"(a2), "r"(b0), "r"(b1), "f"(0.0f));
}

// P*V with P's hi half in rows 0-7 and its lo half in rows 8-15 of one
// m16n8k16 (A = {hi k0-7, lo k0-7, hi k8-15, lo k8-15}): the two products come
// out of one MMA, and the lo rows are added into the hi rows' accumulators.
__device__ __forceinline__ void mma_f16_k16_hl(float &d0, float &d1, uint32_t h0, uint32_t l0, uint32_t h2,
                                               uint32_t l2, uint32_t b0, uint32_t b1) {
    float x2, x3;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%10,%10};"
        : "+f"(d0), "+f"(d1), "=f"(x2), "=f"(x3)
        : "r"(h0), "r"(l0), "r"(h2), "r"(l2), "r"(b0), "r"(b1), "f"(0.0f));
    d0 += x2;
    d1 += x3;
}

// Packed fp32 pairs (Blackwell f32x2 ALU ops, each lane of the pair rounded
// like the scalar instruction).
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pk2(float x, float y) {
    f32x2 r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(x), "f"(y));
    return r;
}
__device__ __forceinline__ void upk2(f32x2 v, float &x, float &y) { asm("mov.b64 {%0,%1}, %2;" : "=f"(x), "=f"(y) : "l"(v)); }
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// Two fp32 -> packed f16x2 (x0 in the low half), round to nearest.
__device__ __forceinline__ uint32_t pack_f16x2(float x0, float x1) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x1), "f"(x0));
    return r;
}
__device__ __forceinline__ void unpack_f16x2(uint32_t h, float &x0, float &x1) {
    asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tcvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
        : "=f"(x0), "=f"(x1)
        : "r"(h));
}
// hi + lo fp16 split of a pair x (values in [0, 1]): hi = x truncated to 10
// mantissa bits (exact in fp16 for normal values), lo = f16(x - hi) with
// |x - hi| < 2^-10 |x|, so hi + lo carries ~21 bits of x.
__device__ __forceinline__ void split_f16x2(f32x2 x, uint32_t &hi, uint32_t &lo) {
    float x0, x1;
    upk2(x, x0, x1);
    const float h0 = __uint_as_float(__float_as_uint(x0) & 0xFFFFE000u);
    const float h1 = __uint_as_float(__float_as_uint(x1) & 0xFFFFE000u);
    float r0, r1;
    upk2(sub2(x, pk2(h0, h1)), r0, r1);
    hi = pack_f16x2(h0, h1);
    lo = pack_f16x2(r0, r1);
}

// Byte jj of a and of b (signed int8) -> exact f16x2 {a_jj, b_jj}: bias to
// unsigned (xor 0x80), drop into the mantissa of 1024.0 (0x6400) and subtract 1152.
template <int JJ>
__device__ __forceinline__ uint32_t s8pair_to_f16x2(uint32_t a, uint32_t b) {
    const uint32_t t = __byte_perm(a, b, JJ | ((4 + JJ) << 8));
    const uint32_t h = (t & 0x00FF00FFu) ^ 0x64806480u;
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));
    return r;
}

__device__ __forceinline__ float exp2_int(int k) {  // 2^k, k in [-126, 127]
    return __int_as_float((k + 127) << 23);
}

// Per-warp state of the tensor-core decode for one (item, kv-head slice) run:
// q fragments, running row max / sum (base 2) and the P*V accumulators.
template <int NB, bool HI>
struct SliceState {
    static constexpr int NACC = HI ? 4 : 2;  // d0,d1 (rows g) [+ d2,d3 (rows g+8)]
    uint32_t qa[NB][4];
    f32x2 qdl2[NB], qdh2[NB];
    float m_lo, l_lo, m_hi, l_hi;
    int kscale;  // running power-of-two exponent of the PV operand scale, in [-125, 126]
    float acc[NB][4][NACC];

    // Loads this lane's q fragments (rows g, g+8) from a quantised [16][HD] int8
    // tile with scales [16][NB], and clears the softmax / accumulator state.
    __device__ __forceinline__ void begin(const int8_t *qq, const float *qd, int g, int t) {
        constexpr int HD = NB * QK;
#pragma unroll
        for (int b = 0; b < NB; b++) {
            qa[b][0] = *reinterpret_cast<const uint32_t *>(qq + g * HD + b * QK + 4 * t);
            qa[b][2] = *reinterpret_cast<const uint32_t *>(qq + g * HD + b * QK + 16 + 4 * t);
            qa[b][1] = HI ? *reinterpret_cast<const uint32_t *>(qq + (g + 8) * HD + b * QK + 4 * t) : 0u;
            qa[b][3] = HI ? *reinterpret_cast<const uint32_t *>(qq + (g + 8) * HD + b * QK + 16 + 4 * t) : 0u;
            const float lo = qd[g * NB + b];
            const float hi = HI ? qd[(g + 8) * NB + b] : 0.0f;
            qdl2[b] = pk2(lo, lo);
            qdh2[b] = pk2(hi, hi);
        }
        m_lo = m_hi = -INFINITY;
        l_lo = l_hi = 0.0f;
        kscale = -125;
#pragma unroll
        for (int b = 0; b < NB; b++)
#pragma unroll
            for (int jj = 0; jj < 4; jj++)
#pragma unroll
                for (int e = 0; e < NACC; e++) acc[b][jj][e] = 0.0f;
    }
};

// One 16-token slice (K rows at ks, V rows at vs, 144*NB/4-byte rows): scores,
// online softmax (log2 domain), P*V into st.  FULL slices skip all masking;
// partial ones mask tokens >= nvalid.  g = lane/4, t = lane%4.
template <int NB, bool HI, bool FULL>
__device__ __forceinline__ void mma_slice(SliceState<NB, HI> &st, const uint8_t *ks, const uint8_t *vs, int nvalid,
                                          float scale, int g, int t) {
    constexpr int ROW = NB * BLOCK_BYTES;
    constexpr int NACC = SliceState<NB, HI>::NACC;
    const f32x2 scale2 = pk2(scale, scale);
    const f32x2 log2e2 = pk2(1.4426950408889634f, 1.4426950408889634f);
    // ---- scores: two 8-token n-tiles; lane holds tokens nt*8 + 2t + {0,1}
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; nt++) {
        const uint8_t *kb = ks + (nt * 8 + g) * ROW;       // B fragment row (token nt*8+g)
        const uint8_t *kda = ks + (nt * 8 + 2 * t) * ROW;  // scale rows of the lane's tokens
        // st.acc += (float)dot * (qd*kd) per block, for the lane's token pair,
        // with separately rounded products and sums as in the reference
        f32x2 alo = pk2(0.0f, 0.0f), ahi = pk2(0.0f, 0.0f);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            const uint32_t b0 = *reinterpret_cast<const uint32_t *>(kb + b * BLOCK_BYTES + 4 + 4 * t);
            const uint32_t b1 = *reinterpret_cast<const uint32_t *>(kb + b * BLOCK_BYTES + 20 + 4 * t);
            int c[4];
            mma_s8_k32(c, st.qa[b], b0, b1);
            const f32x2 kd = pk2(*reinterpret_cast<const float *>(kda + b * BLOCK_BYTES),
                                 *reinterpret_cast<const float *>(kda + ROW + b * BLOCK_BYTES));
            alo = add2(alo, mul2(pk2(__int2float_rn(c[0]), __int2float_rn(c[1])), mul2(st.qdl2[b], kd)));
            if constexpr (HI)
                ahi = add2(ahi, mul2(pk2(__int2float_rn(c[2]), __int2float_rn(c[3])), mul2(st.qdh2[b], kd)));
        }
        // the reference's score (st.acc * scale, bit-exact), then to log2 units
        upk2(mul2(mul2(alo, scale2), log2e2), sc[nt][0], sc[nt][1]);
        if constexpr (HI) upk2(mul2(mul2(ahi, scale2), log2e2), sc[nt][2], sc[nt][3]);
        else sc[nt][2] = sc[nt][3] = 0.0f;
        if constexpr (!FULL) {
            const int tk = nt * 8 + 2 * t;
            if (tk >= nvalid) sc[nt][0] = sc[nt][2] = -INFINITY;
            if (tk + 1 >= nvalid) sc[nt][1] = sc[nt][3] = -INFINITY;
        }
    }

    // ---- online softmax per q-head row (the quad of lanes sharing g), base 2
    float pr[2][4];
    float corr_lo, corr_hi = 1.0f;
    {
        float mx = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(st.m_lo, mx);
        corr_lo = mn == st.m_lo ? 1.0f : ex2f(st.m_lo - mn);
        pr[0][0] = ex2f(sc[0][0] - mn);
        pr[0][1] = ex2f(sc[0][1] - mn);
        pr[1][0] = ex2f(sc[1][0] - mn);
        pr[1][1] = ex2f(sc[1][1] - mn);
        float sum = (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        st.l_lo = st.l_lo * corr_lo + sum;
        st.m_lo = mn;
    }
    if constexpr (HI) {
        float mx = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(st.m_hi, mx);
        corr_hi = mn == st.m_hi ? 1.0f : ex2f(st.m_hi - mn);
        pr[0][2] = ex2f(sc[0][2] - mn);
        pr[0][3] = ex2f(sc[0][3] - mn);
        pr[1][2] = ex2f(sc[1][2] - mn);
        pr[1][3] = ex2f(sc[1][3] - mn);
        float sum = (pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        st.l_hi = st.l_hi * corr_hi + sum;
        st.m_hi = mn;
    } else {
        pr[0][2] = pr[0][3] = pr[1][2] = pr[1][3] = 0.0f;
    }

    // ---- V scales of the lane's tokens (2t, 2t+1, 8+2t, 9+2t); masked rows are 0
    float vd[4][NB];
    float vmax = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int tk = (q >> 1) * 8 + 2 * t + (q & 1);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float d = *reinterpret_cast<const float *>(vs + tk * ROW + b * BLOCK_BYTES);
            if constexpr (!FULL) d = tk < nvalid ? d : 0.0f;
            vd[q][b] = d;
            vmax = fmaxf(vmax, d);
        }
    }
    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
    // exponent of the slice's largest scale (warp-uniform); zero/denormal -> keep the running one
    const int kt = vmax >= 1.17549435e-38f ? ((__float_as_int(vmax) >> 23) & 0xFF) - 127 + 1 : -125;
    const int knew = max(st.kscale, min(kt, 126));
    const bool rescale = __any_sync(0xffffffffu, corr_lo != 1.0f || corr_hi != 1.0f || knew != st.kscale);
    if (rescale) {
        const int df = st.kscale - knew;                     // <= 0
        const float f = df < -126 ? 0.0f : exp2_int(df);  // exact power of two <= 1
        const float flo = corr_lo * f, fhi = corr_hi * f;
#pragma unroll
        for (int b = 0; b < NB; b++)
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                st.acc[b][jj][0] *= flo;
                st.acc[b][jj][1] *= flo;
                if constexpr (HI) {
                    st.acc[b][jj][NACC - 2] *= fhi;
                    st.acc[b][jj][NACC - 1] *= fhi;
                }
            }
        st.kscale = knew;
    }
    const float inv_k = exp2_int(-st.kscale);
    const f32x2 ik2 = pk2(inv_k, inv_k);
    const f32x2 p00 = mul2(pk2(pr[0][0], pr[0][1]), ik2), p10 = mul2(pk2(pr[1][0], pr[1][1]), ik2);
    const f32x2 p02 = HI ? mul2(pk2(pr[0][2], pr[0][3]), ik2) : 0ull;
    const f32x2 p12 = HI ? mul2(pk2(pr[1][2], pr[1][3]), ik2) : 0ull;

    // ---- P*V per block: A = p*vd*2^-K (hi+lo fp16), B = int8 V -> fp16
#pragma unroll
    for (int b = 0; b < NB; b++) {
        uint32_t ah0, al0, ah2, al2, ah1 = 0, al1 = 0, ah3 = 0, al3 = 0;
        const f32x2 vd01 = pk2(vd[0][b], vd[1][b]), vd23 = pk2(vd[2][b], vd[3][b]);
        split_f16x2(mul2(p00, vd01), ah0, al0);
        split_f16x2(mul2(p10, vd23), ah2, al2);
        if constexpr (HI) {
            split_f16x2(mul2(p02, vd01), ah1, al1);
            split_f16x2(mul2(p12, vd23), ah3, al3);
        }
        const uint8_t *vw = vs + b * BLOCK_BYTES + 4 + 4 * g;
        const uint32_t w0 = *reinterpret_cast<const uint32_t *>(vw + (2 * t) * ROW);
        const uint32_t w1 = *reinterpret_cast<const uint32_t *>(vw + (2 * t + 1) * ROW);
        const uint32_t w8 = *reinterpret_cast<const uint32_t *>(vw + (2 * t + 8) * ROW);
        const uint32_t w9 = *reinterpret_cast<const uint32_t *>(vw + (2 * t + 9) * ROW);
#define TQK_PV_NTILE(JJ)                                                                               \
{                                                                                                  \
    const uint32_t bb0 = s8pair_to_f16x2<JJ>(w0, w1), bb1 = s8pair_to_f16x2<JJ>(w8, w9);           \
    float *a = st.acc[b][JJ];                                                                         \
    if constexpr (HI) {                                                                            \
        mma_f16_k16(a[0], a[1], a[2], a[3], ah0, ah1, ah2, ah3, bb0, bb1);                         \
        mma_f16_k16(a[0], a[1], a[2], a[3], al0, al1, al2, al3, bb0, bb1);                         \
    } else {                                                                                       \
        mma_f16_k16_hl(a[0], a[1], ah0, al0, ah2, al2, bb0, bb1);                                  \
    }                                                                                              \
}
        TQK_PV_NTILE(0)
        TQK_PV_NTILE(1)
        TQK_PV_NTILE(2)
        TQK_PV_NTILE(3)
#undef TQK_PV_NTILE
    }
}

template <int NB, int GPAD>
__global__ void __launch_bounds__(MMA_THREADS) decode_q8_mma_kernel(const DecodeParams p) {
    using L = MmaLayout<NB, GPAD>;
    constexpr int HD = L::HD, ROW = L::ROW, STAGES = L::STAGES;
    constexpr bool HI = GPAD > 8;

    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // programmatic dependent launch: everything this kernel reads (q, new rows,
    // lengths, cache rows) may come from earlier kernels of the stream, so wait
    // for them first; then the next kernel may start its own prefetch
    grid_dependency_wait();
    grid_dependents_launch();

    const int item = blockIdx.z;
    const int pair = blockIdx.y;
    const int kvh = pair / p.head_slices;
    const int slice = pair - kvh * p.head_slices;
    const int g0 = slice * p.heads_per_cta;
    const int G = min(p.heads_per_cta, p.group - g0);
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
    if (s >= (n_splits > 0 ? n_splits : 1)) return;
    const int qh0 = kvh * p.group + g0;
    float *out_item = p.out + (long long)item * p.out_item_stride;

    if (len == 0) {  // empty context: zeros, like the reference's accum over no tokens
        for (int i = tid; i < G * HD; i += MMA_THREADS) {
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
    const int n_tiles = (t_end - t_begin + MMA_T - 1) / MMA_T;
    const long long head_off = (long long)kvh * p.max_tokens * ROW;
    const uint8_t *kbase = p.k + (long long)item * p.item_stride + head_off;
    const uint8_t *vbase = p.v + (long long)item * p.item_stride + head_off;

    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t *empty = full + STAGES;
    int8_t *qq = reinterpret_cast<int8_t *>(smem + L::OFF_QQ);
    float *qd = reinterpret_cast<float *>(smem + L::OFF_QD);
    uint8_t *newrow = smem + L::OFF_NEW;
    int *flag = reinterpret_cast<int *>(smem + L::OFF_FLAG);
    int *timeout = flag + 1;

    auto issue = [&](int j) {
        const int slot = j % STAGES;
        const int t0 = t_begin + j * MMA_T;
        const int rows = min(MMA_T, t_end - t0);
        const uint32_t bytes = (uint32_t)(rows * ROW);
        uint8_t *ks = smem + slot * L::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[slot], 2 * bytes);
        bulk_copy_g2s(ks, kbase + (long long)t0 * ROW, bytes, &full[slot]);
        bulk_copy_g2s(ks + L::TILE, vbase + (long long)t0 * ROW, bytes, &full[slot]);
    };

    const int producer = MMA_WARPS * 32;
    if (tid == producer) {
#pragma unroll
        for (int st = 0; st < STAGES; st++) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], MMA_WARPS);
        }
        fence_barrier_init();
        for (int j = 0; j < min(STAGES, n_tiles); j++) issue(j);
        *timeout = 0;
    }

    const bool do_append = p.k_new != nullptr && s == n_splits - 1;
    const int pos = len - 1;
    if (warp < MMA_WARPS) {
        // quantise this CTA's G q heads (quant_x.c:12-34), one row per warp with
        // the row's loads issued together; the padding rows G..15 are zero
        const float *qsrc = p.q + (long long)item * p.q_item_stride + (long long)qh0 * HD;
        float *pro = reinterpret_cast<float *>(smem + L::OFF_PRO) + warp * pro_stride<NB>();
        for (int g = warp; g < 16; g += MMA_WARPS) {
            if (g < G) {
                float x[NB];
#pragma unroll
                for (int b = 0; b < NB; b++) x[b] = __ldg(qsrc + g * HD + b * QK + lane);
                row_prologue<NB>(p, item, false, x, pro, lane);  // fused prologue, if asked for
                int8_t q8[NB];
                float dq[NB];
                warp_quantize_blocks<NB>(x, q8, dq);
#pragma unroll
                for (int b = 0; b < NB; b++) {
                    qq[g * HD + b * QK + lane] = q8[b];
                    if (lane == 0) qd[g * NB + b] = dq[b];
                }
            } else {
#pragma unroll
                for (int b = 0; b < NB; b++) qq[g * HD + b * QK + lane] = 0;
                if (lane < NB) qd[g * NB + lane] = 0.0f;
            }
        }
        // fused append (store_kv, attention_layer.c:66-90) by the split holding len-1
        if (do_append && warp < 2) {
            const float *src = (warp == 0 ? p.k_new : p.v_new) + (long long)item * p.kv_new_item_stride +
                               (long long)kvh * HD;
            uint8_t *nrow = newrow + warp * ROW;
            uint8_t *grow = (warp == 0 ? p.kw : p.vw) + (long long)item * p.item_stride + head_off +
                            (long long)pos * ROW;
            float x[NB];
#pragma unroll
            for (int b = 0; b < NB; b++) x[b] = __ldg(src + b * QK + lane);
            if (warp == 0) row_prologue<NB>(p, item, true, x, pro, lane);
            int8_t q8[NB];
            float dq[NB];
            warp_quantize_blocks<NB>(x, q8, dq);
#pragma unroll
            for (int b = 0; b < NB; b++) {
                const float d = dq[b];
                const int8_t v8 = q8[b];
                nrow[b * BLOCK_BYTES + 4 + lane] = (uint8_t)v8;
                if (lane == 0) *reinterpret_cast<float *>(nrow + b * BLOCK_BYTES) = d;
                if (slice == 0) {
                    grow[b * BLOCK_BYTES + 4 + lane] = (uint8_t)v8;
                    if (lane == 0) *reinterpret_cast<float *>(grow + b * BLOCK_BYTES) = d;
                }
            }
        }
    }
    __syncthreads();

    if (warp == MMA_WARPS) {
        // producer: the rest of the tiles, each once its slot has been released
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
    SliceState<NB, HI> st;
    st.begin(qq, qd, g, t);
    constexpr int NACC = SliceState<NB, HI>::NACC;

    const int r0 = warp * 16;
    bool timed_out = false;
    for (int j = 0; j < n_tiles; j++) {
        const int slot = j % STAGES;
        const int t0 = t_begin + j * MMA_T;
        const int rows = min(MMA_T, t_end - t0);
        const bool ok = mbar_wait_bounded(&full[slot], (uint32_t)((j / STAGES) & 1), WAIT_NS, p.err);
        if (!__all_sync(0xffffffffu, ok)) {
            timed_out = true;
            break;
        }
        const int nvalid = rows - r0;  // tokens of this warp's slice present in the tile
        if (nvalid > 0) {
            uint8_t *ks = smem + slot * L::STAGE_BYTES + r0 * ROW;
            uint8_t *vs = ks + L::TILE;
            if (do_append && pos >= t0 + r0 && pos < t0 + r0 + 16) {
                // substitute the freshly quantised row for the cache row at len-1
                const int r = pos - t0 - r0;
                for (int i = lane; i < ROW / 4; i += 32) {
                    reinterpret_cast<uint32_t *>(ks + r * ROW)[i] = reinterpret_cast<const uint32_t *>(newrow)[i];
                    reinterpret_cast<uint32_t *>(vs + r * ROW)[i] = reinterpret_cast<const uint32_t *>(newrow + ROW)[i];
                }
                __syncwarp();
            }
            if (nvalid >= 16)
                mma_slice<NB, HI, true>(st, ks, vs, 16, p.scale, g, t);
            else
                mma_slice<NB, HI, false>(st, ks, vs, nvalid, p.scale, g, t);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_release(&empty[slot]);
    }

    // ------------------------------------------------------------------ epilogue
    if (timed_out) *timeout = 1;
    cta_sync<1, MMA_WARPS * 32>();
    if (*timeout) return;  // a tile never arrived (DEVERR_TIMEOUT recorded): leave without output

    float *red = reinterpret_cast<float *>(smem);          // [W][GPAD][HD]
    float *wm = red + L::RED_FLOATS;                       // [W][GPAD] row max
    float *wl = wm + MMA_WARPS * GPAD;                     // [W][GPAD] row sum
    float *wsc = wl + MMA_WARPS * GPAD;                    // [W][GPAD] merge weight
    float *fm = wsc + MMA_WARPS * GPAD;                    // [GPAD]
    float *fl = fm + GPAD;                                 // [GPAD]
    float *wts = fl + GPAD;                                // [MAX_SPLITS][GPAD]
    const float unscale = exp2_int(st.kscale);
    if (t == 0) {
        wm[warp * GPAD + g] = st.m_lo;
        wl[warp * GPAD + g] = st.l_lo;
        if (HI) {
            wm[warp * GPAD + g + 8] = st.m_hi;
            wl[warp * GPAD + g + 8] = st.l_hi;
        }
    }
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            // permuted n-tile column n holds block column 4n + jj; this lane's d0/d1 are n = 2t, 2t+1
            const int c = b * QK + 8 * t + jj;
            red[(warp * GPAD + g) * HD + c] = st.acc[b][jj][0] * unscale;
            red[(warp * GPAD + g) * HD + c + 4] = st.acc[b][jj][1] * unscale;
            if constexpr (HI) {
                red[(warp * GPAD + g + 8) * HD + c] = st.acc[b][jj][NACC - 2] * unscale;
                red[(warp * GPAD + g + 8) * HD + c + 4] = st.acc[b][jj][NACC - 1] * unscale;
            }
        }
    cta_sync<1, MMA_WARPS * 32>();
    if (tid < GPAD) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < MMA_WARPS; w++) M = fmaxf(M, wm[w * GPAD + tid]);
        float Lsum = 0.0f;
#pragma unroll
        for (int w = 0; w < MMA_WARPS; w++) {
            const float mw = wm[w * GPAD + tid];  // base-2 units
            const float e = mw == -INFINITY ? 0.0f : exp2f(mw - M);
            wsc[w * GPAD + tid] = e;
            Lsum += wl[w * GPAD + tid] * e;
        }
        fm[tid] = M * 0.6931471805599453f;  // back to natural-log units for partials / merges
        fl[tid] = Lsum;
    }
    cta_sync<1, MMA_WARPS * 32>();
    auto acc_of = [&](int gg, int c) {
        float a = 0.0f;
#pragma unroll
        for (int w = 0; w < MMA_WARPS; w++) a = fmaf(red[(w * GPAD + gg) * HD + c], wsc[w * GPAD + gg], a);
        return a;
    };
    finish_split<HD, GPAD, MMA_WARPS * 32, 1>(p, tid, item, pair, s, n_splits, qh0, G, out_item, acc_of, fm, fl, wts,
                                              flag);
}

}  // namespace tqk
