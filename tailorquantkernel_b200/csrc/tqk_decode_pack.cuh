// tqk_decode_pack.cuh -- tensor-core Q8 decode with two kv heads packed into
// one MMA row block, for the 4-q-heads-per-kv-head grouping (Llama-3-8B:
// 32 q / 8 kv heads).  Included by tqk_decode.cu after tqk_decode_mma.cuh.
//
// With 4 q heads per kv head, the m16n8 fragments of tqk_decode_mma.cuh leave
// q rows 4-7 empty, so half of every lane's scalar work (score combine,
// softmax, P*vd) is spent on padding.  Here a CTA serves kv heads A = 2h and
// B = 2h+1 and a warp step covers 8 tokens of each:
//   QK  rows 0-3 = A's q heads, rows 4-7 = B's; one m16n8k32 against A's 8
//       K rows and one against B's, each lane keeping the one that matches its
//       row (lanes g < 4: A, g >= 4: B) -- every lane holds useful scores;
//   PV  the k = 16 dimension of m16n8k16 is A's 8 tokens then B's 8 tokens:
//       rows 0-3 carry P_A*vd in k 0-7 and zeros in k 8-15, rows 4-7 the
//       opposite, and the B operand stacks V_A over V_B, so one MMA (hi + lo)
//       accumulates both heads without wasted products.
// Everything else -- TMA ring, exact scores, base-2 online softmax, hi/lo fp16
// split, power-of-two PV scale, split merge -- is as in tqk_decode_mma.cuh.
#pragma once

namespace tqk {

constexpr int PK_WARPS = 4;                    // consumer warps
constexpr int PK_THREADS = (PK_WARPS + 1) * 32;
constexpr int PK_T = 8 * PK_WARPS;             // tokens per tile, per kv head

template <int NB>
struct PackLayout {
    static constexpr int HD = NB * QK;
    static constexpr int ROW = NB * BLOCK_BYTES;
    static constexpr int TILE = PK_T * ROW;       // one plane of one kv head
    static constexpr int STAGES = 3;
    static constexpr int STAGE_BYTES = 4 * TILE;  // K_A, K_B, V_A, V_B
    static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
    static constexpr int OFF_QQ = OFF_BAR + ((2 * STAGES * 8 + 15) / 16) * 16;  // int8 [16][HD] (rows 8-15 zero)
    static constexpr int OFF_QD = OFF_QQ + 16 * HD;                             // float [16][NB]
    static constexpr int OFF_NEW = OFF_QD + ((16 * NB * 4 + 15) / 16) * 16;    // appended rows [head][K,V][ROW]
    static constexpr int OFF_FLAG = OFF_NEW + ((4 * ROW + 15) / 16) * 16;
    static constexpr int BYTES = OFF_FLAG + 16;
    static constexpr int RED_FLOATS = PK_WARPS * 8 * HD;
    static constexpr int SCRATCH_FLOATS = RED_FLOATS + 3 * PK_WARPS * 8 + 2 * 8 + 2 * MAX_SPLITS * 8;
    static_assert(SCRATCH_FLOATS * 4 <= OFF_BAR, "stage ring too small for the epilogue scratch");
};

template <int NB>
__global__ void __launch_bounds__(PK_THREADS) decode_q8_pack_kernel(const DecodeParams p) {
    using L = PackLayout<NB>;
    constexpr int HD = L::HD, ROW = L::ROW, STAGES = L::STAGES;

    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const int item = blockIdx.z;
    const int pair = blockIdx.y;  // kv heads 2*pair and 2*pair+1
    const int kvh_a = 2 * pair;
    const int G = 8;              // q heads served: 4 of each kv head
    int len = p.lens ? p.lens[item] : p.len0 + item * p.len_step;
    if (len < 0 || len > p.max_tokens) {
        if (tid == 0) record_error(p.err, DEVERR_BADLEN);
        len = len < 0 ? 0 : p.max_tokens;
    }
    int n_splits = (len + p.split_tokens - 1) / p.split_tokens;
    if (n_splits > p.max_splits) {
        if (tid == 0) record_error(p.err, DEVERR_BADLEN);
        n_splits = p.max_splits;
        len = p.max_splits * p.split_tokens;
    }
    const int s = blockIdx.x;
    if (s >= (n_splits > 0 ? n_splits : 1)) return;
    const int qh0 = kvh_a * p.group;  // q heads qh0..qh0+7 are contiguous (group == 4)
    float *out_item = p.out + (long long)item * p.out_item_stride;

    if (len == 0) {
        for (int i = tid; i < G * HD; i += PK_THREADS) {
            const int g = i / HD, c = i - g * HD;
            if (p.out_mode == TQK_OUT_NORMALIZED) {
                out_item[(long long)(qh0 + g) * HD + c] = 0.0f;
            } else {
                float *o = out_item + (long long)(qh0 + g) * (HD + 2);
                o[c] = 0.0f;
                if (c == 0) { o[HD] = -INFINITY; o[HD + 1] = 0.0f; }
            }
        }
        return;
    }

    const int t_begin = s * p.split_tokens;
    const int t_end = min(len, t_begin + p.split_tokens);
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
        bulk_copy_g2s(st + L::TILE, ka + head_bytes + o, bytes, &full[slot]);
        bulk_copy_g2s(st + 2 * L::TILE, va + o, bytes, &full[slot]);
        bulk_copy_g2s(st + 3 * L::TILE, va + head_bytes + o, bytes, &full[slot]);
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
        // quantise the 8 q heads (quant_x.c:12-34), two rows per warp, loads first; rows 8-15 zero
        const float *qsrc = p.q + (long long)item * p.q_item_stride + (long long)qh0 * HD;
        float x[2][NB];
#pragma unroll
        for (int r = 0; r < 2; r++)
#pragma unroll
            for (int b = 0; b < NB; b++) x[r][b] = __ldg(qsrc + (warp + 4 * r) * HD + b * QK + lane);
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const int g = warp + 4 * r;
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float d;
                const int8_t v8 = warp_quantize_block(x[r][b], &d);
                qq[g * HD + b * QK + lane] = v8;
                qq[(g + 8) * HD + b * QK + lane] = 0;
                if (lane == 0) {
                    qd[g * NB + b] = d;
                    qd[(g + 8) * NB + b] = 0.0f;
                }
            }
        }
        // fused append (store_kv, attention_layer.c:66-90): warp 0/1 K/V of head A, 2/3 of head B
        if (do_append) {
            const int hb = warp >> 1, plane = warp & 1;
            const int kvh = kvh_a + hb;
            const float *src = (plane == 0 ? p.k_new : p.v_new) + (long long)item * p.kv_new_item_stride +
                               (long long)kvh * HD;
            uint8_t *nrow = newrow + (hb * 2 + plane) * ROW;
            uint8_t *grow = (plane == 0 ? p.kw : p.vw) + (long long)item * p.item_stride + (long long)kvh * head_bytes +
                            (long long)pos * ROW;
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float d;
                const int8_t v8 = warp_quantize_block(__ldg(src + b * QK + lane), &d);
                nrow[b * BLOCK_BYTES + 4 + lane] = (uint8_t)v8;
                grow[b * BLOCK_BYTES + 4 + lane] = (uint8_t)v8;
                if (lane == 0) {
                    *reinterpret_cast<float *>(nrow + b * BLOCK_BYTES) = d;
                    *reinterpret_cast<float *>(grow + b * BLOCK_BYTES) = d;
                }
            }
        }
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
    SliceState<NB, false> st;
    st.begin(qq, qd, g, t);

    const int r0 = warp * 8;  // this warp's 8 tokens of each head in a tile
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
            uint8_t *k_a = stg + r0 * ROW, *k_b = stg + L::TILE + r0 * ROW;
            uint8_t *v_a = stg + 2 * L::TILE + r0 * ROW, *v_b = stg + 3 * L::TILE + r0 * ROW;
            if (do_append && pos >= t0 + r0 && pos < t0 + r0 + 8) {
                const int r = pos - t0 - r0;
                uint8_t *dsts[4] = {k_a + r * ROW, v_a + r * ROW, k_b + r * ROW, v_b + r * ROW};
#pragma unroll
                for (int q = 0; q < 4; q++)
                    for (int i = lane; i < ROW / 4; i += 32)
                        reinterpret_cast<uint32_t *>(dsts[q])[i] = reinterpret_cast<const uint32_t *>(newrow + q * ROW)[i];
                __syncwarp();
            }
            const uint8_t *kmine = hb ? k_b : k_a;  // the lane's own head for scales
            const uint8_t *vmine = hb ? v_b : v_a;

            // ---- scores of the lane's row g for tokens 2t, 2t+1 (exact reference rounding)
            f32x2 acc2 = pk2(0.0f, 0.0f);
            {
                const uint8_t *kba = k_a + g * ROW, *kbb = k_b + g * ROW;  // B fragment token g of each head
#pragma unroll
                for (int b = 0; b < NB; b++) {
                    int ca[4], cb[4];
                    mma_s8_k32(ca, st.qa[b], *reinterpret_cast<const uint32_t *>(kba + b * BLOCK_BYTES + 4 + 4 * t),
                               *reinterpret_cast<const uint32_t *>(kba + b * BLOCK_BYTES + 20 + 4 * t));
                    mma_s8_k32(cb, st.qa[b], *reinterpret_cast<const uint32_t *>(kbb + b * BLOCK_BYTES + 4 + 4 * t),
                               *reinterpret_cast<const uint32_t *>(kbb + b * BLOCK_BYTES + 20 + 4 * t));
                    const int c0 = hb ? cb[0] : ca[0], c1 = hb ? cb[1] : ca[1];
                    const f32x2 kd = pk2(*reinterpret_cast<const float *>(kmine + (2 * t) * ROW + b * BLOCK_BYTES),
                                         *reinterpret_cast<const float *>(kmine + (2 * t + 1) * ROW + b * BLOCK_BYTES));
                    acc2 = add2(acc2, mul2(pk2(__int2float_rn(c0), __int2float_rn(c1)), mul2(st.qdl2[b], kd)));
                }
            }
            float s0, s1;
            upk2(mul2(mul2(acc2, pk2(p.scale, p.scale)), pk2(1.4426950408889634f, 1.4426950408889634f)), s0, s1);
            if (2 * t >= nvalid) s0 = -INFINITY;
            if (2 * t + 1 >= nvalid) s1 = -INFINITY;

            // ---- online softmax of the row over its 8 tokens (the quad)
            float mx = fmaxf(s0, s1);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mn = fmaxf(st.m_lo, mx);
            const float corr = exp2f(st.m_lo - mn);
            const float p0 = exp2f(s0 - mn), p1 = exp2f(s1 - mn);
            float sum = p0 + p1;
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            st.l_lo = st.l_lo * corr + sum;
            st.m_lo = mn;

            // ---- V scales of the lane's tokens (own head); slice max over both heads
            float vd0[NB], vd1[NB];
            float vmax = 0.0f;
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float d0 = *reinterpret_cast<const float *>(vmine + (2 * t) * ROW + b * BLOCK_BYTES);
                float d1 = *reinterpret_cast<const float *>(vmine + (2 * t + 1) * ROW + b * BLOCK_BYTES);
                if (2 * t >= nvalid) d0 = 0.0f;
                if (2 * t + 1 >= nvalid) d1 = 0.0f;
                vd0[b] = d0;
                vd1[b] = d1;
                vmax = fmaxf(vmax, fmaxf(d0, d1));
            }
            vmax = warp_max(vmax);
            const int kt = vmax >= 1.17549435e-38f ? ((__float_as_int(vmax) >> 23) & 0xFF) - 127 + 1 : -125;
            const int knew = max(st.kscale, min(kt, 126));
            if (__any_sync(0xffffffffu, corr != 1.0f || knew != st.kscale)) {
                const int df = st.kscale - knew;
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
            const f32x2 pp = mul2(pk2(p0, p1), pk2(inv_k, inv_k));

            // ---- P*V: k 0-7 = head A's tokens, k 8-15 = head B's; lanes fill their own half
#pragma unroll
            for (int b = 0; b < NB; b++) {
                uint32_t ah, al;
                split_f16x2(mul2(pp, pk2(vd0[b], vd1[b])), ah, al);
                const uint32_t ah0 = hb ? 0u : ah, ah2 = hb ? ah : 0u;
                const uint32_t al0 = hb ? 0u : al, al2 = hb ? al : 0u;
                const int wo = b * BLOCK_BYTES + 4 + 4 * g;
                const uint32_t w0 = *reinterpret_cast<const uint32_t *>(v_a + (2 * t) * ROW + wo);
                const uint32_t w1 = *reinterpret_cast<const uint32_t *>(v_a + (2 * t + 1) * ROW + wo);
                const uint32_t w8 = *reinterpret_cast<const uint32_t *>(v_b + (2 * t) * ROW + wo);
                const uint32_t w9 = *reinterpret_cast<const uint32_t *>(v_b + (2 * t + 1) * ROW + wo);
#define TQK_PK_NTILE(JJ)                                                                        \
    {                                                                                           \
        const uint32_t bb0 = s8pair_to_f16x2<JJ>(w0, w1), bb1 = s8pair_to_f16x2<JJ>(w8, w9);    \
        float *a = st.acc[b][JJ];                                                               \
        mma_f16_k16_lo(a[0], a[1], ah0, ah2, bb0, bb1);                                         \
        mma_f16_k16_lo(a[0], a[1], al0, al2, bb0, bb1);                                         \
    }
                TQK_PK_NTILE(0)
                TQK_PK_NTILE(1)
                TQK_PK_NTILE(2)
                TQK_PK_NTILE(3)
#undef TQK_PK_NTILE
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_release(&empty[slot]);
    }

    // ------------------------------------------------------------------ epilogue
    if (timed_out) *timeout = 1;
    cta_sync<1, PK_WARPS * 32>();
    if (*timeout) return;

    float *red = reinterpret_cast<float *>(smem);  // [W][8][HD]
    float *wm = red + L::RED_FLOATS;               // [W][8]
    float *wl = wm + PK_WARPS * 8;
    float *wsc = wl + PK_WARPS * 8;
    float *fm = wsc + PK_WARPS * 8;                // [8]
    float *fl = fm + 8;
    float *wts = fl + 8;                           // [2][MAX_SPLITS][8]
    const float unscale = exp2_int(st.kscale);
    if (t == 0) {
        wm[warp * 8 + g] = st.m_lo;
        wl[warp * 8 + g] = st.l_lo;
    }
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            const int c = b * QK + 8 * t + jj;  // permuted n-tile column n = 2t, 2t+1 -> 4n + jj
            red[(warp * 8 + g) * HD + c] = st.acc[b][jj][0] * unscale;
            red[(warp * 8 + g) * HD + c + 4] = st.acc[b][jj][1] * unscale;
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
    auto acc_of = [&](int gg, int c) {
        float a = 0.0f;
#pragma unroll
        for (int w = 0; w < PK_WARPS; w++) a = fmaf(red[(w * 8 + gg) * HD + c], wsc[w * 8 + gg], a);
        return a;
    };
    finish_split<HD, 8, PK_WARPS * 32, 1>(p, tid, item, pair, s, n_splits, qh0, G, out_item, acc_of, fm, fl, wts, flag);
}

}  // namespace tqk
