// tqk_decode.cu -- fused Q8 GQA decode attention for sm_100a (the hot path).
//
// Replaces attend_q8 (reference model/attention_layer.c:125-150) and, fused,
// store_kv's Q8 branch (:66-90).  Design (one CTA = one contiguous token range
// of one kv head of one item, serving all q heads of the group):
//
//   * K/V rows (144 B for head_dim 128 = 4 blocks of 36 B, 16-byte aligned) of
//     a 64-token tile are one contiguous byte range per plane; thread 0 streams
//     them into a STAGES-deep shared-memory ring with 1-D TMA bulk copies
//     (cp.async.bulk, no multicast) completing on mbarriers, so each K/V byte
//     leaves HBM exactly once per launch.
//   * q is quantised in-kernel with the bit-exact device quantiser; scores use
//     dp4a on int8 (exact int32 block sums) and then the reference's rounding
//     sequence acc += (float)sum * (qd*kd), acc * scale with explicitly rounded
//     intrinsics, so every score equals attn_scores_q8_scalar's bit for bit.
//   * online softmax in FP32 per q head; V accumulation o += (p*vd) * (float)q
//     with threads owning 4-column slices and warps owning token subsets.
//   * splits write (m, l, acc) partials; the last CTA of an (item, kv head)
//     (atomic ticket, no waiting) merges them by log-sum-exp in split order, so
//     results are deterministic.
#include "tqk_internal.h"

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <mutex>

namespace tqk {

constexpr int DEC_THREADS = 128;
constexpr int DEC_WARPS = DEC_THREADS / 32;
constexpr int DEC_T = 64;          // tokens per tile
constexpr int MAX_SPLITS = 128;    // bound on splits per (item, kv head)
constexpr int MERGE_GROUP = 16;    // up to 16 splits merge in one level; more in groups of 16
constexpr int CL_MAX = 16;         // largest cluster of the cluster merge (non-portable above 8)
// ints per (item, head unit) in the ticket region: the final ticket and one per
// group; the stride is kept at 17 so that caller workspaces keep their layout
constexpr int TICKETS_PER_UNIT = 17;
static_assert(1 + (MAX_SPLITS + MERGE_GROUP - 1) / MERGE_GROUP <= TICKETS_PER_UNIT, "ticket block too small");

// Number of splits of an item of len tokens at split tokens per split: the
// whole splits, plus one for a remainder above a quarter split; a smaller
// remainder joins the last whole split, so that no CTA is spent on a sliver
// (4097 tokens at 256 per split are 16 splits, the last of 257 tokens, not
// 17).  Non-decreasing in len.  Split s covers [s*split, s*split + split),
// the last one [s*split, len).
__host__ __device__ __forceinline__ int n_splits_of(int len, int split) {
    if (len <= 0) return 0;
    const int n = len / split, rem = len - n * split;
    return n == 0 ? 1 : n + (rem > split / 4 ? 1 : 0);
}
__host__ __device__ __forceinline__ int split_end(int s, int n_splits, int split, int len) {
    return s == n_splits - 1 ? len : (s + 1) * split;
}
constexpr uint64_t WAIT_NS = 1000000000ull;   // 1 s bound on any mbarrier wait
constexpr uint64_t DRAIN_NS = 20000000ull;    // 20 ms bound when draining after a timeout

struct DecodeParams {
    const uint8_t *k, *v;        // planes of item 0 (bytes)
    uint8_t *kw, *vw;            // the same planes, writable (fused append)
    long long item_stride;       // bytes between items' planes
    int n_items, n_kv, group, max_tokens;
    int heads_per_cta, head_slices, pairs;  // pairs = n_kv * head_slices
    const int *lens;
    int len0, len_step;
    const float *q;
    long long q_item_stride;     // floats
    float *out;
    long long out_item_stride;   // floats
    const float *k_new, *v_new;
    long long kv_new_item_stride;  // floats
    const float *q_norm, *k_norm;  // optional prologue: RMSNorm weights [head_dim] per item
    long long norm_item_stride;    // floats
    float norm_eps;
    const float *rope_cos, *rope_sin;  // optional prologue: RoPE tables [head_dim/2] per item
    long long rope_item_stride;        // floats
    int out_mode;
    int split_tokens;            // multiple of DEC_T
    int max_splits;
    float scale;
    float *part;                 // [n_items][pairs][max_splits][GMAX][HD+2]; balanced: [ctas + units][8][HD+2]
    int *counters;               // tickets: [n_items][pairs][TICKETS_PER_UNIT]; balanced: [..][tickets_per_unit]
    int *err;
    int tickets_per_unit;        // balanced schedule only
    // fused gather of the kv-head-group split (tqk_decode_q8_gather; g_world == 0: off).  The
    // normalised output of local flat q head f = item * n_q_heads + qh goes to every rank r's
    // buffer g_out[r] at [f / g_chunk][g_rank][f % g_chunk][HD] as {value bits, g_epoch} pairs,
    // each written by one 64-bit store, so a reader that sees the epoch sees the value.
    int g_world, g_rank, g_chunk, g_epoch;
    uint2 *g_out[8];
    // the packed kernel's split merge through a thread-block cluster (the max_splits CTAs of one
    // unit, cluster dims (cluster, 1, 1)); 0 = tickets and partials in global memory
    int cluster;
};

// One element of the call's normalised output: head qh (of the item) column c.
template <int HD>
__device__ __forceinline__ void store_out(const DecodeParams &p, float *out_item, int item, int qh, int c, float v) {
    if (p.g_world == 0) {
        out_item[(long long)qh * HD + c] = v;
        return;
    }
    // 32-bit index arithmetic (n_items * n_q_heads < 2^31): the division is by a runtime value
    const unsigned f = (unsigned)item * (unsigned)(p.n_kv * p.group) + (unsigned)qh;
    const unsigned grp = f / (unsigned)p.g_chunk, w = f - grp * (unsigned)p.g_chunk;
    const size_t off = ((size_t)(grp * (unsigned)p.g_world + (unsigned)p.g_rank) * (unsigned)p.g_chunk + w) * HD + c;
    // {value bits, epoch} as one 64-bit access: single-copy atomic, so a reader that sees the
    // epoch sees the value
    const unsigned long long pr = ((unsigned long long)(unsigned)p.g_epoch << 32) | __float_as_uint(v);
    for (int r = 0; r < p.g_world; r++)  // one store per rank, over NVLink for the peers
        asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p.g_out[r] + off), "l"(pr) : "memory");
}

template <int NB>
constexpr int stages_for() { return NB >= 8 ? 2 : 3; }

// Shared-memory layout of one CTA (bytes; every region 16-byte aligned).
template <int NB, int GMAX>
struct DecLayout {
    static constexpr int HD = NB * QK;
    static constexpr int ROW = NB * BLOCK_BYTES;
    static constexpr int TILE = DEC_T * ROW;   // one plane's tile
    static constexpr int STAGES = stages_for<NB>();
    static constexpr int STAGE_BYTES = 2 * TILE;
    static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
    static constexpr int OFF_QQ = OFF_BAR + 64;
    static constexpr int OFF_QD = OFF_QQ + GMAX * HD;
    static constexpr int OFF_SC = OFF_QD + ((GMAX * NB * 4 + 15) / 16) * 16;
    static constexpr int OFF_PV = OFF_SC + GMAX * DEC_T * 4;
    static constexpr int OFF_STATE = OFF_PV + DEC_T * NB * GMAX * 4;  // m, l, corr
    static constexpr int OFF_NEW = OFF_STATE + ((3 * GMAX * 4 + 15) / 16) * 16;
    static constexpr int OFF_PRO = OFF_NEW + ((2 * ROW + 15) / 16) * 16;  // prologue row per warp
    static constexpr int OFF_FLAG = OFF_PRO + DEC_WARPS * pro_stride<NB>() * 4;
    static constexpr int BYTES = OFF_FLAG + 16;
    // after the pipeline drains, the stage ring is reused for the cross-warp
    // reduction and the merge weights
    static constexpr int RED_BYTES = DEC_WARPS * GMAX * HD * 4;
    static constexpr int WTS_BYTES = 2 * MAX_SPLITS * GMAX * 4;  // merge weights + split sums
    static_assert(RED_BYTES + WTS_BYTES <= OFF_BAR, "stage ring too small for the epilogue scratch");
    static_assert(TILE % 16 == 0, "tiles must be whole 16-byte units");
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Score of one cached K row against one quantised q head, with the rounding
// sequence of attn_scores_q8_scalar (reference model/attn_q8.c:24-31).
template <int NB>
__device__ __forceinline__ float score_row(const uint8_t *row, const uint32_t (&qw)[NB * 8], const float (&qds)[NB],
                                           float scale) {
    float acc = 0.0f;
    if constexpr (NB % 4 == 0) {
#pragma unroll
        for (int b4 = 0; b4 < NB / 4; b4++) {
            uint32_t w[36];
            const uint4 *r4 = reinterpret_cast<const uint4 *>(row + b4 * 4 * BLOCK_BYTES);
#pragma unroll
            for (int i = 0; i < 9; i++) {
                const uint4 u = r4[i];
                w[4 * i + 0] = u.x; w[4 * i + 1] = u.y; w[4 * i + 2] = u.z; w[4 * i + 3] = u.w;
            }
#pragma unroll
            for (int bb = 0; bb < 4; bb++) {
                const int b = b4 * 4 + bb;
                int sum = 0;
#pragma unroll
                for (int k = 0; k < 8; k++) sum = __dp4a((int)w[bb * 9 + 1 + k], (int)qw[b * 8 + k], sum);
                const float kd = __uint_as_float(w[bb * 9]);
                acc = __fadd_rn(acc, __fmul_rn(__int2float_rn(sum), __fmul_rn(qds[b], kd)));
            }
        }
    } else {
        const uint32_t *rw = reinterpret_cast<const uint32_t *>(row);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            int sum = 0;
#pragma unroll
            for (int k = 0; k < 8; k++) sum = __dp4a((int)rw[b * 9 + 1 + k], (int)qw[b * 8 + k], sum);
            const float kd = __uint_as_float(rw[b * 9]);
            acc = __fadd_rn(acc, __fmul_rn(__int2float_rn(sum), __fmul_rn(qds[b], kd)));
        }
    }
    return __fmul_rn(acc, scale);
}

// The call's fused prologue (norm_heads + rope_heads, attention_layer.c:183-189)
// on R q rows (is_k false) or the appended K row of `item`, held by a warp as
// x[r][b] = row_r[b*32 + lane]; `scratch` is the warp's R * pro_stride<NB>()
// floats.  A no-op when the call asks for none.
template <int NB, int R>
__device__ __forceinline__ void row_prologue(const DecodeParams &p, int item, bool is_k, float (&x)[R][NB],
                                             float *scratch, int lane) {
    const float *w = is_k ? p.k_norm : p.q_norm;
    if (!w && !p.rope_cos) return;
    const long long ni = (long long)item * p.norm_item_stride, ri = (long long)item * p.rope_item_stride;
    warp_norm_rope<NB, R>(x, w ? w + ni : nullptr, p.rope_cos ? p.rope_cos + ri : nullptr,
                          p.rope_cos ? p.rope_sin + ri : nullptr, p.norm_eps, scratch, lane);
}
template <int NB>
__device__ __forceinline__ void row_prologue(const DecodeParams &p, int item, bool is_k, float (&x)[NB],
                                             float *scratch, int lane) {
    row_prologue<NB, 1>(p, item, is_k, reinterpret_cast<float(&)[1][NB]>(x), scratch, lane);
}

// Tickets and the arrival test of the split merge.  A CTA that wrote its
// partial takes a ticket; the one that draws the last number of its group
// merges (never a wait).
// The CTA's barrier orders every thread's partial writes before thread 0's
// gpu-scope acquire-release ticket increment (fence cumulativity), so one
// thread publishes for the whole CTA; the CTA that draws the last ticket
// acquires every earlier CTA's writes through the same atomic.
__device__ __forceinline__ int ticket_add_acq_rel(int *ticket) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(ticket) : "memory");
    return old;
}

template <int BAR, int NT>
__device__ __forceinline__ bool last_arrival(int *ticket, int n, int tid, int *flag) {
    cta_sync<BAR, NT>();
    if (tid == 0) *flag = (ticket_add_acq_rel(ticket) == n - 1);
    cta_sync<BAR, NT>();
    return *flag;  // read by every thread before the next arrival's sync
}

// Log-sum-exp merge, in slot order, of the n partials {acc[HD], m, l} in slots
// first, first + stride, ... of one (item, head unit)'s partial area pb
// ([slot][GROWS][HD + 2] floats).  to_part: the merged partial goes back into
// slot `first`; otherwise into the call's output (normalised, or as a partial
// in TQK_OUT_PARTIAL mode).  Each thread owns the same EPT elements across the
// slots.  The loads are the latency: the accumulators of up to KB slots are
// loaded in one batch, the first batch together with every slot's (m, l), so
// a merge of up to KB slots costs one L2 round trip.
template <int HD, int GROWS, int NT, int BAR>
__device__ __forceinline__ void merge_slots(const DecodeParams &p, float *pb, int first, int stride, int n, int G,
                                            int tid, float *wts, float *ms, float *ls, bool to_part, float *out_item,
                                            int item, int qh0) {
    constexpr int RS = HD + 2;
    constexpr int EPT = (GROWS * HD + NT - 1) / NT;
    constexpr int KB = EPT >= 64 ? 1 : 64 / EPT;  // slots per batch of loads in flight
    const int lane = tid & 31, warp = tid >> 5;
    float *lall = wts + MAX_SPLITS * GROWS;
    float xb[KB][EPT];
    auto load_batch = [&](int k0) {
#pragma unroll
        for (int kk = 0; kk < KB; kk++) {
            const int k = k0 + kk;
            const float *src = pb + (long long)(first + k * stride) * GROWS * RS;
#pragma unroll
            for (int e = 0; e < EPT; e++) {
                const int i = tid + e * NT, g = i / HD, c = i - g * HD;
                xb[kk][e] = (k < n && i < G * HD) ? __ldcg(src + g * RS + c) : 0.0f;
            }
        }
    };
    load_batch(0);
    for (int i = tid; i < n * G; i += NT) {  // every slot's (m, l), in the same round trip
        const int k = i / G, g = i - k * G;
        const float2 ml =
            __ldcg(reinterpret_cast<const float2 *>(pb + ((long long)(first + k * stride) * GROWS + g) * RS + HD));
        wts[k * GROWS + g] = ml.x;
        lall[k * GROWS + g] = ml.y;
    }
    cta_sync<BAR, NT>();
    for (int g = warp; g < G; g += NT / 32) {
        float M = -INFINITY;
        for (int k = lane; k < n; k += 32) M = fmaxf(M, wts[k * GROWS + g]);
        M = warp_max(M);
        float Lsum = 0.0f;
        for (int k = lane; k < n; k += 32) {
            const float w = expf(wts[k * GROWS + g] - M);
            wts[k * GROWS + g] = w;
            Lsum += lall[k * GROWS + g] * w;
        }
        Lsum = warp_sum(Lsum);
        if (lane == 0) { ms[g] = M; ls[g] = Lsum; }
    }
    cta_sync<BAR, NT>();
    float a[EPT];
#pragma unroll
    for (int e = 0; e < EPT; e++) a[e] = 0.0f;
    for (int k0 = 0; k0 < n; k0 += KB) {
        if (k0 > 0) load_batch(k0);
#pragma unroll
        for (int kk = 0; kk < KB; kk++) {
            const int k = k0 + kk;
            if (k >= n) break;
#pragma unroll
            for (int e = 0; e < EPT; e++) {
                const int i = tid + e * NT, g = i / HD;
                if (i < G * HD) a[e] = fmaf(wts[k * GROWS + g], xb[kk][e], a[e]);
            }
        }
    }
#pragma unroll
    for (int e = 0; e < EPT; e++) {
        const int i = tid + e * NT, g = i / HD, c = i - g * HD;
        if (i >= G * HD) continue;
        if (to_part) {
            float *d = pb + ((long long)first * GROWS + g) * RS;
            d[c] = a[e];
            if (c == 0) { d[HD] = ms[g]; d[HD + 1] = ls[g]; }
        } else if (p.out_mode == TQK_OUT_NORMALIZED) {
            store_out<HD>(p, out_item, item, qh0 + g, c, a[e] / ls[g]);
        } else {
            float *o = out_item + (long long)(qh0 + g) * RS;
            o[c] = a[e];
            if (c == 0) { o[HD] = ms[g]; o[HD + 1] = ls[g]; }
        }
    }
}

// Finishes one split of one (item, kv-head slice).  acc(g, c) is the CTA's
// unnormalised sum for its q head g and column c, relative to the running max
// ms[g], with softmax denominator ls[g].  A single split writes the output (or
// the partial, in TQK_OUT_PARTIAL mode); otherwise the split's partial goes to
// the workspace and the splits are merged by log-sum-exp without any wait:
//   n_splits <= MERGE_GROUP: the last-arriving split merges them all;
//   more: the last arrival of each group of MERGE_GROUP splits merges its group
//   into the group's first slot, and the last group to finish merges the
//   groups -- two short merges instead of one long serial one.
// Merges run in slot order, so results are deterministic.  ms/ls are
// overwritten by the merge; the tickets used are left at zero.
// pb: the unit's partial slots ([slot][GROWS][HD + 2] floats); tickets: its
// ticket block ([0] final, [1 + i] group i).
template <int HD, int GROWS, int NT, int BAR, typename AccFn>
__device__ __forceinline__ void finish_split_at(const DecodeParams &p, int tid, float *pb, int *tickets, int s,
                                                int n_splits, int item, int qh0, int G, float *out_item, AccFn acc,
                                                float *ms, float *ls, float *wts, int *flag) {
    const bool single = n_splits == 1;
    for (int i = tid; i < G * HD; i += NT) {
        const int g = i / HD, c = i - g * HD;
        const float a = acc(g, c);
        if (single) {
            if (p.out_mode == TQK_OUT_NORMALIZED) {
                store_out<HD>(p, out_item, item, qh0 + g, c, a / ls[g]);
            } else {
                float *o = out_item + (long long)(qh0 + g) * (HD + 2);
                o[c] = a;
                if (c == 0) { o[HD] = ms[g]; o[HD + 1] = ls[g]; }
            }
        } else {
            float *pp = pb + ((long long)s * GROWS + g) * (HD + 2);
            pp[c] = a;
            if (c == 0) { pp[HD] = ms[g]; pp[HD + 1] = ls[g]; }
        }
    }
    if (single) return;

    if (n_splits > MERGE_GROUP) {
        const int gi = s / MERGE_GROUP, first = gi * MERGE_GROUP;
        const int gsz = min(MERGE_GROUP, n_splits - first);
        if (!last_arrival<BAR, NT>(tickets + 1 + gi, gsz, tid, flag)) return;
        merge_slots<HD, GROWS, NT, BAR>(p, pb, first, 1, gsz, G, tid, wts, ms, ls, true, out_item, item, qh0);
        if (tid == 0) tickets[1 + gi] = 0;
        const int n_groups = (n_splits + MERGE_GROUP - 1) / MERGE_GROUP;
        if (!last_arrival<BAR, NT>(tickets, n_groups, tid, flag)) return;
        merge_slots<HD, GROWS, NT, BAR>(p, pb, 0, MERGE_GROUP, n_groups, G, tid, wts, ms, ls, false, out_item, item,
                                        qh0);
    } else {
        if (!last_arrival<BAR, NT>(tickets, n_splits, tid, flag)) return;
        merge_slots<HD, GROWS, NT, BAR>(p, pb, 0, 1, n_splits, G, tid, wts, ms, ls, false, out_item, item, qh0);
    }
    if (tid == 0) tickets[0] = 0;  // ready for the next launch
}

// The fixed-split layout: unit (item, pair) owns max_splits slots and
// TICKETS_PER_UNIT tickets.
template <int HD, int GROWS, int NT, int BAR, typename AccFn>
__device__ __forceinline__ void finish_split(const DecodeParams &p, int tid, int item, int pair, int s, int n_splits,
                                             int qh0, int G, float *out_item, AccFn acc, float *ms, float *ls,
                                             float *wts, int *flag) {
    const long long unit = (long long)item * p.pairs + pair;
    finish_split_at<HD, GROWS, NT, BAR>(p, tid, p.part + unit * p.max_splits * GROWS * (HD + 2),
                                        p.counters + unit * TICKETS_PER_UNIT, s, n_splits, item, qh0, G, out_item, acc,
                                        ms, ls, wts, flag);
}

template <int NB, int GMAX>
__global__ void __launch_bounds__(DEC_THREADS) decode_q8_kernel(const DecodeParams p) {
    using L = DecLayout<NB, GMAX>;
    constexpr int HD = L::HD, ROW = L::ROW, STAGES = L::STAGES;
    constexpr bool kTma = (NB % 4 == 0);  // 144-byte rows: every tile is 16-byte aligned
    constexpr int CPL = (HD / 32 < 4) ? 4 : HD / 32;  // V columns per lane
    constexpr int LPT = HD / CPL;                     // lanes per token row
    constexpr int TPW = 32 / LPT;                     // token rows per warp pass

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
        for (int i = tid; i < G * HD; i += DEC_THREADS) {
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
    const int n_tiles = (t_end - t_begin + DEC_T - 1) / DEC_T;
    const long long head_off = (long long)kvh * p.max_tokens * ROW;
    const uint8_t *kbase = p.k + (long long)item * p.item_stride + head_off;
    const uint8_t *vbase = p.v + (long long)item * p.item_stride + head_off;

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    int8_t *qq = reinterpret_cast<int8_t *>(smem + L::OFF_QQ);
    float *qd = reinterpret_cast<float *>(smem + L::OFF_QD);
    float *sc = reinterpret_cast<float *>(smem + L::OFF_SC);
    float *pv = reinterpret_cast<float *>(smem + L::OFF_PV);
    float *m_s = reinterpret_cast<float *>(smem + L::OFF_STATE);
    float *l_s = m_s + GMAX;
    float *corr_s = l_s + GMAX;
    uint8_t *newrow = smem + L::OFF_NEW;
    float *pro = reinterpret_cast<float *>(smem + L::OFF_PRO) + warp * pro_stride<NB>();
    int *flag = reinterpret_cast<int *>(smem + L::OFF_FLAG);

    auto issue = [&](int j) {
        const int slot = j % STAGES;
        const int t0 = t_begin + j * DEC_T;
        const int rows = min(DEC_T, t_end - t0);
        const uint32_t bytes = (uint32_t)(rows * ROW);
        uint8_t *ks = smem + slot * L::STAGE_BYTES;
        mbar_arrive_expect_tx(&bars[slot], 2 * bytes);
        bulk_copy_g2s(ks, kbase + (long long)t0 * ROW, bytes, &bars[slot]);
        bulk_copy_g2s(ks + L::TILE, vbase + (long long)t0 * ROW, bytes, &bars[slot]);
    };

    if (kTma && tid == 0) {
#pragma unroll
        for (int st = 0; st < STAGES; st++) mbar_init(&bars[st], 1);
        fence_barrier_init();
        for (int j = 0; j < min(STAGES - 1, n_tiles); j++) issue(j);
    }
    for (int i = tid; i < GMAX; i += DEC_THREADS) {
        m_s[i] = -INFINITY;
        l_s[i] = 0.0f;
        corr_s[i] = 1.0f;
    }
    for (int i = tid; i < DEC_T * NB * GMAX; i += DEC_THREADS) pv[i] = 0.0f;

    // quantise this CTA's q heads: one warp per 32-float block (quant_x.c:12-34)
    const float *qsrc = p.q + (long long)item * p.q_item_stride + (long long)qh0 * HD;
    if (p.q_norm || p.rope_cos) {
        // with the fused prologue, which needs whole rows: one warp per q row
        for (int g = warp; g < GMAX; g += DEC_WARPS) {
            float x[NB];
#pragma unroll
            for (int b = 0; b < NB; b++) x[b] = g < G ? __ldg(qsrc + g * HD + b * QK + lane) : 0.0f;
            if (g < G) row_prologue<NB>(p, item, false, x, pro, lane);
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float d;
                const int8_t v8 = warp_quantize_block(x[b], &d);
                qq[g * HD + b * QK + lane] = v8;
                if (lane == 0) qd[g * NB + b] = d;
            }
        }
    } else {
        for (int blk = warp; blk < GMAX * NB; blk += DEC_WARPS) {
            const int g = blk / NB, b = blk - g * NB;
            const float x = g < G ? __ldg(qsrc + g * HD + b * QK + lane) : 0.0f;
            float d;
            const int8_t v8 = warp_quantize_block(x, &d);
            qq[g * HD + b * QK + lane] = v8;
            if (lane == 0) qd[g * NB + b] = d;
        }
    }

    // fused append (store_kv, attention_layer.c:66-90): the split holding
    // position len-1 quantises the new K/V rows, writes them to the cache and
    // substitutes them for that row of its staged tile
    const bool do_append = p.k_new != nullptr && s == n_splits - 1;
    const int pos = len - 1;
    if (do_append && warp < 2) {
        const float *src = (warp == 0 ? p.k_new : p.v_new) + (long long)item * p.kv_new_item_stride +
                           (long long)kvh * HD;
        uint8_t *nrow = newrow + warp * ROW;
        uint8_t *grow = (warp == 0 ? p.kw : p.vw) + (long long)item * p.item_stride + head_off + (long long)pos * ROW;
        float x[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) x[b] = __ldg(src + b * QK + lane);
        if (warp == 0) row_prologue<NB>(p, item, true, x, pro, lane);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float d;
            const int8_t v8 = warp_quantize_block(x[b], &d);
            nrow[b * BLOCK_BYTES + 4 + lane] = (uint8_t)v8;
            if (lane == 0) *reinterpret_cast<float *>(nrow + b * BLOCK_BYTES) = d;
            if (slice == 0) {
                grow[b * BLOCK_BYTES + 4 + lane] = (uint8_t)v8;
                if (lane == 0) *reinterpret_cast<float *>(grow + b * BLOCK_BYTES) = d;
            }
        }
    }
    __syncthreads();

    // this thread's q head for the score phase (DEC_THREADS % GMAX == 0, so it is fixed)
    const int gq = tid % GMAX;
    uint32_t qw[NB * 8];
    float qds[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) {
        qds[b] = qd[gq * NB + b];
#pragma unroll
        for (int k = 0; k < 8; k++) qw[b * 8 + k] = reinterpret_cast<const uint32_t *>(qq + gq * HD + b * QK)[k];
    }

    const int sub_t = lane / LPT;
    const int c0 = (lane % LPT) * CPL;
    const int vb = c0 / QK;
    float acc[GMAX][CPL];
#pragma unroll
    for (int g = 0; g < GMAX; g++)
#pragma unroll
        for (int c = 0; c < CPL; c++) acc[g][c] = 0.0f;

    for (int j = 0; j < n_tiles; j++) {
        const int slot = j % STAGES;
        const int t0 = t_begin + j * DEC_T;
        const int rows = min(DEC_T, t_end - t0);
        uint8_t *ks = smem + slot * L::STAGE_BYTES;
        uint8_t *vs = ks + L::TILE;
        bool ok = true;
        if constexpr (kTma) {
            // slot (j-1)%STAGES was released by the trailing barrier of iteration j-1
            if (tid == 0 && j + STAGES - 1 < n_tiles) issue(j + STAGES - 1);
            ok = mbar_wait_bounded(&bars[slot], (uint32_t)((j / STAGES) & 1), WAIT_NS, p.err);
        } else {
            // rows of 36 or 72 bytes are only 4-byte aligned: cooperative word copy
            const uint32_t *gk = reinterpret_cast<const uint32_t *>(kbase + (long long)t0 * ROW);
            const uint32_t *gv = reinterpret_cast<const uint32_t *>(vbase + (long long)t0 * ROW);
            uint32_t *sk = reinterpret_cast<uint32_t *>(ks);
            uint32_t *sv = reinterpret_cast<uint32_t *>(vs);
            const int words = rows * ROW / 4;
            for (int i = tid; i < words; i += DEC_THREADS) {
                sk[i] = __ldg(gk + i);
                sv[i] = __ldg(gv + i);
            }
        }
        const bool has_new = do_append && pos >= t0 && pos < t0 + rows;  // CTA-uniform
        if (!kTma || has_new) {
            if (has_new) {
                __syncthreads();  // every thread has seen the tile land before it is patched
                const int r = pos - t0;
                for (int i = tid; i < ROW / 4; i += DEC_THREADS) {
                    reinterpret_cast<uint32_t *>(ks + r * ROW)[i] = reinterpret_cast<const uint32_t *>(newrow)[i];
                    reinterpret_cast<uint32_t *>(vs + r * ROW)[i] =
                        reinterpret_cast<const uint32_t *>(newrow + ROW)[i];
                }
            }
            __syncthreads();
        }

        // scores: thread -> (q head gq, tokens tid/GMAX + k*DEC_THREADS/GMAX)
        for (int it = tid; it < DEC_T * GMAX; it += DEC_THREADS) {
            const int tt = it / GMAX;
            float sv = -INFINITY;
            if (gq < G && tt < rows) sv = score_row<NB>(ks + tt * ROW, qw, qds, p.scale);
            sc[gq * DEC_T + tt] = sv;
        }
        if (!__syncthreads_and(ok)) {
            // a tile never arrived: drain our outstanding copies (bounded) and leave
            if (kTma && tid == 0) {
                for (int jj = j; jj < min(j + STAGES - 1, n_tiles); jj++)
                    mbar_wait_bounded(&bars[jj % STAGES], (uint32_t)((jj / STAGES) & 1), DRAIN_NS, p.err);
            }
            return;
        }

        // online softmax (one warp per q head) and pv[t][b][g] = p * vd
        for (int g = warp; g < G; g += DEC_WARPS) {
            const float s0 = sc[g * DEC_T + lane], s1 = sc[g * DEC_T + lane + 32];
            const float m_old = m_s[g];
            const float m_new = fmaxf(m_old, warp_max(fmaxf(s0, s1)));
            const float corr = expf(m_old - m_new);
            const float p0 = expf(s0 - m_new), p1 = expf(s1 - m_new);
            const float psum = warp_sum(p0 + p1);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int t = lane + 32 * h;
                const float pt = h ? p1 : p0;
                if (t < rows) {
#pragma unroll
                    for (int b = 0; b < NB; b++) {
                        const float vd = *reinterpret_cast<const float *>(vs + t * ROW + b * BLOCK_BYTES);
                        pv[(t * NB + b) * GMAX + g] = pt * vd;
                    }
                }
            }
            if (lane == 0) {
                l_s[g] = l_s[g] * corr + psum;
                m_s[g] = m_new;
                corr_s[g] = corr;
            }
        }
        __syncthreads();

        // V accumulation: lane owns CPL columns, warp owns a token subset
        {
            float cr[GMAX];
#pragma unroll
            for (int g = 0; g < GMAX; g++) cr[g] = corr_s[g];
#pragma unroll
            for (int g = 0; g < GMAX; g++)
#pragma unroll
                for (int c = 0; c < CPL; c++) acc[g][c] *= cr[g];
            for (int tt = warp * TPW + sub_t; tt < rows; tt += DEC_WARPS * TPW) {
                const uint8_t *vrow = vs + tt * ROW + vb * BLOCK_BYTES + 4 + (c0 % QK);
                float pvv[GMAX];
                const float *pvt = pv + (tt * NB + vb) * GMAX;
                if constexpr (GMAX >= 4) {
#pragma unroll
                    for (int g = 0; g < GMAX; g += 4) {
                        const float4 f = *reinterpret_cast<const float4 *>(pvt + g);
                        pvv[g] = f.x; pvv[g + 1] = f.y; pvv[g + 2] = f.z; pvv[g + 3] = f.w;
                    }
                } else {
#pragma unroll
                    for (int g = 0; g < GMAX; g++) pvv[g] = pvt[g];
                }
#pragma unroll
                for (int w = 0; w < CPL / 4; w++) {
                    const uint32_t word = *reinterpret_cast<const uint32_t *>(vrow + 4 * w);
                    float f[4];
                    s8x4_to_f32(word, f[0], f[1], f[2], f[3]);
#pragma unroll
                    for (int g = 0; g < GMAX; g++)
#pragma unroll
                        for (int c = 0; c < 4; c++) acc[g][4 * w + c] = fmaf(pvv[g], f[c], acc[g][4 * w + c]);
                }
            }
        }
        __syncthreads();
    }

    // ---- epilogue: reduce the token subsets, then finish or hand off the split
#pragma unroll
    for (int o = LPT; o < 32; o <<= 1)
#pragma unroll
        for (int g = 0; g < GMAX; g++)
#pragma unroll
            for (int c = 0; c < CPL; c++) acc[g][c] += __shfl_xor_sync(0xffffffffu, acc[g][c], o);
    float *red = reinterpret_cast<float *>(smem);  // stage ring is idle now
    if (sub_t == 0) {
#pragma unroll
        for (int g = 0; g < GMAX; g++)
#pragma unroll
            for (int c = 0; c < CPL; c++) red[(warp * GMAX + g) * HD + c0 + c] = acc[g][c];
    }
    __syncthreads();
    auto acc_of = [&](int g, int c) {
        float a = 0.0f;
#pragma unroll
        for (int w = 0; w < DEC_WARPS; w++) a += red[(w * GMAX + g) * HD + c];
        return a;
    };
    finish_split<HD, GMAX, DEC_THREADS, 0>(p, tid, item, pair, s, n_splits, qh0, G, out_item, acc_of, m_s, l_s,
                                          red + DEC_WARPS * GMAX * HD, flag);
}

}  // namespace tqk

#include "tqk_decode_mma.cuh"
#include "tqk_decode_pack.cuh"

namespace tqk {

// Cross-part log-sum-exp merge (tqk_merge_partials): one CTA per head.
__global__ void merge_partials_kernel(const float *__restrict__ parts, int n_parts, long long part_stride,
                                      int head_dim, float *__restrict__ out) {
    const int h = blockIdx.x;
    const int stride = head_dim + 2;
    __shared__ float s_m, s_l;
    if (threadIdx.x < 32) {
        float M = -INFINITY;
        for (int pi = threadIdx.x; pi < n_parts; pi += 32) M = fmaxf(M, parts[pi * part_stride + (long long)h * stride + head_dim]);
        M = warp_max(M);
        float Lsum = 0.0f;
        for (int pi = threadIdx.x; pi < n_parts; pi += 32) {
            const float *pp = parts + pi * part_stride + (long long)h * stride;
            if (pp[head_dim + 1] > 0.0f) Lsum += pp[head_dim + 1] * expf(pp[head_dim] - M);
        }
        Lsum = warp_sum(Lsum);
        if (threadIdx.x == 0) { s_m = M; s_l = Lsum; }
    }
    __syncthreads();
    const float M = s_m, Lsum = s_l;
    for (int c = threadIdx.x; c < head_dim; c += blockDim.x) {
        float a = 0.0f;
        for (int pi = 0; pi < n_parts; pi++) {
            const float *pp = parts + pi * part_stride + (long long)h * stride;
            if (pp[head_dim + 1] > 0.0f) a = fmaf(expf(pp[head_dim] - M), pp[c], a);
        }
        out[(long long)h * head_dim + c] = Lsum > 0.0f ? a / Lsum : 0.0f;
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

int gmax_for(int group) { return group <= 1 ? 1 : group <= 2 ? 2 : group <= 4 ? 4 : 8; }

// Tensor-core kernel (head_dim 128 / 256): up to 16 q heads per CTA.
template <int NB, int GPAD>
int launch_mma(const DecodeParams &p, dim3 grid, cudaStream_t stream, int *ctas_per_sm) {
    using L = MmaLayout<NB, GPAD>;
    static std::mutex mu;
    static int occ_by_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return fail_cuda(e, "decode: cudaGetDevice");
    int occ = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (occ_by_dev[dev] == 0) {
            e = cudaFuncSetAttribute(decode_q8_mma_kernel<NB, GPAD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     L::BYTES);
            int o = 0;
            if (e == cudaSuccess)
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, decode_q8_mma_kernel<NB, GPAD>, MMA_THREADS,
                                                                  L::BYTES);
            if (e != cudaSuccess) return fail_cuda(e, "decode_q8_mma_kernel attributes");
            occ_by_dev[dev] = o > 0 ? o : -1;
        }
        occ = occ_by_dev[dev] > 0 ? occ_by_dev[dev] : 0;
    }
    if (ctas_per_sm) {
        *ctas_per_sm = occ;
        return TQK_OK;
    }
    return launch_pdl(decode_q8_mma_kernel<NB, GPAD>, grid, dim3(MMA_THREADS), L::BYTES, stream, p);
}

// Two-kv-heads-per-CTA kernel for 4 q heads per kv head.
// How many clusters of cx CTAs of `kernel` the device `dev` holds at once (cached per device and
// cluster size; sizes above 8 are opted in as non-portable); 0 when it holds none, or with
// TQK_DECODE_CLUSTER=0 in the environment.
template <typename K>
int max_active_clusters(K kernel, int dev, unsigned cx, int threads, int smem) {
    static std::mutex mu;
    static int count_by[64][CL_MAX + 1];  // 0 = unknown, -1 = none, n = n clusters
    static const bool enabled = [] {
        const char *e = getenv("TQK_DECODE_CLUSTER");
        return !(e && e[0] == '0');
    }();
    if (!enabled || dev < 0 || dev >= 64 || cx > (unsigned)CL_MAX) return 0;
    std::lock_guard<std::mutex> lock(mu);
    int &count = count_by[dev][cx];
    if (count == 0) {
        cudaError_t e = cudaSuccess;
        if (cx > 8) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        int n = 0;
        if (e == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(cx, 1, 1);
            cfg.blockDim = dim3(threads);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = cx;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
        }
        if (e != cudaSuccess) (void)cudaGetLastError();  // not an error of the call: no clusters
        count = (e == cudaSuccess && n > 0) ? n : -1;
    }
    return count > 0 ? count : 0;
}

template <int NB>
int launch_pack(const DecodeParams &p, dim3 grid, cudaStream_t stream, int *ctas_per_sm) {
    using L = PackLayout<NB>;
    static std::mutex mu;
    static int occ_by_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return fail_cuda(e, "decode: cudaGetDevice");
    int occ = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (occ_by_dev[dev] == 0) {
            e = cudaFuncSetAttribute(decode_q8_pack_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
            int o = 0;
            if (e == cudaSuccess)
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, decode_q8_pack_kernel<NB>, PK_THREADS, L::BYTES);
            if (e != cudaSuccess) return fail_cuda(e, "decode_q8_pack_kernel attributes");
            occ_by_dev[dev] = o > 0 ? o : -1;
        }
        occ = occ_by_dev[dev] > 0 ? occ_by_dev[dev] : 0;
    }
    if (ctas_per_sm) {
        *ctas_per_sm = occ;
        return TQK_OK;
    }
    // the splits of a unit (grid.x of them) merge through a thread-block cluster when they fit one,
    // every item has the same length (with ragged lengths the idle splits of short items would stay
    // resident until their cluster's merge), and the device holds every cluster of the grid at once:
    // a cluster is placed whole within one GPC, so a grid of more clusters than fit runs in two
    // waves (measured on B200: 16 clusters of 16 CTAs took 29 us where the ticket merge took 19 us).
    // TQK_DECODE_CLUSTER=0 in the environment turns it off
    const bool equal_lengths = p.lens == nullptr && p.len_step == 0;
    if (equal_lengths && grid.x >= 2 && grid.x <= (unsigned)CL_MAX &&
        (long long)grid.y * grid.z <=
            max_active_clusters(decode_q8_pack_kernel<NB>, dev, grid.x, PK_THREADS, L::BYTES)) {
        DecodeParams pc = p;
        pc.cluster = (int)grid.x;
        return launch_pdl_cluster(decode_q8_pack_kernel<NB>, grid, dim3(PK_THREADS), L::BYTES, stream, grid.x, pc);
    }
    return launch_pdl(decode_q8_pack_kernel<NB>, grid, dim3(PK_THREADS), L::BYTES, stream, p);
}

// The balanced (stream-K) schedule of the same kernel: a 1-D grid of equal tile runs.
template <int NB>
int launch_pack_bal(const DecodeParams &p, dim3 grid, cudaStream_t stream, int *ctas_per_sm) {
    using L = PackBalLayout<NB>;
    static std::mutex mu;
    static int occ_by_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return fail_cuda(e, "decode: cudaGetDevice");
    int occ = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (occ_by_dev[dev] == 0) {
            e = cudaFuncSetAttribute(decode_q8_pack_bal_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     L::BYTES);
            int o = 0;
            if (e == cudaSuccess)
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, decode_q8_pack_bal_kernel<NB>, PK_THREADS,
                                                                  L::BYTES);
            if (e != cudaSuccess) return fail_cuda(e, "decode_q8_pack_bal_kernel attributes");
            occ_by_dev[dev] = o > 0 ? o : -1;
        }
        occ = occ_by_dev[dev] > 0 ? occ_by_dev[dev] : 0;
    }
    if (ctas_per_sm) {
        *ctas_per_sm = occ;
        return TQK_OK;
    }
    return launch_pdl(decode_q8_pack_bal_kernel<NB>, grid, dim3(PK_THREADS), L::BYTES, stream, p);
}

int dispatch_pack(int nb, const DecodeParams &p, dim3 grid, cudaStream_t stream, int *occ, bool balanced = false) {
    if (nb == 4) return balanced ? launch_pack_bal<4>(p, grid, stream, occ) : launch_pack<4>(p, grid, stream, occ);
    return fail(TQK_EUNSUPPORTED, "decode: packed kernel needs head_dim 128");
}

int dispatch_mma(int nb, int gpad, const DecodeParams &p, dim3 grid, cudaStream_t stream, int *occ) {
    if (nb == 4) return gpad > 8 ? launch_mma<4, 16>(p, grid, stream, occ) : launch_mma<4, 8>(p, grid, stream, occ);
    if (nb == 8) return gpad > 8 ? launch_mma<8, 16>(p, grid, stream, occ) : launch_mma<8, 8>(p, grid, stream, occ);
    return fail(TQK_EUNSUPPORTED, "decode: tensor-core kernel needs head_dim 128 or 256");
}

template <int NB, int GMAX>
int launch_decode(const DecodeParams &p, dim3 grid, cudaStream_t stream, int *ctas_per_sm) {
    using L = DecLayout<NB, GMAX>;
    // the dynamic shared-memory opt-in is a per-device function attribute
    static std::mutex mu;
    static int occ_by_dev[64];  // 0 = not yet set up on that device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return fail_cuda(e, "decode: cudaGetDevice");
    int occ = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (occ_by_dev[dev] == 0) {
            e = cudaFuncSetAttribute(decode_q8_kernel<NB, GMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
            int o = 0;
            if (e == cudaSuccess)
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, decode_q8_kernel<NB, GMAX>, DEC_THREADS, L::BYTES);
            if (e != cudaSuccess) return fail_cuda(e, "decode_q8_kernel attributes");
            occ_by_dev[dev] = o > 0 ? o : -1;
        }
        occ = occ_by_dev[dev] > 0 ? occ_by_dev[dev] : 0;
    }
    if (ctas_per_sm) {
        *ctas_per_sm = occ;
        return TQK_OK;
    }
    return launch_pdl(decode_q8_kernel<NB, GMAX>, grid, dim3(DEC_THREADS), L::BYTES, stream, p);
}

template <int NB>
int dispatch_gmax(int gmax, const DecodeParams &p, dim3 grid, cudaStream_t stream, int *occ) {
    switch (gmax) {
        case 1: return launch_decode<NB, 1>(p, grid, stream, occ);
        case 2: return launch_decode<NB, 2>(p, grid, stream, occ);
        case 4: return launch_decode<NB, 4>(p, grid, stream, occ);
        default: return launch_decode<NB, 8>(p, grid, stream, occ);
    }
}

// CUDA-core kernel: head_dim 32 and 64 (128 and 256 go to the tensor-core kernels).
int dispatch(int nb, int gmax, const DecodeParams &p, dim3 grid, cudaStream_t stream, int *occ) {
    switch (nb) {
        case 1: return dispatch_gmax<1>(gmax, p, grid, stream, occ);
        case 2: return dispatch_gmax<2>(gmax, p, grid, stream, occ);
        default: return fail(TQK_EUNSUPPORTED, "decode: the CUDA-core kernel takes head_dim 32 or 64");
    }
}

struct Plan {
    int nb, gmax, heads_per_cta, head_slices, pairs, split_tokens, max_splits, max_len;
    bool mma;   // tensor-core kernel (head_dim 128/256) or the CUDA-core one (32/64)
    bool pack;  // tensor-core kernel with two kv heads per CTA (4 q heads per kv head)
    bool balanced;          // packed kernel on the balanced schedule: bal_ctas equal tile runs
    int bal_ctas, tickets_per_unit;
    size_t counters_bytes, part_bytes;
};

// Tickets of the split merge: TICKETS_PER_UNIT ints per (item, head unit), at
// the start of a caller workspace, followed by the partials.  Every completed
// call leaves its tickets at zero but writes partials right after them, so the
// region has a fixed floor (16384 units' worth): calls of up to 16384 units
// all use the same ticket bytes and can share a workspace without
// re-initialisation.
constexpr int TICKET_FLOOR_UNITS = 16384;
size_t counters_region(int n_items, int units) {
    const size_t n = (size_t)n_items * units;
    const size_t b = ((n < TICKET_FLOOR_UNITS ? TICKET_FLOOR_UNITS : n) * TICKETS_PER_UNIT * sizeof(int) + 255) / 256 * 256;
    return b;
}

// K/V bytes a call streams with every item at max_len.
long long kv_bytes_of(const tqk_decode_args *a, int max_len) {
    return 2LL * a->n_items * a->n_kv_heads * max_len * (a->head_dim / QK) * BLOCK_BYTES;
}

// Splits per (item, head unit) of the automatic fixed split.  Measured on B200:
//  * equal lengths: as many as keep every CTA in one wave of the resident slots
//    (a second, partly filled wave costs more than the shorter splits save:
//    76 us in one wave against 101 us in 1.15 waves); but a call that streams
//    less than LATENCY_BYTES is bound by its fixed costs, not by bandwidth, and
//    then at most MERGE_GROUP splits (one merge level) win: a Llama-3-8B layer
//    at n = 4097 took 16.4 us with 13 splits against 17.6 us with 64;
//  * unequal lengths (device lengths unknown to the host): about 0.9 waves if
//    the lengths spread evenly up to max_len -- each unit then takes about
//    want / 2 + 1/2 splits, the half for its last, partial split -- and one
//    merge level: ragged config-3 shares of 8 and 16 sequences took 24.6 and
//    40.5 us with splits near that choice against 35.2 and 51.5 us with two
//    CTAs per slot (1.1 waves, two levels).
constexpr long long LATENCY_BYTES = 16LL << 20;
long long auto_splits(bool uniform, long long slots, long long units, long long kv_bytes) {
    long long want = uniform ? slots / units : (9 * slots - 5 * units) / (5 * units);
    if ((!uniform || kv_bytes < LATENCY_BYTES) && want > MERGE_GROUP) want = MERGE_GROUP;
    return want < 1 ? 1 : want;
}

int make_plan(const tqk_decode_args *a, Plan *pl, bool gather = false) {
    if (!a) return fail(TQK_EINVAL, "decode: NULL args");
    if (a->n_items <= 0 || a->n_q_heads <= 0 || a->n_kv_heads <= 0 || a->head_dim <= 0 || a->max_tokens <= 0)
        return fail(TQK_EINVAL, "decode: non-positive shape");
    if (a->n_q_heads % a->n_kv_heads) return fail(TQK_EINVAL, "decode: n_q_heads % n_kv_heads != 0");
    if (a->head_dim % QK) return fail(TQK_EINVAL, "decode: head_dim % 32 != 0");
    const int nb = a->head_dim / QK;
    if (nb != 1 && nb != 2 && nb != 4 && nb != 8) return fail(TQK_EUNSUPPORTED, "decode: head_dim must be 32, 64, 128 or 256");
    if (!a->k || !a->v || !a->q || !a->out) return fail(TQK_EINVAL, "decode: NULL pointer");
    if ((a->k_new == nullptr) != (a->v_new == nullptr)) return fail(TQK_EINVAL, "decode: k_new and v_new go together");
    if (a->out_mode != TQK_OUT_NORMALIZED && a->out_mode != TQK_OUT_PARTIAL) return fail(TQK_EINVAL, "decode: out_mode");
    if ((a->q_norm == nullptr) != (a->k_norm == nullptr)) return fail(TQK_EINVAL, "decode: q_norm and k_norm go together");
    if ((a->rope_cos == nullptr) != (a->rope_sin == nullptr))
        return fail(TQK_EINVAL, "decode: rope_cos and rope_sin go together");
    if (a->n_items > 65535) return fail(TQK_EINVAL, "decode: n_items > 65535");
    int max_len;
    if (a->lens) {
        max_len = a->max_len;
        if (max_len < 0 || max_len > a->max_tokens) return fail(TQK_EINVAL, "decode: max_len outside [0, max_tokens]");
    } else {
        const long long first = a->len0, last = a->len0 + (long long)(a->n_items - 1) * a->len_step;
        const long long lo = first < last ? first : last, hi = first < last ? last : first;
        if (lo < 0 || hi > a->max_tokens) return fail(TQK_EPOS, "decode: length outside [0, max_tokens]");
        if (a->k_new && lo < 1) return fail(TQK_EPOS, "decode: append needs length >= 1");
        max_len = (int)hi;
    }
    if (nb % 4 == 0) {
        if ((reinterpret_cast<uintptr_t>(a->k) & 15) || (reinterpret_cast<uintptr_t>(a->v) & 15) ||
            ((a->item_stride * BLOCK_BYTES) & 15))
            return fail(TQK_EALIGN, "decode: planes and item stride must be 16-byte aligned");
    } else if ((reinterpret_cast<uintptr_t>(a->k) & 3) || (reinterpret_cast<uintptr_t>(a->v) & 3)) {
        return fail(TQK_EALIGN, "decode: planes must be 4-byte aligned");
    }
    const int group = a->n_q_heads / a->n_kv_heads;
    pl->nb = nb;
    pl->mma = nb % 4 == 0;
    pl->pack = nb == 4 && group == 4 && a->n_kv_heads % 2 == 0;  // head_dim 128 only (register budget)
    pl->gmax = pl->pack ? 8 : pl->mma ? (group <= 8 ? 8 : 16) : gmax_for(group);
    pl->heads_per_cta = pl->pack ? 8 : (group < pl->gmax ? group : pl->gmax);
    pl->head_slices = pl->pack ? 1 : (group + pl->heads_per_cta - 1) / pl->heads_per_cta;
    pl->pairs = pl->pack ? a->n_kv_heads / 2 : a->n_kv_heads * pl->head_slices;
    pl->max_len = max_len;

    int split = a->split_tokens;
    pl->balanced = false;
    pl->bal_ctas = 0;
    pl->tickets_per_unit = TICKETS_PER_UNIT;
    if (split <= 0) {
        const int rc = ensure_device();
        if (rc) return rc;
        const DeviceInfo *d = device_info();
        // the balanced schedule pays a segment switch mid-run (about 7 us of a
        // CTA's time); it wins where the fixed split cannot even out the work --
        // unequal lengths across items -- and every CTA's run is long enough to
        // absorb its switches: at least BAL_MIN_TILES tiles per resident slot,
        // counted with every unit at max_len (the host does not see device
        // lengths).  TQK_SPLIT_BALANCED asks for it whenever the call qualifies.
        const bool ragged = a->n_items > 1 && (a->lens != nullptr || a->len_step != 0);
        const bool can_balance = !gather && pl->pack && a->n_items <= BAL_MAX_ITEMS;
        const long long pairs_total = (long long)a->n_items * pl->pairs;
        bool balanced = can_balance && (split == TQK_SPLIT_BALANCED || ragged);
        int occ = 0;
        DecodeParams dummy{};
        int orc = pl->pack  ? dispatch_pack(nb, dummy, dim3(1), nullptr, &occ, balanced)
                  : pl->mma ? dispatch_mma(nb, pl->gmax, dummy, dim3(1), nullptr, &occ)
                            : dispatch(nb, pl->gmax, dummy, dim3(1), nullptr, &occ);
        if (orc) return orc;
        long long slots = (long long)(d ? d->sm_count : 148) * (occ > 0 ? occ : 1);
        if (balanced && split != TQK_SPLIT_BALANCED &&
            pairs_total * ((max_len + PK_T - 1) / PK_T) < (long long)BAL_MIN_TILES * slots) {
            balanced = false;
            orc = dispatch_pack(nb, dummy, dim3(1), nullptr, &occ, false);
            if (orc) return orc;
            slots = (long long)(d ? d->sm_count : 148) * (occ > 0 ? occ : 1);
        }
        if (balanced) {
            // one CTA per resident slot (never more than there are tiles), each
            // streaming an equal run of the units' tiles
            const long long tiles = pairs_total * ((max_len + PK_T - 1) / PK_T);
            long long ctas = slots < tiles ? slots : tiles;
            if (ctas > BAL_MAX_CTAS) ctas = BAL_MAX_CTAS;
            if (ctas < 1) ctas = 1;
            pl->balanced = true;
            pl->bal_ctas = (int)ctas;
            pl->tickets_per_unit = 1 + (int)((ctas + MERGE_GROUP - 1) / MERGE_GROUP);
            pl->split_tokens = 0;
            pl->max_splits = (int)ctas;
            // tickets inside the fixed-floor region (so workspaces stay shareable
            // across calls), then one partial slot per (CTA, unit) segment
            pl->counters_bytes = counters_region(a->n_items, pl->pairs);
            if ((size_t)pairs_total * pl->tickets_per_unit * sizeof(int) > pl->counters_bytes)
                return fail(TQK_EINVAL, "decode: balanced schedule tickets exceed the ticket region");
            pl->part_bytes = (size_t)(ctas + pairs_total) * 8 * (a->head_dim + 2) * sizeof(float);
            return TQK_OK;
        }
        const bool uniform = !a->lens && a->len_step == 0;
        const long long want = auto_splits(uniform, slots, pairs_total, kv_bytes_of(a, max_len));
        split = (int)((max_len + want - 1) / want);
    }
    split = ((split + DEC_T - 1) / DEC_T) * DEC_T;
    if (split < DEC_T) split = DEC_T;
    while (n_splits_of(max_len, split) > MAX_SPLITS) split += DEC_T;
    pl->split_tokens = split;
    pl->max_splits = max_len > 0 ? n_splits_of(max_len, split) : 1;
    if (pl->max_splits > 1) {
        pl->counters_bytes = counters_region(a->n_items, pl->pairs);
        pl->part_bytes = (size_t)a->n_items * pl->pairs * pl->max_splits * pl->gmax * (a->head_dim + 2) * sizeof(float);
    } else {
        pl->counters_bytes = 0;
        pl->part_bytes = 0;
    }
    return TQK_OK;
}

// Kernel parameters of a validated call (everything but the scratch pointers).
DecodeParams fill_params(const tqk_decode_args *a, const Plan &pl) {
    DecodeParams p{};
    p.k = reinterpret_cast<const uint8_t *>(a->k);
    p.v = reinterpret_cast<const uint8_t *>(a->v);
    p.kw = reinterpret_cast<uint8_t *>(a->k);
    p.vw = reinterpret_cast<uint8_t *>(a->v);
    p.item_stride = a->item_stride * BLOCK_BYTES;
    p.n_items = a->n_items;
    p.n_kv = a->n_kv_heads;
    p.group = a->n_q_heads / a->n_kv_heads;
    p.max_tokens = a->max_tokens;
    p.heads_per_cta = pl.heads_per_cta;
    p.head_slices = pl.head_slices;
    p.pairs = pl.pairs;
    p.lens = a->lens;
    p.len0 = a->len0;
    p.len_step = a->len_step;
    p.q = a->q;
    p.q_item_stride = a->q_item_stride;
    p.out = a->out;
    p.out_item_stride = a->out_item_stride;
    p.k_new = a->k_new;
    p.v_new = a->v_new;
    p.kv_new_item_stride = a->kv_new_item_stride;
    p.q_norm = a->q_norm;
    p.k_norm = a->k_norm;
    p.norm_item_stride = a->norm_item_stride;
    p.norm_eps = a->norm_eps;
    p.rope_cos = a->rope_cos;
    p.rope_sin = a->rope_sin;
    p.rope_item_stride = a->rope_item_stride;
    p.out_mode = a->out_mode;
    p.split_tokens = pl.split_tokens;
    p.max_splits = pl.max_splits;
    p.tickets_per_unit = pl.tickets_per_unit;
    p.scale = 1.0f / sqrtf((float)a->head_dim);  // as attend_q8 computes it (attention_layer.c:131)
    return p;
}


}  // namespace
}  // namespace tqk

using namespace tqk;

extern "C" int tqk_decode_workspace_size(const tqk_decode_args *a, size_t *bytes) {
    Plan pl;
    int rc = make_plan(a, &pl);
    if (rc) return rc;
    if (bytes) *bytes = pl.counters_bytes + pl.part_bytes;
    return TQK_OK;
}

namespace tqk {
namespace {

// tqk_decode_q8 and tqk_decode_q8_gather: the plan, the scratch and the launch.
int decode_impl(const tqk_decode_args *a, const tqk_gather_dst *gd, void *workspace, size_t workspace_bytes,
                tqk_stream_t stream) {
    Plan pl;
    int rc = make_plan(a, &pl, gd != nullptr);  // validates before touching the device
    if (rc) return rc;
    rc = ensure_device();
    if (rc) return rc;
    const size_t need = pl.counters_bytes + pl.part_bytes;
    cudaStream_t st = (cudaStream_t)stream;
    int *counters = nullptr;
    float *part = nullptr;
    if (need) {
        if (!workspace) {
            // library-owned: tickets in a buffer of their own, which partials never touch
            counters = library_counters(st, pl.counters_bytes);
            part = reinterpret_cast<float *>(library_workspace(st, pl.part_bytes));
            if (!counters || !part) return fail(TQK_ECUDA, "decode: cannot allocate the library workspace");
        } else if (workspace_bytes < need) {
            return fail(TQK_EWORKSPACE, "decode: workspace smaller than tqk_decode_workspace_size()");
        } else {
            counters = reinterpret_cast<int *>(workspace);
            part = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(workspace) + pl.counters_bytes);
        }
    }
    DecodeParams p = fill_params(a, pl);
    p.counters = counters;
    p.part = part;
    p.err = device_info()->err_word;
    if (gd) {
        p.g_world = gd->world;
        p.g_rank = gd->rank;
        p.g_chunk = gd->chunk_heads;
        p.g_epoch = gd->epoch;
        for (int r = 0; r < gd->world; r++) p.g_out[r] = reinterpret_cast<uint2 *>(gd->out[r]);
    }
    if (pl.balanced) return dispatch_pack(pl.nb, p, dim3((unsigned)pl.bal_ctas), st, nullptr, true);
    const dim3 grid((unsigned)pl.max_splits, (unsigned)pl.pairs, (unsigned)a->n_items);
    if (pl.pack) return dispatch_pack(pl.nb, p, grid, st, nullptr);
    return pl.mma ? dispatch_mma(pl.nb, pl.gmax, p, grid, st, nullptr) : dispatch(pl.nb, pl.gmax, p, grid, st, nullptr);
}

}  // namespace
}  // namespace tqk

extern "C" int tqk_decode_q8(const tqk_decode_args *a, void *workspace, size_t workspace_bytes,
                             tqk_stream_t stream) {
    return decode_impl(a, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int tqk_decode_unit_count(const tqk_decode_args *a, int *units) {
    if (!units) return fail(TQK_EINVAL, "tqk_decode_unit_count: NULL units");
    Plan pl;
    int rc = make_plan(a, &pl, true);
    if (rc) return rc;
    *units = a->n_items * pl.pairs;
    return TQK_OK;
}

extern "C" int tqk_decode_q8_gather(const tqk_decode_args *a, const tqk_gather_dst *g, void *workspace,
                                    size_t workspace_bytes, tqk_stream_t stream) {
    if (!a || !g) return fail(TQK_EINVAL, "tqk_decode_q8_gather: NULL arguments");
    if (g->world < 1 || g->world > 8 || g->rank < 0 || g->rank >= g->world || g->chunk_heads <= 0)
        return fail(TQK_EINVAL, "tqk_decode_q8_gather: bad world, rank or chunk_heads");
    if (a->out_mode != TQK_OUT_NORMALIZED)
        return fail(TQK_EINVAL, "tqk_decode_q8_gather: the gather carries normalised outputs only");
    if (((long long)a->n_items * a->n_q_heads) % g->chunk_heads)
        return fail(TQK_EINVAL, "tqk_decode_q8_gather: n_items * n_q_heads must be a multiple of chunk_heads");
    if (g->epoch < 1) return fail(TQK_EINVAL, "tqk_decode_q8_gather: epochs count from 1");
    for (int r = 0; r < g->world; r++)
        if (!g->out[r] || (reinterpret_cast<uintptr_t>(g->out[r]) & 7))
            return fail(TQK_EALIGN, "tqk_decode_q8_gather: every rank needs an 8-byte aligned output buffer");
    return decode_impl(a, g, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free decode (tqk_decode_q8_static): the split tickets and
// partials live in file-scope device arrays of fixed size, so a call makes no
// device allocation of any kind (no workspace, no library buffers, no error
// word).  Their device addresses are looked up once per device.
// ---------------------------------------------------------------------------
namespace tqk {
namespace {

constexpr int STATIC_TICKETS = 16384;               // (item, head unit) pairs per call
constexpr size_t STATIC_PART_FLOATS = 1u << 20;     // 4 MiB of split partials

static __device__ __align__(256) int g_static_tickets[STATIC_TICKETS * TICKETS_PER_UNIT];
static __device__ __align__(256) float g_static_part[STATIC_PART_FLOATS];

struct StaticScratch {
    bool ready = false;
    int *tickets = nullptr;
    float *part = nullptr;
};

// Device addresses of the static arrays for the current device (set up on the
// first call made with that device current).
int static_scratch(int dev, StaticScratch *out) {
    static std::mutex mu;
    static StaticScratch by_dev[64];
    if (dev < 0 || dev >= 64) return fail(TQK_ENODEV, "tqk_decode_q8_static: device ordinal out of range");
    std::lock_guard<std::mutex> lock(mu);
    StaticScratch &s = by_dev[dev];
    if (!s.ready) {
        void *t = nullptr, *q = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&t, g_static_tickets);
        if (e != cudaSuccess) return fail_cuda(e, "tqk_decode_q8_static: cudaGetSymbolAddress(tickets)");
        e = cudaGetSymbolAddress(&q, g_static_part);
        if (e != cudaSuccess) return fail_cuda(e, "tqk_decode_q8_static: cudaGetSymbolAddress(partials)");
        s.tickets = static_cast<int *>(t);
        s.part = static_cast<float *>(q);
        s.ready = true;
    }
    *out = s;
    return TQK_OK;
}

}  // namespace
}  // namespace tqk

extern "C" int tqk_decode_q8_static(const tqk_decode_args *args, tqk_stream_t stream) {
    if (!args) return fail(TQK_EINVAL, "tqk_decode_q8_static: NULL args");
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda(e, "tqk_decode_q8_static: cudaGetDevice");
    // plan with a provisional split (no device queries), then pick the split
    // the way tqk_decode_q8 does, from the SM count and the kernel's occupancy
    tqk_decode_args a = *args;
    if (a.split_tokens <= 0) a.split_tokens = a.max_tokens > 0 ? a.max_tokens : 1;
    Plan pl;
    int rc = make_plan(&a, &pl);
    if (rc) return rc;
    if (args->split_tokens <= 0) {
        int sms = 0, occ = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return fail_cuda(e, "tqk_decode_q8_static: SM count");
        DecodeParams dummy{};
        rc = pl.pack  ? dispatch_pack(pl.nb, dummy, dim3(1), nullptr, &occ)
             : pl.mma ? dispatch_mma(pl.nb, pl.gmax, dummy, dim3(1), nullptr, &occ)
                      : dispatch(pl.nb, pl.gmax, dummy, dim3(1), nullptr, &occ);
        if (rc) return rc;
        const long long slots = (long long)sms * (occ > 0 ? occ : 1);
        const long long units = (long long)a.n_items * pl.pairs;
        const bool uniform = !a.lens && a.len_step == 0;
        const long long want = auto_splits(uniform, slots, units, kv_bytes_of(&a, pl.max_len));
        a.split_tokens = (int)((pl.max_len + want - 1) / want);
        if (a.split_tokens < 1) a.split_tokens = 1;
        rc = make_plan(&a, &pl);
        if (rc) return rc;
    }
    const long long units = (long long)a.n_items * pl.pairs;
    if (pl.max_splits > 1) {
        if (units > STATIC_TICKETS)
            return fail(TQK_EWORKSPACE, "tqk_decode_q8_static: more than 16384 (item, head unit) pairs to split; "
                                        "use tqk_decode_q8 with a workspace");
        if (pl.part_bytes > STATIC_PART_FLOATS * sizeof(float))
            return fail(TQK_EWORKSPACE, "tqk_decode_q8_static: split partials exceed the 4 MiB static scratch; "
                                        "use tqk_decode_q8 with a workspace or a larger split_tokens");
    }
    StaticScratch sc;
    rc = static_scratch(dev, &sc);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (pl.max_splits > 1) {
        // the tickets must start at zero: clear this call's range on the stream
        e = cudaMemsetAsync(sc.tickets, 0, (size_t)units * TICKETS_PER_UNIT * sizeof(int), st);
        if (e != cudaSuccess) return fail_cuda(e, "tqk_decode_q8_static: clearing the tickets");
    }
    DecodeParams p = fill_params(&a, pl);
    p.counters = pl.max_splits > 1 ? sc.tickets : nullptr;
    p.part = pl.max_splits > 1 ? sc.part : nullptr;
    p.err = nullptr;  // no device error word: device-side checks still clamp or stop safely
    const dim3 grid((unsigned)pl.max_splits, (unsigned)pl.pairs, (unsigned)a.n_items);
    if (pl.pack) return dispatch_pack(pl.nb, p, grid, st, nullptr);
    return pl.mma ? dispatch_mma(pl.nb, pl.gmax, p, grid, st, nullptr) : dispatch(pl.nb, pl.gmax, p, grid, st, nullptr);
}

extern "C" int tqk_attend_q8(const tqk_block_q8 *k_plane, const tqk_block_q8 *v_plane, int n_q_heads,
                             int n_kv_heads, int head_dim, int max_tokens, int pos, const float *q, float *out,
                             tqk_stream_t stream) {
    if (pos < 0 || pos >= max_tokens) return fail(TQK_EPOS, "tqk_attend_q8: position out of range");
    tqk_decode_args a{};
    a.k = const_cast<tqk_block_q8 *>(k_plane);
    a.v = const_cast<tqk_block_q8 *>(v_plane);
    a.n_items = 1;
    a.n_q_heads = n_q_heads;
    a.n_kv_heads = n_kv_heads;
    a.head_dim = head_dim;
    a.max_tokens = max_tokens;
    a.len0 = pos + 1;
    a.q = q;
    a.out = out;
    return tqk_decode_q8(&a, nullptr, 0, stream);
}

extern "C" int tqk_append_attend_q8(tqk_block_q8 *k_plane, tqk_block_q8 *v_plane, int n_q_heads, int n_kv_heads,
                                    int head_dim, int max_tokens, int pos, const float *q, const float *k,
                                    const float *v, float *out, tqk_stream_t stream) {
    if (pos < 0 || pos >= max_tokens) return fail(TQK_EPOS, "tqk_append_attend_q8: position out of range");
    if (!k || !v) return fail(TQK_EINVAL, "tqk_append_attend_q8: NULL k/v");
    tqk_decode_args a{};
    a.k = k_plane;
    a.v = v_plane;
    a.n_items = 1;
    a.n_q_heads = n_q_heads;
    a.n_kv_heads = n_kv_heads;
    a.head_dim = head_dim;
    a.max_tokens = max_tokens;
    a.len0 = pos + 1;
    a.q = q;
    a.out = out;
    a.k_new = k;
    a.v_new = v;
    return tqk_decode_q8(&a, nullptr, 0, stream);
}

extern "C" int tqk_prefill_q8(tqk_block_q8 *k_plane, tqk_block_q8 *v_plane, int n_q_heads, int n_kv_heads,
                              int head_dim, int max_tokens, int pos0, int n, const float *q, const float *k,
                              const float *v, float *out, tqk_stream_t stream) {
    if (n <= 0) return fail(TQK_EINVAL, "tqk_prefill_q8: n must be positive");
    if (pos0 < 0 || (long long)pos0 + n > max_tokens) return fail(TQK_EPOS, "tqk_prefill_q8: range out of cache");
    int rc = tqk_store_kv_q8_batch(k_plane, v_plane, n_kv_heads, head_dim, max_tokens, pos0, n, k, v, stream);
    if (rc) return rc;
    // tensor-core path (head_dim 128, 1/2/4/8 q heads per kv head); other shapes use the decode kernel
    rc = prefill_attend_tc(k_plane, v_plane, n_q_heads, n_kv_heads, head_dim, max_tokens, pos0, n, q, out,
                           (cudaStream_t)stream);
    if (rc != TQK_EUNSUPPORTED) return rc;
    tqk_decode_args a{};
    a.k = k_plane;
    a.v = v_plane;
    a.item_stride = 0;
    a.n_items = n;
    a.n_q_heads = n_q_heads;
    a.n_kv_heads = n_kv_heads;
    a.head_dim = head_dim;
    a.max_tokens = max_tokens;
    a.len0 = pos0 + 1;
    a.len_step = 1;
    a.q = q;
    a.q_item_stride = (int64_t)n_q_heads * head_dim;
    a.out = out;
    a.out_item_stride = (int64_t)n_q_heads * head_dim;
    return tqk_decode_q8(&a, nullptr, 0, stream);
}

extern "C" int tqk_merge_partials(const float *parts, int n_parts, int64_t part_stride, int n_heads, int head_dim,
                                  float *out, tqk_stream_t stream) {
    if (!parts || !out || n_parts <= 0 || n_heads <= 0 || head_dim <= 0)
        return fail(TQK_EINVAL, "tqk_merge_partials: bad arguments");
    int rc = ensure_device();
    if (rc) return rc;
    merge_partials_kernel<<<n_heads, 128, 0, (cudaStream_t)stream>>>(parts, n_parts, part_stride, head_dim, out);
    return check_launch("merge_partials_kernel");
}
