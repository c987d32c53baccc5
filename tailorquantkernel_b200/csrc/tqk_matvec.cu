// tqk_matvec.cu -- the projections around the attention: Q8 / Q4 weight rows
// times Q8-quantised activations (MatmulFn / MatmulBatchFn of reference
// kernel/kernel.h:17-24, kernel/q8_scalar.c:3-29, kernel/q4_scalar.c:3-31),
// optionally with the activation quantisation of project_qkv / project_output
// (model/attention_layer.c:38-46, 161-167) fused in.
//
// Bit-exact with the reference's scalar kernels: every output adds, in block
// order, (float)(int dot) * w.d * x.d rounded left to right.  That sum is one
// serial chain per (row, token); the kernel keeps many chains in flight
// instead of reordering it.
//
// Work layout: every warp is its own pipeline.  It owns groups of R
// consecutive rows of one matrix (group g = its global warp index + k * all
// warps), fetches a group with one TMA bulk copy into a two-slot ring of its
// own (plain lane copies when the rows are not whole 16-byte units), and per
// group lanes take 4-block chunks of each row (chunk c on lane c % 32: nine
// conflict-free 16-byte loads for a Q8 chunk, five for Q4) and write every
// (row, token, block) term into the warp's scratch.  After MB groups (or the
// last one) lanes 0 .. MB*R*n_tok - 1 each walk one (row, token) chain over the
// scratch with 16-byte loads and write y.
// The kernel is launched with programmatic stream serialization: before
// griddepcontrol.wait it only issues weight copies (weights are never written
// by kernels), so in a chain of launches its weight prefetch overlaps the
// previous kernel.  Weights must not be modified by kernels on the stream
// while a call that reads them may be in flight.
// The activations sit in shared memory for the whole CTA, per token in
// chunks of four blocks (128 bytes of int8 + 16 bytes of padding, so that the
// lanes' chunk loads hit distinct banks), with the scales and (Q4) int8 sums
// per chunk in 16-byte groups; with one token and one chunk per lane the
// lane's chunk stays in registers for every row.
#include "tqk_internal.h"

#include <mutex>

namespace tqk {
namespace {

constexpr int MV_MAX_JOBS = 4;
constexpr int MV_MAX_TOK = 8;        // tokens per launch; more are looped on the host
// Warps per CTA.  Four (about 80 KB of shared memory at hidden 4096, two CTAs per SM) rather than
// eight (one CTA per SM): a projection's CTAs can then start on SMs that still hold the decode's
// CTAs, whose tail they overlap.  Measured on B200: 32 attention layers per token 1024.5 -> 979.5 us,
// a whole Llama-3-8B token unchanged (2944 / 2947 us); 1-row or 4-row groups were slower.
#ifndef TQK_MV_WARPS
#define TQK_MV_WARPS 4
#endif
#ifndef TQK_MV_GROUP_BYTES
#define TQK_MV_GROUP_BYTES 9216
#endif
#ifndef TQK_MV_CHAINS
#define TQK_MV_CHAINS 8
#endif
constexpr int MV_MAX_WARPS = TQK_MV_WARPS;
constexpr int MV_GROUP_BYTES = TQK_MV_GROUP_BYTES;  // target bytes of one row group (one ring slot)
constexpr int MV_CHAINS = TQK_MV_CHAINS;            // target (row, token) chains per walk
constexpr int MV_SMEM_LIMIT = 227 * 1024;
constexpr uint64_t MV_WAIT_NS = 1000000000ull;  // 1 s bound on a ring wait
constexpr uint64_t MV_DRAIN_NS = 20000000ull;   // 20 ms when draining after a timeout

struct MvJob {
    const uint8_t *w;  // rows of Q8 / Q4 blocks
    float *y;          // [n_tok][rows]
    int rows;
    int group0;        // first global group of this job
};

struct MvParams {
    MvJob job[MV_MAX_JOBS];
    int n_jobs, n_groups;
    int nb, n_tok, R;        // blocks per row, tokens, rows per group
    int row_bytes;
    int sp;                  // floats per scratch chain row
    int mb;                  // groups per chain walk
    int tma;                 // groups start on 16-byte boundaries and span whole 16-byte units
    const float *x;          // fp32 activations [n_tok][nb*32], or NULL
    const uint8_t *xq;       // Q8 activations [n_tok][nb] (when x is NULL)
    int *err;
};

// Shared-memory carve-up, computed identically on host and device.
struct MvLayout {
    int nch, x_w, x_d, x_s, warp0, warp_bytes, slot_bytes, scr_off, bytes;
    __host__ __device__ MvLayout(int nb, int n_tok, int R, int row_bytes, int sp, int mb, int warps) {
        nch = (nb + 3) / 4;                       // chunks of 4 blocks per token
        const int nc = n_tok * nch;
        x_w = 0;                                  // uint32 [n_tok][nch][36]: 4 blocks x 8 words + pad
        x_d = x_w + nc * 144;                     // float  [n_tok][nch][4]
        x_s = x_d + nc * 16;                      // int    [n_tok][nch][4] (Q4: sum of the block's int8)
        warp0 = x_s + nc * 16;
        slot_bytes = ((R * row_bytes + 15) / 16) * 16;
        scr_off = 16 + 2 * slot_bytes;            // after 2 mbarriers and 2 slots
        warp_bytes = scr_off + mb * R * n_tok * sp * 4;
        bytes = warp0 + warps * warp_bytes;
    }
};

// Word offset of block b of token t in the activation words.
__device__ __forceinline__ int xw_off(int t, int b, int nch) { return (t * nch + (b >> 2)) * 36 + (b & 3) * 8; }

// Two independent dp4a chains per block (integer sums: exact in any order).
__device__ __forceinline__ int dot_q8_block(const uint32_t (&w)[8], uint4 x0, uint4 x1) {
    int s = dp4a(w[0], x0.x, 0), u = dp4a(w[4], x1.x, 0);
    s = dp4a(w[1], x0.y, s);
    u = dp4a(w[5], x1.y, u);
    s = dp4a(w[2], x0.z, s);
    u = dp4a(w[6], x1.z, u);
    s = dp4a(w[3], x0.w, s);
    u = dp4a(w[7], x1.w, u);
    return s + u;
}

// sum_j (lo_j - 8) * x_j + (hi_j - 8) * x_{j+16}: the nibbles 0..15 are valid
// signed bytes, so signed dp4a on the masked words, minus 8 * sum(x).
__device__ __forceinline__ int dot_q4_block(const uint32_t (&w)[4], uint4 x0, uint4 x1, int xsum) {
    int s = dp4a(w[0] & 0x0F0F0F0Fu, x0.x, 0), u = dp4a((w[0] >> 4) & 0x0F0F0F0Fu, x1.x, 0);
    s = dp4a(w[1] & 0x0F0F0F0Fu, x0.y, s);
    u = dp4a((w[1] >> 4) & 0x0F0F0F0Fu, x1.y, u);
    s = dp4a(w[2] & 0x0F0F0F0Fu, x0.z, s);
    u = dp4a((w[2] >> 4) & 0x0F0F0F0Fu, x1.z, u);
    s = dp4a(w[3] & 0x0F0F0F0Fu, x0.w, s);
    u = dp4a((w[3] >> 4) & 0x0F0F0F0Fu, x1.w, u);
    return s + u - 8 * xsum;
}

template <int FMT>
__global__ void __launch_bounds__(MV_MAX_WARPS * 32, 1) matvec_kernel(const MvParams p) {
    constexpr int BB = FMT == TQK_FMT_Q8 ? 36 : 20;  // bytes per weight block
    constexpr int NW = FMT == TQK_FMT_Q8 ? 8 : 4;    // int8 / nibble words per block
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int nb = p.nb, T = p.n_tok, R = p.R, sp = p.sp;
    const int mb = p.mb;
    const MvLayout L(nb, T, R, p.row_bytes, sp, mb, nwarps);
    const int nch = L.nch;
    uint32_t *xw = reinterpret_cast<uint32_t *>(smem + L.x_w);
    float *xd = reinterpret_cast<float *>(smem + L.x_d);
    int *xs = reinterpret_cast<int *>(smem + L.x_s);

    // this warp's ring; its first copy goes out before the activations are staged
    uint8_t *wbase = smem + L.warp0 + warp * L.warp_bytes;
    uint64_t *bar = reinterpret_cast<uint64_t *>(wbase);
    uint8_t *slots = wbase + 16;  // slot s at slots + s * L.slot_bytes
    float *scr = reinterpret_cast<float *>(wbase + L.scr_off);
    const int gw = blockIdx.x * nwarps + warp, TW = gridDim.x * nwarps;
    const bool active = gw < p.n_groups;
    if (active && p.tma) {
        if (lane == 0) {
            mbar_init(&bar[0], 1);
            mbar_init(&bar[1], 1);
            fence_barrier_init();
        }
        __syncwarp();
    }

    // group g -> its job (selected without a dynamically indexed parameter
    // array), first row and row count
    auto locate = [&](int g, MvJob &job, int &r0, int &rows) {
        job = p.job[0];
#pragma unroll
        for (int k = 1; k < MV_MAX_JOBS; k++)
            if (k < p.n_jobs && g >= p.job[k].group0) job = p.job[k];
        r0 = (g - job.group0) * R;
        rows = min(R, job.rows - r0);
    };
    unsigned pending = 0;  // bit s: a copy into slot s is in flight
    auto fetch = [&](int g, int slot) {
        MvJob job;
        int r0, rows;
        locate(g, job, r0, rows);
        const uint8_t *src = job.w + (long long)r0 * p.row_bytes;
        const uint32_t bytes = (uint32_t)(rows * p.row_bytes);
        if (p.tma) {
            if (lane == 0) {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&bar[slot], bytes);
                bulk_copy_g2s(slots + slot * L.slot_bytes, src, bytes, &bar[slot]);
            }
            pending |= 1u << slot;
        } else {
            uint32_t *dst = reinterpret_cast<uint32_t *>(slots + slot * L.slot_bytes);
            const uint32_t *s32 = reinterpret_cast<const uint32_t *>(src);
            for (uint32_t i = lane; i < bytes / 4; i += 32) dst[i] = __ldg(s32 + i);
        }
    };
    if (active && p.tma) fetch(gw, 0);
    // programmatic dependent launch: the weights (which no kernel writes) are
    // already in flight; the activations below may come from earlier kernels,
    // so they are read only after those completed.  Then the next kernel may
    // start its own weight prefetch.
    grid_dependency_wait();
    grid_dependents_launch();

    // the activations, quantised here when fp32 x is given: one thread per
    // 32-float block (quant_x.c:12-34), all blocks at once
    const int nx = T * nb;
    for (int i = threadIdx.x; i < nx; i += blockDim.x) {
        const int t = i / nb, b = i - t * nb;
        uint32_t wv[8];
        float d;
        if (p.x) {
            const float4 *src = reinterpret_cast<const float4 *>(p.x + (long long)i * QK);
            float v[QK];
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const float4 f = __ldg(src + k);
                v[4 * k] = f.x;
                v[4 * k + 1] = f.y;
                v[4 * k + 2] = f.z;
                v[4 * k + 3] = f.w;
            }
            float amax = 0.0f;
#pragma unroll
            for (int e = 0; e < QK; e++) amax = q8_absmax(amax, v[e]);
            d = q8_scale(amax);
            const float inv = q8_inverse(d);
#pragma unroll
            for (int k = 0; k < 8; k++)
                wv[k] = (uint32_t)(uint8_t)q8_round(v[4 * k], inv) |
                        ((uint32_t)(uint8_t)q8_round(v[4 * k + 1], inv) << 8) |
                        ((uint32_t)(uint8_t)q8_round(v[4 * k + 2], inv) << 16) |
                        ((uint32_t)(uint8_t)q8_round(v[4 * k + 3], inv) << 24);
        } else {
            const uint8_t *src = p.xq + (long long)i * 36;
            d = __ldg(reinterpret_cast<const float *>(src));
#pragma unroll
            for (int k = 0; k < 8; k++) wv[k] = __ldg(reinterpret_cast<const uint32_t *>(src + 4 + 4 * k));
        }
        int qs = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) qs = dp4a(wv[k], 0x01010101, qs);
        uint4 *dst = reinterpret_cast<uint4 *>(xw + xw_off(t, b, nch));
        dst[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        dst[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
        const int si = (t * nch + (b >> 2)) * 4 + (b & 3);
        xd[si] = d;
        xs[si] = qs;
    }
    __syncthreads();
    if (!active) return;
    if (!p.tma) fetch(gw, 0);

    // rows of whole 16-byte units (nb % 4 == 0) take the chunk path
    constexpr int CW = FMT == TQK_FMT_Q8 ? 9 : 5;  // 16-byte loads per weight chunk (4 blocks)
    const bool chunked = (nb & 3) == 0;
    // one token and at most one chunk per lane: the lane's x chunk in registers
    const bool xreg = chunked && T == 1 && nch <= 32;
    uint32_t xr[32];
    float4 xdr = make_float4(0.f, 0.f, 0.f, 0.f);
    int4 xsr = make_int4(0, 0, 0, 0);
    if (xreg && lane < nch) {
        const uint4 *xv = reinterpret_cast<const uint4 *>(xw + lane * 36);
#pragma unroll
        for (int m = 0; m < 8; m++) {
            const uint4 u = xv[m];
            xr[4 * m] = u.x;
            xr[4 * m + 1] = u.y;
            xr[4 * m + 2] = u.z;
            xr[4 * m + 3] = u.w;
        }
        xdr = *reinterpret_cast<const float4 *>(xd + lane * 4);
        xsr = *reinterpret_cast<const int4 *>(xs + lane * 4);
    }

    // the (row, token, 4 blocks) terms of chunk c of one weight row into scratch
    // row srow, against the activation chunk xl (int8 words), dd (scales), ss (sums)
    auto chunk_terms = [&](const uint8_t *wrow, int c, const uint32_t (&xl)[32], float4 dd, int4 ss, float *srow) {
        const uint4 *wc = reinterpret_cast<const uint4 *>(wrow + c * (CW * 16));
        const float xdv[4] = {dd.x, dd.y, dd.z, dd.w};
        const int xsv[4] = {ss.x, ss.y, ss.z, ss.w};
        float out[4];
        // two halves of the chunk (blocks 0-1, then 2-3), to keep fewer words live
#pragma unroll
        for (int h = 0; h < 2; h++) {
            constexpr int HW = FMT == TQK_FMT_Q8 ? 5 : 3;          // 16-byte loads per half
            const int u0 = h == 0 ? 0 : (FMT == TQK_FMT_Q8 ? 4 : 2);  // first load of the half
            uint32_t ww[HW * 4];
#pragma unroll
            for (int m = 0; m < HW; m++) {
                const uint4 u = wc[u0 + m];
                ww[4 * m] = u.x;
                ww[4 * m + 1] = u.y;
                ww[4 * m + 2] = u.z;
                ww[4 * m + 3] = u.w;
            }
#pragma unroll
            for (int jj = 0; jj < 2; jj++) {
                const int jb = 2 * h + jj;
                const int w0 = jb * CW - 4 * u0;  // block jb's first word within ww
                const float wd = __uint_as_float(ww[w0]);
                const uint4 x0 = make_uint4(xl[8 * jb], xl[8 * jb + 1], xl[8 * jb + 2], xl[8 * jb + 3]);
                const uint4 x1 = make_uint4(xl[8 * jb + 4], xl[8 * jb + 5], xl[8 * jb + 6], xl[8 * jb + 7]);
                int sdot;
                if constexpr (FMT == TQK_FMT_Q8) {
                    const uint32_t q[8] = {ww[w0 + 1], ww[w0 + 2], ww[w0 + 3], ww[w0 + 4],
                                           ww[w0 + 5], ww[w0 + 6], ww[w0 + 7], ww[w0 + 8]};
                    sdot = dot_q8_block(q, x0, x1);
                } else {
                    const uint32_t q[4] = {ww[w0 + 1], ww[w0 + 2], ww[w0 + 3], ww[w0 + 4]};
                    sdot = dot_q4_block(q, x0, x1, xsv[jb]);
                }
                out[jb] = __fmul_rn(__fmul_rn((float)sdot, wd), xdv[jb]);
            }
        }
        *reinterpret_cast<float4 *>(srow + 4 * c) = make_float4(out[0], out[1], out[2], out[3]);
    };

    int k = 0, m = 0;        // groups done, groups in the current chain batch
    float *dst = nullptr;    // this lane's chain destination in the batch
    for (int g = gw; g < p.n_groups; g += TW, k++) {
        const int slot = k & 1;
        if (g + TW < p.n_groups) fetch(g + TW, slot ^ 1);
        if (p.tma) {
            const bool ok = mbar_wait_bounded(&bar[slot], (uint32_t)((k >> 1) & 1), MV_WAIT_NS, p.err);
            if (!__all_sync(0xffffffffu, ok)) {
                // stop: let the other slot's copy (if any) land before the CTA exits
                if (pending & (1u << (slot ^ 1)))
                    mbar_wait_bounded(&bar[slot ^ 1], (uint32_t)(((k + 1) >> 1) & 1), MV_DRAIN_NS, p.err);
                return;
            }
            pending &= ~(1u << slot);
        } else {
            __syncwarp();
        }
        MvJob job;
        int r0, rows;
        locate(g, job, r0, rows);
        const uint8_t *st = slots + slot * L.slot_bytes;
        const int cbase = m * R * T;  // this group's first chain row
        for (int i = 0; i < rows; i++) {
            const uint8_t *wrow = st + i * p.row_bytes;
            for (int t = 0; t < T; t++) {
                float *srow = scr + (cbase + i * T + t) * sp;
                if (xreg) {
                    if (lane < nch) chunk_terms(wrow, lane, xr, xdr, xsr, srow);
                } else if (chunked) {
                    for (int c = lane; c < nch; c += 32) {
                        uint32_t xl[32];
                        const uint4 *xv = reinterpret_cast<const uint4 *>(xw + (t * nch + c) * 36);
#pragma unroll
                        for (int q = 0; q < 8; q++) {
                            const uint4 u = xv[q];
                            xl[4 * q] = u.x;
                            xl[4 * q + 1] = u.y;
                            xl[4 * q + 2] = u.z;
                            xl[4 * q + 3] = u.w;
                        }
                        chunk_terms(wrow, c, xl, *reinterpret_cast<const float4 *>(xd + (t * nch + c) * 4),
                                    *reinterpret_cast<const int4 *>(xs + (t * nch + c) * 4), srow);
                    }
                } else {
                    for (int b = lane; b < nb; b += 32) {
                        const uint8_t *blk = wrow + b * (FMT == TQK_FMT_Q8 ? 36 : 20);
                        const float wd = *reinterpret_cast<const float *>(blk);
                        const uint4 *xv = reinterpret_cast<const uint4 *>(xw + xw_off(t, b, nch));
                        const uint4 x0 = xv[0], x1 = xv[1];
                        const int si = (t * nch + (b >> 2)) * 4 + (b & 3);
                        int sdot;
                        if constexpr (FMT == TQK_FMT_Q8) {
                            uint32_t q[8];
#pragma unroll
                            for (int w = 0; w < 8; w++) q[w] = *reinterpret_cast<const uint32_t *>(blk + 4 + 4 * w);
                            sdot = dot_q8_block(q, x0, x1);
                        } else {
                            uint32_t q[4];
#pragma unroll
                            for (int w = 0; w < 4; w++) q[w] = *reinterpret_cast<const uint32_t *>(blk + 4 + 4 * w);
                            sdot = dot_q4_block(q, x0, x1, xs[si]);
                        }
                        srow[b] = __fmul_rn(__fmul_rn((float)sdot, wd), xd[si]);
                    }
                }
            }
        }
        if (lane >= cbase && lane < cbase + R * T) {
            const int q = lane - cbase, i = q / T, t = q - i * T;
            dst = i < rows ? job.y + (long long)t * job.rows + r0 + i : nullptr;
        }
        __syncwarp();  // the slot is read: it may be refilled; the scratch rows are written
        m++;
        if (m == mb || g + TW >= p.n_groups) {
            if (lane < m * R * T && dst) {  // one (row, token) chain per lane, blocks in order
                const float *row = scr + lane * sp;
                float sum = 0.0f;
                int b = 0;
#pragma unroll 8
                for (; b + 4 <= nb; b += 4) {
                    const float4 v = *reinterpret_cast<const float4 *>(row + b);
                    sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, v.x), v.y), v.z), v.w);
                }
                for (; b < nb; b++) sum = __fadd_rn(sum, row[b]);
                *dst = sum;
            }
            __syncwarp();
            m = 0;
            dst = nullptr;
        }
    }
}

struct MvConfig {
    int tok, R, mb, warps, sp, smem;
};

// Launch geometry for (format, blocks per row, tokens): groups of about
// MV_GROUP_BYTES, chain walks of about MV_CHAINS rows, as many warps (up to
// MV_MAX_WARPS) as shared memory allows.
template <int FMT>
int mv_config(int nb, int n_tok, MvConfig *c) {
    const int BB = FMT == TQK_FMT_Q8 ? 36 : 20;
    const int row_bytes = nb * BB;
    int tok = n_tok < MV_MAX_TOK ? n_tok : MV_MAX_TOK;
    // chain rows are 16-byte aligned and an odd number of 16-byte units apart (the
    // walking lanes' 16-byte loads then fall into distinct bank groups)
    int sp = ((nb + 3) / 4) * 4;
    if ((sp / 4) % 2 == 0) sp += 4;
    for (;;) {
        int R = MV_GROUP_BYTES / row_bytes;
        if (R < 1) R = 1;
        if (R * tok > 32) R = 32 / tok;
        int mb = MV_CHAINS / (R * tok);
        if (mb < 1) mb = 1;
        for (; mb >= 1; mb--) {
            for (int warps = MV_MAX_WARPS; warps >= 4 || (warps >= 1 && mb == 1); warps--) {
                const MvLayout L(nb, tok, R, row_bytes, sp, mb, warps);
                if (L.bytes <= MV_SMEM_LIMIT) {
                    *c = MvConfig{tok, R, mb, warps, sp, L.bytes};
                    return TQK_OK;
                }
            }
        }
        if (tok == 1) break;
        tok = (tok + 1) / 2;
    }
    return fail(TQK_EUNSUPPORTED, "matmul: a row of this many blocks does not fit in shared memory");
}

template <int FMT>
int mv_occupancy(const MvConfig &c, int *per_sm) {
    static std::mutex mu;
    static bool attr_set[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return fail_cuda(e, "matmul: cudaGetDevice");
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!attr_set[dev]) {
            e = cudaFuncSetAttribute(matvec_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, MV_SMEM_LIMIT);
            if (e != cudaSuccess) return fail_cuda(e, "matvec_kernel attributes");
            attr_set[dev] = true;
        }
    }
    int o = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, matvec_kernel<FMT>, c.warps * 32, c.smem);
    if (e != cudaSuccess) return fail_cuda(e, "matvec_kernel occupancy");
    *per_sm = o > 0 ? o : 1;
    return TQK_OK;
}

template <int FMT>
int matvec_run(const tqk_proj_job *jobs, int n_jobs, const float *x, const uint8_t *xq, int cols, int n_tok,
               cudaStream_t stream) {
    const int nb = cols / QK;
    const int BB = FMT == TQK_FMT_Q8 ? 36 : 20;
    const int row_bytes = nb * BB;
    MvConfig c;
    int rc = mv_config<FMT>(nb, n_tok, &c);
    if (rc) return rc;
    int per_sm = 1;
    rc = mv_occupancy<FMT>(c, &per_sm);
    if (rc) return rc;
    const DeviceInfo *d = device_info();
    const int sms = d ? d->sm_count : 148;

    MvParams p{};
    p.n_jobs = n_jobs;
    p.nb = nb;
    p.R = c.R;
    p.mb = c.mb;
    p.row_bytes = row_bytes;
    p.sp = c.sp;
    p.err = d ? d->err_word : nullptr;
    bool aligned = row_bytes % 16 == 0;
    long long groups = 0;
    for (int j = 0; j < n_jobs; j++) {
        p.job[j].w = static_cast<const uint8_t *>(jobs[j].w);
        p.job[j].rows = jobs[j].rows;
        p.job[j].group0 = (int)groups;
        groups += (jobs[j].rows + c.R - 1) / c.R;
        if (reinterpret_cast<uintptr_t>(jobs[j].w) % 16) aligned = false;
    }
    if (groups > 0x7fffffff) return fail(TQK_EINVAL, "matmul: too many rows");
    p.n_groups = (int)groups;
    p.tma = aligned ? 1 : 0;
    // fp32 activations: quantised inside the kernel (one thread per block) while
    // every thread has at most one block and x is 16-byte aligned, otherwise
    // first by the grid-wide quantiser into a library buffer (then every CTA
    // only copies the Q8 rows)
    if (x && ((long long)c.tok * nb > 32LL * c.warps || reinterpret_cast<uintptr_t>(x) % 16)) {
        void *buf = library_scratch(stream, (size_t)n_tok * nb * 36);
        if (!buf) return fail(TQK_ECUDA, "matmul: cannot allocate the activation buffer");
        rc = tqk_quantize_rows_q8(x, static_cast<tqk_block_q8 *>(buf), n_tok, cols, stream);
        if (rc) return rc;
        xq = static_cast<const uint8_t *>(buf);
        x = nullptr;
    }
    const long long warps_needed = groups;
    long long ctas = (warps_needed + c.warps - 1) / c.warps;
    const long long cap = (long long)sms * per_sm;
    if (ctas > cap) ctas = cap;
    for (int t0 = 0; t0 < n_tok; t0 += c.tok) {
        const int tl = n_tok - t0 < c.tok ? n_tok - t0 : c.tok;
        p.n_tok = tl;
        p.x = x ? x + (long long)t0 * cols : nullptr;
        p.xq = xq ? xq + (long long)t0 * nb * 36 : nullptr;
        for (int j = 0; j < n_jobs; j++) p.job[j].y = jobs[j].y + (long long)t0 * jobs[j].rows;
        const MvLayout L(nb, tl, c.R, row_bytes, c.sp, c.mb, c.warps);
        rc = launch_pdl(matvec_kernel<FMT>, dim3((unsigned)ctas), dim3(c.warps * 32), L.bytes, stream, p);
        if (rc) return rc;
        rc = check_launch("matvec_kernel");
        if (rc) return rc;
    }
    return TQK_OK;
}

int matvec_entry(const tqk_proj_job *jobs, int n_jobs, int format, const float *x, const void *xq, int cols,
                 int n_tok, tqk_stream_t stream) {
    if (!jobs || n_jobs <= 0 || n_jobs > MV_MAX_JOBS) return fail(TQK_EINVAL, "matmul: 1 to 4 jobs");
    if (format != TQK_FMT_Q8 && format != TQK_FMT_Q4) return fail(TQK_EINVAL, "matmul: format");
    if (cols <= 0 || cols % QK) return fail(TQK_EINVAL, "matmul: cols must be a positive multiple of 32");
    if (n_tok < 0) return fail(TQK_EINVAL, "matmul: n_tok < 0");
    if (!x && !xq) return fail(TQK_EINVAL, "matmul: NULL activations");
    for (int j = 0; j < n_jobs; j++) {
        if (jobs[j].rows < 0) return fail(TQK_EINVAL, "matmul: rows < 0");
        if (jobs[j].rows > 0 && (!jobs[j].w || !jobs[j].y)) return fail(TQK_EINVAL, "matmul: NULL weights or output");
        if (reinterpret_cast<uintptr_t>(jobs[j].w) % 4) return fail(TQK_EINVAL, "matmul: weights not 4-byte aligned");
    }
    if (xq && reinterpret_cast<uintptr_t>(xq) % 4) return fail(TQK_EINVAL, "matmul: xq not 4-byte aligned");
    // jobs without rows drop out
    tqk_proj_job live[MV_MAX_JOBS];
    int n_live = 0;
    for (int j = 0; j < n_jobs; j++)
        if (jobs[j].rows > 0) live[n_live++] = jobs[j];
    if (n_live == 0 || n_tok == 0) return TQK_OK;
    int rc = ensure_device();
    if (rc) return rc;
    const uint8_t *xq8 = static_cast<const uint8_t *>(xq);
    cudaStream_t st = (cudaStream_t)stream;
    return format == TQK_FMT_Q8 ? matvec_run<TQK_FMT_Q8>(live, n_live, x, xq8, cols, n_tok, st)
                                : matvec_run<TQK_FMT_Q4>(live, n_live, x, xq8, cols, n_tok, st);
}

}  // namespace
}  // namespace tqk

using namespace tqk;

extern "C" int tqk_matmul_q8_batch(const tqk_block_q8 *W, const tqk_block_q8 *xq, float *y, int rows, int cols,
                                   int n_tok, tqk_stream_t stream) {
    const tqk_proj_job j{W, y, rows};
    return matvec_entry(&j, 1, TQK_FMT_Q8, nullptr, xq, cols, n_tok, stream);
}

extern "C" int tqk_matmul_q4_batch(const tqk_block_q4 *W, const tqk_block_q8 *xq, float *y, int rows, int cols,
                                   int n_tok, tqk_stream_t stream) {
    const tqk_proj_job j{W, y, rows};
    return matvec_entry(&j, 1, TQK_FMT_Q4, nullptr, xq, cols, n_tok, stream);
}

extern "C" int tqk_matmul_q8(const tqk_block_q8 *W, const tqk_block_q8 *xq, float *y, int rows, int cols,
                             tqk_stream_t stream) {
    return tqk_matmul_q8_batch(W, xq, y, rows, cols, 1, stream);
}

extern "C" int tqk_matmul_q4(const tqk_block_q4 *W, const tqk_block_q8 *xq, float *y, int rows, int cols,
                             tqk_stream_t stream) {
    return tqk_matmul_q4_batch(W, xq, y, rows, cols, 1, stream);
}

extern "C" int tqk_project(const tqk_proj_job *jobs, int n_jobs, int format, const float *x, int cols, int n_tok,
                           tqk_stream_t stream) {
    if (!x) return fail(TQK_EINVAL, "tqk_project: NULL x");
    return matvec_entry(jobs, n_jobs, format, x, nullptr, cols, n_tok, stream);
}
