// tqk_exchange.cu -- the exchange step of a context split by sequence over the
// GPUs of one box (the multi-GPU form of attend_q8, reference
// model/attention_layer.c:125-150, whose single CPU has no such step): every
// rank holds log-sum-exp partials {acc[head_dim], m, l} of its token range and
// every rank needs the merged output.
//
// tqk_exchange_merge does it in one kernel over peer memory, without a
// collective library:
//   * each rank owns a mailbox (tqk_peer_buffer_alloc) that the others map
//     through CUDA IPC handles (tqk_ipc_get_handle / tqk_ipc_open_handle);
//   * the rank's decode writes its partial records straight into its own
//     mailbox, in the slot of the step's epoch parity (tqk_exchange_slot_offset);
//   * the kernel raises this rank's flag in every peer's mailbox to the epoch
//     number (the records are complete: the decode grid has finished), waits
//     until every peer's flag in the local mailbox shows the epoch (a spin
//     with a 1 s limit that records TQK_ETIMEOUT in the device error word
//     and skips the merge instead of hanging), then reads the peers' records
//     of the epoch over NVLink with plain loads and merges head h of all
//     ranks as tqk_merge_partials does.
// Slots alternate by epoch parity: a rank's decode overwrites its slot of
// epoch e only at epoch e+2, after its exchange of epoch e+1 has seen every
// peer's flag e+1, which each peer raises only once it has finished merging
// epoch e.  No TMA, no multicast, no NVLS: plain loads and stores.
//
// tqk_exchange_gather runs the same protocol for the kv-head-group split of
// one sequence (the decode's q heads divided over the ranks by kv head): each
// rank's slot holds its output heads of every layer, and the kernel
// concatenates every rank's slice into the full output instead of merging.
#include "tqk_internal.h"

#include <cstring>

namespace tqk {
namespace {

constexpr int EX_MAX_WORLD = 8;
constexpr uint64_t EX_WAIT_NS = 1000000000ull;

struct MailboxLayout {
    size_t rec;         // floats per head record {acc[head_dim], m, l}
    size_t slot;        // floats per parity slot: n_heads * rec
    size_t flags_off;   // bytes: int flags[2][world]
    size_t bytes;
};

// Layout of a mailbox whose two parity slots hold slot_floats floats each,
// followed by the flags int[2][world] (every part 256-byte aligned).
MailboxLayout mailbox_layout_floats(int world, size_t slot_floats) {
    MailboxLayout m{};
    m.rec = 0;
    m.slot = slot_floats;
    const size_t data = 2 * m.slot * sizeof(float);
    m.flags_off = (data + 255) & ~(size_t)255;
    m.bytes = m.flags_off + (((size_t)2 * world * sizeof(int) + 255) & ~(size_t)255);
    return m;
}

MailboxLayout mailbox_layout(int world, int n_heads, int head_dim) {
    MailboxLayout m = mailbox_layout_floats(world, (size_t)n_heads * ((size_t)head_dim + 2));
    m.rec = (size_t)head_dim + 2;
    return m;
}

struct ExchangeParams {
    float *mbox[EX_MAX_WORLD];  // every rank's mailbox as mapped in this process (mbox[rank] is local)
    float *out;                 // [n_heads][head_dim]
    int world, rank, n_heads, head_dim;
    int epoch;                  // >= 1, one more per step
    long long slot, flags_off;
    int *err;
};

__device__ __forceinline__ void st_release_sys(int *p, int v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float ld_relaxed_sys(const float *p) {
    float v;
    asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

// Raises this rank's flag of the epoch in every peer's mailbox (block 0) and
// waits, in thread 0 of every block, until every peer's flag of the epoch has
// arrived in the local mailbox (1 s limit: DEVERR_TIMEOUT, returns false).
// Called after grid_dependency_wait, so this rank's slot is complete.
__device__ bool raise_and_wait_flags(float *const *mbox, int world, int rank, int epoch, long long flags_off,
                                     int *err) {
    __shared__ int s_ok;
    const int tid = threadIdx.x, par = epoch & 1;
    if (blockIdx.x == 0 && tid < world && tid != rank) {
        int *flags = reinterpret_cast<int *>(reinterpret_cast<char *>(mbox[tid]) + flags_off);
        st_release_sys(flags + par * world + rank, epoch);
    }
    if (tid == 0) {
        const int *flags = reinterpret_cast<const int *>(reinterpret_cast<const char *>(mbox[rank]) + flags_off);
        int ok = 1;
        const uint64_t t0 = world > 1 ? globaltimer_ns() : 0;
        for (int peer = 0; peer < world && ok; peer++) {
            if (peer == rank) continue;
            for (uint32_t it = 0; ld_acquire_sys(flags + par * world + peer) != epoch; it++) {
                if ((it & 63u) == 63u && globaltimer_ns() - t0 > EX_WAIT_NS) {
                    record_error(err, DEVERR_TIMEOUT);
                    ok = 0;
                    break;
                }
                __nanosleep(32);
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

__global__ void __launch_bounds__(128) exchange_merge_kernel(const ExchangeParams p) {
    const int h = blockIdx.x, tid = threadIdx.x;
    const int rec = p.head_dim + 2, par = p.epoch & 1;

    // launched with programmatic stream serialization: the records come from the decode grid before
    grid_dependency_wait();
    grid_dependents_launch();  // the next kernel waits for this grid before it touches anything
    // this rank's records of the epoch are in its slot: tell every peer, then wait for theirs
    if (!raise_and_wait_flags(p.mbox, p.world, p.rank, p.epoch, p.flags_off, p.err)) return;

    // ---- merge head h: out = sum_r acc_r e^(m_r - M) / sum_r l_r e^(m_r - M), M = max_r m_r
    //      (tqk_merge_partials' arithmetic).  Every thread issues all its loads of the ranks'
    //      records (m, l and its column of acc) together, so the peers' records cost one
    //      NVLink round trip, and derives M and L itself.
    auto rec_of = [&](int r) -> const float * { return p.mbox[r] + (long long)par * p.slot + (long long)h * rec; };
    float mr[EX_MAX_WORLD], lr[EX_MAX_WORLD], ar[EX_MAX_WORLD];
    const int c = tid;  // head_dim <= 128 = blockDim.x (checked on the host)
#pragma unroll
    for (int r = 0; r < EX_MAX_WORLD; r++) {
        if (r < p.world) {
            const float *rp = rec_of(r);
            mr[r] = ld_relaxed_sys(rp + p.head_dim);
            lr[r] = ld_relaxed_sys(rp + p.head_dim + 1);
            ar[r] = c < p.head_dim ? ld_relaxed_sys(rp + c) : 0.0f;
        }
    }
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < EX_MAX_WORLD; r++)
        if (r < p.world) M = fmaxf(M, mr[r]);
    float L = 0.0f, a = 0.0f;
#pragma unroll
    for (int r = 0; r < EX_MAX_WORLD; r++) {
        if (r < p.world && lr[r] > 0.0f) {
            const float e = expf(mr[r] - M);
            L += lr[r] * e;
            a = fmaf(e, ar[r], a);
        }
    }
    if (c < p.head_dim) p.out[(long long)h * p.head_dim + c] = L > 0.0f ? a / L : 0.0f;
}

struct GatherParams {
    float *mbox[EX_MAX_WORLD];  // every rank's mailbox as mapped in this process (mbox[rank] is local)
    float *out;                 // [n_groups][world][chunk]
    int world, rank, n_groups, chunk;
    int epoch;
    long long slot, flags_off;
    int *err;
};

__device__ __forceinline__ float4 ld_relaxed_sys_v4(const float4 *p) {
    float4 v;
    asm volatile("ld.relaxed.sys.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// All-gather of the kv-head-group split: rank r's slot of the epoch holds
// [n_groups][chunk] floats (its head slice of every layer); out[g][r][:] =
// slot_r[g][:] on every rank.  Block g copies group g of every rank; each
// thread issues the loads of all its float4 columns before it stores any, so
// the peers' slices cost one NVLink round trip.  chunk % 4 == 0 (host-checked).
constexpr int GATHER_THREADS = 256;
constexpr int GATHER_MAX_V4 = 8;  // float4 per thread: world * chunk <= 8192 floats per group

__global__ void __launch_bounds__(GATHER_THREADS) exchange_gather_kernel(const GatherParams p) {
    grid_dependency_wait();
    grid_dependents_launch();  // the next kernel waits for this grid before it touches anything
    if (!raise_and_wait_flags(p.mbox, p.world, p.rank, p.epoch, p.flags_off, p.err)) return;
    const int g = blockIdx.x, tid = threadIdx.x, par = p.epoch & 1;
    const int c4 = p.chunk >> 2, total = p.world * c4;
    float4 v[GATHER_MAX_V4];
#pragma unroll
    for (int k = 0; k < GATHER_MAX_V4; k++) {
        const int i = tid + k * GATHER_THREADS;
        if (i < total) {
            const int r = i / c4, c = i - r * c4;
            const float4 *src = reinterpret_cast<const float4 *>(p.mbox[r] + (long long)par * p.slot +
                                                                 (long long)g * p.chunk) + c;
            v[k] = ld_relaxed_sys_v4(src);
        }
    }
    float4 *dst = reinterpret_cast<float4 *>(p.out + (long long)g * p.world * p.chunk);
#pragma unroll
    for (int k = 0; k < GATHER_MAX_V4; k++) {
        const int i = tid + k * GATHER_THREADS;
        if (i < total) dst[i] = v[k];
    }
}

// One {value bits, epoch} pair as a single 64-bit access (the writer's is one too).
__device__ __forceinline__ uint2 ld_relaxed_sys_pair(const uint2 *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return make_uint2((uint32_t)v, (uint32_t)(v >> 32));
}

// tqk_gather_collect: launched with programmatic dependent launch behind the
// decode, so its blocks are resident early; they first wait for that decode
// grid to complete (this rank's own pairs are then written, and the stream's
// next kernel may reuse the decode's workspace), and only then poll -- polling
// during the decode would put every thread's re-reads on the memory system the
// decode is streaming through.  Every thread loads its {value, epoch} pairs,
// re-reads a pair (bounded: 1 s in all) until it shows the step's epoch, and
// writes the value.
constexpr int COLLECT_THREADS = 256, COLLECT_PER = 4;

__global__ void __launch_bounds__(COLLECT_THREADS) gather_collect_kernel(const uint2 *pairs, long long n, int epoch,
                                                                        float *out, int *err) {
    grid_dependency_wait();
    // the next step's decode may launch now: it waits for this grid before it reads or writes
    // anything, and its CTAs find the SMs the finished decode left
    grid_dependents_launch();
    const long long base = (long long)blockIdx.x * COLLECT_THREADS * COLLECT_PER + threadIdx.x;
    uint2 v[COLLECT_PER];
#pragma unroll
    for (int k = 0; k < COLLECT_PER; k++) {
        const long long i = base + (long long)k * COLLECT_THREADS;
        if (i < n) v[k] = ld_relaxed_sys_pair(pairs + i);
    }
    bool ok = true;
    uint64_t t0 = 0;
#pragma unroll
    for (int k = 0; k < COLLECT_PER; k++) {
        const long long i = base + (long long)k * COLLECT_THREADS;
        if (i >= n) continue;
        for (uint32_t it = 0; ok && v[k].y != (uint32_t)epoch; it++) {
            if (t0 == 0) t0 = globaltimer_ns();
            if ((it & 15u) == 15u && globaltimer_ns() - t0 > EX_WAIT_NS) {
                record_error(err, DEVERR_TIMEOUT);
                ok = false;
                break;
            }
            __nanosleep(64);
            v[k] = ld_relaxed_sys_pair(pairs + i);
        }
        out[i] = __uint_as_float(v[k].x);
    }
}

}  // namespace
}  // namespace tqk

using namespace tqk;

extern "C" size_t tqk_exchange_mailbox_bytes(int world, int n_heads, int head_dim) {
    if (world < 1 || world > EX_MAX_WORLD || n_heads <= 0 || head_dim <= 0) return 0;
    return mailbox_layout(world, n_heads, head_dim).bytes;
}

extern "C" size_t tqk_exchange_slot_offset(int n_heads, int head_dim, int epoch) {
    if (n_heads <= 0 || head_dim <= 0 || epoch < 1) return 0;
    return (size_t)(epoch & 1) * mailbox_layout(1, n_heads, head_dim).slot * sizeof(float);
}

extern "C" int tqk_peer_buffer_alloc(size_t bytes, void **ptr) {
    if (!ptr || bytes == 0) return fail(TQK_EINVAL, "tqk_peer_buffer_alloc: bad arguments");
    *ptr = nullptr;
    int rc = ensure_device();
    if (rc) return rc;
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);  // a whole allocation: its IPC handle maps exactly this buffer
    if (e != cudaSuccess) return fail_cuda(e, "tqk_peer_buffer_alloc: cudaMalloc");
    e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail_cuda(e, "tqk_peer_buffer_alloc: cudaMemset");
    }
    *ptr = p;
    return TQK_OK;
}

extern "C" int tqk_peer_buffer_free(void *ptr) {
    if (!ptr) return TQK_OK;
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? TQK_OK : fail_cuda(e, "tqk_peer_buffer_free");
}

extern "C" int tqk_ipc_get_handle(void *ptr, unsigned char *handle) {
    if (!ptr || !handle) return fail(TQK_EINVAL, "tqk_ipc_get_handle: bad arguments");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
    if (e != cudaSuccess) return fail_cuda(e, "tqk_ipc_get_handle: cudaIpcGetMemHandle");
    static_assert(sizeof(h) == TQK_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof h);
    return TQK_OK;
}

extern "C" int tqk_ipc_open_handle(const unsigned char *handle, void **ptr) {
    if (!ptr || !handle) return fail(TQK_EINVAL, "tqk_ipc_open_handle: bad arguments");
    *ptr = nullptr;
    int rc = ensure_device();
    if (rc) return rc;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? TQK_OK : fail_cuda(e, "tqk_ipc_open_handle: cudaIpcOpenMemHandle");
}

extern "C" int tqk_ipc_close_handle(void *ptr) {
    if (!ptr) return TQK_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? TQK_OK : fail_cuda(e, "tqk_ipc_close_handle");
}

extern "C" int tqk_exchange_merge(int n_heads, int head_dim, int world, int rank, void *const *mailboxes, int epoch,
                                  float *out, tqk_stream_t stream) {
    if (!out || !mailboxes || n_heads <= 0 || head_dim <= 0 || head_dim > 128 || world < 1 || world > EX_MAX_WORLD ||
        rank < 0 || rank >= world || epoch < 1)
        return fail(TQK_EINVAL, "tqk_exchange_merge: bad arguments");
    int rc = ensure_device();
    if (rc) return rc;
    const MailboxLayout m = mailbox_layout(world, n_heads, head_dim);
    ExchangeParams p{};
    for (int r = 0; r < world; r++) {
        if (!mailboxes[r] || (reinterpret_cast<uintptr_t>(mailboxes[r]) & 255))
            return fail(TQK_EALIGN, "tqk_exchange_merge: every mailbox must be a whole tqk_peer_buffer_alloc buffer");
        p.mbox[r] = static_cast<float *>(mailboxes[r]);
    }
    p.out = out;
    p.world = world;
    p.rank = rank;
    p.n_heads = n_heads;
    p.head_dim = head_dim;
    p.epoch = epoch;
    p.slot = (long long)m.slot;
    p.flags_off = (long long)m.flags_off;
    p.err = device_info()->err_word;
    return launch_pdl(exchange_merge_kernel, dim3((unsigned)n_heads), dim3(128), 0, (cudaStream_t)stream, p);
}

extern "C" size_t tqk_gather_mailbox_bytes(int world, int n_groups, int chunk_floats) {
    if (world < 1 || world > EX_MAX_WORLD || n_groups <= 0 || chunk_floats <= 0) return 0;
    return mailbox_layout_floats(world, (size_t)n_groups * chunk_floats).bytes;
}

extern "C" size_t tqk_gather_slot_offset(int n_groups, int chunk_floats, int epoch) {
    if (n_groups <= 0 || chunk_floats <= 0 || epoch < 1) return 0;
    return (size_t)(epoch & 1) * (size_t)n_groups * chunk_floats * sizeof(float);
}

extern "C" int tqk_exchange_gather(int n_groups, int chunk_floats, int world, int rank, void *const *mailboxes,
                                   int epoch, float *out, tqk_stream_t stream) {
    if (!out || !mailboxes || n_groups <= 0 || n_groups > 65535 || chunk_floats <= 0 || world < 1 ||
        world > EX_MAX_WORLD || rank < 0 || rank >= world || epoch < 1)
        return fail(TQK_EINVAL, "tqk_exchange_gather: bad arguments");
    if (chunk_floats % 4 || (long long)world * chunk_floats > (long long)GATHER_MAX_V4 * GATHER_THREADS * 4)
        return fail(TQK_EUNSUPPORTED, "tqk_exchange_gather: chunk_floats must be a multiple of 4 and "
                                      "world * chunk_floats at most 8192");
    if (reinterpret_cast<uintptr_t>(out) & 15) return fail(TQK_EALIGN, "tqk_exchange_gather: out must be 16-byte aligned");
    int rc = ensure_device();
    if (rc) return rc;
    const MailboxLayout m = mailbox_layout_floats(world, (size_t)n_groups * chunk_floats);
    GatherParams p{};
    for (int r = 0; r < world; r++) {
        if (!mailboxes[r] || (reinterpret_cast<uintptr_t>(mailboxes[r]) & 255))
            return fail(TQK_EALIGN, "tqk_exchange_gather: every mailbox must be a whole tqk_peer_buffer_alloc buffer");
        p.mbox[r] = static_cast<float *>(mailboxes[r]);
    }
    p.out = out;
    p.world = world;
    p.rank = rank;
    p.n_groups = n_groups;
    p.chunk = chunk_floats;
    p.epoch = epoch;
    p.slot = (long long)m.slot;
    p.flags_off = (long long)m.flags_off;
    p.err = device_info()->err_word;
    return launch_pdl(exchange_gather_kernel, dim3((unsigned)n_groups), dim3(GATHER_THREADS), 0, (cudaStream_t)stream,
                      p);
}

extern "C" int tqk_gather_collect(const void *pairs, size_t n, int epoch, float *out, tqk_stream_t stream) {
    if (!pairs || !out || (reinterpret_cast<uintptr_t>(pairs) & 7) || epoch < 1)
        return fail(TQK_EINVAL, "tqk_gather_collect: bad pairs, out or epoch");
    if (n == 0) return TQK_OK;
    int rc = ensure_device();
    if (rc) return rc;
    const long long per_block = (long long)COLLECT_THREADS * COLLECT_PER;
    const long long blocks = ((long long)n + per_block - 1) / per_block;
    if (blocks > 0x7fffffffLL) return fail(TQK_EINVAL, "tqk_gather_collect: n too large");
    return launch_pdl(gather_collect_kernel, dim3((unsigned)blocks), dim3(COLLECT_THREADS), 0, (cudaStream_t)stream,
                      static_cast<const uint2 *>(pairs), (long long)n, epoch, out, device_info()->err_word);
}
