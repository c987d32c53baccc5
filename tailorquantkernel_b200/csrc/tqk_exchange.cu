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

MailboxLayout mailbox_layout(int world, int n_heads, int head_dim) {
    MailboxLayout m{};
    m.rec = (size_t)head_dim + 2;
    m.slot = (size_t)n_heads * m.rec;
    const size_t data = 2 * m.slot * sizeof(float);
    m.flags_off = (data + 255) & ~(size_t)255;
    m.bytes = m.flags_off + (((size_t)2 * world * sizeof(int) + 255) & ~(size_t)255);
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

__global__ void __launch_bounds__(128) exchange_merge_kernel(const ExchangeParams p) {
    const int h = blockIdx.x, tid = threadIdx.x;
    const int rec = p.head_dim + 2, par = p.epoch & 1;
    __shared__ int s_ok;

    // launched with programmatic stream serialization: the records come from the decode grid before
    grid_dependency_wait();
    // this rank's records of the epoch are in its slot: tell every peer
    if (h == 0 && tid < p.world && tid != p.rank) {
        int *flags = reinterpret_cast<int *>(reinterpret_cast<char *>(p.mbox[tid]) + p.flags_off);
        st_release_sys(flags + par * p.world + p.rank, p.epoch);
    }
    if (tid == 0) {
        // wait until every peer's records of this epoch are in its slot
        const int *flags = reinterpret_cast<const int *>(reinterpret_cast<const char *>(p.mbox[p.rank]) + p.flags_off);
        int ok = 1;
        const uint64_t t0 = p.world > 1 ? globaltimer_ns() : 0;
        for (int peer = 0; peer < p.world && ok; peer++) {
            if (peer == p.rank) continue;
            for (uint32_t it = 0; ld_acquire_sys(flags + par * p.world + peer) != p.epoch; it++) {
                if ((it & 63u) == 63u && globaltimer_ns() - t0 > EX_WAIT_NS) {
                    record_error(p.err, DEVERR_TIMEOUT);
                    ok = 0;
                    break;
                }
                __nanosleep(32);
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;

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
