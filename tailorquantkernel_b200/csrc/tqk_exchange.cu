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
//   * phase 1: CTA h stores head h's record of this rank into every peer's
//     mailbox slot [epoch parity][this rank] with plain P2P stores over
//     NVLink, fences at system scope and takes a ticket; the last CTA raises
//     this rank's flag in every peer's mailbox to the epoch number;
//   * phase 2: each CTA waits until every peer's flag in the local mailbox
//     shows this epoch (a spin with a 1 s limit that records TQK_ETIMEOUT in
//     the device error word and skips the merge instead of hanging), then
//     merges head h of all ranks' records as tqk_merge_partials does.
// Slots alternate by epoch parity: a rank overwrites a peer's slot of epoch e
// only after that peer's flag for epoch e+1 showed that it had finished
// merging epoch e.  No TMA, no multicast, no NVLS: plain loads and stores.
#include "tqk_internal.h"

#include <cstring>

namespace tqk {
namespace {

constexpr int EX_MAX_WORLD = 8;
constexpr uint64_t EX_WAIT_NS = 1000000000ull;

struct MailboxLayout {
    size_t rec;         // floats per (rank, head) record
    size_t slot;        // floats per (parity, rank) slot: n_heads * rec
    size_t flags_off;   // bytes: int flags[2][world]
    size_t ticket_off;  // bytes: unsigned tickets[2]
    size_t bytes;
};

MailboxLayout mailbox_layout(int world, int n_heads, int head_dim) {
    MailboxLayout m{};
    m.rec = (size_t)head_dim + 2;
    m.slot = (size_t)n_heads * m.rec;
    const size_t data = 2 * (size_t)world * m.slot * sizeof(float);
    m.flags_off = (data + 255) & ~(size_t)255;
    m.ticket_off = m.flags_off + 256;
    m.bytes = m.ticket_off + 256;
    return m;
}

struct ExchangeParams {
    float *mbox[EX_MAX_WORLD];  // every rank's mailbox as mapped in this process (mbox[rank] is local)
    const float *partial;       // this rank's records [n_heads][head_dim + 2]
    float *out;                 // [n_heads][head_dim]
    int world, rank, n_heads, head_dim;
    int epoch;                  // >= 1, one more per step
    long long slot, flags_off, ticket_off;
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

__global__ void __launch_bounds__(128) exchange_merge_kernel(const ExchangeParams p) {
    const int h = blockIdx.x, tid = threadIdx.x;
    const int rec = p.head_dim + 2, par = p.epoch & 1;
    __shared__ int s_ok;
    __shared__ float s_m, s_l;

    // ---- phase 1: this rank's record of head h into every peer's slot [par][rank]
    const float *src = p.partial + (long long)h * rec;
    for (int peer = 0; peer < p.world; peer++) {
        if (peer == p.rank) continue;
        float *dst = p.mbox[peer] + ((long long)par * p.world + p.rank) * p.slot + (long long)h * rec;
        for (int c = tid; c < rec; c += blockDim.x) dst[c] = src[c];
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
        unsigned *ticket = reinterpret_cast<unsigned *>(reinterpret_cast<char *>(p.mbox[p.rank]) + p.ticket_off) + par;
        if (atomicAdd(ticket, 1u) == (unsigned)(p.n_heads - 1)) {
            // every CTA's stores are fenced before its ticket: publish the epoch to the peers
            *ticket = 0u;  // the next use of this ticket is two epochs later, in a later launch
            __threadfence_system();
            for (int peer = 0; peer < p.world; peer++) {
                if (peer == p.rank) continue;
                int *flags = reinterpret_cast<int *>(reinterpret_cast<char *>(p.mbox[peer]) + p.flags_off);
                st_release_sys(flags + par * p.world + p.rank, p.epoch);
            }
        }
        // ---- phase 2: wait until every peer's record of this epoch has arrived here
        const int *flags = reinterpret_cast<const int *>(reinterpret_cast<const char *>(p.mbox[p.rank]) + p.flags_off);
        int ok = 1;
        const uint64_t t0 = globaltimer_ns();
        for (int peer = 0; peer < p.world && ok; peer++) {
            if (peer == p.rank) continue;
            for (uint32_t it = 0; ld_acquire_sys(flags + par * p.world + peer) != p.epoch; it++) {
                if ((it & 63u) == 63u && globaltimer_ns() - t0 > EX_WAIT_NS) {
                    record_error(p.err, DEVERR_TIMEOUT);
                    ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    __threadfence();

    // ---- merge head h: out = sum_r acc_r e^(m_r - M) / sum_r l_r e^(m_r - M), M = max_r m_r
    //      (tqk_merge_partials' arithmetic; this rank's record is read from its own buffer)
    auto rec_of = [&](int r) -> const float * {
        return r == p.rank ? src : p.mbox[p.rank] + ((long long)par * p.world + r) * p.slot + (long long)h * rec;
    };
    if (tid < 32) {
        float M = -INFINITY;
        if (tid < p.world) M = __ldcg(rec_of(tid) + p.head_dim);
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.0f;
        if (tid < p.world) {
            const float *rp = rec_of(tid);
            const float l = __ldcg(rp + p.head_dim + 1);
            if (l > 0.0f) L = l * expf(__ldcg(rp + p.head_dim) - M);
        }
        for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        if (tid == 0) {
            s_m = M;
            s_l = L;
        }
    }
    __syncthreads();
    const float M = s_m, L = s_l;
    for (int c = tid; c < p.head_dim; c += blockDim.x) {
        float a = 0.0f;
        for (int r = 0; r < p.world; r++) {
            const float *rp = rec_of(r);
            if (__ldcg(rp + p.head_dim + 1) > 0.0f) a = fmaf(expf(__ldcg(rp + p.head_dim) - M), __ldcg(rp + c), a);
        }
        p.out[(long long)h * p.head_dim + c] = L > 0.0f ? a / L : 0.0f;
    }
}

}  // namespace
}  // namespace tqk

using namespace tqk;

extern "C" size_t tqk_exchange_mailbox_bytes(int world, int n_heads, int head_dim) {
    if (world < 1 || world > EX_MAX_WORLD || n_heads <= 0 || head_dim <= 0) return 0;
    return mailbox_layout(world, n_heads, head_dim).bytes;
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

extern "C" int tqk_exchange_merge(const float *partial, int n_heads, int head_dim, int world, int rank,
                                  void *const *mailboxes, int epoch, float *out, tqk_stream_t stream) {
    if (!partial || !out || !mailboxes || n_heads <= 0 || head_dim <= 0 || world < 1 || world > EX_MAX_WORLD ||
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
    p.partial = partial;
    p.out = out;
    p.world = world;
    p.rank = rank;
    p.n_heads = n_heads;
    p.head_dim = head_dim;
    p.epoch = epoch;
    p.slot = (long long)m.slot;
    p.flags_off = (long long)m.flags_off;
    p.ticket_off = (long long)m.ticket_off;
    p.err = device_info()->err_word;
    exchange_merge_kernel<<<n_heads, 128, 0, (cudaStream_t)stream>>>(p);
    return check_launch("exchange_merge_kernel");
}
