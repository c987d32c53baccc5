// tqk_runtime.cu -- status codes, per-thread error text, per-device state and
// the library-owned workspaces behind the tqk C ABI.
#include "tqk_internal.h"

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

namespace tqk {

namespace {
thread_local char t_last_error[512] = "";

std::mutex g_mutex;
DeviceInfo g_devices[64];

struct Workspace {
    void *ptr = nullptr;
    size_t bytes = 0;
};
std::map<std::pair<int, cudaStream_t>, Workspace> g_workspaces;
std::map<std::pair<int, cudaStream_t>, Workspace> g_counters;
std::map<std::pair<int, cudaStream_t>, Workspace> g_scratch;
std::map<std::pair<int, cudaStream_t>, Workspace> g_prefill_stage;

// Grows `w` to at least `bytes` (minimum 1 MiB), zeroing the new buffer on `stream`.
void *grow_zeroed(Workspace &w, cudaStream_t stream, size_t bytes) {
    if (w.bytes >= bytes && w.ptr) return w.ptr;
    if (w.ptr) {
        // the old buffer may still be in use by work queued on `stream`
        cudaStreamSynchronize(stream);
        cudaFree(w.ptr);
        w.ptr = nullptr;
        w.bytes = 0;
    }
    size_t grow = bytes < (size_t(1) << 20) ? (size_t(1) << 20) : bytes;
    if (cudaMalloc(&w.ptr, grow) != cudaSuccess) {
        w.ptr = nullptr;
        return nullptr;
    }
    if (cudaMemsetAsync(w.ptr, 0, grow, stream) != cudaSuccess) return nullptr;
    w.bytes = grow;
    return w.ptr;
}
}  // namespace

int fail(int status, const char *msg) {
    std::snprintf(t_last_error, sizeof t_last_error, "%s", msg);
    return status;
}

int fail_cuda(cudaError_t e, const char *what) {
    std::snprintf(t_last_error, sizeof t_last_error, "%s: %s (%s)", what, cudaGetErrorName(e),
                  cudaGetErrorString(e));
    return e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ? TQK_ENODEV : TQK_ECUDA;
}

int check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TQK_OK : fail_cuda(e, what);
}

const DeviceInfo *device_info() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceInfo &d = g_devices[dev];
    if (d.device < 0) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return nullptr;
        int *err = nullptr;
        if (cudaMalloc(&err, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(err, 0, sizeof(int)) != cudaSuccess) return nullptr;
        d.sm_count = prop.multiProcessorCount;
        d.smem_optin = prop.sharedMemPerBlockOptin;
        d.err_word = err;
        d.device = dev;
    }
    return &d;
}

int ensure_device() {
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetDeviceCount");
    if (n <= 0) return fail(TQK_ENODEV, "no CUDA device");
    if (!device_info()) return fail(TQK_ECUDA, "cannot initialise the current CUDA device");
    return TQK_OK;
}

void *library_workspace(cudaStream_t stream, size_t bytes) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    return grow_zeroed(g_workspaces[{dev, stream}], stream, bytes);
}

int *library_counters(cudaStream_t stream, size_t bytes) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    return static_cast<int *>(grow_zeroed(g_counters[{dev, stream}], stream, bytes));
}

void *library_scratch(cudaStream_t stream, size_t bytes) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    return grow_zeroed(g_scratch[{dev, stream}], stream, bytes);
}

void *library_prefill_stage(cudaStream_t stream, size_t bytes) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    return grow_zeroed(g_prefill_stage[{dev, stream}], stream, bytes);
}

}  // namespace tqk

using namespace tqk;

extern "C" const char *tqk_status_string(int status) {
    switch (status) {
        case TQK_OK: return "ok";
        case TQK_EPOS: return "position out of range";
        case TQK_EINVAL: return "invalid argument";
        case TQK_EALIGN: return "device pointer not 16-byte aligned";
        case TQK_EWORKSPACE: return "workspace too small";
        case TQK_ECUDA: return "CUDA error";
        case TQK_ENODEV: return "no CUDA device";
        case TQK_ETIMEOUT: return "device wait timed out";
        case TQK_EUNSUPPORTED: return "unsupported shape";
        case TQK_EDEVLEN: return "a device-side length was outside [0, max_tokens] and was clamped";
        default: return "unknown status";
    }
}

extern "C" const char *tqk_last_error(void) { return t_last_error; }

extern "C" const char *tqk_version(void) { return "tqk 0.1 sm_100a"; }

extern "C" int tqk_device_status(int *device_error, int clear) {
    int rc = ensure_device();
    if (rc) return rc;
    const DeviceInfo *d = device_info();
    int v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail_cuda(e, "tqk_device_status: synchronize");
    e = cudaMemcpy(&v, d->err_word, sizeof v, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail_cuda(e, "tqk_device_status: read");
    if (clear) {
        e = cudaMemset(d->err_word, 0, sizeof(int));
        if (e != cudaSuccess) return fail_cuda(e, "tqk_device_status: clear");
    }
    if (device_error) *device_error = v;
    return TQK_OK;
}

extern "C" int tqk_device_status_async(int *host_dst, tqk_stream_t stream) {
    if (!host_dst) return fail(TQK_EINVAL, "tqk_device_status_async: NULL destination");
    int rc = ensure_device();
    if (rc) return rc;
    const DeviceInfo *d = device_info();
    if (!d) return fail(TQK_ENODEV, "tqk_device_status_async: no device state");
    const cudaError_t e = cudaMemcpyAsync(host_dst, d->err_word, sizeof(int), cudaMemcpyDeviceToHost,
                                          (cudaStream_t)stream);
    return e == cudaSuccess ? TQK_OK : fail_cuda(e, "tqk_device_status_async");
}

extern "C" int tqk_device_error_status(int device_error) {
    switch (device_error) {
        case 0: return TQK_OK;
        case DEVERR_TIMEOUT: return TQK_ETIMEOUT;
        case DEVERR_BADLEN: return TQK_EDEVLEN;
        default: return TQK_ECUDA;
    }
}

extern "C" int tqk_workspace_init(void *workspace, size_t bytes, tqk_stream_t stream) {
    if (!workspace && bytes) return fail(TQK_EINVAL, "tqk_workspace_init: NULL workspace");
    int rc = ensure_device();
    if (rc) return rc;
    const cudaError_t e = cudaMemsetAsync(workspace, 0, bytes, (cudaStream_t)stream);
    return e == cudaSuccess ? TQK_OK : fail_cuda(e, "tqk_workspace_init");
}
