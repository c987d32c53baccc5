// tqk_internal.h -- host-side runtime shared by the tqk_*.cu translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "tqk_common.cuh"

namespace tqk {

// Records `msg` as the calling thread's last error and returns `status`.
int fail(int status, const char *msg);
// Maps a CUDA error to TQK_ECUDA with a message naming `what`.
int fail_cuda(cudaError_t e, const char *what);
// Checks the launch that was just issued (configuration errors only; async).
int check_launch(const char *what);
// Makes sure a CUDA device is usable from this thread; TQK_ENODEV otherwise.
int ensure_device();

struct DeviceInfo {
    int device = -1;
    int sm_count = 0;
    size_t smem_optin = 0;  // max dynamic shared memory per block
    int *err_word = nullptr;  // sticky device error word (device memory)
};
// Cached properties of the current device (initialised on first use).
const DeviceInfo *device_info();

// Library-owned decode partials buffer for (current device, stream), grown on
// demand and zeroed when (re)allocated.  Returns nullptr on allocation failure.
void *library_workspace(cudaStream_t stream, size_t bytes);
// Library-owned split-merge tickets for (current device, stream): a buffer that
// holds nothing but tickets, zeroed when (re)allocated; every completed decode
// leaves its tickets at zero, so the buffer stays zero between calls.
int *library_counters(cudaStream_t stream, size_t bytes);
// Library-owned staging buffer per (device, stream) for intermediate rows that
// one call produces and consumes (e.g. quantised activations); grows on demand.
void *library_scratch(cudaStream_t stream, size_t bytes);
// Library-owned buffer per (device, stream) for the prefill's staged K/V tiles
// (MMA-ready images of the cache rows, written and read within one call).
void *library_prefill_stage(cudaStream_t stream, size_t bytes);

// Launches `kernel` with programmatic stream serialization, so that it may
// start while the previous kernel of the stream finishes (the kernel must call
// grid_dependency_wait before it reads anything that kernel wrote).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
    if (e != cudaSuccess) return fail_cuda(e, "kernel launch");
    return check_launch("kernel launch");
}

// launch_pdl with thread-block clusters of (cluster_x, 1, 1) CTAs.
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       unsigned cluster_x, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
    if (e != cudaSuccess) return fail_cuda(e, "kernel launch (cluster)");
    return check_launch("kernel launch (cluster)");
}

// Tensor-core prefill attention over the chunk [pos0, pos0 + n) whose K/V rows
// are already in the planes (tqk_prefill.cu).  TQK_EUNSUPPORTED for shapes it
// does not cover (the caller then uses the decode kernel).
int prefill_attend_tc(const tqk_block_q8 *k_plane, const tqk_block_q8 *v_plane, int n_q_heads, int n_kv_heads,
                      int head_dim, int max_tokens, int pos0, int n, const float *q, float *out, cudaStream_t stream);

}  // namespace tqk
