// Host-side helpers of the C ABI: per-thread error messages, argument checks and kernel launches with programmatic
// dependent launch (PDL), so a kernel's prologue (weight prefetch) overlaps the tail of the kernel before it.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "../../include/espalier_b200.h"

namespace esp {

int set_error(int code, const char* fmt, ...);   // records the message, returns code
bool pdl_enabled();                               // ESPALIER_PDL (default 1): programmatic dependent launch
int ok();                                         // clears the message, returns ESP_OK
int device_sms();                                 // SM count of the current device (cached per device)

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

#define ESP_REQUIRE(cond, code, ...) \
    do {                             \
        if (!(cond)) return ::esp::set_error((code), __VA_ARGS__); \
    } while (0)

inline int cuda_status(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ESP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return ESP_OK;
}

// Launch with the programmatic-stream-serialization attribute: the kernel may start while the previous kernel on the
// stream finishes; it must execute griddepcontrol.wait before touching that kernel's outputs.
template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void* stream, bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = (pdl && pdl_enabled()) ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) return set_error(ESP_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
    return ESP_OK;
}

// The same with a thread-block cluster of `cluster` CTAs along x (cluster > 1; the grid is a multiple of it).
template <typename... KArgs, typename... Args>
int launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void* stream, bool pdl, int cluster,
                   Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = (pdl && pdl_enabled()) ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) return set_error(ESP_ERR_CUDA, "cluster kernel launch: %s", cudaGetErrorString(e));
    return ESP_OK;
}

// Opt a kernel into more than 48 KB of dynamic shared memory (once per kernel).
template <typename K>
int allow_smem(K kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return ESP_OK;
    const cudaError_t e =
        cudaFuncSetAttribute(reinterpret_cast<const void*>(kernel), cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(bytes));
    if (e != cudaSuccess) return set_error(ESP_ERR_CUDA, "shared memory opt-in (%zu B): %s", bytes, cudaGetErrorString(e));
    return ESP_OK;
}

}  // namespace esp
