// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <utility>

#include "exl3_b200.h"

namespace exl3 {

// SM count of the current device (cached per device id).
int device_sm_count();

// 0 when the current device is compute capability 10.x, else EXL3_E_DEVICE.
int check_device();

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int launch_status()
{
    return cudaGetLastError() == cudaSuccess ? EXL3_OK : EXL3_E_CUDA;
}

// Programmatic dependent launch (on unless EXL3_PDL=0): the kernel may start while the previous
// kernel in the stream is still running; it runs its independent prologue (the GEMV's first weight
// loads), then waits in griddepcontrol.wait until the previous kernel has completed and its writes
// are visible. Every kernel of this library that is launched this way makes that wait before it
// touches anything the previous kernel may write or read.
inline bool pdl_enabled()
{
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("EXL3_PDL");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) == cudaSuccess ? EXL3_OK : EXL3_E_CUDA;
}

// launch_pdl with thread-block clusters of cluster_x CTAs along x (grid.x a multiple of cluster_x).
template <typename... KArgs, typename... Args>
inline int launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster_x,
                              cudaStream_t s, Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster_x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) == cudaSuccess ? EXL3_OK : EXL3_E_CUDA;
}

}  // namespace exl3
