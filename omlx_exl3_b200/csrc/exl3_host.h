// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

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

}  // namespace exl3
