// C-ABI utilities: status strings, version, device queries.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "exl3_b200.h"
#include "exl3_host.h"

namespace exl3 {

int device_sm_count()
{
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
    if (dev < 64 && cached[dev]) return cached[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev < 64) cached[dev] = n;
    return n;
}

int check_device()
{
    static int cached[64] = {0};   // 1 ok, 2 bad
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return EXL3_E_CUDA;
    if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev] == 1 ? EXL3_OK : EXL3_E_DEVICE;
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return EXL3_E_CUDA;
    const int ok = major == 10;
    if (dev >= 0 && dev < 64) cached[dev] = ok ? 1 : 2;
    return ok ? EXL3_OK : EXL3_E_DEVICE;
}

}  // namespace exl3

PFN_cuTensorMapEncodeTiled_v12000 exl3_get_tensormap_encoder()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

extern "C" const char* exl3_strerror(int status)
{
    switch (status) {
    case EXL3_OK: return "ok";
    case EXL3_E_SHAPE: return "shape out of range or not a required multiple";
    case EXL3_E_BITS: return "bits per weight must be in 1..8";
    case EXL3_E_CODEBOOK: return "codebook must be 0 (3inst), 1 (mcg) or 2 (mul1)";
    case EXL3_E_DTYPE: return "unsupported dtype";
    case EXL3_E_ALIGN: return "pointer not aligned as required";
    case EXL3_E_NULL: return "required pointer is NULL";
    case EXL3_E_CUDA: return "CUDA launch or attribute call failed";
    case EXL3_E_WORKSPACE: return "scratch workspace too small";
    case EXL3_E_DEVICE: return "device is not an sm_100 (B200-class) GPU";
    default: return "unknown status";
    }
}

extern "C" int exl3_version(void) { return (1 << 16) | 0; }
