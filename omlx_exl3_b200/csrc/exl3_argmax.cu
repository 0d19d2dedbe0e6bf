// Greedy token selection of the decode step: per row, the largest of the first n logits and its index
// (the first one on ties), read straight from the head GEMV's fp16 / bf16 / fp32 output.
//
// Replaces the framework's cast-to-fp32 + max-reduction pair at the end of the decode step (the
// reference samples in oMLX's generate loop; this is this package's greedy step). One CTA of 1024
// threads per row: 16-byte loads of the whole row, a (value, index) reduction per thread, then across
// the warps. No scratch.
#include <cuda_runtime.h>

#include <cstdint>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_host.h"

namespace exl3 {

constexpr int kArgThreads = 1024;

__device__ __forceinline__ void arg_better(float& bv, int& bi, float v, int i)
{
    // larger value wins; equal values: smaller index; NaN never wins
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

template <typename T>
__global__ void __launch_bounds__(kArgThreads) argmax_kernel(const T* __restrict__ x, int ld, int n, int index_base,
                                                             float* __restrict__ val, long long* __restrict__ idx)
{
    pdl_trigger();
    pdl_wait();                                      // the logits come from the previous kernel
    __shared__ float sv[kArgThreads / 32];
    __shared__ int si[kArgThreads / 32];
    const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const T* row = x + (size_t)r * ld;
    constexpr int V = 16 / sizeof(T);                // elements per 16-byte load
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    const bool vec = (reinterpret_cast<uintptr_t>(row) % 16) == 0;
    const int nv = vec ? n / V : 0;
    for (int j = tid; j < nv; j += kArgThreads) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(row) + j);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int t = 0; t < V; ++t) arg_better(bv, bi, to_f32(e[t]), j * V + t);
    }
    for (int c = nv * V + tid; c < n; c += kArgThreads) arg_better(bv, bi, to_f32(row[c]), c);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        arg_better(bv, bi, ov, oi);
    }
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < kArgThreads / 32; ++w) arg_better(bv, bi, sv[w], si[w]);
        if (bi == 0x7fffffff) bi = 0;                // every logit NaN: index 0
        val[r] = bv;
        idx[r] = (long long)bi + index_base;
    }
}

}  // namespace exl3

using namespace exl3;

extern "C" int exl3_argmax(const void* x, int dtype, int rows, int ld, int n, int index_base, float* val,
                           long long* idx, void* stream)
{
    if (!x || !val || !idx) return EXL3_E_NULL;
    if (rows < 1 || n < 1 || ld < n) return EXL3_E_SHAPE;
    if (!aligned(val, 4) || !aligned(idx, 8)) return EXL3_E_ALIGN;
    if (int e = check_device()) return e;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (dtype) {
    case EXL3_F16:
        if (int e_ = launch_pdl(argmax_kernel<__half>, rows, kArgThreads, 0, s, static_cast<const __half*>(x), ld, n,
                                index_base, val, idx))
            return e_;
        break;
    case EXL3_BF16:
        if (int e_ = launch_pdl(argmax_kernel<__nv_bfloat16>, rows, kArgThreads, 0, s,
                                static_cast<const __nv_bfloat16*>(x), ld, n, index_base, val, idx))
            return e_;
        break;
    case EXL3_F32:
        if (int e_ = launch_pdl(argmax_kernel<float>, rows, kArgThreads, 0, s, static_cast<const float*>(x), ld, n,
                                index_base, val, idx))
            return e_;
        break;
    default: return EXL3_E_DTYPE;
    }
    return launch_status();
}
