// Decode-path input rotations: xh = fp16(had128(x * suh) / sqrt(128)) for 1..3 members, alone
// (rot), fused with the RMSNorm that produces x (norm_rot), or fused with SwiGLU (swiglu_rot).
// Replaces daig/omlx-exl3 src/omlx/exl3/kernels.py:354-483.
//
// One warp rotates one 128-element block of one row: lane holds columns lane + 32 i (i = 0..3),
// butterflies h = 1..16 go through shuffles and h = 32, 64 stay in registers. The stage order
// (h = 1, 2, ..., 64) and the butterfly (lower a0 + a1, upper a0 - a1) are the reference's, so for
// equal fp32 inputs the rotated values are bit-identical.
#include <cuda_runtime.h>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_host.h"

namespace exl3 {

__device__ __forceinline__ void fwht128_warp(float (&v)[4], int lane)
{
#pragma unroll
    for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float p = __shfl_xor_sync(0xffffffffu, v[i], h);
            v[i] = (lane & h) ? p - v[i] : v[i] + p;
        }
    }
    float a0 = v[0], a1 = v[1];
    v[0] = a0 + a1; v[1] = a0 - a1;
    a0 = v[2]; a1 = v[3];
    v[2] = a0 + a1; v[3] = a0 - a1;
    a0 = v[0]; a1 = v[2];
    v[0] = a0 + a1; v[2] = a0 - a1;
    a0 = v[1]; a1 = v[3];
    v[1] = a0 + a1; v[3] = a0 - a1;
}

// Rotate the row block held in xv for every member and store fp16 xh (member-major).
__device__ __forceinline__ void rotate_members(const float (&xv)[4], int lane, const __half* suh, int nm, int kd,
                                               int rows, int r, int c0, __half* xh)
{
    for (int m = 0; m < nm; ++m) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = xv[i] * __half2float(suh[(size_t)m * kd + c0 + lane + 32 * i]);
        fwht128_warp(v, lane);
        __half* o = xh + ((size_t)m * rows + r) * kd + c0;
#pragma unroll
        for (int i = 0; i < 4; ++i) o[lane + 32 * i] = __float2half_rn(v[i] * kHadScale);
    }
}

template <typename T>
__global__ void __launch_bounds__(128) rot_kernel(const T* __restrict__ x, const __half* __restrict__ suh, int nm,
                                                  int rows, int kd, __half* __restrict__ xh)
{
    pdl_trigger();                                   // the next kernel may start launching
    pdl_wait();                                      // inputs written by the previous kernel
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * 4 + (threadIdx.x >> 5);   // (row, block)
    const int nblk = kd / 128;
    if (item >= rows * nblk) return;
    const int r = item / nblk, c0 = (item - r * nblk) * 128;
    float xv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) xv[i] = to_f32(x[(size_t)r * kd + c0 + lane + 32 * i]);
    rotate_members(xv, lane, suh, nm, kd, rows, r, c0, xh);
}

// One CTA per (row, group of 8 column blocks). Each CTA recomputes the row's sum of squares
// (fp32, fixed order) so that the row can be split across CTAs without a second launch.
template <typename T>
__global__ void __launch_bounds__(256) norm_rot_kernel(const T* __restrict__ x, const T* __restrict__ w, float eps,
                                                       const __half* __restrict__ suh, int nm, int rows, int kd,
                                                       T* __restrict__ xn, __half* __restrict__ xh)
{
    pdl_trigger();                                   // the next kernel may start launching
    pdl_wait();                                      // inputs written by the previous kernel
    __shared__ float part[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = blockIdx.y;
    const T* xr = x + (size_t)r * kd;
    float ss = row_sumsq<T>(xr, nullptr, kd, threadIdx.x, 256);
#pragma unroll
    for (int h = 16; h >= 1; h >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, h);
    if (lane == 0) part[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += part[i];
    const float inv = 1.0f / sqrtf(tot / (float)kd + eps);

    const int nblk = kd / 128;
    const int blk = blockIdx.x * 8 + warp;
    if (blk >= nblk) return;
    const int c0 = blk * 128;
    float xv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = c0 + lane + 32 * i;
        const T t = from_f32<T>(to_f32(xr[c]) * inv);
        const T o = from_f32<T>(to_f32(w[c]) * to_f32(t));
        xn[(size_t)r * kd + c] = o;
        xv[i] = to_f32(o);
    }
    rotate_members(xv, lane, suh, nm, kd, rows, r, c0, xh);
}

template <typename T>
__global__ void __launch_bounds__(128) swiglu_rot_kernel(const T* __restrict__ gu, const __half* __restrict__ suh,
                                                         int rows, int n, __half* __restrict__ xh)
{
    pdl_trigger();                                   // the next kernel may start launching
    pdl_wait();                                      // inputs written by the previous kernel
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int nblk = n / 128;
    if (item >= rows * nblk) return;
    const int r = item / nblk, c0 = (item - r * nblk) * 128;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = c0 + lane + 32 * i;
        const float gv = to_f32(gu[(size_t)r * 2 * n + c]);
        const float uv = to_f32(gu[(size_t)r * 2 * n + n + c]);
        v[i] = gv / (1.0f + expf(-gv)) * uv * __half2float(suh[c]);
    }
    fwht128_warp(v, lane);
    __half* o = xh + (size_t)r * n + c0;
#pragma unroll
    for (int i = 0; i < 4; ++i) o[lane + 32 * i] = __float2half_rn(v[i] * kHadScale);
}

// Output rotation of the prefill path: out = OT(had128(y) / sqrt(128) * svh) (linear.py:105).
template <typename T, typename OT>
__global__ void __launch_bounds__(128) had_svh_kernel(const T* __restrict__ y, const __half* __restrict__ svh,
                                                      int rows, int n, OT* __restrict__ out)
{
    pdl_trigger();                                   // the next kernel may start launching
    pdl_wait();                                      // inputs written by the previous kernel
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int nblk = n / 128;
    if (item >= rows * nblk) return;
    const int r = item / nblk, c0 = (item - r * nblk) * 128;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = to_f32(y[(size_t)r * n + c0 + lane + 32 * i]);
    fwht128_warp(v, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = c0 + lane + 32 * i;
        out[(size_t)r * n + c] = from_f32<OT>(v[i] * kHadScale * __half2float(svh[c]));
    }
}

template <typename T>
static int launch_had_svh(const void* y, int rows, int n, const __half* svh, void* out, int out_dtype, int grid,
                          cudaStream_t s)
{
    const T* yy = static_cast<const T*>(y);
    switch (out_dtype) {
    case EXL3_F16: if (int e_ = launch_pdl(had_svh_kernel<T, __half>, grid, 128, 0, s, yy, svh, rows, n, static_cast<__half*>(out))) return e_; break;
    case EXL3_BF16:
        if (int e_ = launch_pdl(had_svh_kernel<T, __nv_bfloat16>, grid, 128, 0, s, yy, svh, rows, n, static_cast<__nv_bfloat16*>(out))) return e_;
        break;
    case EXL3_F32: if (int e_ = launch_pdl(had_svh_kernel<T, float>, grid, 128, 0, s, yy, svh, rows, n, static_cast<float*>(out))) return e_; break;
    default: return EXL3_E_DTYPE;
    }
    return launch_status();
}

}  // namespace exl3

using namespace exl3;

extern "C" int exl3_had_svh(const void* y, int y_dtype, int rows, int n, const void* svh, void* out, int out_dtype,
                            void* stream)
{
    if (!y || !svh || !out) return EXL3_E_NULL;
    if (rows < 1 || n <= 0 || n % 128) return EXL3_E_SHAPE;
    if (int e = check_device()) return e;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int grid = (rows * (n / 128) + 3) / 4;
    const __half* sv = static_cast<const __half*>(svh);
    switch (y_dtype) {
    case EXL3_F16: return launch_had_svh<__half>(y, rows, n, sv, out, out_dtype, grid, s);
    case EXL3_BF16: return launch_had_svh<__nv_bfloat16>(y, rows, n, sv, out, out_dtype, grid, s);
    case EXL3_F32: return launch_had_svh<float>(y, rows, n, sv, out, out_dtype, grid, s);
    default: return EXL3_E_DTYPE;
    }
}

extern "C" int exl3_rot(const void* x, int x_dtype, int rows, int k, const void* suh, int n_members, void* xh,
                        void* stream)
{
    if (!x || !suh || !xh) return EXL3_E_NULL;
    if (rows < 1 || k <= 0 || k % 128 || n_members < 1 || n_members > 3) return EXL3_E_SHAPE;
    if (int e = check_device()) return e;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int items = rows * (k / 128);
    const int grid = (items + 3) / 4;
    const __half* sh = static_cast<const __half*>(suh);
    __half* o = static_cast<__half*>(xh);
    switch (x_dtype) {
    case EXL3_F16: if (int e_ = launch_pdl(rot_kernel<__half>, grid, 128, 0, s, static_cast<const __half*>(x), sh, n_members, rows, k, o)) return e_; break;
    case EXL3_BF16:
        if (int e_ = launch_pdl(rot_kernel<__nv_bfloat16>, grid, 128, 0, s, static_cast<const __nv_bfloat16*>(x), sh, n_members, rows, k, o)) return e_;
        break;
    case EXL3_F32: if (int e_ = launch_pdl(rot_kernel<float>, grid, 128, 0, s, static_cast<const float*>(x), sh, n_members, rows, k, o)) return e_; break;
    default: return EXL3_E_DTYPE;
    }
    return launch_status();
}

extern "C" int exl3_norm_rot(const void* x, const void* w, int dtype, int rows, int k, float eps, const void* suh,
                             int n_members, void* xn, void* xh, void* stream)
{
    if (!x || !w || !suh || !xn || !xh) return EXL3_E_NULL;
    if (rows < 1 || k <= 0 || k % 128 || n_members < 1 || n_members > 3) return EXL3_E_SHAPE;
    if (int e = check_device()) return e;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid((k / 128 + 7) / 8, rows);
    const __half* sh = static_cast<const __half*>(suh);
    __half* o = static_cast<__half*>(xh);
    switch (dtype) {
    case EXL3_F16:
        if (int e_ = launch_pdl(norm_rot_kernel<__half>, grid, 256, 0, s, static_cast<const __half*>(x), static_cast<const __half*>(w), eps,
                                                     sh, n_members, rows, k, static_cast<__half*>(xn), o)) return e_;
        break;
    case EXL3_BF16:
        if (int e_ = launch_pdl(norm_rot_kernel<__nv_bfloat16>, grid, 256, 0, s, 
            static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), eps, sh, n_members, rows, k,
            static_cast<__nv_bfloat16*>(xn), o)) return e_;
        break;
    default: return EXL3_E_DTYPE;
    }
    return launch_status();
}

extern "C" int exl3_swiglu_rot(const void* gu, int gu_dtype, int rows, int n, const void* suh, void* xh, void* stream)
{
    if (!gu || !suh || !xh) return EXL3_E_NULL;
    if (rows < 1 || n <= 0 || n % 128) return EXL3_E_SHAPE;
    if (int e = check_device()) return e;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int items = rows * (n / 128);
    const int grid = (items + 3) / 4;
    const __half* sh = static_cast<const __half*>(suh);
    __half* o = static_cast<__half*>(xh);
    switch (gu_dtype) {
    case EXL3_F16: if (int e_ = launch_pdl(swiglu_rot_kernel<__half>, grid, 128, 0, s, static_cast<const __half*>(gu), sh, rows, n, o)) return e_; break;
    case EXL3_BF16:
        if (int e_ = launch_pdl(swiglu_rot_kernel<__nv_bfloat16>, grid, 128, 0, s, static_cast<const __nv_bfloat16*>(gu), sh, rows, n, o)) return e_;
        break;
    case EXL3_F32: if (int e_ = launch_pdl(swiglu_rot_kernel<float>, grid, 128, 0, s, static_cast<const float*>(gu), sh, rows, n, o)) return e_; break;
    default: return EXL3_E_DTYPE;
    }
    return launch_status();
}
