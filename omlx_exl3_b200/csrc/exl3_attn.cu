// Decode-step glue around the EXL3 linears, fused so a layer is a handful of launches:
//
//   exl3_qkv_post       q/k per-head RMSNorm (MLX rounding), rotary embedding (rotate-half),
//                       k and v written into the fp16 KV cache at each row's position, q out in fp16.
//                       Replaces the per-head norms, RoPE, casts and cache writes of the attention
//                       block (about 20 small framework kernels per layer).
//   exl3_add_norm_rot   residual add fused into the RMSNorm + input-rotation kernel (kernels.py:408-425
//                       norm_rot semantics): x <- x + d (stored), xn = T(w * T(x * rsqrt(mean(x^2)+eps))),
//                       xh[m] = fp16(had128(xn * suh[m]) / sqrt(128)).
//
// One warp per (row, 128-element head or block); lane holds elements lane + 32 i (i = 0..3), so the
// rotate-half partner of element c (< 64) is element c + 64 in the same lane.
#include <cuda_runtime.h>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_host.h"

namespace exl3 {

template <typename T>
__global__ void __launch_bounds__(128) qkv_post_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                       const T* __restrict__ v_in, int sq, int sk, int sv,
                                                       int rows, int hq, int hkv,
                                                       const T* __restrict__ qw, const T* __restrict__ kw, float eps,
                                                       const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                                       const long long* __restrict__ pos, __half* __restrict__ kc,
                                                       __half* __restrict__ vc, int max_len, __half* __restrict__ qout)
{
    pdl_trigger();                                   // the next kernel may start launching
    pdl_wait();                                      // inputs written by the previous kernel
    const int lane = threadIdx.x & 31;
    const int heads = hq + 2 * hkv;
    const int item = blockIdx.x * 4 + (threadIdx.x >> 5);
    if (item >= rows * heads) return;
    const int r = item / heads, hd = item - r * heads;
    const T* src = hd < hq ? q + (size_t)r * sq + (size_t)hd * 128
                 : hd < hq + hkv ? k + (size_t)r * sk + (size_t)(hd - hq) * 128
                                 : v_in + (size_t)r * sv + (size_t)(hd - hq - hkv) * 128;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = to_f32(src[lane + 32 * i]);
    const long long p = pos[r];
    const float* cs = cos_t + (size_t)p * 64;
    const float* sn = sin_t + (size_t)p * 64;
    if (hd < hq) {                                   // query head
        head_rms<T>(v, qw, eps, lane);
        rope_half(v, cs, sn, lane);
        __half* o = qout + ((size_t)r * hq + hd) * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) o[lane + 32 * i] = __float2half_rn(to_f32(from_f32<T>(v[i])));
    } else if (hd < hq + hkv) {                      // key head: norm, rope, cache
        head_rms<T>(v, kw, eps, lane);
        rope_half(v, cs, sn, lane);
        __half* o = kc + ((size_t)(hd - hq) * max_len + p) * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) o[lane + 32 * i] = __float2half_rn(to_f32(from_f32<T>(v[i])));
    } else {                                         // value head: cache
        __half* o = vc + ((size_t)(hd - hq - hkv) * max_len + p) * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) o[lane + 32 * i] = __float2half_rn(v[i]);
    }
}

// One CTA per (row, group of 8 column blocks), as norm_rot. Every CTA of a row reads the whole row
// of x and d for the sum of squares, so the new residual goes to a separate buffer x_out (x_out must
// not alias x or d). A warp issues every load of its own block (x, d, w, each member's suh) before
// the row reduction, so their latency overlaps it. xn may be null (not stored).
template <typename T>
__global__ void __launch_bounds__(256) add_norm_rot_kernel(const T* __restrict__ x, const T* __restrict__ d,
                                                           const T* __restrict__ w, float eps,
                                                           const __half* __restrict__ suh, int nm, int rows, int kd,
                                                           T* __restrict__ x_out, T* __restrict__ xn,
                                                           __half* __restrict__ xh)
{
    pdl_trigger();                                   // the next kernel may start launching
    pdl_wait();                                      // inputs written by the previous kernel
    __shared__ float part[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r = blockIdx.y;
    const T* xr = x + (size_t)r * kd;
    const T* dr = d + (size_t)r * kd;
    const int blk = blockIdx.x * 8 + warp;
    const bool active = blk < kd / 128;
    const int c0 = blk * 128;
    float xs[4], ds[4], ws[4], su[3][4];
    if (active) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = c0 + lane + 32 * i;
            xs[i] = to_f32(xr[c]);
            ds[i] = to_f32(dr[c]);
            ws[i] = to_f32(w[c]);
        }
#pragma unroll
        for (int m = 0; m < 3; ++m)
            if (m < nm)
#pragma unroll
                for (int i = 0; i < 4; ++i) su[m][i] = __half2float(suh[(size_t)m * kd + c0 + lane + 32 * i]);
    }
    float ss = row_sumsq<T>(xr, dr, kd, threadIdx.x, 256);
    ss = warp_sum(ss);
    if (lane == 0) part[warp] = ss;
    __syncthreads();
    if (!active) return;
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += part[i];
    const float inv = 1.0f / sqrtf(tot / (float)kd + eps);
    float xv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = c0 + lane + 32 * i;
        const T s = from_f32<T>(xs[i] + ds[i]);
        const T t = from_f32<T>(to_f32(s) * inv);
        const T o = from_f32<T>(ws[i] * to_f32(t));
        x_out[(size_t)r * kd + c] = s;
        if (xn) xn[(size_t)r * kd + c] = o;
        xv[i] = to_f32(o);
    }
#pragma unroll
    for (int m = 0; m < 3; ++m) {
        if (m >= nm) break;
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = xv[i] * su[m][i];
#pragma unroll
        for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pp = __shfl_xor_sync(0xffffffffu, v[i], h);
                v[i] = (lane & h) ? pp - v[i] : v[i] + pp;
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
        __half* o = xh + ((size_t)m * rows + r) * kd + c0;
#pragma unroll
        for (int i = 0; i < 4; ++i) o[lane + 32 * i] = __float2half_rn(v[i] * kHadScale);
    }
}

}  // namespace exl3

using namespace exl3;

extern "C" int exl3_qkv_post(const void* q, const void* k, const void* v, int q_stride, int k_stride, int v_stride,
                             int dtype, int rows, int hq, int hkv, const void* q_norm_w, const void* k_norm_w, float eps,
                             const float* cos_table, const float* sin_table, const long long* pos, void* k_cache,
                             void* v_cache, int max_len, void* q_out, void* stream)
{
    if (!q || !k || !v || !q_norm_w || !k_norm_w || !cos_table || !sin_table || !pos || !k_cache || !v_cache || !q_out)
        return EXL3_E_NULL;
    if (rows < 1 || hq < 1 || hkv < 1 || max_len < 1) return EXL3_E_SHAPE;
    if (int e = check_device()) return e;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int items = rows * (hq + 2 * hkv);
    const int grid = (items + 3) / 4;
    __half* kc = static_cast<__half*>(k_cache);
    __half* vc = static_cast<__half*>(v_cache);
    __half* qo = static_cast<__half*>(q_out);
    switch (dtype) {
    case EXL3_F16:
        if (int e_ = launch_pdl(qkv_post_kernel<__half>, grid, 128, 0, s, static_cast<const __half*>(q), static_cast<const __half*>(k),
                                                     static_cast<const __half*>(v), q_stride, k_stride, v_stride,
                                                     rows, hq, hkv,
                                                     static_cast<const __half*>(q_norm_w),
                                                     static_cast<const __half*>(k_norm_w), eps, cos_table, sin_table,
                                                     pos, kc, vc, max_len, qo)) return e_;
        break;
    case EXL3_BF16:
        if (int e_ = launch_pdl(qkv_post_kernel<__nv_bfloat16>, grid, 128, 0, s, 
            static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
            static_cast<const __nv_bfloat16*>(v), q_stride, k_stride, v_stride, rows, hq, hkv, static_cast<const __nv_bfloat16*>(q_norm_w),
            static_cast<const __nv_bfloat16*>(k_norm_w), eps, cos_table, sin_table, pos, kc, vc, max_len, qo)) return e_;
        break;
    default: return EXL3_E_DTYPE;
    }
    return launch_status();
}

extern "C" int exl3_add_norm_rot(const void* x, const void* d, const void* w, int dtype, int rows, int k, float eps,
                                 const void* suh, int n_members, void* x_out, void* xn, void* xh, void* stream)
{
    if (!x || !d || !w || !suh || !x_out || !xh) return EXL3_E_NULL;   // xn may be null
    if (rows < 1 || k <= 0 || k % 128 || n_members < 1 || n_members > 3) return EXL3_E_SHAPE;
    if (x_out == x || x_out == d) return EXL3_E_SHAPE;
    if (int e = check_device()) return e;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid((k / 128 + 7) / 8, rows);
    const __half* sh = static_cast<const __half*>(suh);
    __half* o = static_cast<__half*>(xh);
    switch (dtype) {
    case EXL3_F16:
        if (int e_ = launch_pdl(add_norm_rot_kernel<__half>, grid, 256, 0, s, 
            static_cast<const __half*>(x), static_cast<const __half*>(d), static_cast<const __half*>(w), eps, sh,
            n_members, rows, k, static_cast<__half*>(x_out), static_cast<__half*>(xn), o)) return e_;
        break;
    case EXL3_BF16:
        if (int e_ = launch_pdl(add_norm_rot_kernel<__nv_bfloat16>, grid, 256, 0, s, 
            static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(d),
            static_cast<const __nv_bfloat16*>(w), eps, sh, n_members, rows, k, static_cast<__nv_bfloat16*>(x_out),
            static_cast<__nv_bfloat16*>(xn), o)) return e_;
        break;
    default: return EXL3_E_DTYPE;
    }
    return launch_status();
}
