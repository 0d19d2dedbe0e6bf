// Tensor-parallel all-reduce fused with its consumer, over NVLink peer memory.
//
// In the decode step every row-parallel projection (o_proj, down_proj) is followed by an all-reduce
// of its (rows x hidden) partial output and then by the residual add + RMSNorm + input rotation of
// the next projection group (exl3_add_norm_rot). Here that is one kernel per rank:
//
//   1. the rank's partial was written by its GEMV straight into its slot of a peer buffer (one
//      cudaMalloc per rank, mapped into every other rank's process with CUDA IPC);
//   2. one thread stores "slot ready for epoch e" into every rank's flag block (plain P2P stores with
//      system-scope release ordering) and every CTA waits, with a time limit, until all ranks have;
//   3. each CTA reads its row of every rank's partial over NVLink (plain loads, L2 only), sums them in
//      rank order in fp32 (every rank computes the identical sum), then does the residual add,
//      RMSNorm (MLX rounding) and the 128-point rotations of exl3_add_norm_rot.
//
// No multicast and no NCCL: the only cross-GPU traffic is the flag stores and the partial reads.
// The epoch is a counter in each rank's own flag block, advanced by the last CTA of every call, so
// the kernel can be captured in a CUDA graph. Slots alternate between calls (the caller passes the
// parity): a rank can only reach the call that rewrites a slot after every rank has finished the
// previous call that reads it, because each call waits for all ranks' flags of the call before it.
// The reference has no counterpart (it runs on one Apple GPU); this replaces the NCCL all-reduce +
// exl3_add_norm_rot pair of this package's tensor-parallel decode step.
#include <cuda_runtime.h>

#include <cstring>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_host.h"

namespace exl3 {

constexpr int kArThreads = 256;
constexpr int kArChunk = 1024;            // output columns per CTA
constexpr int kArVec = 3;                 // 16-byte loads per thread per rank in flight (k <= 6144 in one pass)
enum : uint32_t { kStatusPeerTimeout = 4u };

// flag block (uint32 words): [0, 8) arrival epoch per source rank, [8] epoch of the last completed
// call, [9] CTAs finished in the current call, [10] status bits
constexpr int kFlagEpoch = 8, kFlagDone = 9, kFlagStatus = 10;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// g.base[i] by selects: a runtime index into the parameter struct would copy it to the stack
__device__ __forceinline__ void* peer_base(const exl3_peer_group& g, int i)
{
    void* b = g.base[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) b = i == j ? g.base[j] : b;
    return b;
}

// 8 consecutive values of a row as fp32 (one 16-byte load, L2 only: peer data changes between calls)
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8])
{
    const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = to_f32(e[i]);
}

// One CTA per (row, 1024-column chunk). Every CTA of a row sums the whole row over the ranks (the
// RMSNorm needs the full sum of squares; the extra NVLink reads are a few tens of KB) and writes the
// outputs of its own chunk only.
template <typename T>
__global__ void __launch_bounds__(kArThreads) ar_add_norm_rot_kernel(const exl3_peer_group g, int slot,
                                                                     const T* __restrict__ x,
                                                                     const T* __restrict__ w, float eps,
                                                                     const __half* __restrict__ suh, int nm, int rows,
                                                                     int kd, T* __restrict__ x_out,
                                                                     T* __restrict__ xn, __half* __restrict__ xh)
{
    pdl_trigger();                                   // the next kernel may start launching
    pdl_wait();                                      // inputs written by the previous kernel
    __shared__ float hbuf[kArChunk];                     // the chunk after add, then after norm
    __shared__ float part[kArThreads / 32];
    __shared__ uint32_t s_epoch;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r = blockIdx.y, c0 = blockIdx.x * kArChunk;
    const int cn = min(kArChunk, kd - c0);
    uint32_t* my_flags =
        reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(peer_base(g, g.rank)) + g.flag_off);

    if (tid == 0) {
        const uint32_t e = *reinterpret_cast<volatile uint32_t*>(&my_flags[kFlagEpoch]) + 1u;
        s_epoch = e;
        if (blockIdx.x == 0 && r == 0) {
            __threadfence_system();                      // the partial in our slot before the flags
#pragma unroll
            for (int p = 0; p < 8; ++p)                  // static indices: g stays in the parameter space
                if (p < g.world)
                    st_release_sys(reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(g.base[p]) + g.flag_off) + g.rank, e);
        }
        const uint64_t t0 = global_ns();
        bool ok = true;
        for (int p = 0; p < g.world && ok; ++p) {
            for (uint32_t it = 0; ld_acquire_sys(&my_flags[p]) < e; ++it) {
                if ((it & 63u) == 63u && global_ns() - t0 > 2000000000ull) {
                    atomicOr(&my_flags[kFlagStatus], kStatusPeerTimeout);
                    ok = false;
                    break;
                }
            }
        }
    }
    __syncthreads();

    // whole row: sum of the ranks' partials (rank order, fp32), residual add, sum of squares
    const size_t row_off = (size_t)r * kd;
    const size_t slot_off = g.data_off + (size_t)slot * g.slot_bytes;
    float ss = 0.f;
    for (int v0 = 0; v0 < kd / 8; v0 += kArThreads * kArVec) {
        float acc[kArVec][8];
#pragma unroll
        for (int j = 0; j < kArVec; ++j)
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[j][i] = 0.f;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
            if (p >= g.world) break;
            const T* d = reinterpret_cast<const T*>(static_cast<const uint8_t*>(g.base[p]) + slot_off) + row_off;
            float dv[kArVec][8];
#pragma unroll
            for (int j = 0; j < kArVec; ++j) {              // all loads of this rank before any use
                const int v = v0 + j * kArThreads + tid;
                if (v < kd / 8) load8(d + 8 * v, dv[j]);
            }
#pragma unroll
            for (int j = 0; j < kArVec; ++j)
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[j][i] += dv[j][i];
        }
#pragma unroll
        for (int j = 0; j < kArVec; ++j) {
            const int v = v0 + j * kArThreads + tid;
            if (v >= kd / 8) continue;
            const int c = 8 * v;
            float xv[8];
            load8(x + row_off + c, xv);
            T hv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                hv[i] = from_f32<T>(xv[i] + to_f32(from_f32<T>(acc[j][i])));
                const float hf = to_f32(hv[i]);
                ss = fmaf(hf, hf, ss);
            }
            if (c >= c0 && c < c0 + cn) {
                *reinterpret_cast<uint4*>(x_out + row_off + c) = *reinterpret_cast<const uint4*>(hv);
#pragma unroll
                for (int i = 0; i < 8; ++i) hbuf[c - c0 + i] = to_f32(hv[i]);
            }
        }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) part[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kArThreads / 32; ++i) tot += part[i];
    const float inv = 1.0f / sqrtf(tot / (float)kd + eps);
    for (int c = tid; c < cn; c += kArThreads) {
        const T t = from_f32<T>(hbuf[c] * inv);
        const T o = from_f32<T>(to_f32(w[c0 + c]) * to_f32(t));
        xn[row_off + c0 + c] = o;
        hbuf[c] = to_f32(o);
    }
    __syncthreads();

    // rotations of the chunk's 128-column blocks, every member
    for (int item = warp; item < (cn / 128) * nm; item += kArThreads / 32) {
        const int blk = item % (cn / 128), m = item / (cn / 128);
        const int b0 = blk * 128;
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            v[i] = hbuf[b0 + lane + 32 * i] * __half2float(suh[(size_t)m * kd + c0 + b0 + lane + 32 * i]);
#pragma unroll
        for (int hs = 1; hs < 32; hs <<= 1) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pp = __shfl_xor_sync(0xffffffffu, v[i], hs);
                v[i] = (lane & hs) ? pp - v[i] : v[i] + pp;
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
        __half* o = xh + ((size_t)m * rows + r) * kd + c0 + b0;
#pragma unroll
        for (int i = 0; i < 4; ++i) o[lane + 32 * i] = __float2half_rn(v[i] * kHadScale);
    }

    // the last CTA of the call publishes the epoch for the next call
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t done = atomicAdd(&my_flags[kFlagDone], 1u);
        if (done == gridDim.x * gridDim.y - 1) {
            my_flags[kFlagDone] = 0u;
            __threadfence();
            *reinterpret_cast<volatile uint32_t*>(&my_flags[kFlagEpoch]) = s_epoch;
        }
    }
}

}  // namespace exl3

using namespace exl3;

extern "C" int exl3_peer_create(size_t bytes, void** ptr, void* handle)
{
    if (!ptr || !handle) return EXL3_E_NULL;
    if (bytes < 256) return EXL3_E_SHAPE;
    if (int e = check_device()) return e;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return EXL3_E_CUDA;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        return EXL3_E_CUDA;
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return EXL3_E_CUDA;
    }
    static_assert(sizeof(h) == EXL3_PEER_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return EXL3_OK;
}

extern "C" int exl3_peer_destroy(void* ptr)
{
    if (!ptr) return EXL3_E_NULL;
    return cudaFree(ptr) == cudaSuccess ? EXL3_OK : EXL3_E_CUDA;
}

extern "C" int exl3_peer_open(const void* handle, void** ptr)
{
    if (!handle || !ptr) return EXL3_E_NULL;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return EXL3_E_CUDA;
    *ptr = p;
    return EXL3_OK;
}

extern "C" int exl3_peer_close(void* ptr)
{
    if (!ptr) return EXL3_E_NULL;
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? EXL3_OK : EXL3_E_CUDA;
}

extern "C" int exl3_peer_status(const exl3_peer_group* g, uint32_t* status)
{
    if (!g || !status || !g->base[g->rank]) return EXL3_E_NULL;
    const uint32_t* f = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(g->base[g->rank]) + g->flag_off);
    return cudaMemcpy(status, f + kFlagStatus, sizeof(uint32_t), cudaMemcpyDeviceToHost) == cudaSuccess ? EXL3_OK
                                                                                                   : EXL3_E_CUDA;
}

extern "C" int exl3_ar_add_norm_rot(const exl3_peer_group* g, int slot, const void* x, const void* w, int dtype,
                                    int rows, int k, float eps, const void* suh, int n_members, void* x_out,
                                    void* xn, void* xh, void* stream)
{
    if (!g || !x || !w || !suh || !x_out || !xn || !xh) return EXL3_E_NULL;
    if (g->world < 1 || g->world > 8 || g->rank < 0 || g->rank >= g->world) return EXL3_E_SHAPE;
    for (int p = 0; p < g->world; ++p)
        if (!g->base[p]) return EXL3_E_NULL;
    if (rows < 1 || rows > 8 || k <= 0 || k % 128 || k > 16384 || n_members < 1 || n_members > 3 || slot < 0 ||
        slot > 1)
        return EXL3_E_SHAPE;
    if ((size_t)rows * k * 2 > g->slot_bytes) return EXL3_E_WORKSPACE;
    if (g->flag_off % 64 || g->data_off % 16 || g->slot_bytes % 16) return EXL3_E_ALIGN;
    if (x_out == x) return EXL3_E_SHAPE;
    if (!aligned(x, 16) || !aligned(x_out, 16)) return EXL3_E_ALIGN;
    if (int e = check_device()) return e;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid((k + kArChunk - 1) / kArChunk, rows);
    const __half* sh = static_cast<const __half*>(suh);
    __half* o = static_cast<__half*>(xh);
    switch (dtype) {
    case EXL3_F16:
        if (int e_ = launch_pdl(ar_add_norm_rot_kernel<__half>, grid, kArThreads, 0, s, 
            *g, slot, static_cast<const __half*>(x), static_cast<const __half*>(w), eps, sh, n_members, rows, k,
            static_cast<__half*>(x_out), static_cast<__half*>(xn), o)) return e_;
        break;
    case EXL3_BF16:
        if (int e_ = launch_pdl(ar_add_norm_rot_kernel<__nv_bfloat16>, grid, kArThreads, 0, s, 
            *g, slot, static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), eps, sh,
            n_members, rows, k, static_cast<__nv_bfloat16*>(x_out), static_cast<__nv_bfloat16*>(xn), o)) return e_;
        break;
    default: return EXL3_E_DTYPE;
    }
    return launch_status();
}
