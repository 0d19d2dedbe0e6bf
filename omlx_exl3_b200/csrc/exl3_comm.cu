// Tensor-parallel all-reduce fused with its consumer, over NVLink peer memory.
//
// In the decode step every row-parallel projection (o_proj, down_proj) is followed by an all-reduce
// of its (rows x hidden) partial output and then by the residual add + RMSNorm + input rotation of
// the next projection group (exl3_add_norm_rot). Here that is:
//
//   1. the producer (the row-parallel GEMV, exl3_gemv_peer, or exl3_peer_put) pushes the rank's
//      partial into inbox (slot, rank) of every rank's buffer as LL words (exl3_peer.cuh): P2P stores
//      over NVLink that carry the call's epoch next to the data;
//   2. exl3_ar_add_norm_rot polls only its own buffer until every word of every source rank carries
//      this call's epoch (bounded: 2 s, then a status bit), sums the ranks in rank order in fp32
//      (every rank computes the identical sum), then does the residual add, RMSNorm (MLX rounding) and
//      the 128-point rotations of exl3_add_norm_rot.
//
// One thread-block cluster per row: each CTA of the cluster owns a chunk of the row's columns, so no
// word is read twice, and the CTAs exchange their sums of squares through distributed shared memory.
// The norm weight and the rotation signs are constants, so they are staged into shared memory before
// the dependency wait, overlapping the producer's tail. No multicast and no NCCL: the only cross-GPU
// traffic is the producers' stores. The epoch is a counter in each rank's own flag block, advanced by
// the last CTA of every call, so the kernels can be captured in a CUDA graph. Slots alternate between
// calls (the caller passes the parity): a rank can only push into a slot again after every rank has
// finished the call that read it, because its previous call waited for every rank's data.
// The reference has no counterpart (it runs on one Apple GPU); this replaces the NCCL all-reduce +
// exl3_add_norm_rot pair of this package's tensor-parallel decode step.
#include <cuda_runtime.h>

#include <cstring>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_host.h"
#include "exl3_peer.cuh"

namespace exl3 {

constexpr int kArThreads = 256;
constexpr int kArPairs = 2;               // column pairs per thread per pass

// own buffer by selects: a runtime index into the parameter struct would copy it to the stack
__device__ __forceinline__ void* peer_base(const exl3_peer_group& g, int i)
{
    void* b = g.base[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) b = i == j ? g.base[j] : b;
    return b;
}

__device__ __forceinline__ float ld_cluster_f32(const float* p, uint32_t rank)
{
    uint32_t a, v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_addr(p)), "r"(rank));
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return __uint_as_float(v);
}

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

template <typename T> __device__ __forceinline__ T from_bits16(uint32_t b);
template <> __device__ __forceinline__ __half from_bits16<__half>(uint32_t b) { return __ushort_as_half((unsigned short)b); }
template <> __device__ __forceinline__ __nv_bfloat16 from_bits16<__nv_bfloat16>(uint32_t b)
{
    return __ushort_as_bfloat16((unsigned short)b);
}
template <typename T> __device__ __forceinline__ uint32_t bits16(T v);
template <> __device__ __forceinline__ uint32_t bits16<__half>(__half v) { return __half_as_ushort(v); }
template <> __device__ __forceinline__ uint32_t bits16<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat16_as_ushort(v); }

// grid (C, rows), clusters of C CTAs along x; CTA x owns columns [x * chunk, (x + 1) * chunk).
// Dynamic shared memory: the chunk after add (then after norm) as fp32, w's chunk, each member's suh chunk.
template <typename T>
__global__ void __launch_bounds__(kArThreads) ar_add_norm_rot_kernel(const exl3_peer_group g, int slot,
                                                                     const T* __restrict__ x,
                                                                     const T* __restrict__ w, float eps,
                                                                     const __half* __restrict__ suh, int nm, int rows,
                                                                     int kd, int chunk, T* __restrict__ x_out,
                                                                     T* __restrict__ xn, __half* __restrict__ xh)
{
    extern __shared__ __align__(16) uint8_t ar_smem[];
    float* hbuf = reinterpret_cast<float*>(ar_smem);
    T* wbuf = reinterpret_cast<T*>(hbuf + chunk);
    __half* sbuf = reinterpret_cast<__half*>(wbuf + chunk);
    __shared__ float part[kArThreads / 32];
    __shared__ float cta_ss;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r = blockIdx.y, c0 = blockIdx.x * chunk;
    const uint32_t C = gridDim.x;

    // weights first: they do not depend on the previous kernel
    for (int i = tid; i < chunk / 8; i += kArThreads) cp_async16(wbuf + 8 * i, w + c0 + 8 * i);
    for (int m = 0; m < nm; ++m)
        for (int i = tid; i < chunk / 8; i += kArThreads)
            cp_async16(sbuf + (size_t)m * chunk + 8 * i, suh + (size_t)m * kd + c0 + 8 * i);
    cp_async_commit();

    pdl_trigger();                                   // the next kernel may start launching
    pdl_wait();                                      // inputs written by the previous kernel
    void* own = peer_base(g, g.rank);
    uint32_t* my_flags = peer_flags(own, g);
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(&my_flags[kFlagEpoch]) + 1u;

    // this CTA's pairs of every source rank's inbox (same offsets in each)
    const size_t pair0 = ((size_t)r * kd + c0) / 2;
    const uint64_t* ib[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) ib[p] = peer_inbox(own, g, slot, p < g.world ? p : 0) + pair0;
    const uint32_t* xp = reinterpret_cast<const uint32_t*>(x + (size_t)r * kd + c0);
    uint32_t* xop = reinterpret_cast<uint32_t*>(x_out + (size_t)r * kd + c0);
    const int np = chunk / 2;
    float ss = 0.f;
    for (int j0 = 0; j0 < np; j0 += kArThreads * kArPairs) {
        uint64_t wv[kArPairs][8];
        uint32_t xv[kArPairs];
#pragma unroll
        for (int i = 0; i < kArPairs; ++i) {
            const int j = j0 + i * kArThreads + tid;
            xv[i] = 0u;
#pragma unroll
            for (int p = 0; p < 8; ++p) wv[i][p] = (uint64_t)e << 32;
            if (j < np) {
                xv[i] = xp[j];
#pragma unroll
                for (int p = 0; p < 8; ++p)
                    if (p < g.world) wv[i][p] = ld_ll(ib[p] + j);
            }
        }
        // until every word carries this call's epoch
        uint64_t t0 = 0;
        for (uint32_t it = 0;; ++it) {
            bool all = true;
#pragma unroll
            for (int i = 0; i < kArPairs; ++i) {
                const int j = j0 + i * kArThreads + tid;
#pragma unroll
                for (int p = 0; p < 8; ++p)
                    if (p < g.world && j < np && (uint32_t)(wv[i][p] >> 32) != e) {
                        all = false;
                        wv[i][p] = ld_ll(ib[p] + j);
                    }
            }
            if (all) break;
            if (it == 0) t0 = global_ns();
            if ((it & 31u) == 31u && global_ns() - t0 > 2000000000ull) {
                atomicOr(&my_flags[kFlagStatus], kStatusPeerTimeout);
                break;
            }
        }
#pragma unroll
        for (int i = 0; i < kArPairs; ++i) {
            const int j = j0 + i * kArThreads + tid;
            if (j >= np) continue;
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int p = 0; p < 8; ++p) {
                if (p >= g.world) break;
                const uint32_t d = (uint32_t)wv[i][p];
                s0 += to_f32(from_bits16<T>(d & 0xffffu));
                s1 += to_f32(from_bits16<T>(d >> 16));
            }
            const T h0 = from_f32<T>(to_f32(from_bits16<T>(xv[i] & 0xffffu)) + to_f32(from_f32<T>(s0)));
            const T h1 = from_f32<T>(to_f32(from_bits16<T>(xv[i] >> 16)) + to_f32(from_f32<T>(s1)));
            const float f0 = to_f32(h0), f1 = to_f32(h1);
            ss = fmaf(f0, f0, ss);
            ss = fmaf(f1, f1, ss);
            xop[j] = bits16(h0) | (bits16(h1) << 16);
            hbuf[2 * j] = f0;
            hbuf[2 * j + 1] = f1;
        }
    }
    ss = warp_sum(ss);
    if (lane == 0) part[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < kArThreads / 32; ++i) t += part[i];
        cta_ss = t;
    }
    // every CTA's sum of squares, added in cluster-rank order (the same on every CTA and every rank)
    cluster_arrive();
    cluster_wait();
    float tot = 0.f;
    for (uint32_t q = 0; q < C; ++q) tot += ld_cluster_f32(&cta_ss, q);
    cluster_arrive();                                // this CTA is done reading the others' shared memory
    const float inv = 1.0f / sqrtf(tot / (float)kd + eps);
    cp_async_wait<0>();
    __syncthreads();
    for (int c = tid; c < chunk; c += kArThreads) {
        const T t = from_f32<T>(hbuf[c] * inv);
        const T o = from_f32<T>(to_f32(wbuf[c]) * to_f32(t));
        if (xn) xn[(size_t)r * kd + c0 + c] = o;
        hbuf[c] = to_f32(o);
    }
    __syncthreads();

    // rotations of the chunk's 128-column blocks, every member
    const int nb = chunk / 128;
    for (int item = warp; item < nb * nm; item += kArThreads / 32) {
        const int blk = item % nb, m = item / nb;
        const int b0 = blk * 128;
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            v[i] = hbuf[b0 + lane + 32 * i] * __half2float(sbuf[(size_t)m * chunk + b0 + lane + 32 * i]);
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
        const uint32_t done = atomicAdd(&my_flags[kFlagDone], 1u);
        if (done == gridDim.x * gridDim.y - 1) {
            my_flags[kFlagDone] = 0u;
            *reinterpret_cast<volatile uint32_t*>(&my_flags[kFlagEpoch]) = e;
        }
    }
    cluster_wait();                                  // no CTA leaves while another may read its cta_ss
}

// exl3_peer_put: n pairs of 16-bit values from src into inbox (slot, rank) of every rank.
__global__ void __launch_bounds__(256) peer_put_kernel(const exl3_peer_group g, int slot,
                                                       const uint32_t* __restrict__ src, int n)
{
    pdl_trigger();
    pdl_wait();
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(&peer_flags(peer_base(g, g.rank), g)[kFlagEpoch]) + 1u;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
        const uint32_t v = src[j];
#pragma unroll
        for (int p = 0; p < 8; ++p)
            if (p < g.world) st_ll(peer_inbox(g.base[p], g, slot, g.rank) + j, v, e);
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
    if (!g || !status) return EXL3_E_NULL;
    if (g->rank < 0 || g->rank >= 8) return EXL3_E_SHAPE;
    if (!g->base[g->rank]) return EXL3_E_NULL;
    const uint32_t* f = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(g->base[g->rank]) + g->flag_off);
    return cudaMemcpy(status, f + kFlagStatus, sizeof(uint32_t), cudaMemcpyDeviceToHost) == cudaSuccess ? EXL3_OK
                                                                                                   : EXL3_E_CUDA;
}

extern "C" int exl3_peer_put(const exl3_peer_group* g, int slot, const void* src, int rows, int k, void* stream)
{
    if (int e = check_peer_group(g, slot)) return e;
    if (!src) return EXL3_E_NULL;
    if (rows < 1 || k <= 0 || k % 2) return EXL3_E_SHAPE;
    if ((size_t)rows * k * 4 > g->inbox_bytes) return EXL3_E_WORKSPACE;
    if (!aligned(src, 4)) return EXL3_E_ALIGN;
    if (int e = check_device()) return e;
    const int n = rows * k / 2;
    const int grid = (n + 255) / 256 < 2 * device_sm_count() ? (n + 255) / 256 : 2 * device_sm_count();
    if (int e_ = launch_pdl(peer_put_kernel, grid, 256, 0, static_cast<cudaStream_t>(stream), *g, slot,
                            static_cast<const uint32_t*>(src), n))
        return e_;
    return launch_status();
}

extern "C" int exl3_ar_add_norm_rot(const exl3_peer_group* g, int slot, const void* x, const void* w, int dtype,
                                    int rows, int k, float eps, const void* suh, int n_members, void* x_out,
                                    void* xn, void* xh, void* stream)
{
    if (int e = check_peer_group(g, slot)) return e;
    if (!x || !w || !suh || !x_out || !xh) return EXL3_E_NULL;   // xn may be null
    if (rows < 1 || rows > 8 || k <= 0 || k % 128 || k > 16384 || n_members < 1 || n_members > 3)
        return EXL3_E_SHAPE;
    if ((size_t)rows * k * 4 > g->inbox_bytes) return EXL3_E_WORKSPACE;
    if (x_out == x) return EXL3_E_SHAPE;
    if (!aligned(x, 16) || !aligned(x_out, 16) || !aligned(w, 16) || !aligned(suh, 16)) return EXL3_E_ALIGN;
    if (int e = check_device()) return e;
    // a cluster of C CTAs per row, C the largest of 8, 4, 2, 1 that splits the row into whole blocks
    const int nblk = k / 128;
    const int C = nblk % 8 == 0 ? 8 : (nblk % 4 == 0 ? 4 : (nblk % 2 == 0 ? 2 : 1));
    const int chunk = k / C;
    const size_t smem = (size_t)chunk * (4 + 2 + 2 * n_members);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(C, rows);
    const __half* sh = static_cast<const __half*>(suh);
    __half* o = static_cast<__half*>(xh);
    switch (dtype) {
    case EXL3_F16:
        if (smem > 48 * 1024 && cudaFuncSetAttribute(ar_add_norm_rot_kernel<__half>,
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return EXL3_E_CUDA;
        if (int e_ = launch_pdl_cluster(ar_add_norm_rot_kernel<__half>, grid, kArThreads, smem, C, s, *g, slot,
                                        static_cast<const __half*>(x), static_cast<const __half*>(w), eps, sh,
                                        n_members, rows, k, chunk, static_cast<__half*>(x_out),
                                        static_cast<__half*>(xn), o))
            return e_;
        break;
    case EXL3_BF16:
        if (smem > 48 * 1024 && cudaFuncSetAttribute(ar_add_norm_rot_kernel<__nv_bfloat16>,
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return EXL3_E_CUDA;
        if (int e_ = launch_pdl_cluster(ar_add_norm_rot_kernel<__nv_bfloat16>, grid, kArThreads, smem, C, s, *g,
                                        slot, static_cast<const __nv_bfloat16*>(x),
                                        static_cast<const __nv_bfloat16*>(w), eps, sh, n_members, rows, k, chunk,
                                        static_cast<__nv_bfloat16*>(x_out), static_cast<__nv_bfloat16*>(xn), o))
            return e_;
        break;
    default: return EXL3_E_DTYPE;
    }
    return launch_status();
}
