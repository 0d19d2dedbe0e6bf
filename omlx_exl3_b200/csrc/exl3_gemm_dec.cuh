// Pieces shared by the two prefill kernels that decode the trellis into shared memory: the one-CTA
// kernel (exl3_gemm.cu) and the SM-pair kernel (exl3_gemm_pair.cu). A decoder warp writes its tiles'
// exact fp16 weights straight into the K-major, 128-byte-swizzled B tile the tensor core reads.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "exl3_common.cuh"

namespace exl3 {

constexpr int kGemmBN = 128;                  // output columns per CTA
constexpr int kGemmBK = 64;                   // k per pipeline stage (128 bytes of fp16: one swizzle row)
constexpr int kGemmDecWarps = 16;
constexpr int kGemmThreads = 32 * (2 + kGemmDecWarps);
constexpr int kGemmBBytes = kGemmBN * kGemmBK * 2;   // 16 KB
constexpr int kGemmDecDepth = 4;              // trellis k-steps in flight per decoder warp

struct GemmParams {
    const uint32_t* trellis;
    const __half* svh;
    void* y;
    uint32_t* status;
    uint32_t* counters;      // [row tiles][column blocks] arrival tickets of the k split (zero at rest)
    float* partials;         // [row tiles][column blocks][split][BM x 128 fp32, epilogue-thread order]
    int M, k, n, KT, NT, out_dtype;
    int split;               // k parts (grid z); 1 = every CTA runs all of k
};

// ------------------------------------------------------------------------------ decode into B
// Byte offset of (row n, k) inside a K-major 128B-swizzled tile whose rows are 128 bytes (64 fp16):
// 16-byte chunk index XOR (row mod 8), 8-row groups of 1024 bytes.
__device__ __forceinline__ uint32_t sw128_offset(int n, int kbyte)
{
    return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + ((((kbyte >> 4) ^ (n & 7))) << 4) + (kbyte & 15));
}

template <int CB>
__device__ __forceinline__ uint32_t pack_weights(uint32_t sa, uint32_t sb)
{
    if constexpr (CB == 2) {
        return __byte_perm(sa, sb, 0x5410);        // (w_a, w_b): the mul1 split word is (w, 0)
    } else {
        const uint32_t lo = __byte_perm(sa, sb, 0x5410), hi = __byte_perm(sa, sb, 0x7632);
        const __half2 w = __hadd2(*reinterpret_cast<const __half2*>(&lo), *reinterpret_cast<const __half2*>(&hi));
        return *reinterpret_cast<const uint32_t*>(&w);
    }
}

template <typename OT>
__device__ __forceinline__ void store_row64(OT* dst, const float (&v)[64], const __half* svh)
{
#pragma unroll
    for (int c = 0; c < 64; c += 8) {
        if constexpr (sizeof(OT) == 4) {
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[c + i] = from_f32<OT>(v[c + i] * kHadScale * __half2float(svh[c + i]));
        } else {
            uint32_t pk[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const OT a = from_f32<OT>(v[c + 2 * i] * kHadScale * __half2float(svh[c + 2 * i]));
                const OT b = from_f32<OT>(v[c + 2 * i + 1] * kHadScale * __half2float(svh[c + 2 * i + 1]));
                pk[i] = (uint32_t)(*reinterpret_cast<const uint16_t*>(&a)) |
                        ((uint32_t)(*reinterpret_cast<const uint16_t*>(&b)) << 16);
            }
            *reinterpret_cast<uint4*>(dst + c) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
    }
}

// Launch of the SM-pair kernel (exl3_gemm_pair.cu): grid (2 x n / 256, m_tiles, split), `nacc` M=256
// accumulators per pair tile (1: 256 rows, 2: 512 rows); xmap boxes are 64 k x 128 rows.
int launch_gemm_pair(int bits, int codebook, int nacc, const CUtensorMap& xmap, const GemmParams& prm, int m_tiles,
                     cudaStream_t s);

}  // namespace exl3
