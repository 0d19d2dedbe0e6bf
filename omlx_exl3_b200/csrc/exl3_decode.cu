// Trellis -> W^T fp16 decode, bit-exact with the reference's decode kernel
// (daig/omlx-exl3 src/omlx/exl3/kernels.py:304-351).
//
// One CTA = one 16-column n-tile x up to 64 k-tiles. Each warp decodes whole tiles, one lane per
// eight consecutive stream positions (exl3_common.cuh), into a padded shared-memory strip of
// 16 output rows; the strip then leaves in 16-byte coalesced stores along k.
#include <cuda_runtime.h>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_host.h"

namespace exl3 {

constexpr int kDecKC = 64;                   // k-tiles per CTA
constexpr int kDecRowWords = kDecKC * 8 + 4; // strip row stride in 32-bit words (== 4 mod 32)

template <int K, int CB>
__global__ void __launch_bounds__(256) decode_wt_kernel(const uint32_t* __restrict__ trellis, int KT, int NT,
                                                        int nt0, __half* __restrict__ w)
{
    constexpr int TW = 8 * K;
    __shared__ __align__(16) uint32_t strip[16 * kDecRowWords];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int ntl = blockIdx.x;
    const int kt0 = blockIdx.y * kDecKC;
    const int nkt = min(kDecKC, KT - kt0);
    const LaneWindow<K> lw(lane);

    // The windows of all the warp's tiles are loaded before any is decoded, so their global-memory
    // latencies overlap instead of following one another tile by tile.
    constexpr int kTilesPerWarp = kDecKC / 8;
    uint32_t win[kTilesPerWarp][3];
#pragma unroll
    for (int i = 0; i < kTilesPerWarp; ++i) {
        const int t = warp + 8 * i;
        if (t < nkt) window_words<K>(trellis + ((size_t)(kt0 + t) * NT + nt0 + ntl) * TW, lw, win[i]);
    }
#pragma unroll
    for (int i = 0; i < kTilesPerWarp; ++i) {
        const int t = warp + 8 * i;
        if (t < nkt) {
            // states as the GEMV extracts them (state_at), each decoded bit-exactly (dec1)
            const uint32_t m[2] = {__funnelshift_r(win[i][0], win[i][1], 16), __funnelshift_r(win[i][1], win[i][2], 16)};
            __half d[8];
            d[0] = dec1<CB>(state_at<K, 7 * K>(win[i], m));
            d[1] = dec1<CB>(state_at<K, 6 * K>(win[i], m));
            d[2] = dec1<CB>(state_at<K, 5 * K>(win[i], m));
            d[3] = dec1<CB>(state_at<K, 4 * K>(win[i], m));
            d[4] = dec1<CB>(state_at<K, 3 * K>(win[i], m));
            d[5] = dec1<CB>(state_at<K, 2 * K>(win[i], m));
            d[6] = dec1<CB>(state_at<K, 1 * K>(win[i], m));
            d[7] = dec1<CB>(state_at<K, 0>(win[i], m));
            // position j -> (row g or g+8, k 2q, 2q+1, 2q+8, 2q+9): pairs are adjacent in k
            const int col = t * 8 + q;   // word column of k 2q within this tile's 16 k
            strip[g * kDecRowWords + col] = (uint32_t)__half_as_ushort(d[0]) | ((uint32_t)__half_as_ushort(d[1]) << 16);
            strip[g * kDecRowWords + col + 4] = (uint32_t)__half_as_ushort(d[2]) | ((uint32_t)__half_as_ushort(d[3]) << 16);
            strip[(g + 8) * kDecRowWords + col] = (uint32_t)__half_as_ushort(d[4]) | ((uint32_t)__half_as_ushort(d[5]) << 16);
            strip[(g + 8) * kDecRowWords + col + 4] =
                (uint32_t)__half_as_ushort(d[6]) | ((uint32_t)__half_as_ushort(d[7]) << 16);
        }
    }
    __syncthreads();

    const size_t k = (size_t)KT * 16;
    const int vec_per_row = nkt * 2;            // 16-byte vectors (8 halves) per row
    for (int i = threadIdx.x; i < 16 * vec_per_row; i += 256) {
        const int row = i / vec_per_row, vcol = i - row * vec_per_row;
        const uint4 val = *reinterpret_cast<const uint4*>(&strip[row * kDecRowWords + vcol * 4]);
        *reinterpret_cast<uint4*>(w + ((size_t)ntl * 16 + row) * k + (size_t)kt0 * 16 + vcol * 8) = val;
    }
}

template <int K>
static void launch_decode(int cb, dim3 grid, cudaStream_t s, const uint32_t* t, int KT, int NT, int nt0, __half* w)
{
    switch (cb) {
    case 0: decode_wt_kernel<K, 0><<<grid, 256, 0, s>>>(t, KT, NT, nt0, w); break;
    case 1: decode_wt_kernel<K, 1><<<grid, 256, 0, s>>>(t, KT, NT, nt0, w); break;
    default: decode_wt_kernel<K, 2><<<grid, 256, 0, s>>>(t, KT, NT, nt0, w); break;
    }
}

}  // namespace exl3

extern "C" int exl3_decode_wt(const uint32_t* trellis, int k, int n, int bits, int codebook, int nt0, int ntc,
                              void* w, void* stream)
{
    using namespace exl3;
    if (!trellis || !w) return EXL3_E_NULL;
    if (k <= 0 || n <= 0 || k % 16 || n % 16) return EXL3_E_SHAPE;
    if (bits < 1 || bits > 8) return EXL3_E_BITS;
    if (codebook < 0 || codebook > 2) return EXL3_E_CODEBOOK;
    const int NT = n / 16, KT = k / 16;
    if (ntc < 0) ntc = NT - nt0;
    if (nt0 < 0 || ntc < 0 || nt0 + ntc > NT) return EXL3_E_SHAPE;
    if (ntc == 0) return EXL3_OK;
    if (!aligned(trellis, 4) || !aligned(w, 16)) return EXL3_E_ALIGN;
    if (int e = check_device()) return e;
    const dim3 grid(ntc, (KT + kDecKC - 1) / kDecKC);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    __half* out = static_cast<__half*>(w);
    switch (bits) {
    case 1: launch_decode<1>(codebook, grid, s, trellis, KT, NT, nt0, out); break;
    case 2: launch_decode<2>(codebook, grid, s, trellis, KT, NT, nt0, out); break;
    case 3: launch_decode<3>(codebook, grid, s, trellis, KT, NT, nt0, out); break;
    case 4: launch_decode<4>(codebook, grid, s, trellis, KT, NT, nt0, out); break;
    case 5: launch_decode<5>(codebook, grid, s, trellis, KT, NT, nt0, out); break;
    case 6: launch_decode<6>(codebook, grid, s, trellis, KT, NT, nt0, out); break;
    case 7: launch_decode<7>(codebook, grid, s, trellis, KT, NT, nt0, out); break;
    default: launch_decode<8>(codebook, grid, s, trellis, KT, NT, nt0, out); break;
    }
    return launch_status();
}
