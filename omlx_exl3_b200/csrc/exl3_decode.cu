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

    for (int t = warp; t < nkt; t += 8) {
        const uint32_t* tile = trellis + ((size_t)(kt0 + t) * NT + nt0 + ntl) * TW;
        const Window96<K> v = load_window<K>(tile, lw);
        __half d[8];
        d[0] = dec1<CB>(lane_state<K, 0>(v));
        d[1] = dec1<CB>(lane_state<K, 1>(v));
        d[2] = dec1<CB>(lane_state<K, 2>(v));
        d[3] = dec1<CB>(lane_state<K, 3>(v));
        d[4] = dec1<CB>(lane_state<K, 4>(v));
        d[5] = dec1<CB>(lane_state<K, 5>(v));
        d[6] = dec1<CB>(lane_state<K, 6>(v));
        d[7] = dec1<CB>(lane_state<K, 7>(v));
        // position j -> (row g or g+8, k 2q, 2q+1, 2q+8, 2q+9): pairs are adjacent in k
        const int col = t * 8 + q;   // word column of k 2q within this tile's 16 k
        strip[g * kDecRowWords + col] = (uint32_t)__half_as_ushort(d[0]) | ((uint32_t)__half_as_ushort(d[1]) << 16);
        strip[g * kDecRowWords + col + 4] = (uint32_t)__half_as_ushort(d[2]) | ((uint32_t)__half_as_ushort(d[3]) << 16);
        strip[(g + 8) * kDecRowWords + col] = (uint32_t)__half_as_ushort(d[4]) | ((uint32_t)__half_as_ushort(d[5]) << 16);
        strip[(g + 8) * kDecRowWords + col + 4] = (uint32_t)__half_as_ushort(d[6]) | ((uint32_t)__half_as_ushort(d[7]) << 16);
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
