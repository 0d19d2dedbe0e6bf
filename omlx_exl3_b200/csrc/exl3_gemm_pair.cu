// EXL3 prefill GEMM with the trellis decoded in shared memory, on pairs of SMs (a cluster of two CTAs,
// tcgen05 cta_group::2): y = had128(xh @ W) / sqrt(128) * svh, the same product as exl3_gemm.cu's
// one-CTA kernel, for outputs whose width is a multiple of 256.
//
// Pair tile: NACC x 256 rows x 256 output columns (two Hadamard blocks), k-steps of 64. The pair's MMA
// (M=256, N=256, K=16) reads 128 rows of xh and 128 columns of W from each CTA's shared memory, so a
// CTA stages NACC x 16 KB of xh and 16 KB of decoded weights per k-step: half of what the one-CTA
// kernel's 512-row tile needs, which leaves room for 4-6 stages instead of 2 (the one-CTA kernel's
// decoders and TMA loads wait on its two stages). Each weight is still decoded once per NACC x 256 rows,
// each CTA decoding its own 128 columns. Per CTA:
//   - warp 0 (one lane): TMA loads of its NACC 128-row halves of xh, counted on the leader's "full"
//     barrier (no multicast);
//   - warp 1 of the leader (one lane): per stage 4 x NACC tcgen05.mma, committed to both CTAs' "empty"
//     barriers;
//   - warps 2..17: decode the CTA's 4 x 8 trellis tiles of the step into its B half (exl3_gemm_dec.cuh),
//     arrive on the leader's "decoded" barrier, then run the epilogue on the CTA's accumulator rows
//     (128 per M=256 accumulator, all 256 columns): FWHT stages 1..32 in registers, stage 64 through
//     shared memory, * 1/sqrt(128) * svh, store; or, with a k split, the partial / ticket / ordered sum
//     of exl3_gemm.cu.
// All waits are bounded polls (exl3_tc.cuh mbar_wait_pair): a lost completion sets a status bit.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_gemm_dec.cuh"
#include "exl3_host.h"
#include "exl3_tc.cuh"

namespace exl3 {

// Shared memory: [barriers, 1 KB][stages: A (NACC x 16 KB) + B (16 KB) each][decoder rings]; the
// epilogue's exchange buffer (2 column blocks x 128 rows x 129 floats) reuses stages + rings.
template <int NACC>
struct PairTile {
    static constexpr int ABYTES = NACC * 128 * kGemmBK * 2;
    static constexpr int SBYTES = ABYTES + kGemmBBytes;
    static constexpr int STAGES = NACC == 2 ? 4 : 6;
    static constexpr int RING = kGemmDecWarps * kGemmDecDepth * 2 * 256;
    static constexpr int SMEM = 1024 + 1024 + STAGES * SBYTES + RING;
    static constexpr int TMEM_COLS = NACC * 256;
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(2 * 128 * 129 * 4 <= STAGES * SBYTES + RING, "epilogue exchange buffer");
    static_assert(3 * STAGES * 8 + 8 + 12 <= 1024, "barrier area");
};

// Warps 2..17 of both CTAs: decode this CTA's 128 columns of every k-step into its B half, then the
// epilogue on the CTA's accumulator rows.
template <int K, int CB, int NACC>
__device__ __forceinline__ void pair_decode_and_finish(const GemmParams& p, uint8_t* stages, uint8_t* rings,
                                                       uint64_t* decoded, uint64_t* empty, uint64_t* accum,
                                                       uint32_t* words, uint32_t tmem, uint32_t rank, int pair_n,
                                                       int nb, int m0, int s0, int nsteps)
{
    using TL = PairTile<NACC>;
    constexpr int S = TL::STAGES;
    constexpr int TW = 8 * K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int dw = warp - 2;                        // 0..15
    const int g = lane >> 2, q = lane & 3;
    const LaneWindow<K> lw(lane);
    const HashRegs hr = hash_regs<CB>();
    // warp dw decodes k-slice dw / 4 and the two n-tiles 2 * (dw % 4) + {0, 1} of the CTA's block
    constexpr int kTiles = 2;
    const int ktl = dw >> 2, nt_base = (dw & 3) * kTiles;
    uint32_t* dring = reinterpret_cast<uint32_t*>(rings) + (size_t)dw * kGemmDecDepth * kTiles * TW;
    const uint32_t dec0 = cluster_addr(decoded, 0);
    int fstep = 0, fslot = 0, cslot = 0;
    const uint32_t* tsrc =
        p.trellis + ((size_t)(s0 * (kGemmBK / 16) + ktl) * p.NT + (size_t)nb * 8 + nt_base) * TW;
    const size_t tstep = (size_t)(kGemmBK / 16) * p.NT * TW;
    auto fetch = [&]() {
        if (fstep < nsteps) {
            const uint32_t* src = tsrc + (size_t)fstep * tstep;
            uint32_t* dst = dring + (size_t)fslot * kTiles * TW;
            for (int c = lane; c < kTiles * TW / 4; c += 32) cp_async16(dst + c * 4, src + c * 4);
        }
        ++fstep;
        cp_async_commit();
        fslot = fslot + 1 == kGemmDecDepth ? 0 : fslot + 1;
    };
#pragma unroll 1
    for (int d = 0; d < kGemmDecDepth - 1; ++d) fetch();
    bool ok = true;
    for (int i = 0; i < nsteps && ok; ++i) {
        const int s = i % S;
        fetch();
        if (i >= S && !mbar_wait_pair(&empty[s], ((i / S) - 1) & 1)) {
            atomicOr(p.status, kStatusPipeTimeout);
            ok = false;
        }
        cp_async_wait<kGemmDecDepth - 1>();
        __syncwarp();
        const uint32_t* stage_tiles = dring + (size_t)cslot * kTiles * TW;
        cslot = cslot + 1 == kGemmDecDepth ? 0 : cslot + 1;
        uint8_t* B = stages + s * TL::SBYTES + TL::ABYTES;
#pragma unroll
        for (int t = 0; t < kTiles; ++t) {
            const int ntl = nt_base + t;
            const uint32_t* tile = stage_tiles + t * TW;
            uint32_t w[3], hsh[8], a[8];
            window_words<K>(tile, lw, w);
            hashes8<K, CB>(w, hsh, hr);
#pragma unroll
            for (int j = 0; j < 8; ++j) a[j] = split_from_hash<CB>(hsh[j], hr);
            // lane holds column g (positions 0..3) and g+8 (4..7) at k 2q, 2q+1, 2q+8, 2q+9
            const int n_lo = ntl * 16 + g, n_hi = n_lo + 8;
            const int kb = ktl * 32 + 4 * q;
            *reinterpret_cast<uint32_t*>(B + sw128_offset(n_lo, kb)) = pack_weights<CB>(a[0], a[1]);
            *reinterpret_cast<uint32_t*>(B + sw128_offset(n_lo, kb + 16)) = pack_weights<CB>(a[2], a[3]);
            *reinterpret_cast<uint32_t*>(B + sw128_offset(n_hi, kb)) = pack_weights<CB>(a[4], a[5]);
            *reinterpret_cast<uint32_t*>(B + sw128_offset(n_hi, kb + 16)) = pack_weights<CB>(a[6], a[7]);
        }
        fence_proxy_async_smem();                   // generic-proxy writes -> tensor core reads
        __syncwarp();                               // also: the ring slot may be refilled
        if (lane == 0) mbar_arrive_cluster(dec0 + 8u * s);
    }
    cp_async_wait<0>();                             // no copy in flight past this point

    // ---- epilogue: per M=256 accumulator a (one pass each), warp dw takes TMEM lane quarter warp % 4
    // and (column block cb, 64-column half ch) = dw / 4 of the CTA's 128 rows x 256 columns
    const int j = dw >> 2, cb = j >> 1, ch = j & 1;
    const int quarter = warp & 3;
    const int lrow = quarter * 32 + lane;
    uint32_t* vote = words + 2;
    if (!mbar_wait_pair(accum, 0, 200)) {
        atomicOr(p.status, kStatusPipeTimeout);
        atomicOr(vote, 1u);
    }
    named_bar_sync(1, 32 * kGemmDecWarps);          // the wait's outcome, uniform before any barrier below
    const bool done = *vote == 0u;
    tc_fence_after();
    float* xbuf = reinterpret_cast<float*>(stages);  // stages and rings are free once the MMAs completed
    constexpr int kRow = 129;
    constexpr int kPassF4 = 16 * 16 * 32;           // float4s of one pass: 16 warps x 16 quads x 32 lanes
    const size_t tile = ((size_t)blockIdx.y * (gridDim.x >> 1) + pair_n) * 2 + rank;
    const float4* parts =
        p.split > 1 ? reinterpret_cast<const float4*>(p.partials) + tile * p.split * (NACC * kPassF4) : nullptr;
    const size_t my_slot = (size_t)dw * 16 * 32 + lane;
    const uint32_t tlane = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(cb * 128 + ch * 64);
    bool finish = done;
    if (p.split > 1 && done) {
        // k split: this part's accumulators to the workspace in thread order, a ticket on the tile's
        // counter; the last part sums all parts in part order
        float4* mine = const_cast<float4*>(parts) + (size_t)blockIdx.z * (NACC * kPassF4) + my_slot;
#pragma unroll 1
        for (int a = 0; a < NACC; ++a) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float part[32];
                tc_ld32(tlane + a * 256 + c * 32, part);
                tc_wait_ld();
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4)
                    __stcg(mine + (size_t)a * kPassF4 + (size_t)(8 * c + q4) * 32,
                           make_float4(part[4 * q4], part[4 * q4 + 1], part[4 * q4 + 2], part[4 * q4 + 3]));
            }
        }
        __threadfence();
        named_bar_sync(1, 32 * kGemmDecWarps);
        uint32_t* flag = words + 1;
        if (dw == 0 && lane == 0) {
            const uint32_t ticket = atomicAdd(p.counters + tile, 1u);
            const bool last = ticket == (uint32_t)p.split - 1;
            if (last) {
                p.counters[tile] = 0u;              // zero at rest for the next call
                __threadfence();
            }
            *flag = last ? 1u : 0u;
        }
        named_bar_sync(1, 32 * kGemmDecWarps);
        finish = *flag != 0u;
    }
    if (!finish) return;
#pragma unroll 1
    for (int a = 0; a < NACC; ++a) {
        float v[64];
        if (p.split == 1) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float part[32];
                tc_ld32(tlane + a * 256 + c * 32, part);
                tc_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) v[c * 32 + i] = part[i];
            }
        } else {
            const float4* src = parts + (size_t)a * kPassF4 + my_slot;
#pragma unroll
            for (int q4 = 0; q4 < 16; ++q4) {
                const float4 w = __ldcg(src + (size_t)q4 * 32);
                v[4 * q4] = w.x;
                v[4 * q4 + 1] = w.y;
                v[4 * q4 + 2] = w.z;
                v[4 * q4 + 3] = w.w;
            }
#pragma unroll 1
            for (int z = 1; z < p.split; ++z) {
                const float4* sz = src + (size_t)z * (NACC * kPassF4);
#pragma unroll
                for (int q4 = 0; q4 < 16; ++q4) {
                    const float4 w = __ldcg(sz + (size_t)q4 * 32);
                    v[4 * q4] += w.x;
                    v[4 * q4 + 1] += w.y;
                    v[4 * q4 + 2] += w.z;
                    v[4 * q4 + 3] += w.w;
                }
            }
        }
        // FWHT stages h = 1..32 inside the 64-column half
#pragma unroll
        for (int hs = 1; hs < 64; hs <<= 1) {
#pragma unroll
            for (int b = 0; b < 32; ++b) {
                const int i0 = (b / hs) * (2 * hs) + (b % hs), i1 = i0 + hs;
                const float a0 = v[i0], a1 = v[i1];
                v[i0] = a0 + a1;
                v[i1] = a0 - a1;
            }
        }
        // stage h = 64 pairs column c with c + 64 of the same block: exchange halves in shared memory
        if (a > 0) named_bar_sync(1, 32 * kGemmDecWarps);     // the previous pass's reads are done
        float* xrow = xbuf + (size_t)(cb * 128 + lrow) * kRow;
#pragma unroll
        for (int i = 0; i < 64; ++i) xrow[ch * 64 + i] = v[i];
        named_bar_sync(1, 32 * kGemmDecWarps);
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            const float other = xrow[(ch ^ 1) * 64 + i];
            v[i] = ch == 0 ? v[i] + other : other - v[i];
        }
        const int row = m0 + a * 256 + (int)rank * 128 + lrow;
        const int col = (2 * pair_n + cb) * 128 + ch * 64;
        if (row < p.M) {
            const size_t off = (size_t)row * p.n + col;
            if (p.out_dtype == EXL3_F16) store_row64(static_cast<__half*>(p.y) + off, v, p.svh + col);
            else if (p.out_dtype == EXL3_BF16) store_row64(static_cast<__nv_bfloat16*>(p.y) + off, v, p.svh + col);
            else store_row64(static_cast<float*>(p.y) + off, v, p.svh + col);
        }
    }
}

template <int K, int CB, int NACC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap xmap, const GemmParams p)
{
    using TL = PairTile<NACC>;
    constexpr int S = TL::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    uint64_t* full = bars;                          // [S] leader: both CTAs' xh halves landed
    uint64_t* decoded = bars + S;                   // [S] leader: both CTAs' B halves written
    uint64_t* empty = bars + 2 * S;                 // [S] both: the stage's MMAs completed
    uint64_t* accum = bars + 3 * S;                 // both: all MMAs completed
    uint32_t* words = reinterpret_cast<uint32_t*>(bars + 3 * S + 1);   // [0] TMEM, [1] last-part flag, [2] vote
    uint8_t* stages = smem + 1024;
    uint8_t* rings = stages + S * TL::SBYTES;

    constexpr int TW = 8 * K;
    const uint32_t rank = cluster_rank();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pair_n = blockIdx.x >> 1;             // 256-column pair tile
    const int nb = 2 * pair_n + (int)rank;          // the 128-column block this CTA decodes
    const int m0 = blockIdx.y * (256 * NACC);
    const int ktot = p.k / kGemmBK;
    const int s0 = (int)blockIdx.z * ktot / p.split;
    const int nsteps = ((int)blockIdx.z + 1) * ktot / p.split - s0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&decoded[s], 2 * kGemmDecWarps);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        words[1] = 0u;
        words[2] = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(words)),
                     "n"(TL::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync_all();                             // both CTAs' barriers initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = words[0];

    if (warp == 0) {
        // ---------------------------------------------------------------- xh producer (TMA)
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
            const uint32_t full0 = cluster_addr(full, 0);
            bool ok = true;
            for (int i = 0; i < nsteps; ++i) {
                const int s = i % S;
                if (i >= S && !mbar_wait_pair(&empty[s], ((i / S) - 1) & 1)) {
                    atomicOr(p.status, kStatusPipeTimeout);
                    ok = false;
                    break;
                }
                if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * TL::ABYTES);
#pragma unroll
                for (int a = 0; a < NACC; ++a)
                    tma_load_2d_pair(stages + s * TL::SBYTES + a * 128 * 128, &xmap, (s0 + i) * kGemmBK,
                                     m0 + a * 256 + (int)rank * 128, full0 + 8u * s);
            }
            // no copy of this CTA in flight when the pair exits: the MMAs of the last stages read them
            if (ok)
                for (int j = nsteps > S ? nsteps - S : 0; j < nsteps; ++j)
                    if (!mbar_wait_pair(&empty[j % S], (j / S) & 1)) {
                        atomicOr(p.status, kStatusPipeTimeout);
                        break;
                    }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (leader)
        if (rank == 0 && lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(256, 256);
            bool ok = true;
            for (int i = 0; i < nsteps; ++i) {
                const int s = i % S;
                const uint32_t par = (i / S) & 1;
                if (!mbar_wait_pair(&full[s], par) || !mbar_wait_pair(&decoded[s], par)) {
                    atomicOr(p.status, kStatusPipeTimeout);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint8_t* st = stages + s * TL::SBYTES;
#pragma unroll
                for (int kk = 0; kk < kGemmBK / 16; ++kk) {
                    const uint64_t bdesc = smem_desc_sw128(st + TL::ABYTES + kk * 32);
#pragma unroll
                    for (int a = 0; a < NACC; ++a)
                        tc_mma_f16_pair(tmem + a * 256, smem_desc_sw128(st + a * 128 * 128 + kk * 32), bdesc, idesc,
                                        (i > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit_pair(&empty[s]);
            }
            if (ok) tc_commit_pair(accum);
        }
    } else {
        pair_decode_and_finish<K, CB, NACC>(p, stages, rings, decoded, empty, accum, words, tmem, rank, pair_n, nb,
                                            m0, s0, nsteps);
    }

    tc_fence_before();
    cluster_sync_all();                             // no MMA, copy or arrival of the pair is pending
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(TL::TMEM_COLS));
    }
}

// ------------------------------------------------------------------------------ host
template <int K, int CB, int NACC>
static int launch_pair_t(const CUtensorMap& xmap, const GemmParams& prm, int m_tiles, cudaStream_t s)
{
    constexpr int SMEM = PairTile<NACC>::SMEM;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(gemm_pair_kernel<K, CB, NACC>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) !=
            cudaSuccess)
            return EXL3_E_CUDA;
        attr_set[dev] = true;
    }
    const dim3 grid(2 * (prm.n / 256), m_tiles, prm.split);
    gemm_pair_kernel<K, CB, NACC><<<grid, kGemmThreads, SMEM, s>>>(xmap, prm);
    return launch_status();
}

template <int K, int CB>
static int launch_pair_n(int nacc, const CUtensorMap& xmap, const GemmParams& prm, int m_tiles, cudaStream_t s)
{
    return nacc == 2 ? launch_pair_t<K, CB, 2>(xmap, prm, m_tiles, s) : launch_pair_t<K, CB, 1>(xmap, prm, m_tiles, s);
}

template <int K>
static int launch_pair_cb(int cb, int nacc, const CUtensorMap& xmap, const GemmParams& prm, int m_tiles,
                          cudaStream_t s)
{
    switch (cb) {
    case 0: return launch_pair_n<K, 0>(nacc, xmap, prm, m_tiles, s);
    case 1: return launch_pair_n<K, 1>(nacc, xmap, prm, m_tiles, s);
    default: return launch_pair_n<K, 2>(nacc, xmap, prm, m_tiles, s);
    }
}

int launch_gemm_pair(int bits, int codebook, int nacc, const CUtensorMap& xmap, const GemmParams& prm, int m_tiles,
                     cudaStream_t s)
{
    switch (bits) {
    case 1: return launch_pair_cb<1>(codebook, nacc, xmap, prm, m_tiles, s);
    case 2: return launch_pair_cb<2>(codebook, nacc, xmap, prm, m_tiles, s);
    case 3: return launch_pair_cb<3>(codebook, nacc, xmap, prm, m_tiles, s);
    case 4: return launch_pair_cb<4>(codebook, nacc, xmap, prm, m_tiles, s);
    case 5: return launch_pair_cb<5>(codebook, nacc, xmap, prm, m_tiles, s);
    case 6: return launch_pair_cb<6>(codebook, nacc, xmap, prm, m_tiles, s);
    case 7: return launch_pair_cb<7>(codebook, nacc, xmap, prm, m_tiles, s);
    default: return launch_pair_cb<8>(codebook, nacc, xmap, prm, m_tiles, s);
    }
}

}  // namespace exl3
