// EXL3 prefill GEMM for sm_100a: y = had128(xh @ W) / sqrt(128) * svh, W decoded from the trellis
// inside the kernel and fed to the 5th-generation tensor cores.
//
// Replaces the reference's prefill path (daig/omlx-exl3 src/omlx/exl3/linear.py:97-121: decode_wt
// of 16384-column chunks to fp16 in memory, MLX matmul, _had128, * svh). Here nothing but xh, the
// trellis and y touch HBM.
//
// CTA tile: BM rows of xh (BM / 128 M=128 accumulators: 256 rows for M <= 256, else 512) x 128 output
// columns (one Hadamard block) x the whole k, in k-steps of 64. Per k-step and pipeline stage:
//   - warp 0 (one lane) loads the BM x 64 fp16 xh tile with TMA tensor loads of 256 rows (128B swizzle);
//   - warps 2..17 decode the 4 x 8 trellis tiles of the step (16 k-rows x 16 columns each; one lane =
//     8 consecutive stream positions, exl3_common.cuh) to exact fp16 weights and store them straight
//     into the 128 x 64 B tile in the same K-major 128B-swizzled layout the tensor core reads;
//   - warp 1 (one lane) issues BM / 128 x 4 tcgen05.mma (M=128, N=128, K=16, fp16 in, fp32 accumulate
//     in tensor memory) and commits them to the stage's "empty" barrier.
// The weight decode is the kernel's bound, so a taller row tile serves more MMAs per decoded tile: at
// BM = 512 each weight of an M <= 512 GEMM is decoded once, and the 512 TMEM columns hold the four
// accumulators. The epilogue warps read one accumulator row half per thread (tcgen05.ld 32x32b), run
// the 128-point FWHT in registers (stage order 1..64, as the reference), scale by 1/sqrt(128) and svh,
// and store y. Every wait is bounded (exl3_common.cuh mbar_wait): a lost completion sets a status
// bit instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_host.h"
#include "exl3_gemm_dec.cuh"
#include "exl3_tc.cuh"

namespace exl3 {

// BM rows per CTA: shared memory = operand stages + barriers + per decoder warp a ring of
// kGemmDecDepth x 2 tiles x 32 K bytes (K <= 8: 256 bytes per tile)
template <int BM>
struct GemmTile {
    static constexpr int NH = BM / 128;                           // M=128 accumulators
    static constexpr int STAGES = BM == 512 ? 2 : 3;
    static constexpr int ABYTES = BM * kGemmBK * 2;              // 32 or 64 KB
    static constexpr int SMEM = 1024 + STAGES * (ABYTES + kGemmBBytes) + 256 + kGemmDecWarps * kGemmDecDepth * 2 * 256;
    static constexpr int TMEM_COLS = NH * kGemmBN;
    static_assert(256 * 129 * 4 <= STAGES * (ABYTES + kGemmBBytes), "epilogue exchange buffer");
    static_assert(SMEM <= 227 * 1024, "shared memory");
};

template <int K, int CB, int BM>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap xmap, const GemmParams p)
{
    using TL = GemmTile<BM>;
    constexpr int kGemmStages = TL::STAGES;
    constexpr int kGemmABytes = TL::ABYTES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* As = smem;                                         // stages x BM x 128 bytes
    uint8_t* Bs = smem + kGemmStages * kGemmABytes;             // stages x 16 KB
    uint64_t* bars = reinterpret_cast<uint64_t*>(Bs + kGemmStages * kGemmBBytes);
    uint64_t* full = bars;                                      // xh tile landed
    uint64_t* decoded = bars + kGemmStages;                     // B tile written by the decoders
    uint64_t* empty = bars + 2 * kGemmStages;                   // MMAs of the stage done
    uint64_t* accum = bars + 3 * kGemmStages;                   // all MMAs done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * kGemmStages + 1);

    constexpr int TW = 8 * K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = blockIdx.x;                                  // 128-column block
    const int m0 = blockIdx.y * BM;
    // this CTA's k part: k-steps [s0, s0 + nsteps)
    const int ktot = p.k / kGemmBK;
    const int s0 = (int)blockIdx.z * ktot / p.split;
    const int nsteps = ((int)blockIdx.z + 1) * ktot / p.split - s0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kGemmStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&decoded[s], kGemmDecWarps);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        tmem_slot[1] = 0u;                                      // last-part flag
        tmem_slot[2] = 0u;                                      // epilogue's timeout vote
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        // NH x 128 TMEM columns: the 128 x 128 fp32 accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "n"(TL::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- xh producer (TMA)
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
            for (int i = 0; i < nsteps; ++i) {
                const int s = i % kGemmStages;
                if (i >= kGemmStages && !mbar_wait(&empty[s], ((i / kGemmStages) - 1) & 1)) {
                    atomicOr(p.status, kStatusPipeTimeout);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], kGemmABytes);
#pragma unroll
                for (int t = 0; t < BM / 256; ++t)                // boxes of 256 rows
                    tma_load_2d(As + s * kGemmABytes + t * 256 * 128, &xmap, (s0 + i) * kGemmBK, m0 + 256 * t,
                                &full[s]);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(128, kGemmBN);
            bool ok = true;
            for (int i = 0; i < nsteps && ok; ++i) {
                const int s = i % kGemmStages;
                const uint32_t par = (i / kGemmStages) & 1;
                if (!mbar_wait(&full[s], par) || !mbar_wait(&decoded[s], par)) {
                    atomicOr(p.status, kStatusPipeTimeout);
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kGemmBK / 16; ++kk) {
                    const uint64_t bdesc = smem_desc_sw128(Bs + s * kGemmBBytes + kk * 32);
#pragma unroll
                    for (int h = 0; h < TL::NH; ++h) {
                        const uint64_t adesc = smem_desc_sw128(As + s * kGemmABytes + h * 128 * 128 + kk * 32);
                        tc_mma_f16(tmem + h * kGemmBN, adesc, bdesc, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                tc_commit(&empty[s]);
            }
            tc_commit(accum);
        }
    } else {
        // ---------------------------------------------------------------- decoders, then epilogue
        const int dw = warp - 2;                                // 0..7
        const int g = lane >> 2, q = lane & 3;
        const LaneWindow<K> lw(lane);
        const HashRegs hr = hash_regs<CB>();
        // warp dw decodes k-slice dw / 4 and the two n-tiles 2 * (dw % 4) + {0, 1} of every k-step
        constexpr int kTiles = 2;
        const int ktl = dw >> 2, nt_base = (dw & 3) * kTiles;
        // The warp's tiles of a k-step are contiguous (kTiles * TW words); they are streamed into a
        // private ring of kGemmDecDepth slots with cp.async, kGemmDecDepth - 1 steps ahead.
        uint32_t* dring = reinterpret_cast<uint32_t*>(Bs + kGemmStages * kGemmBBytes + 256) +
                          (size_t)dw * kGemmDecDepth * kTiles * TW;
        int fstep = 0, fslot = 0, cslot = 0;
        // the warp's tiles of this part's first k-step; one k-step further is kGemmBK / 16 tile rows
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
            const int s = i % kGemmStages;
            fetch();
            if (i >= kGemmStages && !mbar_wait(&empty[s], ((i / kGemmStages) - 1) & 1)) {
                atomicOr(p.status, kStatusPipeTimeout);
                ok = false;
            }
            cp_async_wait<kGemmDecDepth - 1>();
            __syncwarp();
            const uint32_t* stage_tiles = dring + (size_t)cslot * kTiles * TW;
            cslot = cslot + 1 == kGemmDecDepth ? 0 : cslot + 1;
            uint8_t* B = Bs + s * kGemmBBytes;
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
                const int kb = ktl * 32 + 4 * q;                // byte of k = 16*ktl + 2q in the 128-byte row
                const uint32_t o0 = sw128_offset(n_lo, kb), o1 = sw128_offset(n_lo, kb + 16);
                const uint32_t o2 = sw128_offset(n_hi, kb), o3 = sw128_offset(n_hi, kb + 16);
                const uint32_t w0 = pack_weights<CB>(a[0], a[1]), w1 = pack_weights<CB>(a[2], a[3]);
                const uint32_t w2 = pack_weights<CB>(a[4], a[5]), w3 = pack_weights<CB>(a[6], a[7]);
                *reinterpret_cast<uint32_t*>(B + o0) = w0;
                *reinterpret_cast<uint32_t*>(B + o1) = w1;
                *reinterpret_cast<uint32_t*>(B + o2) = w2;
                *reinterpret_cast<uint32_t*>(B + o3) = w3;
            }
            fence_proxy_async_smem();                           // generic-proxy writes -> tensor core reads
            __syncwarp();                                       // also: the ring slot may be refilled
            if (lane == 0) mbar_arrive(&decoded[s]);
        }
        cp_async_wait<0>();                                     // no copy in flight past this point

        // ---- epilogue: each thread takes 64 columns of one accumulator row; per pass the 16 decoder
        // warps cover (two accumulators, column half) x the 4 TMEM lane quarters
        const int j = dw >> 2;                                  // 0..3
        const int chalf = j & 1;
        const int quarter = warp & 3;                           // TMEM lanes this warp may access
        // the accumulator wait's outcome, made uniform over the epilogue warps before any named
        // barrier below (a wait that gave up in some threads only must not split the barriers)
        uint32_t* vote = tmem_slot + 2;
        if (!mbar_wait(accum, 0)) {
            atomicOr(p.status, kStatusPipeTimeout);
            atomicOr(vote, 1u);
        }
        named_bar_sync(1, 32 * kGemmDecWarps);
        const bool done = *vote == 0u;
        tc_fence_after();
        float* xbuf = reinterpret_cast<float*>(smem);           // operand stages are free once the MMAs completed
        constexpr int kRow = 129;
        // k split: this CTA's accumulator goes to the workspace in thread order ([pass][warp][column
        // quad][lane] float4s: a warp's stores of one quad are 512 contiguous bytes) and the CTA takes a
        // ticket; the last of the tile's parts sums all parts in part order and finishes.
        const size_t tile = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
        const float4* parts = p.split > 1 ? reinterpret_cast<const float4*>(p.partials) + tile * p.split * (BM * 32)
                                          : nullptr;
        const size_t my_slot = (size_t)dw * 16 * 32 + lane;    // + pass * 16 warps * 16 quads * 32 lanes
        bool finish = done;
        if (p.split > 1 && done) {
            float4* mine = const_cast<float4*>(parts) + (size_t)blockIdx.z * (BM * 32) + my_slot;
#pragma unroll 1
            for (int pass = 0; pass < TL::NH / 2; ++pass) {
                const int h = 2 * pass + (j >> 1);
                const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(h * kGemmBN + chalf * 64);
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    float part[32];
                    tc_ld32(tbase + c * 32, part);
                    tc_wait_ld();
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4)
                        __stcg(mine + (size_t)pass * (16 * 16 * 32) + (size_t)(8 * c + q4) * 32,
                               make_float4(part[4 * q4], part[4 * q4 + 1], part[4 * q4 + 2], part[4 * q4 + 3]));
                }
            }
            __threadfence();                                    // this thread's partial before the ticket
            named_bar_sync(1, 32 * kGemmDecWarps);
            uint32_t* flag = tmem_slot + 1;
            if (dw == 0 && lane == 0) {
                const uint32_t ticket = atomicAdd(p.counters + tile, 1u);
                const bool last = ticket == (uint32_t)p.split - 1;
                if (last) {
                    p.counters[tile] = 0u;                      // zero at rest for the next call
                    __threadfence();
                }
                *flag = last ? 1u : 0u;
            }
            named_bar_sync(1, 32 * kGemmDecWarps);
            finish = *flag != 0u;
        }
        if (finish) {
#pragma unroll 1
            for (int pass = 0; pass < TL::NH / 2; ++pass) {
                const int h = 2 * pass + (j >> 1);
                const int rpass = (j >> 1) * 128 + quarter * 32 + lane;     // row inside this pass's 256
                const int row = m0 + h * 128 + quarter * 32 + lane;
                float v[64];
                if (p.split == 1) {
                    const uint32_t tbase =
                        tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(h * kGemmBN + chalf * 64);
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        float part[32];
                        tc_ld32(tbase + c * 32, part);
                        tc_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[c * 32 + i] = part[i];
                    }
                } else {
                    const float4* src = parts + my_slot + (size_t)pass * (16 * 16 * 32);
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
                        const float4* sz = src + (size_t)z * (BM * 32);
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
                // FWHT stages h = 1..32 stay inside a 64-column half
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
                // stage h = 64 pairs column c with c + 64: exchange halves through shared memory, rows
                // padded to 129 floats
                if (pass > 0) named_bar_sync(1, 32 * kGemmDecWarps);     // the previous pass's reads are done
#pragma unroll
                for (int i = 0; i < 64; ++i) xbuf[rpass * kRow + chalf * 64 + i] = v[i];
                named_bar_sync(1, 32 * kGemmDecWarps);
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    const float other = xbuf[rpass * kRow + (chalf ^ 1) * 64 + i];
                    v[i] = chalf == 0 ? v[i] + other : other - v[i];
                }
                if (row < p.M) {
                    const __half* sv = p.svh + (size_t)nb * kGemmBN + chalf * 64;
                    const size_t off = (size_t)row * p.n + (size_t)nb * kGemmBN + chalf * 64;
                    if (p.out_dtype == EXL3_F16) store_row64(static_cast<__half*>(p.y) + off, v, sv);
                    else if (p.out_dtype == EXL3_BF16) store_row64(static_cast<__nv_bfloat16*>(p.y) + off, v, sv);
                    else store_row64(static_cast<float*>(p.y) + off, v, sv);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(TL::TMEM_COLS));
    }
}

// ------------------------------------------------------------------------------ host
// Grid of one call: BM-row tiles x 128-column blocks x `split` k parts.
//   - Without a split: 512-row tiles once a second 256-row tile would be needed (each weight decoded
//     once per 512 rows), as long as they still give about one CTA per SM; else 256-row tiles.
//   - When the tiles fill at most half of the SMs (narrow outputs: 17408 -> 5120 has 40 column
//     blocks) and a workspace is given, k is split so that tiles x parts still fit one CTA per SM
//     (at least 16 k-steps per part), with 512-row tiles above 256 rows so every weight is decoded
//     once. The parts' fp32 partials go through the workspace and the last part of each tile sums
//     them in part order.
struct GemmPlan {
    bool pair;      // the SM-pair kernel (exl3_gemm_pair.cu): n % 256 == 0
    int bm;         // rows per tile: one-CTA 256 / 512; pair 256 x nacc
    int nacc;       // pair: M=256 accumulators per pair tile
    int m_tiles, split;
    int units;      // CTAs per k part (each has its own arrival counter and partial)
};

// The SM-pair kernel runs only when the environment sets EXL3_GEMM_PAIR=1 (read at every call): it is
// correct for every output width that is a multiple of 256 but measured slower than the one-CTA kernel
// (M=512, 5120->17408: 620 against 732 TFLOP/s; M=4096: 732 against 884).
static bool pair_enabled()
{
    const char* e = getenv("EXL3_GEMM_PAIR");
    return e && e[0] == '1';
}

static GemmPlan plan_gemm(int M, int k, int n, bool may_split)
{
    const int sms = device_sm_count(), nb = n / kGemmBN, ktot = k / kGemmBK;
    GemmPlan pl{};
    pl.split = 1;
    if (n % 256 == 0 && pair_enabled()) {
        pl.pair = true;
        pl.nacc = M > 256 ? 2 : 1;
        pl.bm = 256 * pl.nacc;
        pl.m_tiles = (M + pl.bm - 1) / pl.bm;
        pl.units = pl.m_tiles * (n / 256) * 2;
        if (may_split && 2 * pl.units <= sms) {
            const int s = std::min(std::min(8, sms / pl.units), ktot / 16);
            if (s > 1) pl.split = s;
        }
        return pl;
    }
    const long long ctas512 = (long long)nb * ((M + 511) / 512);
    pl.bm = (M > 256 && ctas512 * 8 >= (long long)sms * 7) ? 512 : 256;
    pl.m_tiles = (M + pl.bm - 1) / pl.bm;
    if (may_split) {
        const int bm = M > 256 ? 512 : 256;
        const int tiles = nb * ((M + bm - 1) / bm);
        if (2 * tiles <= sms) {
            const int s = std::min(std::min(8, sms / tiles), ktot / 16);
            if (s > 1) {
                pl.bm = bm;
                pl.m_tiles = (M + bm - 1) / bm;
                pl.split = s;
            }
        }
    }
    pl.units = pl.m_tiles * nb;
    return pl;
}

// [counters: one per CTA of a part, rounded up to 256 bytes][partials: units x split x a CTA's
// accumulators (one-CTA: BM x 128 fp32; pair: 128 rows x 256 columns per accumulator)]
static size_t gemm_counter_bytes(const GemmPlan& pl) { return ((size_t)pl.units * 4 + 255) / 256 * 256; }

static size_t gemm_workspace_bytes(const GemmPlan& pl)
{
    if (pl.split == 1) return 0;
    const size_t per_cta = pl.pair ? (size_t)pl.nacc * 128 * 256 : (size_t)pl.bm * kGemmBN;
    return gemm_counter_bytes(pl) + (size_t)pl.units * pl.split * per_cta * 4;
}

template <int K, int CB, int BM>
static int launch_gemm_bm(const CUtensorMap& map, const GemmParams& prm, int m_tiles, cudaStream_t s)
{
    constexpr int SMEM = GemmTile<BM>::SMEM;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(gemm_kernel<K, CB, BM>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
            return EXL3_E_CUDA;
        attr_set[dev] = true;
    }
    const dim3 grid(prm.n / kGemmBN, m_tiles, prm.split);
    gemm_kernel<K, CB, BM><<<grid, kGemmThreads, SMEM, s>>>(map, prm);
    return launch_status();
}

template <int K, int CB>
static int launch_gemm_k(const CUtensorMap& map, const GemmParams& prm, const GemmPlan& pl, cudaStream_t s)
{
    return pl.bm == 512 ? launch_gemm_bm<K, CB, 512>(map, prm, pl.m_tiles, s)
                        : launch_gemm_bm<K, CB, 256>(map, prm, pl.m_tiles, s);
}

template <int K>
static int launch_gemm_cb(int cb, const CUtensorMap& map, const GemmParams& prm, const GemmPlan& pl, cudaStream_t s)
{
    switch (cb) {
    case 0: return launch_gemm_k<K, 0>(map, prm, pl, s);
    case 1: return launch_gemm_k<K, 1>(map, prm, pl, s);
    default: return launch_gemm_k<K, 2>(map, prm, pl, s);
    }
}

}  // namespace exl3

extern "C" int exl3_gemm_workspace(int M, int k, int n, size_t* bytes)
{
    using namespace exl3;
    if (!bytes) return EXL3_E_NULL;
    if (M < 1 || k <= 0 || n <= 0 || k % kGemmBK || n % kGemmBN) return EXL3_E_SHAPE;
    if (int e = check_device()) return e;
    *bytes = gemm_workspace_bytes(plan_gemm(M, k, n, true));
    return EXL3_OK;
}

extern "C" int exl3_gemm(const void* xh, int M, int k, int n, const uint32_t* trellis, int bits, int codebook,
                         const void* svh, void* y, int out_dtype, void* workspace, size_t workspace_bytes,
                         uint32_t* status, void* stream)
{
    using namespace exl3;
    if (!xh || !trellis || !svh || !y || !status) return EXL3_E_NULL;
    if (M < 1 || k <= 0 || n <= 0 || k % kGemmBK || n % kGemmBN) return EXL3_E_SHAPE;
    if (bits < 1 || bits > 8) return EXL3_E_BITS;
    if (codebook < 0 || codebook > 2) return EXL3_E_CODEBOOK;
    if (out_dtype != EXL3_F16 && out_dtype != EXL3_BF16 && out_dtype != EXL3_F32) return EXL3_E_DTYPE;
    if (!aligned(xh, 16) || !aligned(trellis, 16) || !aligned(y, 16) || !aligned(svh, 2) || !aligned(status, 4) ||
        !aligned(workspace, 256))
        return EXL3_E_ALIGN;
    if (int e = check_device()) return e;
    GemmPlan pl = plan_gemm(M, k, n, workspace != nullptr);
    if (pl.split > 1 && workspace_bytes < gemm_workspace_bytes(pl)) pl = plan_gemm(M, k, n, false);
    auto encode = exl3_get_tensormap_encoder();
    if (!encode) return EXL3_E_CUDA;

    // xh: fp16 (M, k) row-major -> 2D map {k, M}, 128-byte swizzle, zero fill past M; boxes of 64 k x
    // 256 rows for the one-CTA kernel (a 512-row tile takes two), 128 rows for the pair kernel (each CTA
    // loads its half of every 256-row accumulator)
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kGemmBK, pl.pair ? 128u : 256u};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(xh), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return EXL3_E_CUDA;

    GemmParams prm{};
    prm.trellis = trellis;
    prm.svh = static_cast<const __half*>(svh);
    prm.y = y;
    prm.status = status;
    prm.M = M;
    prm.k = k;
    prm.n = n;
    prm.KT = k / 16;
    prm.NT = n / 16;
    prm.out_dtype = out_dtype;
    prm.split = pl.split;
    if (pl.split > 1) {
        prm.counters = static_cast<uint32_t*>(workspace);
        prm.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + gemm_counter_bytes(pl));
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (pl.pair) return launch_gemm_pair(bits, codebook, pl.nacc, map, prm, pl.m_tiles, s);
    switch (bits) {
    case 1: return launch_gemm_cb<1>(codebook, map, prm, pl, s);
    case 2: return launch_gemm_cb<2>(codebook, map, prm, pl, s);
    case 3: return launch_gemm_cb<3>(codebook, map, prm, pl, s);
    case 4: return launch_gemm_cb<4>(codebook, map, prm, pl, s);
    case 5: return launch_gemm_cb<5>(codebook, map, prm, pl, s);
    case 6: return launch_gemm_cb<6>(codebook, map, prm, pl, s);
    case 7: return launch_gemm_cb<7>(codebook, map, prm, pl, s);
    default: return launch_gemm_cb<8>(codebook, map, prm, pl, s);
    }
}
