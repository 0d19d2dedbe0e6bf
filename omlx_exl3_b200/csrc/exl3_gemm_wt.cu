// Prefill GEMM on decoded weights for sm_100a: y = had128(xh @ Wt^T) / sqrt(128) * svh, with Wt the fp16
// (n, k) matrix exl3_decode_wt writes. The large-M half of the reference's prefill path (daig/omlx-exl3
// src/omlx/exl3/linear.py:97-105: decode_wt chunks, matmul, _had128, * svh) as one kernel after the
// decode: the weights are decoded once per column chunk, so above a few hundred rows the product is
// bound by the tensor cores, not by the trellis decode that limits the fused kernel (exl3_gemm.cu).
//
// Pair tiles on two SMs (a cluster of 2 CTAs, tcgen05 cta_group::2): 256 rows x 256 output columns
// (two Hadamard blocks) per tile, k-steps of 64. Each CTA of the pair holds half of each operand in its
// own shared memory (rows 128 * rank .. of xh, columns 128 * rank .. of the tile's Wt rows) and half of
// the accumulator in its tensor memory (its 128 rows x 256 columns). Per CTA:
//   - warp 0 (one lane) loads its two 128 x 64 fp16 halves per stage with TMA (128-byte swizzle, no
//     multicast), counted on the leader CTA's "full" barrier of the stage;
//   - warp 1 of the leader (one lane) issues 4 tcgen05.mma (M=256, N=256, K=16, fp32 accumulate) per
//     stage and commits them to both CTAs' "empty" barriers;
//   - warps 2..5 are the epilogue: a thread owns one accumulator row (its TMEM lane), reads 128 columns
//     (tcgen05.ld 32x32b), runs the 128-point FWHT in registers (stages 1..64, the reference's order),
//     scales by 1/sqrt(128) and svh, and stores.
// The kernel is persistent (one pair per two SMs, tiles strided over the pairs) and the 512 TMEM columns
// hold two accumulators, so a tile's epilogue runs while the next tile's MMAs accumulate in the other
// buffer. Every wait is a bounded poll (mbar_wait_pair): a lost completion sets a status bit instead
// of hanging.
//
// k split: when the tiles do not fill the pairs evenly (narrow outputs: 17408 -> 5120 has 20 column
// tiles), each tile's k range is cut into S parts that run as separate work units. A unit's epilogue
// writes its fp32 accumulator to the caller's workspace and takes an arrival ticket on the tile's
// counter (zero at rest); the unit that arrives last sums the S partials in part order (the result does
// not depend on which unit finished last), rotates, scales, stores and resets the counter. No unit waits
// for another.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_host.h"
#include "exl3_tc.cuh"

namespace exl3 {

constexpr int kWtRows = 128;                          // xh rows per CTA (pair tile: 256)
constexpr int kWtCols = 128;                          // Wt rows = output columns per CTA (pair tile: 256)
constexpr int kWtBK = 64;                             // k per stage: one 128-byte swizzle row of fp16
constexpr int kWtStages = 6;
constexpr int kWtHalfBytes = kWtRows * kWtBK * 2;     // 16 KB
constexpr int kWtStageBytes = 2 * kWtHalfBytes;       // A half + B half of one CTA
constexpr int kWtEpiWarps = 4;
constexpr int kWtThreads = 32 * (2 + kWtEpiWarps);
constexpr int kWtBarBytes = 256;
constexpr int kWtSmem = 1024 + kWtStages * kWtStageBytes + kWtBarBytes;
static_assert(kWtSmem <= 227 * 1024, "shared memory");
static_assert((2 * kWtStages + 4) * 8 + 8 <= kWtBarBytes, "barrier area");

struct GemmWtParams {
    const __half* svh;
    void* y;
    uint32_t* status;
    uint32_t* counters;      // [split tiles][2] arrival tickets of the k split (zero at rest)
    float* partials;         // [split tiles][2][split][64 column quads][128 rows][4] fp32
    int M, k, n, ldy, out_dtype;
    int tiles_m, n_tiles;
    int n_whole;             // tiles 0 .. n_whole - 1 run whole; the others in `split` k parts each
    int split;
    int n_units;             // n_whole + (n_tiles - n_whole) * split
};

constexpr size_t kWtPartialFloats = 2 * kWtCols * kWtRows;     // one CTA's accumulator

// Work unit u -> its tile, its k part and the tile's part count; k-steps [first, last) of the part.
struct WtUnit {
    int t, part, parts, first, last;
};

__device__ __forceinline__ WtUnit unit_of(const GemmWtParams& p, int u, int nsteps)
{
    WtUnit w;
    if (u < p.n_whole) {
        w.t = u;
        w.part = 0;
        w.parts = 1;
    } else {
        const int v = u - p.n_whole;
        w.t = p.n_whole + v / p.split;
        w.part = v % p.split;
        w.parts = p.split;
    }
    w.first = w.part * nsteps / w.parts;
    w.last = (w.part + 1) * nsteps / w.parts;
    return w;
}

template <typename OT>
__device__ __forceinline__ void store_row128(OT* dst, const float (&v)[128], const __half* svh)
{
#pragma unroll
    for (int c = 0; c < 128; c += 8) {
        if constexpr (sizeof(OT) == 4) {
            float4 a, b;
            a.x = v[c] * kHadScale * __half2float(svh[c]);
            a.y = v[c + 1] * kHadScale * __half2float(svh[c + 1]);
            a.z = v[c + 2] * kHadScale * __half2float(svh[c + 2]);
            a.w = v[c + 3] * kHadScale * __half2float(svh[c + 3]);
            b.x = v[c + 4] * kHadScale * __half2float(svh[c + 4]);
            b.y = v[c + 5] * kHadScale * __half2float(svh[c + 5]);
            b.z = v[c + 6] * kHadScale * __half2float(svh[c + 6]);
            b.w = v[c + 7] * kHadScale * __half2float(svh[c + 7]);
            *reinterpret_cast<float4*>(dst + c) = a;
            *reinterpret_cast<float4*>(dst + c + 4) = b;
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

// 128-point FWHT of one accumulator row block in registers (stages 1..64, the reference's butterfly),
// then * 1/sqrt(128) * svh and the store of columns col .. col + 127 of `row` (skipped outside y).
__device__ __forceinline__ void fwht128_store(float (&v)[128], const GemmWtParams& p, int row, int col)
{
#pragma unroll
    for (int hs = 1; hs < 128; hs <<= 1) {
#pragma unroll
        for (int q = 0; q < 64; ++q) {
            const int i0 = (q / hs) * (2 * hs) + (q % hs), i1 = i0 + hs;
            const float a0 = v[i0], a1 = v[i1];
            v[i0] = a0 + a1;
            v[i1] = a0 - a1;
        }
    }
    if (row < p.M && col < p.n) {
        const size_t off = (size_t)row * p.ldy + col;
        if (p.out_dtype == EXL3_F16) store_row128(static_cast<__half*>(p.y) + off, v, p.svh + col);
        else if (p.out_dtype == EXL3_BF16) store_row128(static_cast<__nv_bfloat16*>(p.y) + off, v, p.svh + col);
        else store_row128(static_cast<float*>(p.y) + off, v, p.svh + col);
    }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kWtThreads, 1)
    gemm_wt_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                   const GemmWtParams p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWtStages * kWtStageBytes);
    uint64_t* full = bars;                          // [stages] leader: both CTAs' halves of the stage landed
    uint64_t* empty = bars + kWtStages;             // [stages] both CTAs: the stage's MMAs completed
    uint64_t* tfull = bars + 2 * kWtStages;         // [2] both CTAs: accumulator b complete
    uint64_t* tempty = bars + 2 * kWtStages + 2;    // [2] leader: both epilogues have read accumulator b
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kWtStages + 4);

    const uint32_t rank = cluster_rank();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int nsteps = p.k / kWtBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kWtStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * kWtEpiWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        // both accumulators: 2 x 256 fp32 columns of this CTA's 128 lanes (one warp of each CTA allocates)
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(tmem_slot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync_all();                              // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer (both CTAs)
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&amap)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&bmap)) : "memory");
            const uint32_t full0 = cluster_addr(full, 0);
            int g = 0;
            bool ok = true;
            for (int u = pair; u < p.n_units && ok; u += npairs) {
                const WtUnit w = unit_of(p, u, nsteps);
                const int tm = w.t % p.tiles_m, tn = w.t / p.tiles_m;
                const int arow = tm * 2 * kWtRows + (int)rank * kWtRows;
                const int brow = tn * 2 * kWtCols + (int)rank * kWtCols;
                for (int i = w.first; i < w.last; ++i, ++g) {
                    const int s = g % kWtStages;
                    if (g >= kWtStages && !mbar_wait_pair(&empty[s], ((g / kWtStages) - 1) & 1)) {
                        atomicOr(p.status, kStatusPipeTimeout);
                        ok = false;
                        break;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * kWtStageBytes);
                    uint8_t* st = smem + s * kWtStageBytes;
                    tma_load_2d_pair(st, &amap, i * kWtBK, arow, full0 + 8u * s);
                    tma_load_2d_pair(st + kWtHalfBytes, &bmap, i * kWtBK, brow, full0 + 8u * s);
                }
            }
            // no copy of this CTA may still be in flight when the pair exits: the MMAs of the last
            // stages read them
            if (ok)
                for (int j = g > kWtStages ? g - kWtStages : 0; j < g; ++j)
                    if (!mbar_wait_pair(&empty[j % kWtStages], (j / kWtStages) & 1)) {
                        atomicOr(p.status, kStatusPipeTimeout);
                        break;
                    }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (leader CTA)
        if (rank == 0 && lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(2 * kWtRows, 2 * kWtCols);
            int g = 0, j = 0;
            bool ok = true;
            for (int u = pair; u < p.n_units && ok; u += npairs, ++j) {
                const int b = j & 1;
                if (j >= 2 && !mbar_wait_pair(&tempty[b], ((j >> 1) - 1) & 1)) {
                    atomicOr(p.status, kStatusPipeTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * 2 * kWtCols);
                const WtUnit w = unit_of(p, u, nsteps);
                for (int i = w.first; i < w.last; ++i, ++g) {
                    const int s = g % kWtStages;
                    if (!mbar_wait_pair(&full[s], (g / kWtStages) & 1)) {
                        atomicOr(p.status, kStatusPipeTimeout);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t* st = smem + s * kWtStageBytes;
#pragma unroll
                    for (int kk = 0; kk < kWtBK / 16; ++kk)
                        tc_mma_f16_pair(d, smem_desc_sw128(st + kk * 32), smem_desc_sw128(st + kWtHalfBytes + kk * 32),
                                        idesc, (i > w.first || kk > 0) ? 1u : 0u);
                    tc_commit_pair(&empty[s]);
                }
                if (ok) tc_commit_pair(&tfull[b]);
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue (both CTAs)
        const int quarter = warp & 3;                    // TMEM lanes 32 quarter .. this warp may read
        const int lrow = quarter * 32 + lane;
        const int etid = threadIdx.x - 64;               // 0..127 over the epilogue warps
        const uint32_t tempty0 = cluster_addr(tempty, 0);
        uint32_t* last_flag = tmem_slot + 1;
        // accumulator b read out by this warp: once all eight epilogue warps of the pair arrived, the
        // leader may accumulate into it again
        auto release = [&](int b) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty0 + 8u * b);
        };
        int j = 0;
        for (int u = pair; u < p.n_units; u += npairs, ++j) {
            const int b = j & 1;
            const WtUnit w = unit_of(p, u, nsteps);
            const int t = w.t, part = w.part;
            const int tm = t % p.tiles_m, tn = t / p.tiles_m;
            if (!mbar_wait_pair(&tfull[b], (j >> 1) & 1, 200)) {
                atomicOr(p.status, kStatusPipeTimeout);
                break;
            }
            tc_fence_after();
            const int row = tm * 2 * kWtRows + (int)rank * kWtRows + lrow;
            const uint32_t tlane = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * 2 * kWtCols);
            const float4* tile_part = w.parts == 1 ? nullptr : reinterpret_cast<const float4*>(
                p.partials + ((size_t)(t - p.n_whole) * 2 + rank) * p.split * kWtPartialFloats);
            bool finish = true;
            if (w.parts > 1) {
                // this part's accumulator as [column quad][row][4] (a warp's 16-byte stores of one quad
                // are 512 contiguous bytes), 32 columns at a time straight from tensor memory
                float4* dst = const_cast<float4*>(tile_part) + (size_t)part * (kWtPartialFloats / 4) + lrow;
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    float pv[32];
                    tc_ld32(tlane + c * 32, pv);
                    tc_wait_ld();
#pragma unroll
                    for (int c4 = 0; c4 < 8; ++c4)
                        __stcg(dst + (size_t)(8 * c + c4) * kWtRows,
                               make_float4(pv[4 * c4], pv[4 * c4 + 1], pv[4 * c4 + 2], pv[4 * c4 + 3]));
                }
                release(b);
                __threadfence();                         // this thread's partial before the ticket
                named_bar_sync(1, 32 * kWtEpiWarps);
                if (etid == 0) {
                    uint32_t* cnt = p.counters + (size_t)(t - p.n_whole) * 2 + rank;
                    const uint32_t ticket = atomicAdd(cnt, 1u);
                    const bool last = ticket == (uint32_t)p.split - 1;
                    if (last) {
                        *cnt = 0u;                       // zero at rest for the next call
                        __threadfence();
                    }
                    *last_flag = last ? 1u : 0u;
                }
                named_bar_sync(1, 32 * kWtEpiWarps);
                finish = *last_flag != 0u;
                named_bar_sync(1, 32 * kWtEpiWarps);     // the flag is read before the next unit writes it
            }
            if (!finish) continue;
#pragma unroll 1
            for (int blk = 0; blk < 2; ++blk) {
                float v[128];
                if (w.parts == 1) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        float pv[32];
                        tc_ld32(tlane + blk * 128 + c * 32, pv);
                        tc_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[c * 32 + i] = pv[i];
                    }
                    if (blk == 1) release(b);
                } else {
                    // the parts' partials summed in part order, whichever unit arrived last
                    const float4* src = tile_part + (size_t)blk * 32 * kWtRows + lrow;
#pragma unroll
                    for (int c4 = 0; c4 < 32; ++c4) {
                        const float4 w = __ldcg(src + (size_t)c4 * kWtRows);
                        v[4 * c4] = w.x;
                        v[4 * c4 + 1] = w.y;
                        v[4 * c4 + 2] = w.z;
                        v[4 * c4 + 3] = w.w;
                    }
#pragma unroll 1
                    for (int q = 1; q < p.split; ++q) {
                        const float4* sq = src + (size_t)q * (kWtPartialFloats / 4);
#pragma unroll
                        for (int c4 = 0; c4 < 32; ++c4) {
                            const float4 w = __ldcg(sq + (size_t)c4 * kWtRows);
                            v[4 * c4] += w.x;
                            v[4 * c4 + 1] += w.y;
                            v[4 * c4 + 2] += w.z;
                            v[4 * c4 + 3] += w.w;
                        }
                    }
                }
                fwht128_store(v, p, row, tn * 2 * kWtCols + blk * 128);
            }
        }
    }

    tc_fence_before();
    cluster_sync_all();                              // no MMA, copy or arrival of the pair is pending
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    }
}

static bool encode_kmajor(PFN_cuTensorMapEncodeTiled_v12000 encode, CUtensorMap* map, const void* base, int k,
                          int rows)
{
    // fp16 (rows, k) row-major -> 2D map {k, rows}, box {64, 128}, 128-byte swizzle, zero fill past the end
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kWtBK, (cuuint32_t)kWtRows};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


// Schedule: the tiles that fill whole rounds of the pairs run whole; when the last round is partly
// empty, its tiles ("tail") may instead run as `split` k parts each, so that the last round spreads
// over the idle pairs. Cost model in k-steps of the busiest pair: full rounds x k-steps, plus for the
// tail either one more whole round or its split rounds plus kWtSplitCost (writing and summing the
// partials; the tail's epilogues are not hidden behind later MMAs). A part keeps at least
// kWtMinPartSteps k-steps. Splitting a tile that a full round would have run anyway was measured
// slower (M=4096, 17408->5120: 1069 against 1234 TFLOP/s): its partials' traffic competes with the
// operands for L2.
constexpr int kWtSplitCost = 16;
constexpr int kWtMinPartSteps = 64;

struct WtPlan {
    int tiles_m, n_tiles, n_whole, split, n_units, pairs;
};

static WtPlan plan_wt(int M, int k, int n, bool may_split)
{
    WtPlan pl{};
    pl.tiles_m = (M + 2 * kWtRows - 1) / (2 * kWtRows);
    pl.n_tiles = pl.tiles_m * ((n + 2 * kWtCols - 1) / (2 * kWtCols));
    const int P = std::max(1, device_sm_count() / 2);
    const int nsteps = k / kWtBK;
    const int full = pl.n_tiles / P, tail = pl.n_tiles % P;
    pl.n_whole = pl.n_tiles;
    pl.split = 1;
    long long best = (long long)(full + (tail ? 1 : 0)) * nsteps;
    for (int s = 2; may_split && tail && s <= 8 && nsteps / s >= kWtMinPartSteps; ++s) {
        const long long cost =
            (long long)full * nsteps + ((long long)tail * s + P - 1) / P * ((nsteps + s - 1) / s) + kWtSplitCost;
        if (cost < best) {
            best = cost;
            pl.split = s;
            pl.n_whole = full * P;
        }
    }
    pl.n_units = pl.n_whole + (pl.n_tiles - pl.n_whole) * pl.split;
    pl.pairs = std::min(pl.n_units, P);
    return pl;
}

// workspace of a split plan: the arrival counters (2 per split tile) rounded up to 256 bytes, then the
// partials
static size_t wt_counter_bytes(const WtPlan& pl)
{
    return ((size_t)(pl.n_tiles - pl.n_whole) * 2 * 4 + 255) / 256 * 256;
}

static size_t wt_workspace_bytes(const WtPlan& pl)
{
    if (pl.split == 1) return 0;
    return wt_counter_bytes(pl) +
           (size_t)(pl.n_tiles - pl.n_whole) * 2 * pl.split * kWtPartialFloats * sizeof(float);
}

}  // namespace exl3

extern "C" int exl3_gemm_wt_workspace(int M, int k, int n, size_t* bytes)
{
    using namespace exl3;
    if (!bytes) return EXL3_E_NULL;
    if (M < 1 || k <= 0 || n <= 0 || k % kWtBK || n % 128) return EXL3_E_SHAPE;
    if (int e = check_device()) return e;
    *bytes = wt_workspace_bytes(plan_wt(M, k, n, true));
    return EXL3_OK;
}

extern "C" int exl3_gemm_wt(const void* xh, int M, int k, int n, const void* wt, const void* svh, void* y, int ldy,
                            int out_dtype, void* workspace, size_t workspace_bytes, uint32_t* status, void* stream)
{
    using namespace exl3;
    if (!xh || !wt || !svh || !y || !status) return EXL3_E_NULL;
    if (M < 1 || k <= 0 || n <= 0 || k % kWtBK || n % 128 || ldy < n) return EXL3_E_SHAPE;
    if (out_dtype != EXL3_F16 && out_dtype != EXL3_BF16 && out_dtype != EXL3_F32) return EXL3_E_DTYPE;
    const int esz = out_dtype == EXL3_F32 ? 4 : 2;
    if (!aligned(xh, 16) || !aligned(wt, 16) || !aligned(y, 16) || !aligned(svh, 2) || !aligned(status, 4) ||
        !aligned(workspace, 256) || ((size_t)ldy * esz) % 16)
        return EXL3_E_ALIGN;
    if (int e = check_device()) return e;
    // the k split needs the workspace exl3_gemm_wt_workspace sized; without one the call runs unsplit
    WtPlan pl = plan_wt(M, k, n, workspace != nullptr);
    if (pl.split > 1 && workspace_bytes < wt_workspace_bytes(pl)) pl = plan_wt(M, k, n, false);
    auto encode = exl3_get_tensormap_encoder();
    if (!encode) return EXL3_E_CUDA;
    CUtensorMap amap, bmap;
    if (!encode_kmajor(encode, &amap, xh, k, M) || !encode_kmajor(encode, &bmap, wt, k, n)) return EXL3_E_CUDA;

    GemmWtParams prm{};
    prm.svh = static_cast<const __half*>(svh);
    prm.y = y;
    prm.status = status;
    prm.M = M;
    prm.k = k;
    prm.n = n;
    prm.ldy = ldy;
    prm.out_dtype = out_dtype;
    prm.tiles_m = pl.tiles_m;
    prm.n_tiles = pl.n_tiles;
    prm.n_whole = pl.n_whole;
    prm.split = pl.split;
    prm.n_units = pl.n_units;
    if (pl.split > 1) {
        prm.counters = static_cast<uint32_t*>(workspace);
        prm.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + wt_counter_bytes(pl));
    }

    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(gemm_wt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kWtSmem) != cudaSuccess)
            return EXL3_E_CUDA;
        attr_set[dev] = true;
    }
    gemm_wt_kernel<<<2 * pl.pairs, kWtThreads, kWtSmem, static_cast<cudaStream_t>(stream)>>>(amap, bmap, prm);
    return launch_status();
}
