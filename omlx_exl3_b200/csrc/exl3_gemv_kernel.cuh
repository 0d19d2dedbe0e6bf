// EXL3 decode GEMV (1..8 rows) for sm_100a: y = had128(xh @ W) / sqrt(128) * svh in one launch.
//
// Replaces the reference's trellis GEMV (daig/omlx-exl3 src/omlx/exl3/kernels.py:114-299).
//
// Work split (stream-K over "units"): a unit is one 16-row k-slice of one 128-column output block,
// i.e. 8 consecutive trellis tiles = 256*K contiguous bytes. Units are numbered block-major
// (u = block * KT + kt) and each persistent CTA (one per SM) owns the contiguous range
// [c*U/G, (c+1)*U/G), so every SM streams the same number of bytes whatever the shape.
//
// Inside a CTA every warp streams its own units (CTA unit indices w, w + NCW, ...) into a private
// shared-memory ring with 16-byte cp.async copies, DEPTH - 1 units ahead of the unit it decodes (no
// producer thread and no cross-warp handshake: many small copies from all warps keep enough bytes in
// flight). A warp decodes each of the unit's 8 tiles straight into m16n8k16 A fragments (one lane =
// 8 consecutive stream positions, exl3_common.cuh) and, for 2..8 rows, issues two MMAs per tile
// against the rows of xh duplicated across each k pair ("split" operands: the 3inst/mcg weight is
// the sum of two fp16 halves, so A = (lo, hi) and B = (x, x)); accumulators are fp32 registers, as
// the reference's fp32 FMAs (kernels.py:215-218). One row takes the same path, so row r of any call
// has the same bits whatever `rows` is (the reference's row-exact property, kernels.py:13-15).
//
// Reduction, fixed order (bitwise reproducible, row-exact): at the end of each block segment the
// consumer warps sum their accumulators through shared memory in warp order. A block that lies
// entirely inside one CTA is finished right there; otherwise each CTA publishes its partial, and
// the last CTA to arrive (per-block arrival counter, zero at rest) sums the partials in a fixed order
// (CTA order for up to 8 partials; beyond that four interleaved groups of the CTAs, each in CTA order,
// then the groups in order).
// The finishing CTA applies the 128-point FWHT (Sylvester order, stages 1..64 as the reference),
// * 1/sqrt(128) * svh, and writes y in the output dtype. No CTA ever waits on another CTA.
//
// This header holds the kernel and its launch templates; exl3_gemv.cu holds the grid planner and the
// C entry points, exl3_gemv_fused.cu the instantiations of the fused finishes.
#pragma once

#include <cuda_runtime.h>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_host.h"
#include "exl3_peer.cuh"

namespace exl3 {

constexpr int kNCW = 16;                 // warps per CTA

struct GemvParams {
    const uint32_t* trellis[3];
    int nt_member[3];        // n-tiles of each member (row stride of its trellis, in tiles)
    int blk_off[4];          // first global 128-column block of each member; [nm] = total blocks
    int nm;
    const __half* xh;        // (nm, rows, k)
    const __half* svh;       // (n_total)
    void* y;                 // (rows, n_total)
    float* partials;         // grid * J * 8 * 128
    uint32_t* counters;      // one arrival counter per 128-column block, zero at rest
    int k, KT, rows, n_total, blocks, out_bf16, J, gran;
    long long units;
    exl3_qkv_post_args post; // finish kind 1: members are q, k, v (no y)
    int seg_cta[4];          // mixed bitrates: member m owns CTAs [seg_cta[m], seg_cta[m + 1])
    int seg_bits[3];         // mixed bitrates: bits of each member
    int ll_world;            // > 0: rows go as LL words into ll[0..ll_world) (exl3_gemv_peer; no y)
    uint64_t* ll[8];         // inbox (slot, this rank) of every rank of the group
    const uint32_t* epoch;   // own flag block's "last completed" epoch word
    // input prologue (PRO > 0): xh is not given but computed by each CTA for the k it reads, into its
    // own region of xs (laid out as xh: (nm, rows, k) fp16, xs_stride halves per CTA)
    const void* src;         // PRO 1: x (rows, k); PRO 2: gu (rows, 2k) = [gate | up]
    int src_dtype;           // EXL3_F16 / EXL3_BF16 / EXL3_F32
    const __half* suh;       // (nm, k) fp16 input signs
    __half* xs;
    long long xs_stride;
};

// Input prologue kinds: 0 = xh given; 1 = rotation of x (kernels.rot, kernels.py:451-458); 2 = SwiGLU
// of [gate | up] then the rotation (kernels.swiglu_rot, kernels.py:476-483).
enum : int { kProNone = 0, kProRot = 1, kProSwiglu = 2 };

constexpr int kRedStride = 8 * 128;   // floats per warp partial (8 rows x 128 columns)

template <int K, int NCW>
struct GemvShape {
    static constexpr int TW = 8 * K;                 // words per tile
    static constexpr int UW = 8 * TW;                // words per unit (8 tiles)
    static constexpr int UB = UW * 4;                // bytes per unit
    static constexpr int D0 = (96 * 1024) / (NCW * UB);
    static constexpr int DEPTH = D0 < 3 ? 3 : (D0 > 8 ? 8 : D0);   // units in flight per warp
    static constexpr int RING = NCW * DEPTH * UB;
    static constexpr int RED = NCW * kRedStride * 4;
    static constexpr int SMEM = RING + RED;
    static constexpr int THREADS = 32 * NCW;
};

// 32-bit: the host guarantees units * (grid + 1) < 2^32
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(uint32_t* p, unsigned v)
{
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ int owner_cta(unsigned u, unsigned U, unsigned G)
{
    return (int)(((u + 1) * G - 1) / U);
}

__device__ __forceinline__ int cta_start(unsigned c, unsigned U, unsigned G)
{
    return (int)(c * U / G);
}

// Sums of one block's CTA partials in the fixed order shared by every `rows` (row-exact calls stay
// row-exact): four accumulators take the partials c_first + j, c_first + j + 4, ... (CTA order within
// each); the caller adds them in order. NG thread groups per element, 4 / NG accumulators each, so a
// block split over many CTAs costs one round of L2 loads per 8 partials of a group (the loads of a
// round are all in flight before any add). gsum: 4 x E floats (accumulator-major) of shared memory.
template <int NG>
__device__ __forceinline__ void part_sums(const float* __restrict__ partials, int J, int jj0, int c_first, int c_last,
                                          int E, int ctid, int nthreads, float* gsum)
{
    constexpr int NA = 4 / NG;
    for (int it = ctid; it < NG * E; it += nthreads) {
        const int e = it % E, gq = it / E;
        float a[NA];
#pragma unroll
        for (int m = 0; m < NA; ++m) a[m] = 0.f;
        for (int c0 = c_first + gq; c0 <= c_last; c0 += 8 * NG) {
            float t[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int ci = c0 + NG * i;
                t[i] = ci <= c_last ? __ldcg(partials + ((size_t)ci * J + (ci == c_first ? jj0 : 0)) * kRedStride + e)
                                    : 0.f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (c0 + NG * i <= c_last) a[i % NA] += t[i];
        }
#pragma unroll
        for (int m = 0; m < NA; ++m) gsum[(gq + NG * m) * E + e] = a[m];
    }
}

// 128-point FWHT of one row held by one warp as v[i] = column lane + 32 i, then scale, svh, store.
__device__ __forceinline__ void fwht128_rows(float (&v)[4], int lane)
{
#pragma unroll
    for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float p = __shfl_xor_sync(0xffffffffu, v[i], h);
            v[i] = (lane & h) ? p - v[i] : v[i] + p;
        }
    }
    {   // h = 32: columns c, c + 32 are v[i], v[i + 1] for i even
        float a0 = v[0], a1 = v[1];
        v[0] = a0 + a1; v[1] = a0 - a1;
        a0 = v[2]; a1 = v[3];
        v[2] = a0 + a1; v[3] = a0 - a1;
    }
    {   // h = 64
        float a0 = v[0], a1 = v[2];
        v[0] = a0 + a1; v[2] = a0 - a1;
        a0 = v[1]; a1 = v[3];
        v[1] = a0 + a1; v[3] = a0 - a1;
    }
}

__device__ __forceinline__ float src_at(const void* src, int dtype, size_t i)
{
    if (dtype == EXL3_F16) return __half2float(static_cast<const __half*>(src)[i]);
    if (dtype == EXL3_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]);
    return static_cast<const float*>(src)[i];
}

// Input prologue: this CTA's rotated inputs for the 128-column k blocks [kb0, kb1) of every member and
// row, written into its xs region in the layout of xh. One warp per (member, row, block), with the
// arithmetic of exl3_rot / exl3_swiglu_rot (exl3_rot.cu), so the values are bit-identical to theirs.
template <int PRO, int NCW>
__device__ __forceinline__ void gemv_prologue(const GemvParams& p, __half* xs, int kb0, int kb1, int lane, int cw)
{
    const int nkb = kb1 - kb0, k = p.k;
    const int tasks = p.nm * p.rows * nkb;
    // A warp takes up to kBatch of its tasks at a time and issues all their loads before any math, so
    // their L2 round trips overlap instead of following one another.
    constexpr int kBatch = 4;
    constexpr int NV = PRO == kProSwiglu ? 2 : 1;                 // source values per element
    for (int t0 = cw; t0 < tasks; t0 += kBatch * NCW) {
        float in[kBatch][NV][4], sg[kBatch][4];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const int t = t0 + b * NCW;
            if (t >= tasks) break;
            const int kb = kb0 + t % nkb, mr = t / nkb, r = mr % p.rows, m = mr / p.rows;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = kb * 128 + lane + 32 * i;
                if constexpr (PRO == kProRot) {
                    in[b][0][i] = src_at(p.src, p.src_dtype, (size_t)r * k + c);
                } else {
                    in[b][0][i] = src_at(p.src, p.src_dtype, (size_t)r * 2 * k + c);
                    in[b][NV - 1][i] = src_at(p.src, p.src_dtype, (size_t)r * 2 * k + k + c);
                }
                sg[b][i] = __half2float(p.suh[(size_t)m * k + c]);
            }
        }
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const int t = t0 + b * NCW;
            if (t >= tasks) break;
            const int kb = kb0 + t % nkb, mr = t / nkb, r = mr % p.rows, m = mr / p.rows;
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float xv;
                if constexpr (PRO == kProRot) {
                    xv = in[b][0][i];
                } else {
                    const float gv = in[b][0][i], uv = in[b][NV - 1][i];
                    xv = gv / (1.0f + expf(-gv)) * uv;
                }
                v[i] = xv * sg[b][i];
            }
            fwht128_rows(v, lane);
            __half* o = xs + ((size_t)m * p.rows + r) * k + kb * 128;
#pragma unroll
            for (int i = 0; i < 4; ++i) o[lane + 32 * i] = __float2half_rn(v[i] * kHadScale);
        }
    }
}

template <typename OT>
__device__ __forceinline__ void finish_row(float (&v)[4], int lane, const float (&sv)[4], OT* yrow)
{
    fwht128_rows(v, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) yrow[lane + 32 * i] = from_f32<OT>(v[i] * kHadScale * sv[i]);
}

// Peer finish (exl3_gemv_peer): the row's values rounded to OT exactly as a stored y would be, pushed
// as LL words (column pairs + the next all-reduce's epoch) into every rank's inbox. Even lanes pair
// their column with the odd neighbour's.
template <typename OT>
__device__ __forceinline__ void finish_row_peer(float (&v)[4], int lane, const float (&sv)[4], uint32_t e,
                                                const GemvParams& p, int b, int r)
{
    fwht128_rows(v, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = lane + 32 * i;
        const OT o = from_f32<OT>(v[i] * kHadScale * sv[i]);
        const uint32_t lo = *reinterpret_cast<const unsigned short*>(&o);
        const uint32_t hi = __shfl_down_sync(0xffffffffu, lo, 1);
        if (!(lane & 1)) {
            const size_t j = ((size_t)r * p.n_total + (size_t)b * 128 + c) >> 1;
#pragma unroll
            for (int d = 0; d < 8; ++d)
                if (d < p.ll_world) st_ll(p.ll[d] + j, lo | (hi << 16), e);
        }
    }
}

// Per-lane operands of the q/k/v finish for row r of block b: the row's position, the norm weights of
// the block's member and the RoPE cos / sin at that position. The finishing warp loads them at the
// segment end, so their two dependent round trips (position, then the table rows) overlap the
// reduction and the cross-CTA arrival instead of following them.
struct QkvPre {
    long long pos;
    float w[4];
    float co[2], si[2];
};

template <typename T>
__device__ __forceinline__ void qkv_preload(const GemvParams& p, int b, int r, int lane, QkvPre& q)
{
    const exl3_qkv_post_args& a = p.post;
    const int m = b >= p.blk_off[2] ? 2 : (b >= p.blk_off[1] ? 1 : 0);
    q.pos = a.pos[r];
    if (m < 2) {
        const T* w = static_cast<const T*>(m == 0 ? a.q_norm_w : a.k_norm_w);
#pragma unroll
        for (int i = 0; i < 4; ++i) q.w[i] = to_f32(w[lane + 32 * i]);
        const float* cs = a.cos_table + (size_t)q.pos * 64;
        const float* sn = a.sin_table + (size_t)q.pos * 64;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            q.co[i] = cs[lane + 32 * i];
            q.si[i] = sn[lane + 32 * i];
        }
    }
}

// The q/k/v group's finish, fused with exl3_qkv_post: block b is one head of q (member 0), k (1) or
// v (2). The GEMV value is rounded to the model dtype T exactly as a stored y would be, then q/k get
// the per-head RMSNorm (MLX rounding) and rotate-half RoPE and go to q_out / the k cache, v to the v
// cache, all at this row's position. The arithmetic is exl3_qkv_post's (head_rms, rope_half) on the
// operands preloaded by qkv_preload.
template <typename T>
__device__ __forceinline__ void finish_qkv(float (&v)[4], int lane, const float (&sv)[4], const GemvParams& p, int b,
                                           int r, const QkvPre& q)
{
    fwht128_rows(v, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = to_f32(from_f32<T>(v[i] * kHadScale * sv[i]));
    const exl3_qkv_post_args& a = p.post;
    const int m = b >= p.blk_off[2] ? 2 : (b >= p.blk_off[1] ? 1 : 0);
    const int head = b - (m == 0 ? 0 : (m == 1 ? p.blk_off[1] : p.blk_off[2]));
    __half* o;
    if (m < 2) {
        // head RMSNorm (as head_rms), then rotate-half RoPE (as rope_half)
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) ss = fmaf(v[i], v[i], ss);
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / 128.0f + a.eps);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const T t = from_f32<T>(v[i] * inv);
            v[i] = to_f32(from_f32<T>(q.w[i] * to_f32(t)));
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float x1 = v[i], x2 = v[i + 2];
            v[i] = __fsub_rn(__fmul_rn(x1, q.co[i]), __fmul_rn(x2, q.si[i]));
            v[i + 2] = __fadd_rn(__fmul_rn(x2, q.co[i]), __fmul_rn(x1, q.si[i]));
        }
        o = m == 0 ? static_cast<__half*>(a.q_out) + ((size_t)r * a.hq + head) * 128
                   : static_cast<__half*>(a.k_cache) + ((size_t)head * a.max_len + q.pos) * 128;
    } else {
        o = static_cast<__half*>(a.v_cache) + ((size_t)head * a.max_len + q.pos) * 128;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) o[lane + 32 * i] = __float2half_rn(m == 2 ? v[i] : to_f32(from_f32<T>(v[i])));
}

// EPI: the finish of a block: 0 = y (exl3_gemv), 1 = exl3_qkv_post's (exl3_gemv_qkv_post), 2 = LL words
// into the peers' inboxes (exl3_gemv_peer). A template parameter, so the plain GEMV carries no code of
// the other two (measured: ~2.5 % of the sweep when they shared one kernel).
// The GEMV of one CTA: CTA c of the G CTAs that share the U granules of units starting at unit ubase
// (the whole launch, or one member's segment of a mixed-bitrate launch); coff is the launch-wide index
// of the segment's first CTA (its split-k partials).
// Two xh values: through the read-only path when xh is an input, through L2 when the CTA itself wrote
// them in its prologue (the non-coherent path may not see writes made during the kernel).
template <int PRO>
__device__ __forceinline__ uint32_t ld_x(const __half* p)
{
    if constexpr (PRO == kProNone) return __ldg(reinterpret_cast<const unsigned int*>(p));
    else return __ldcg(reinterpret_cast<const unsigned int*>(p));
}

template <int K, int CB, int NCW, int EPI, int PRO = kProNone>
__device__ __forceinline__ void gemv_body(const GemvParams& p, uint8_t* smem, const int c, const int G, const int coff,
                                          const int ubase, const unsigned U)
{
    using S = GemvShape<K, NCW>;
    static_assert(NCW >= 8, "the finish gives each of the up to 8 rows its own warp");
    float* red = reinterpret_cast<float*>(smem + S::RING);
    __shared__ int s_last;

    const int lane = threadIdx.x & 31;
    const int cw = threadIdx.x >> 5;
    const int ctid = threadIdx.x;
    // CTA ranges are whole granules of p.gran units (16 when k is a multiple of 256), so every block
    // segment inside a CTA is a whole number of rounds of the NCW warps
    const int gran = p.gran;
    const int u0 = ubase + cta_start(c, U, G) * gran, u1 = ubase + cta_start(c + 1, U, G) * gran;
    const int n_units = (int)(u1 - u0);
    const int KT = p.KT;
    const int rows = p.rows;
    const int b_first = (int)(u0 / KT), b_last = (int)((u1 - 1) / KT);

    // Every warp streams its own units (CTA unit indices cw, cw + NCW, ...) into a private ring of
    // DEPTH slots with 16-byte cp.async copies, DEPTH - 1 units ahead of the one it decodes. The
    // source pointer (already offset by this lane's first chunk) advances by a fixed stride while
    // the warp stays inside one 128-column block and is recomputed only when it moves to the next.
    constexpr int kChunks = S::UB / 16;                               // 16-byte chunks per unit
    constexpr int kPerLane = (kChunks + 31) / 32;
    uint32_t* wring = reinterpret_cast<uint32_t*>(smem) + (size_t)cw * S::DEPTH * S::UW + lane * 4;
    int fi = cw;                                                      // next unit index to fetch
    int fb = 0, fkt = 0;
    const uint32_t* fsrc = nullptr;
    size_t fstep = 0;                                                 // words between k-slices NCW apart
    auto fseek = [&]() {
        const int u = u0 + fi;
        fb = (int)(u / KT);
        fkt = u - fb * KT;
        const int m = (p.nm > 1 && fb >= p.blk_off[1]) ? ((p.nm > 2 && fb >= p.blk_off[2]) ? 2 : 1) : 0;
        const int ntm = m == 0 ? p.nt_member[0] : (m == 1 ? p.nt_member[1] : p.nt_member[2]);
        const int off = m == 0 ? 0 : (m == 1 ? p.blk_off[1] : p.blk_off[2]);
        const uint32_t* base = m == 0 ? p.trellis[0] : (m == 1 ? p.trellis[1] : p.trellis[2]);
        fsrc = base + ((size_t)fkt * ntm + (size_t)(fb - off) * 8) * S::TW + lane * 4;
        fstep = (size_t)NCW * ntm * S::TW;
    };
    if (fi < n_units) fseek();
    // ring slots as 32-bit shared-window byte offsets (no generic-pointer arithmetic per copy)
    const uint32_t wring32 = smem_addr(wring);
    uint32_t foff = 0;                                                // byte offset of the slot to fill
    auto fetch = [&]() {
        if (fi < n_units) {
            const uint32_t dst = wring32 + foff;
#pragma unroll
            for (int cidx = 0; cidx < kPerLane; ++cidx)
                if (kChunks % 32 == 0 || cidx * 32 + lane < kChunks) cp_async16_s(dst + cidx * 512, fsrc + cidx * 128);
            fi += NCW;
            fkt += NCW;
            if (fkt >= KT) {
                if (fi < n_units) fseek();
            } else {
                fsrc += fstep;
            }
        }
        cp_async_commit();                                    // (possibly empty) group per unit
        foff = foff + S::UB == S::DEPTH * S::UB ? 0u : foff + S::UB;
    };
#pragma unroll 1
    for (int d = 0; d < S::DEPTH - 1; ++d) fetch();
    // The weights are constant; everything from here on (xh, y, the split-k scratch) may be written or
    // read by the previous kernel in the stream, so under programmatic dependent launch the ring fill
    // above overlaps that kernel and the rest waits for it.
    pdl_trigger();
    pdl_wait();
    int cslot = 0;                                            // ring slot of the unit being decoded

    // Input prologue: the rotated inputs of the k blocks this CTA's units read, into its own xs region
    // (redundant across CTAs that read the same k, which costs less than a separate launch)
    __half* xs = nullptr;
    if constexpr (PRO != kProNone) {
        xs = p.xs + (size_t)(coff + c) * p.xs_stride;
        const int KB = p.k / 128;
        const int lo = u0 - b_first * KT, hi = u1 - b_last * KT;          // k-slices [lo, KT) .. [0, hi)
        if (b_first == b_last) {
            gemv_prologue<PRO, NCW>(p, xs, lo / 8, (hi + 7) / 8, lane, cw);
        } else if (b_last == b_first + 1 && hi < lo) {
            gemv_prologue<PRO, NCW>(p, xs, 0, (hi + 7) / 8, lane, cw);
            gemv_prologue<PRO, NCW>(p, xs, lo / 8, KB, lane, cw);
        } else {
            gemv_prologue<PRO, NCW>(p, xs, 0, KB, lane, cw);
        }
        __syncthreads();                                      // xs written by the CTA's warps
    }

    const int g = lane >> 2, q = lane & 3;
    const LaneWindow<K> lw(lane);
    const HashRegs hr = hash_regs<CB>();
    const bool xlane = g < rows;                  // this lane carries a row of xh

    for (int b = b_first; b <= b_last; ++b) {
        const int m = (p.nm > 1 && b >= p.blk_off[1]) ? ((p.nm > 2 && b >= p.blk_off[2]) ? 2 : 1) : 0;
        const __half* xrow = (PRO != kProNone ? xs : p.xh) + ((size_t)m * rows + g) * p.k;
        const int sa = max(u0, b * KT) - u0;
        const int se = min(u1, (b + 1) * KT) - u0;

        // acc[j]: the m16n8 fp32 accumulator of tile j (rows in the n dimension)
        float acc[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

        const int kt_base = u0 - b * KT;                     // k-slice of unit index 0 (may be < 0)
        int i = sa + ((cw - sa) % NCW + NCW) % NCW;
        // the lane's xh values for the next unit are fetched one unit ahead
        const __half* xp = xrow + (kt_base + i) * 16 + 2 * q;
        uint32_t x0n = 0, x1n = 0;
        if (i < se && xlane) {
            x0n = ld_x<PRO>(xp);
            x1n = ld_x<PRO>(xp + 8);
        }
        for (; i < se; i += NCW) {
            const uint32_t x0 = x0n, x1 = x1n;
            xp += NCW * 16;
            if (i + NCW < se && xlane) {
                x0n = ld_x<PRO>(xp);
                x1n = ld_x<PRO>(xp + 8);
            }
            // x duplicated across each k pair: (x[2q], x[2q]), (x[2q+8], ..), (x[2q+1], ..), (x[2q+9], ..)
            const uint32_t be0 = prmt(x0, x0, 0x1010), be1 = prmt(x1, x1, 0x1010);
            const uint32_t bo0 = prmt(x0, x0, 0x3232), bo1 = prmt(x1, x1, 0x3232);
            fetch();                                  // unit + DEPTH - 1 (or an empty group)
            cp_async_wait<S::DEPTH - 1>();            // this unit's copies have landed
            __syncwarp();
            const uint32_t* unit = wring - lane * 4 + (size_t)cslot * S::UW;
            cslot = cslot + 1 == S::DEPTH ? 0 : cslot + 1;
            // Tile j + 1 is decoded before tile j's two MMAs are issued: the source order hands the
            // scheduler the next tile's integer work to interleave with the MMAs (bit-identical,
            // measured 1-3 % faster per launch than decode-then-MMA per tile).
            uint32_t ac[8];
            decode_tile<K, CB>(unit, lw, hr, ac);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint32_t an[8];
                if (j < 7) decode_tile<K, CB>(unit + (j + 1) * S::TW, lw, hr, an);
                // even k of the tile: (g,2q) (g+8,2q) (g,2q+8) (g+8,2q+8); odd k: the +1 neighbours
                mma16816(acc[j], ac[0], ac[4], ac[2], ac[6], be0, be1);
                mma16816(acc[j], ac[1], ac[5], ac[3], ac[7], bo0, bo1);
                if (j < 7) {
#pragma unroll
                    for (int t = 0; t < 8; ++t) ac[t] = an[t];
                }
            }
            __syncwarp();                             // the slot is refilled by the next fetch
        }

        // ---- segment end: warp partials -> shared memory, summed in warp order
        float* rw = red + cw * kRedStride;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int col = 16 * j + g;
            if (2 * q < rows) {
                rw[(2 * q) * 128 + col] = acc[j][0];
                rw[(2 * q) * 128 + col + 8] = acc[j][2];
            }
            if (2 * q + 1 < rows) {
                rw[(2 * q + 1) * 128 + col] = acc[j][1];
                rw[(2 * q + 1) * 128 + col + 8] = acc[j][3];
            }
        }
        // The finish's output scales (and the peer push's epoch) are read now, so their round trip
        // overlaps the reduction and the cross-CTA arrival instead of following them. Warp cw finishes
        // row cw (rows <= 8 < NCW); the epoch is final here, since the all-reduce that advances it runs
        // after this kernel has completed.
        float sv[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t epoch = 0;
        QkvPre qpre;
        if (cw < rows) {
#pragma unroll
            for (int ii = 0; ii < 4; ++ii) sv[ii] = __half2float(p.svh[(size_t)b * 128 + lane + 32 * ii]);
            if constexpr (EPI == 2) epoch = *reinterpret_cast<const volatile uint32_t*>(p.epoch) + 1u;
            if constexpr (EPI == 1) {
                if (p.out_bf16) qkv_preload<__nv_bfloat16>(p, b, cw, lane, qpre);
                else qkv_preload<__half>(p, b, cw, lane, qpre);
            }
        }
        __syncthreads();
        for (int e = ctid; e < rows * 128; e += 32 * NCW) {
            float v = red[e];
#pragma unroll
            for (int w = 1; w < NCW; ++w) v += red[w * kRedStride + e];
            red[e] = v;
        }
        __syncthreads();

        const bool whole = b * KT >= u0 && (b + 1) * KT <= u1;
        bool finish = whole;
        if (!whole) {
            // one warp publishes the CTA's partial and takes the block's arrival ticket
            if (cw == 0) {
                float* gp = p.partials + ((size_t)(coff + c) * p.J + (b - b_first)) * kRedStride;
                for (int e = lane; e < rows * 128; e += 32) gp[e] = red[e];
                __syncwarp();                                // the warp's stores, ordered before lane 0's release
                if (lane == 0) {
                    const int c_first = owner_cta((b * KT - ubase) / gran, U, G);
                    const int c_last = owner_cta(((b + 1) * KT - 1 - ubase) / gran, U, G);
                    // one acquire-release RMW: publishes this CTA's partial and, for the last arriver,
                    // makes every other CTA's partial visible (no separate fences)
                    const unsigned old = atom_add_acq_rel_gpu(&p.counters[b], 1u);
                    s_last = old == (unsigned)(c_last - c_first);
                }
            }
            __syncthreads();
            finish = s_last != 0;
            if (finish) {
                const int c_first = owner_cta((b * KT - ubase) / gran, U, G);
                const int c_last = owner_cta(((b + 1) * KT - 1 - ubase) / gran, U, G);
                const float* parts = p.partials + (size_t)coff * p.J * kRedStride;   // the segment's CTAs
                // CTA c_first holds the block in its slot jj0, every later CTA in its slot 0. Up to 8
                // partials: one round of loads, added in CTA order; more: part_sums' order. The choice
                // depends on the grid only, never on `rows`.
                const int jj0 = b - (ubase + cta_start(c_first, U, G) * gran) / KT;
                const int E = rows * 128;
                if (c_last - c_first < 8) {
                    for (int e = ctid; e < E; e += 32 * NCW) {
                        float t[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int ci = c_first + i;
                            t[i] = ci <= c_last ? __ldcg(parts + ((size_t)ci * p.J + (i == 0 ? jj0 : 0)) * kRedStride + e)
                                                : 0.f;
                        }
                        float v = t[0];
#pragma unroll
                        for (int i = 1; i < 8; ++i)
                            if (c_first + i <= c_last) v += t[i];
                        red[e] = v;
                    }
                } else {
                    float* gsum = red + NCW * kRedStride / 2;
                    if (E <= 128) part_sums<4>(parts, p.J, jj0, c_first, c_last, E, ctid, 32 * NCW, gsum);
                    else if (E <= 256) part_sums<2>(parts, p.J, jj0, c_first, c_last, E, ctid, 32 * NCW, gsum);
                    else part_sums<1>(parts, p.J, jj0, c_first, c_last, E, ctid, 32 * NCW, gsum);
                    __syncthreads();
                    for (int e = ctid; e < E; e += 32 * NCW)
                        red[e] = ((gsum[e] + gsum[E + e]) + gsum[2 * E + e]) + gsum[3 * E + e];
                }
                if (ctid == 0) atomicExch(&p.counters[b], 0u);
                __syncthreads();
            }
        }
        if (finish) {
            if (cw < rows) {
                const int r = cw;
                float v[4];
#pragma unroll
                for (int ii = 0; ii < 4; ++ii) v[ii] = red[r * 128 + lane + 32 * ii];
                const size_t yoff = (size_t)r * p.n_total + (size_t)b * 128;
                if constexpr (EPI == 1) {
                    if (p.out_bf16) finish_qkv<__nv_bfloat16>(v, lane, sv, p, b, r, qpre);
                    else finish_qkv<__half>(v, lane, sv, p, b, r, qpre);
                } else if constexpr (EPI == 2) {
                    if (p.out_bf16) finish_row_peer<__nv_bfloat16>(v, lane, sv, epoch, p, b, r);
                    else finish_row_peer<__half>(v, lane, sv, epoch, p, b, r);
                } else if (p.out_bf16) {
                    finish_row(v, lane, sv, reinterpret_cast<__nv_bfloat16*>(p.y) + yoff);
                } else {
                    finish_row(v, lane, sv, reinterpret_cast<__half*>(p.y) + yoff);
                }
            }
        }
        __syncthreads();   // red is reused by the next segment
    }
}

template <int K, int CB, int NCW, int EPI, int PRO>
__global__ void __launch_bounds__(32 * NCW, 1) gemv_kernel(const GemvParams p)
{
    extern __shared__ __align__(128) uint8_t smem[];
    gemv_body<K, CB, NCW, EPI, PRO>(p, smem, blockIdx.x, gridDim.x, 0, 0, (unsigned)(p.units / p.gran));
}

// Members of different bitrates in one launch (e.g. q/k/v quantised at different bpw): member m owns
// the CTAs [seg_cta[m], seg_cta[m + 1]) and runs the body of its own bitrate over its own blocks, so a
// group still takes one launch (and one fused finish) whatever its members' bitrates.
template <int CB, int NCW, int EPI>
__global__ void __launch_bounds__(32 * NCW, 1) gemv_seg_kernel(const GemvParams p)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const int bx = blockIdx.x;
    const int m = (p.nm > 2 && bx >= p.seg_cta[2]) ? 2 : ((p.nm > 1 && bx >= p.seg_cta[1]) ? 1 : 0);
    const int c0 = m == 0 ? 0 : (m == 1 ? p.seg_cta[1] : p.seg_cta[2]);
    const int c1 = m == 0 ? p.seg_cta[1] : (m == 1 ? p.seg_cta[2] : p.seg_cta[3]);
    const int b0 = m == 0 ? 0 : (m == 1 ? p.blk_off[1] : p.blk_off[2]);
    const int b1 = m + 1 < p.nm ? (m == 0 ? p.blk_off[1] : p.blk_off[2]) : p.blk_off[3];
    const int bits = m == 0 ? p.seg_bits[0] : (m == 1 ? p.seg_bits[1] : p.seg_bits[2]);
    const int ubase = b0 * p.KT;
    const unsigned U = (unsigned)((b1 - b0) * p.KT / p.gran);
    const int c = bx - c0, G = c1 - c0;
    switch (bits) {
    case 1: gemv_body<1, CB, NCW, EPI>(p, smem, c, G, c0, ubase, U); break;
    case 2: gemv_body<2, CB, NCW, EPI>(p, smem, c, G, c0, ubase, U); break;
    case 3: gemv_body<3, CB, NCW, EPI>(p, smem, c, G, c0, ubase, U); break;
    case 4: gemv_body<4, CB, NCW, EPI>(p, smem, c, G, c0, ubase, U); break;
    case 5: gemv_body<5, CB, NCW, EPI>(p, smem, c, G, c0, ubase, U); break;
    case 6: gemv_body<6, CB, NCW, EPI>(p, smem, c, G, c0, ubase, U); break;
    case 7: gemv_body<7, CB, NCW, EPI>(p, smem, c, G, c0, ubase, U); break;
    default: gemv_body<8, CB, NCW, EPI>(p, smem, c, G, c0, ubase, U); break;
    }
}

// Dynamic shared memory of the body for `bits` (a mixed launch takes the largest of its members').
inline int gemv_smem_bytes(int bits)
{
    switch (bits) {
    case 1: return GemvShape<1, kNCW>::SMEM;
    case 2: return GemvShape<2, kNCW>::SMEM;
    case 3: return GemvShape<3, kNCW>::SMEM;
    case 4: return GemvShape<4, kNCW>::SMEM;
    case 5: return GemvShape<5, kNCW>::SMEM;
    case 6: return GemvShape<6, kNCW>::SMEM;
    case 7: return GemvShape<7, kNCW>::SMEM;
    default: return GemvShape<8, kNCW>::SMEM;
    }
}


template <int K, int CB, int EPI, int PRO>
static int launch_gemv_k(const GemvParams& prm, int grid, cudaStream_t s)
{
    using S = GemvShape<K, kNCW>;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(gemv_kernel<K, CB, kNCW, EPI, PRO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 S::SMEM) != cudaSuccess)
            return EXL3_E_CUDA;
        attr_set[dev] = true;
    }
    if (int e_ = launch_pdl(gemv_kernel<K, CB, kNCW, EPI, PRO>, grid, S::THREADS, S::SMEM, s, prm)) return e_;
    return launch_status();
}

template <int K, int EPI, int PRO>
static int launch_gemv_cb(int cb, const GemvParams& prm, int grid, cudaStream_t s)
{
    switch (cb) {
    case 0: return launch_gemv_k<K, 0, EPI, PRO>(prm, grid, s);
    case 1: return launch_gemv_k<K, 1, EPI, PRO>(prm, grid, s);
    default: return launch_gemv_k<K, 2, EPI, PRO>(prm, grid, s);
    }
}

// Every K and codebook for one finish kind; instantiated once per kind (exl3_gemv.cu: 0,
// exl3_gemv_fused.cu: 1 and 2) so the translation units compile in parallel.
template <int EPI, int PRO = kProNone>
int launch_gemv_epi(int bits, int cb, const GemvParams& prm, int grid, cudaStream_t s)
{
    switch (bits) {
    case 1: return launch_gemv_cb<1, EPI, PRO>(cb, prm, grid, s);
    case 2: return launch_gemv_cb<2, EPI, PRO>(cb, prm, grid, s);
    case 3: return launch_gemv_cb<3, EPI, PRO>(cb, prm, grid, s);
    case 4: return launch_gemv_cb<4, EPI, PRO>(cb, prm, grid, s);
    case 5: return launch_gemv_cb<5, EPI, PRO>(cb, prm, grid, s);
    case 6: return launch_gemv_cb<6, EPI, PRO>(cb, prm, grid, s);
    case 7: return launch_gemv_cb<7, EPI, PRO>(cb, prm, grid, s);
    default: return launch_gemv_cb<8, EPI, PRO>(cb, prm, grid, s);
    }
}

template <int CB, int EPI>
static int launch_gemv_seg_v(const GemvParams& prm, int grid, int smem, cudaStream_t s)
{
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        int mx = 0;
        for (int b = 1; b <= 8; ++b) mx = gemv_smem_bytes(b) > mx ? gemv_smem_bytes(b) : mx;
        if (cudaFuncSetAttribute(gemv_seg_kernel<CB, kNCW, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 mx) != cudaSuccess)
            return EXL3_E_CUDA;
        attr_set[dev] = true;
    }
    if (int e_ = launch_pdl(gemv_seg_kernel<CB, kNCW, EPI>, grid, 32 * kNCW, smem, s, prm)) return e_;
    return launch_status();
}

// Mixed-bitrate launch for one finish kind (instantiated in exl3_gemv_mixed.cu).
template <int EPI>
int launch_gemv_seg(int cb, const GemvParams& prm, int grid, int smem, cudaStream_t s)
{
    switch (cb) {
    case 0: return launch_gemv_seg_v<0, EPI>(prm, grid, smem, s);
    case 1: return launch_gemv_seg_v<1, EPI>(prm, grid, smem, s);
    default: return launch_gemv_seg_v<2, EPI>(prm, grid, smem, s);
    }
}

extern template int launch_gemv_seg<0>(int, const GemvParams&, int, int, cudaStream_t);
extern template int launch_gemv_seg<1>(int, const GemvParams&, int, int, cudaStream_t);

extern template int launch_gemv_epi<0>(int, int, const GemvParams&, int, cudaStream_t);
extern template int launch_gemv_epi<1>(int, int, const GemvParams&, int, cudaStream_t);
extern template int launch_gemv_epi<2>(int, int, const GemvParams&, int, cudaStream_t);
extern template int launch_gemv_epi<0, kProRot>(int, int, const GemvParams&, int, cudaStream_t);
extern template int launch_gemv_epi<0, kProSwiglu>(int, int, const GemvParams&, int, cudaStream_t);
extern template int launch_gemv_epi<2, kProSwiglu>(int, int, const GemvParams&, int, cudaStream_t);

}  // namespace exl3
