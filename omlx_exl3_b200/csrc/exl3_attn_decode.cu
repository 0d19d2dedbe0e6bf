// Decode attention (rows new tokens, head_dim 128, GQA) over the fp16 KV cache, fused with o_proj's
// input rotation: xh = fp16(had128(fp16(softmax(q k^T / sqrt(128)) v) * suh) / sqrt(128)).
//
// Replaces, in the decode step, the framework's scaled-dot-product attention call and the exl3_rot
// launch that follows it (the reference has no attention kernel: attention belongs to the model
// library; its rotation is src/omlx/exl3/kernels.py:451-458). Two launches, both dependent launches:
//
//   split kernel    grid (splits, kv heads), 2..8 warps per CTA (about one CTA per SM over all kv
//                   heads), each warp a contiguous range of ppw positions (ppw multiple of 16). The
//                   warp's K and V rows are copied into shared memory with 16-byte asynchronous copies
//                   (two whole rows per warp instruction; one commit group per 16-position step, so
//                   the math on the first step starts while later rows land) into padded rows, so the
//                   fragment reads below are free of bank conflicts. (One bulk copy per 256-byte row
//                   was measured first: the copy engine's per-request rate made issuing them alone
//                   take ~2 us per CTA.) Rows of earlier steps are
//                   copied before the dependency wait (they overlap the previous kernel); only this
//                   step's rows wait for it. m16n8k16 tensor-core MMAs with positions as the 16-row
//                   side: S^T = K Q^T (the GQA group's q vectors, rows x heads per kv head <= 16, are
//                   one or two n8 tiles), the online softmax in fp32 (exp2 with the scale folded in),
//                   then O^T += V^T P^T with P^T moved from accumulator to operand layout by movmatrix.
//                   Warps merge in shared memory; each CTA writes (max, sum, O) per q vector.
//   combine kernel  grid (q vectors, kv heads): merges the splits in split order (max, rescale, sum),
//                   divides, rounds to fp16 (the attention output), multiplies by suh, runs the
//                   128-point FWHT (Sylvester order) and writes xh. (Merging in the last CTA of each
//                   kv head instead was measured at ~13 us per call: one CTA per head serialises what
//                   the q x head CTAs here do in parallel.)
//
// Causal rule: new row i sits at position T - rows + i and sees positions <= that (the framework
// call this replaces used the same mask). Positions >= T are never read.
#include <cuda_runtime.h>

#include <mutex>

#include "exl3_b200.h"
#include "exl3_common.cuh"
#include "exl3_host.h"

namespace exl3 {

constexpr int kAttMaxWarps = 8;
constexpr int kKStride = 320;             // bytes per K row in shared memory (256 + 64)
constexpr int kVStride = 272;             // bytes per V row (256 + 16)
constexpr int kRowBytes = kKStride + kVStride;
constexpr int kAttPart = 132;             // floats per (kv head, split, q vector): max, sum, 2 pad, O[128]
constexpr int kAttMaxQ = 16;              // q vectors per CTA (two n8 tiles)
constexpr int kAttMaxQGroups = 4;         // q groups of kAttMaxQ per kv head: rows x grp <= 64
constexpr int kAttMaxSplits = 512;
constexpr int kAttMaxCta = 384;           // positions per CTA (shared memory: 384 x 592 bytes)
constexpr int kCombThreads = 256;
constexpr int kAttHeader = 16;            // reserved workspace bytes before the partials
constexpr float kAttScaleLog2 = 0.08838834764831845f * 1.4426950408889634f;   // 1/sqrt(128) * log2(e)

struct AttnParams {
    const __half* q;          // (rows, hq, 128)
    const __half* kc;         // (hkv, max_len, 128)
    const __half* vc;
    float* part;              // (hkv, splits, nq, kAttPart)
    int rows, hq, hkv, grp, nq, max_len, T, ppw, splits;
};

__device__ __forceinline__ uint32_t word_of(const uint4& v, int w)
{
    return w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w));
}

// cp.async.wait_group with a run-time count (0 .. 3)
__device__ __forceinline__ void cp_async_wait_upto(int n)
{
    if (n <= 0) cp_async_wait<0>();
    else if (n == 1) cp_async_wait<1>();
    else if (n == 2) cp_async_wait<2>();
    else cp_async_wait<3>();
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a)
{
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi)
{
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// NQT n8 tiles of q vectors (nq <= 8 NQT). Per 16-position step of a warp:
//   S^T (16 positions x 8 q) = K Q^T: A = K rows (lane (g, c) reads 64 contiguous bytes of rows g and
//     g + 8; logical k (2c + e) of k-step ks <-> d = 8c + 32 (ks >> 1) + 4 (ks & 1) + e, k (2c + 8 + e)
//     <-> that d + 2), B = Q^T (the same d map: one 8-byte load per k-step);
//   online softmax per q column (position max over the 8 lanes of a column group);
//   O^T (128 d x 8 q) += V^T P^T: B = P^T, the S^T accumulators transposed per 8 x 8 block by
//     movmatrix; A = V^T, row g of m-tile mt is d = 8g + mt, row g + 8 is d = 64 + 8g + mt, packed
//     from two 16-byte row reads per position with byte permutes.
template <int NQT>
__global__ void __launch_bounds__(32 * kAttMaxWarps, 1) attn_split_kernel(const AttnParams p)
{
    extern __shared__ __align__(128) uint8_t att_sm[];
    __shared__ float wm[kAttMaxWarps][kAttMaxQ], wl[kAttMaxWarps][kAttMaxQ];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int h = blockIdx.y, s = blockIdx.x;
    // q vectors [qg0, qg0 + nql) of this kv head's group (q vector j = new row j / grp, head j % grp)
    const int qg0 = kAttMaxQ * blockIdx.z, nql = min(kAttMaxQ, p.nq - qg0);
    const int ppw = p.ppw;
    uint8_t* kbuf = att_sm + (size_t)warp * ppw * kRowBytes;
    uint8_t* vbuf = kbuf + (size_t)ppw * kKStride;
    const int pos0 = (s * nw + warp) * ppw;
    const int nval = max(0, min(ppw, p.T - pos0));           // positions < T in this warp's range
    const int nsteps = (nval + 15) >> 4;
    const int old_end = p.T - p.rows;                        // rows below this come from earlier steps
    const __half* kh = p.kc + (size_t)h * p.max_len * 128;
    const __half* vh = p.vc + (size_t)h * p.max_len * 128;

    // step t (rows 16t .. 16t + 15) is commit group t; rows of this step's tokens (>= old_end) go in
    // one more group after the dependency wait. Per step and lane: 8 K and 8 V 16-byte copies, a warp
    // instruction covering two whole rows.
    for (int t = 0; t < nsteps; ++t) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int qd = 32 * j + lane, r = 16 * t + (qd >> 4), ch = qd & 15;
            if (r < nval && pos0 + r < old_end) {
                cp_async16(kbuf + (size_t)r * kKStride + 16 * ch, kh + (size_t)(pos0 + r) * 128 + 8 * ch);
                cp_async16(vbuf + (size_t)r * kVStride + 16 * ch, vh + (size_t)(pos0 + r) * 128 + 8 * ch);
            }
        }
        cp_async_commit();
    }
    // V rows past T are never copied; zero them (a zero probability times stale bits could be NaN)
    for (int e = lane; e < (16 * nsteps - nval) * 16; e += 32)
        *reinterpret_cast<uint4*>(vbuf + (size_t)(nval + e / 16) * kVStride + (e % 16) * 16) = make_uint4(0, 0, 0, 0);

    pdl_trigger();
    pdl_wait();                                              // q and this step's k/v rows are written
    const bool fresh = pos0 + nval > old_end;                // this warp holds rows of this step's tokens
    if (fresh) {
        for (int i = (old_end > pos0 ? old_end - pos0 : 0) * 16 + lane; i < nval * 16; i += 32) {
            const int r = i >> 4, ch = i & 15;
            cp_async16(kbuf + (size_t)r * kKStride + 16 * ch, kh + (size_t)(pos0 + r) * 128 + 8 * ch);
            cp_async16(vbuf + (size_t)r * kVStride + 16 * ch, vh + (size_t)(pos0 + r) * 128 + 8 * ch);
        }
    }
    cp_async_commit();

    // Q^T as the B operand; q column jl = 8 qt + g of n-tile qt is q vector qg0 + jl
    uint32_t qb[NQT][8][2];
    int lim[NQT][2];                                         // last visible position of column 8 qt + 2c + e
#pragma unroll
    for (int qt = 0; qt < NQT; ++qt) {
        const int jl = 8 * qt + g, j = qg0 + jl;
        const __half* qv = p.q + ((size_t)(j / p.grp) * p.hq + (size_t)h * p.grp + j % p.grp) * 128;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const int d0 = 8 * c + 32 * (ks >> 1) + 4 * (ks & 1);
            const uint2 v = jl < nql ? *reinterpret_cast<const uint2*>(qv + d0) : make_uint2(0, 0);
            qb[qt][ks][0] = v.x;
            qb[qt][ks][1] = v.y;
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int jj = 8 * qt + 2 * c + e;
            lim[qt][e] = jj < nql ? p.T - p.rows + (qg0 + jj) / p.grp : -1;
        }
    }

    float oacc[8][NQT][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int qt = 0; qt < NQT; ++qt) oacc[mt][qt][0] = oacc[mt][qt][1] = oacc[mt][qt][2] = oacc[mt][qt][3] = 0.f;
    float m[NQT][2], l[NQT][2];
#pragma unroll
    for (int qt = 0; qt < NQT; ++qt) m[qt][0] = m[qt][1] = -INFINITY, l[qt][0] = l[qt][1] = 0.f;

    for (int t = 0; t < nsteps; ++t) {
        // groups after step t may still be in flight (none if this warp holds fresh rows)
        cp_async_wait_upto(fresh ? 0 : nsteps - t);
        __syncwarp();
        const int t0 = 16 * t;
        // S^T for positions t0 .. t0 + 15 (rows g: t0 + g, rows g + 8: t0 + 8 + g)
        uint4 ka[4], kb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ka[i] = *reinterpret_cast<const uint4*>(kbuf + (size_t)(t0 + g) * kKStride + 16 * c + 64 * i);
            kb[i] = *reinterpret_cast<const uint4*>(kbuf + (size_t)(t0 + 8 + g) * kKStride + 16 * c + 64 * i);
        }
        float sacc[NQT][4];
#pragma unroll
        for (int qt = 0; qt < NQT; ++qt) {
            float se[4] = {0.f, 0.f, 0.f, 0.f}, so[4] = {0.f, 0.f, 0.f, 0.f};   // even / odd k-steps: shorter chains
#pragma unroll
            for (int ks = 0; ks < 8; ks += 2) {
                mma16816(se, word_of(ka[ks >> 1], 0), word_of(kb[ks >> 1], 0), word_of(ka[ks >> 1], 1),
                         word_of(kb[ks >> 1], 1), qb[qt][ks][0], qb[qt][ks][1]);
                mma16816(so, word_of(ka[ks >> 1], 2), word_of(kb[ks >> 1], 2), word_of(ka[ks >> 1], 3),
                         word_of(kb[ks >> 1], 3), qb[qt][ks + 1][0], qb[qt][ks + 1][1]);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) sacc[qt][i] = se[i] + so[i];
        }
        // online softmax (log2 domain) per q column; [0], [1]: position t0 + g, [2], [3]: t0 + 8 + g
        const int pa = pos0 + t0 + g, pb = pa + 8;
        uint32_t pbf[NQT][2];
#pragma unroll
        for (int qt = 0; qt < NQT; ++qt) {
            float x[4];
            x[0] = pa <= lim[qt][0] ? sacc[qt][0] * kAttScaleLog2 : -INFINITY;
            x[1] = pa <= lim[qt][1] ? sacc[qt][1] * kAttScaleLog2 : -INFINITY;
            x[2] = pb <= lim[qt][0] ? sacc[qt][2] * kAttScaleLog2 : -INFINITY;
            x[3] = pb <= lim[qt][1] ? sacc[qt][3] * kAttScaleLog2 : -INFINITY;
            float mx0 = fmaxf(x[0], x[2]), mx1 = fmaxf(x[1], x[3]);
#pragma unroll
            for (int o = 4; o <= 16; o <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
            }
            const float n0 = fmaxf(m[qt][0], mx0), n1 = fmaxf(m[qt][1], mx1);
            const float b0 = n0 == -INFINITY ? 0.f : n0, b1 = n1 == -INFINITY ? 0.f : n1;
            const float cr0 = exp2f(m[qt][0] - b0), cr1 = exp2f(m[qt][1] - b1);
            m[qt][0] = n0;
            m[qt][1] = n1;
            const float p0 = exp2f(x[0] - b0), p1 = exp2f(x[1] - b1);
            const float p2 = exp2f(x[2] - b0), p3 = exp2f(x[3] - b1);
            l[qt][0] = l[qt][0] * cr0 + (p0 + p2);
            l[qt][1] = l[qt][1] * cr1 + (p1 + p3);
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                oacc[mt][qt][0] *= cr0;
                oacc[mt][qt][1] *= cr1;
                oacc[mt][qt][2] *= cr0;
                oacc[mt][qt][3] *= cr1;
            }
            // P^T as the B operand: b0 = P^T[t0 + 2c, t0 + 2c + 1][q g], b1 = the same at t0 + 8
            pbf[qt][0] = movmatrix_trans(pack_half2(p0, p1));
            pbf[qt][1] = movmatrix_trans(pack_half2(p2, p3));
        }
        // V rows t0 + {2c, 2c + 1, 2c + 8, 2c + 9}, d 8g .. 8g + 7 and 64 + 8g .. 64 + 8g + 7
        uint4 vq[4][2];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = t0 + 2 * c + (e & 1) + 8 * (e >> 1);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
                vq[e][hh] = *reinterpret_cast<const uint4*>(vbuf + (size_t)row * kVStride + 16 * g + 128 * hh);
        }
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            const uint32_t sel = (mt & 1) ? 0x7632u : 0x5410u;
            const int w = mt >> 1;
            const uint32_t a0 = __byte_perm(word_of(vq[0][0], w), word_of(vq[1][0], w), sel);
            const uint32_t a1 = __byte_perm(word_of(vq[0][1], w), word_of(vq[1][1], w), sel);
            const uint32_t a2 = __byte_perm(word_of(vq[2][0], w), word_of(vq[3][0], w), sel);
            const uint32_t a3 = __byte_perm(word_of(vq[2][1], w), word_of(vq[3][1], w), sel);
#pragma unroll
            for (int qt = 0; qt < NQT; ++qt) mma16816(oacc[mt][qt], a0, a1, a2, a3, pbf[qt][0], pbf[qt][1]);
        }
    }
#pragma unroll
    for (int qt = 0; qt < NQT; ++qt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
#pragma unroll
            for (int o = 4; o <= 16; o <<= 1) l[qt][e] += __shfl_xor_sync(0xffffffffu, l[qt][e], o);

    // the warp's (max, sum, O) into its own (now free) region, then the CTA merge
    __syncwarp();
    float* ob = reinterpret_cast<float*>(kbuf);
#pragma unroll
    for (int qt = 0; qt < NQT; ++qt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int q = 8 * qt + 2 * c + e;                // local to this CTA's q group
            if (q >= nql) continue;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                ob[q * 128 + 8 * g + mt] = oacc[mt][qt][e];
                ob[q * 128 + 64 + 8 * g + mt] = oacc[mt][qt][2 + e];
            }
            if (g == 0) {
                wm[warp][q] = m[qt][e];
                wl[warp][q] = l[qt][e];
            }
        }
    __syncthreads();
    // per q vector: the CTA max, the warps' weights and the CTA sum (one thread each), then O per (q, d)
    if (threadIdx.x < nql) {
        const int q = threadIdx.x;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttMaxWarps; ++w)
            if (w < nw) M = fmaxf(M, wm[w][q]);
        const float base = M == -INFINITY ? 0.f : M;
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < kAttMaxWarps; ++w)
            if (w < nw) {
                const float f = exp2f(wm[w][q] - base);
                wm[w][q] = f;                                // now the warp's weight
                L += f * wl[w][q];
            }
        float* dst = p.part + (((size_t)h * p.splits + s) * p.nq + qg0 + q) * kAttPart;
        dst[0] = M;
        dst[1] = L;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nql * 128; i += blockDim.x) {
        const int q = i >> 7, d = i & 127;
        float O = 0.f;
#pragma unroll
        for (int w = 0; w < kAttMaxWarps; ++w)
            if (w < nw) O += wm[w][q] * reinterpret_cast<const float*>(att_sm + (size_t)w * ppw * kRowBytes)[i];
        p.part[(((size_t)h * p.splits + s) * p.nq + qg0 + q) * kAttPart + 4 + d] = O;
    }

}

// About one CTA per SM over all kv heads: P positions per CTA (a multiple of 16, 128 .. 384), in
// 8 warps of ppw positions (16, 32 or 48: at most 3 commit groups pending per warp).
static int attn_plan(int hkv, int T, int* warps, int* ppw, int* splits)
{
    const int sms = device_sm_count();
    int P = (T * hkv + sms - 1) / sms;
    P = (P + 15) / 16 * 16;
    P = P > kAttMaxCta ? kAttMaxCta : (P < 128 ? 128 : P);      // >= 8 warps of 16: fewer splits to merge
    const int nw = P / 16 < 2 ? 2 : (P / 16 > kAttMaxWarps ? kAttMaxWarps : P / 16);
    int per = ((P + nw - 1) / nw + 15) / 16 * 16;
    if (nw * per > kAttMaxCta) per = kAttMaxCta / nw / 16 * 16;
    const int sp = (T + nw * per - 1) / (nw * per);
    if (sp > kAttMaxSplits) return EXL3_E_SHAPE;
    *warps = nw;
    *ppw = per;
    *splits = sp;
    return EXL3_OK;
}

// One CTA per (q vector, kv head). Every load is issued right after the dependency wait: thread t
// holds (max, sum) of split t and the float4 columns 4 lane .. 4 lane + 3 of splits warp, warp + 8, ...
__global__ void __launch_bounds__(kCombThreads) attn_combine_kernel(const float* __restrict__ part, int splits, int nq,
                                                                   int grp, int hq, const __half* __restrict__ suh,
                                                                   __half* __restrict__ xh)
{
    constexpr int NW = kCombThreads / 32;
    constexpr int OB = 8;                                    // float4 loads per thread in flight
    pdl_trigger();
    pdl_wait();                                              // the split kernel's partials
    __shared__ float wsp[kAttMaxSplits];
    __shared__ float red[NW][128];
    __shared__ float wred[NW];
    __shared__ float vrow[128];
    const int q = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t stride = (size_t)nq * kAttPart;
    const float* base = part + ((size_t)h * splits * nq + q) * kAttPart;

    float4 ov[OB];
#pragma unroll
    for (int i = 0; i < OB; ++i) {
        const int sp = warp + NW * i;
        ov[i] = sp < splits ? __ldcg(reinterpret_cast<const float4*>(base + sp * stride + 4) + lane)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float ms[kAttMaxSplits / kCombThreads], ls[kAttMaxSplits / kCombThreads];
#pragma unroll
    for (int i = 0; i < kAttMaxSplits / kCombThreads; ++i) {
        const int sp = tid + kCombThreads * i;
        const float2 v = sp < splits ? __ldcg(reinterpret_cast<const float2*>(base + sp * stride))
                                     : make_float2(-INFINITY, 0.f);
        ms[i] = v.x;
        ls[i] = v.y;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kAttMaxSplits / kCombThreads; ++i) mx = fmaxf(mx, ms[i]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) wred[warp] = mx;
    __syncthreads();
    float M = wred[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) M = fmaxf(M, wred[w]);
    const float mb = M == -INFINITY ? 0.f : M;
    __syncthreads();
    float lsum = 0.f;
#pragma unroll
    for (int i = 0; i < kAttMaxSplits / kCombThreads; ++i) {
        const int sp = tid + kCombThreads * i;
        if (sp < splits) {
            const float w = exp2f(ms[i] - mb);
            wsp[sp] = w;
            lsum += w * ls[i];
        }
    }
    lsum = warp_sum(lsum);
    if (lane == 0) wred[warp] = lsum;
    __syncthreads();
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) L += wred[w];

    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < splits; s0 += NW * OB) {
        if (s0 > 0) {
#pragma unroll
            for (int i = 0; i < OB; ++i) {
                const int sp = s0 + warp + NW * i;
                ov[i] = sp < splits ? __ldcg(reinterpret_cast<const float4*>(base + sp * stride + 4) + lane)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int i = 0; i < OB; ++i) {
            const int sp = s0 + warp + NW * i;
            if (sp < splits) {
                const float w = wsp[sp];
                acc.x += w * ov[i].x;
                acc.y += w * ov[i].y;
                acc.z += w * ov[i].z;
                acc.w += w * ov[i].w;
            }
        }
    }
    red[warp][4 * lane] = acc.x;
    red[warp][4 * lane + 1] = acc.y;
    red[warp][4 * lane + 2] = acc.z;
    red[warp][4 * lane + 3] = acc.w;
    __syncthreads();
    const int r = q / grp, head = (int)h * grp + q % grp;
    if (tid < 128) {
        float O = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) O += red[w][tid];
        const float o16 = __half2float(__float2half_rn(O / L));        // the attention output in fp16
        vrow[tid] = o16 * __half2float(suh[(size_t)head * 128 + tid]);
    }
    __syncthreads();
    if (warp == 0) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = vrow[lane + 32 * i];
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
        __half* o = xh + (size_t)r * hq * 128 + (size_t)head * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) o[lane + 32 * i] = __float2half_rn(v[i] * kHadScale);
    }
}

static int attn_check(int rows, int hq, int hkv, int max_len, int T)
{
    if (rows < 1 || hq < 1 || hkv < 1 || hq % hkv || max_len < 1 || T < rows || T > max_len) return EXL3_E_SHAPE;
    if (rows * (hq / hkv) > kAttMaxQ * kAttMaxQGroups) return EXL3_E_SHAPE;
    return EXL3_OK;
}

}  // namespace exl3

using namespace exl3;

extern "C" int exl3_attn_workspace(int rows, int hq, int hkv, int max_len, int T, size_t* bytes)
{
    if (!bytes) return EXL3_E_NULL;
    if (int e = attn_check(rows, hq, hkv, max_len, T)) return e;
    int nw = 0, ppw = 0, splits = 0;
    if (int e = attn_plan(hkv, T, &nw, &ppw, &splits)) return e;
    *bytes = (size_t)hkv * splits * rows * (hq / hkv) * kAttPart * sizeof(float) + kAttHeader;
    return EXL3_OK;
}

extern "C" int exl3_attn_decode_rot(const void* q, const void* k_cache, const void* v_cache, int rows, int hq, int hkv,
                                    int max_len, int T, const void* suh, void* xh, void* workspace,
                                    size_t workspace_bytes, void* stream)
{
    if (!q || !k_cache || !v_cache || !suh || !xh || !workspace) return EXL3_E_NULL;
    if (int e = attn_check(rows, hq, hkv, max_len, T)) return e;
    if (!aligned(q, 8) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(workspace, 16) ||
        !aligned(suh, 2) || !aligned(xh, 2))
        return EXL3_E_ALIGN;
    if (int e = check_device()) return e;
    int nw = 0, ppw = 0, splits = 0;
    if (int e = attn_plan(hkv, T, &nw, &ppw, &splits)) return e;
    const int grp = hq / hkv, nq = rows * grp;
    const size_t part_bytes = (size_t)hkv * splits * nq * kAttPart * sizeof(float);
    if (workspace_bytes < part_bytes + kAttHeader) return EXL3_E_WORKSPACE;
    const size_t smem = (size_t)nw * ppw * kRowBytes;
    {
        static std::mutex mu;
        static bool set[64] = {false};
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> lk(mu);
        if (dev >= 0 && dev < 64 && !set[dev]) {
            const int mx = kAttMaxCta * kRowBytes;
            if (cudaFuncSetAttribute(attn_split_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx) != cudaSuccess ||
                cudaFuncSetAttribute(attn_split_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx) != cudaSuccess)
                return EXL3_E_CUDA;
            set[dev] = true;
        }
        if (smem > (size_t)kAttMaxCta * kRowBytes) return EXL3_E_SHAPE;
    }
    AttnParams prm;
    prm.q = static_cast<const __half*>(q);
    prm.kc = static_cast<const __half*>(k_cache);
    prm.vc = static_cast<const __half*>(v_cache);
    prm.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kAttHeader);
    prm.rows = rows;
    prm.hq = hq;
    prm.hkv = hkv;
    prm.grp = grp;
    prm.nq = nq;
    prm.max_len = max_len;
    prm.T = T;
    prm.ppw = ppw;
    prm.splits = splits;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(splits, hkv, (nq + kAttMaxQ - 1) / kAttMaxQ);
    if (int e = nq <= 8 ? launch_pdl(attn_split_kernel<1>, grid, dim3(32 * nw), smem, s, prm)
                        : launch_pdl(attn_split_kernel<2>, grid, dim3(32 * nw), smem, s, prm))
        return e;
    if (int e = launch_pdl(attn_combine_kernel, dim3(nq, hkv), dim3(kCombThreads), 0, s, static_cast<const float*>(prm.part),
                           splits, nq, grp, hq, static_cast<const __half*>(suh), static_cast<__half*>(xh)))
        return e;
    return launch_status();
}
