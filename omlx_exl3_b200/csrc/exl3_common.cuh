// EXL3 (ExLlamaV3 trellis) decode primitives for sm_100a.
//
// Weight format (daig/omlx-exl3 src/omlx/exl3/kernels.py:4-8): a K-bit tensor of shape k x n is
// stored as int16 trellis[k/16][n/16][16K]. Each 16x16 tile is a tail-biting bitstream of 256*K
// bits held as 8K little-endian uint32 words, bits read MSB-first. The 16-bit state of stream
// position t (0..255) is bits [(t+1)K - 16, (t+1)K) of the stream, modulo 256K. Run g (0..7) is
// positions 32g..32g+31; position p of a run holds tile column g + 8*[(p%8) >= 4] and tile k-row
// 2*(p/8) + (p%2) + 8*[(p%4) >= 2] (kernels.py:52-55).
//
// Those eight consecutive positions 8L..8L+7 of lane L = 4g + q are exactly the eight weights
// that lane L holds in the A fragment of an m16n8k16 MMA whose rows are the tile's 16 output
// columns and whose k is the tile's 16 k-rows: (row g | g+8) x (k 2q, 2q+1, 2q+8, 2q+9). So one
// warp decodes one tile straight into MMA fragments, each lane from one small bit window.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace exl3 {

// ------------------------------------------------------------------------------ codebooks
// 16-bit state -> weight (kernels.py:26-48). cb 0 "3inst", 1 "mcg", 2 "mul1".
constexpr uint32_t k3instMul = 89226354u, k3instAdd = 64248484u;
constexpr uint32_t kMcgMul = 0xCBAC1FEDu;
constexpr uint32_t kMul1Mul = 0x83DCD12Du;
constexpr uint16_t kMul1InvBits = 0x1eee, kMul1BiasBits = 0xc931;   // fp16 1/K and bias

// The raw pair of fp16 halves whose sum is the 3inst / mcg weight.
template <int CB>
__device__ __forceinline__ uint32_t hash_pair(uint32_t s)
{
    const uint32_t h = CB == 0 ? s * k3instMul + k3instAdd : s * kMcgMul;
    return (h & 0x8fff8fffu) ^ 0x3b603b60u;
}

// mul1: fp16 bits of 1024 + (sum of the 4 bytes of the hash), in the low half (high half 0).
__device__ __forceinline__ uint32_t mul1_r(uint32_t s)
{
    return __dp4a(s * kMul1Mul, 0x01010101u, 0x6400u);
}

// Bit-exact fp16 weight of one state (the reference's dec1<CB>): one fp16 add or one fp16 fma.
template <int CB>
__device__ __forceinline__ __half dec1(uint32_t s)
{
    if constexpr (CB == 2) {
        const __half r = __ushort_as_half((unsigned short)mul1_r(s));
        return __hfma(r, __ushort_as_half(kMul1InvBits), __ushort_as_half(kMul1BiasBits));
    } else {
        const uint32_t v = hash_pair<CB>(s);
        return __hadd(__ushort_as_half((unsigned short)(v & 0xffffu)), __ushort_as_half((unsigned short)(v >> 16)));
    }
}

// MMA A-operand word for one state in the "split" form used by the GEMV: a half2 (a, b) whose
// a*x + b*x equals the weight times x. For 3inst / mcg that is the hash pair itself (the weight
// is the sum of its halves, here left unrounded); for mul1 it is (fma(r, 1/K, bias), 0).
template <int CB>
__device__ __forceinline__ uint32_t split_word(uint32_t s)
{
    if constexpr (CB == 2) {
        const __half2 r = __halves2half2(__ushort_as_half((unsigned short)mul1_r(s)), __ushort_as_half(0));
        const __half2 a = __halves2half2(__ushort_as_half(kMul1InvBits), __ushort_as_half(0));
        const __half2 c = __halves2half2(__ushort_as_half(kMul1BiasBits), __ushort_as_half(0));
        const __half2 w = __hfma2(r, a, c);
        return *reinterpret_cast<const uint32_t*>(&w);
    } else {
        return hash_pair<CB>(s);
    }
}

// ------------------------------------------------------------------------------ bit windows
// Lane L's positions 8L..8L+7 end at stream bit E = 8K(L+1). Let V be the stream bits just before
// E read as a number whose bit i is stream bit E-1-i. The state of the lane's j-th position is then
// (V >> (7-j)K) & 0xffff. V needs 7K+16 bits: one word (K <= 2), two (K <= 6) or three (K >= 7).
template <int K>
struct LaneWindow {
    static constexpr int TW = 8 * K;                     // words per tile
    static constexpr int NEED = 7 * K + 16;              // bits of V used
    static constexpr bool kAligned = (K % 4) == 0;       // E is a multiple of 32: no shift
    int idx[4];                                          // word indices (mod TW), latest first
    uint32_t shift;                                      // right shift that puts bit E-1 at bit 0

    __device__ __forceinline__ explicit LaneWindow(int lane)
    {
        const int E = 8 * K * (lane + 1);
        const int iw = (E - 1) >> 5;
        shift = kAligned ? 0u : (uint32_t)((32 * (iw + 1) - E) & 31);
#pragma unroll
        for (int q = 0; q < 4; ++q) idx[q] = ((iw - q) % TW + TW) % TW;
    }
};

// V as three 32-bit words (bits [0,32), [32,64), [64,96)) from the tile's words.
template <int K>
struct Window96 {
    uint32_t lo, mid, hi;
};

template <int K>
__device__ __forceinline__ Window96<K> load_window(const uint32_t* tile, const LaneWindow<K>& lw)
{
    constexpr int NEED = LaneWindow<K>::NEED;
    constexpr bool A = LaneWindow<K>::kAligned;
    Window96<K> v;
    const uint32_t w0 = tile[lw.idx[0]];
    uint32_t w1 = 0, w2 = 0, w3 = 0;
    if (!A || NEED > 32) w1 = tile[lw.idx[1]];
    if (NEED > 32 && (!A || NEED > 64)) w2 = tile[lw.idx[2]];
    if (NEED > 64 && !A) w3 = tile[lw.idx[3]];
    if constexpr (A) {
        v.lo = w0; v.mid = w1; v.hi = w2;
    } else {
        v.lo = __funnelshift_r(w0, w1, lw.shift);
        v.mid = NEED > 32 ? __funnelshift_r(w1, w2, lw.shift) : 0u;
        v.hi = NEED > 64 ? __funnelshift_r(w2, w3, lw.shift) : 0u;
    }
    return v;
}

// State of the lane's position j (0..7).
template <int K, int J>
__device__ __forceinline__ uint32_t lane_state(const Window96<K>& v)
{
    constexpr int sh = (7 - J) * K;
    if constexpr (sh + 16 <= 32) {
        return sh == 16 ? (v.lo >> 16) : ((v.lo >> sh) & 0xffffu);
    } else if constexpr (sh < 32) {
        return __funnelshift_r(v.lo, v.mid, sh) & 0xffffu;
    } else if constexpr (sh + 16 <= 64) {
        return sh == 48 ? (v.mid >> 16) : ((v.mid >> (sh - 32)) & 0xffffu);
    } else if constexpr (sh < 64) {
        return __funnelshift_r(v.mid, v.hi, sh - 32) & 0xffffu;
    } else {
        return (v.hi >> (sh - 64)) & 0xffffu;
    }
}

// ------------------------------------------------------------------------------ hashing
// The decode is bound by instruction issue. Per state the floor is one extraction (one or two ops),
// one IMAD for the hash and one LOP3 for the codebook's and/xor. What keeps it there (measured with
// per-pipe instruction counters and CUDA-event timing on B200):
//   * the codebook constants live in registers the compiler cannot see through (HashRegs): as
//     literals, one of them is re-materialised at every LOP3 / IMAD (one extra ALU op per weight,
//     ~8 per tile);
//   * every state is isolated exactly with integer-ALU ops (shift and mask, byte permute, funnel
//     shift); folding the unmasked high bits into a correcting multiply-add costs more issue slots
//     than it saves;
//   * no extraction uses a multiply-high: moving fields to the top of the word and back with two
//     multiplies (IMAD, IMAD.HI), or taking the top half with IMAD.HI, was measured 8-21 % slower per
//     GEMV launch than shifts and masks (K = 2: 29.5 -> 23.3 us, K = 6: 28.0 -> 25.8 us, K = 8:
//     24.3 -> 22.1 us at 5120 -> 17408, one row; the multiply-high also raised dispatch stalls);
//   * with the extraction on the ALU pipe that pipe runs at ~70 % of its peak and limits issue, so a
//     field inside one word is moved to the top by a plain multiply (IMAD on the FMA pipe, by a
//     power of two from constant memory: as a literal the compiler would turn it into an ALU shift)
//     and brought down by one shift: one ALU op instead of two (K = 6: 25.7 -> 23.8 us; issue slots
//     60 -> 65 % busy).

// Powers of two as constant-memory operands (see above).
static __constant__ uint32_t c_pow2[17] = {1u << 0, 1u << 1, 1u << 2, 1u << 3, 1u << 4, 1u << 5, 1u << 6,
                                           1u << 7, 1u << 8, 1u << 9, 1u << 10, 1u << 11, 1u << 12, 1u << 13,
                                           1u << 14, 1u << 15, 1u << 16};

// The 16-bit field at bit SH of the lane's window.
template <int SH>
__device__ __forceinline__ uint32_t state_exact(const uint32_t (&w)[3])
{
    constexpr int wi = SH / 32, o = SH % 32;
    if constexpr (o == 0) {
        return w[wi] & 0xffffu;
    } else if constexpr (o == 16) {
        return w[wi] >> 16;
    } else if constexpr (o == 8) {
        return __byte_perm(w[wi], 0u, 0x4421);
    } else if constexpr (o + 16 <= 32) {
        return (w[wi] * c_pow2[16 - o]) >> 16;
    } else {
        return __funnelshift_r(w[wi], w[wi + 1], o) & 0xffffu;
    }
}

// Codebook constants held in registers the compiler cannot see through (see above). They are read
// from constant memory: a literal routed through an empty asm statement is still a literal to the
// assembler, which then re-materialises it at each use.
struct HashRegs {
    uint32_t mul, add, msk, xr;
};

// [codebook][mul, add, and-mask, xor]
static __constant__ uint32_t c_hash_consts[3][4] = {
    {k3instMul, k3instAdd, 0x8fff8fffu, 0x3b603b60u},
    {kMcgMul, 0u, 0x8fff8fffu, 0x3b603b60u},
    {kMul1Mul, 0u, 0x8fff8fffu, 0x3b603b60u},
};

template <int CB>
__device__ __forceinline__ HashRegs hash_regs()
{
    HashRegs r;
    r.mul = c_hash_consts[CB][0];
    r.add = c_hash_consts[CB][1];
    r.msk = c_hash_consts[CB][2];
    r.xr = c_hash_consts[CB][3];
    return r;
}

// Fields of the lane's window that straddle word boundary 32 B (B = 1, 2).
template <int K, int B>
__host__ __device__ constexpr int cross_count()
{
    int c = 0;
    for (int j = 0; j < 8; ++j) {
        const int sh = (7 - j) * K;
        if (sh < 32 * B && sh + 16 > 32 * B) ++c;
    }
    return c;
}

// The 16-bit field at bit O of one word (O + 16 <= 32), as in state_exact.
template <int O>
__device__ __forceinline__ uint32_t field_in_word(uint32_t x)
{
    if constexpr (O == 0) return x & 0xffffu;
    else if constexpr (O == 8) return __byte_perm(x, 0u, 0x4421);
    else return (x * c_pow2[16 - O]) >> 16;
}

// State at bit SH. Where two or more fields straddle the same word boundary, one funnel shift builds
// the word that starts 16 bits below the boundary (m), and each of those fields is taken from it as an
// in-word field (one ALU op each, plus the shared shift) instead of a funnel shift and a mask each
// (K = 4 / 5: ~3 % per launch).
template <int K, int SH>
__device__ __forceinline__ uint32_t state_at(const uint32_t (&w)[3], const uint32_t (&m)[2])
{
    constexpr int wi = SH / 32, o = SH % 32;
    if constexpr (o + 16 > 32 && cross_count<K, wi + 1>() >= 2) return field_in_word<o - 16>(m[wi]);
    else return state_exact<SH>(w);
}

// The eight raw codebook hashes h_j = s_j * mul + add of a lane (s_j the state of position j).
template <int K, int CB>
__device__ __forceinline__ void hashes8(const uint32_t (&w)[3], uint32_t (&h)[8], const HashRegs& hr)
{
    uint32_t m[2];                           // bits [16, 48) and [48, 80) of the window (unused ones drop out)
    m[0] = __funnelshift_r(w[0], w[1], 16);
    m[1] = __funnelshift_r(w[1], w[2], 16);
#define EXL3_HASH(J) h[J] = state_at<K, (7 - J) * K>(w, m) * hr.mul + hr.add;
    EXL3_HASH(0) EXL3_HASH(1) EXL3_HASH(2) EXL3_HASH(3)
    EXL3_HASH(4) EXL3_HASH(5) EXL3_HASH(6) EXL3_HASH(7)
#undef EXL3_HASH
}

// hash -> split MMA word (see split_word)
template <int CB>
__device__ __forceinline__ uint32_t split_from_hash(uint32_t h, const HashRegs& hr)
{
    if constexpr (CB == 2) {
        const uint32_t r = __dp4a(h, 0x01010101u, 0x6400u);
        const __half2 rr = *reinterpret_cast<const __half2*>(&r);
        const __half2 a = __halves2half2(__ushort_as_half(kMul1InvBits), __ushort_as_half(0));
        const __half2 c = __halves2half2(__ushort_as_half(kMul1BiasBits), __ushort_as_half(0));
        const __half2 w = __hfma2(rr, a, c);
        return *reinterpret_cast<const uint32_t*>(&w);
    } else {
        return (h & hr.msk) ^ hr.xr;
    }
}

// The lane's three window words (V bits [0,32), [32,64), [64,96)) of one tile.
template <int K>
__device__ __forceinline__ void window_words(const uint32_t* tile, const LaneWindow<K>& lw, uint32_t (&w)[3])
{
    const Window96<K> v = load_window<K>(tile, lw);
    w[0] = v.lo;
    w[1] = v.mid;
    w[2] = v.hi;
}

// The eight split MMA words of one lane for one tile (the tile's words start at `tile`, 8-byte
// aligned: the GEMV's shared-memory ring). At K = 8 the window's two newest words are the aligned
// pair (2L, 2L + 1) of lane L, read with one 64-bit load.
template <int K, int CB>
__device__ __forceinline__ void decode_tile(const uint32_t* tile, const LaneWindow<K>& lw, const HashRegs& hr,
                                            uint32_t (&a)[8])
{
    uint32_t w[3], h[8];
    if constexpr (K == 8) {
        const uint2 p = *reinterpret_cast<const uint2*>(tile + lw.idx[1]);
        w[0] = p.y;
        w[1] = p.x;
        w[2] = tile[lw.idx[2]];
    } else {
        window_words<K>(tile, lw, w);
    }
    hashes8<K, CB>(w, h, hr);
#pragma unroll
    for (int t = 0; t < 8; ++t) a[t] = split_from_hash<CB>(h[t], hr);
}

// ------------------------------------------------------------------------------ MMA
// D += A(16x16 fp16, row) * B(16x8 fp16, col), fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// ------------------------------------------------------------------------------ mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_addr(const void* p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// try_wait that lets the hardware suspend the thread for up to `hint_ns` while the phase is pending
// (no issue slots spent polling).
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up (returns false) once `limit_ns` of wall time has passed without the phase
// completing, so a lost completion turns into an error status instead of a hung GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, 100000u)) return true;
        if (global_ns() - t0 > limit_ns) return false;
    }
}

// Global -> shared bulk copy (no multicast), completion counted on `bar` in bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// 16-byte global -> shared copy through L2 only (LDGSTS), tracked by per-thread commit groups.
__device__ __forceinline__ void cp_async16(void* dst, const void* src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// The same copy to a 32-bit shared-window address.
__device__ __forceinline__ void cp_async16_s(uint32_t dst, const void* src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------------------ dependent launch
// Let the next kernel in the stream begin launching (it still waits for this one in pdl_wait).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Wait until the previous kernel in the stream has completed and its writes are visible (a no-op
// when this kernel was launched without programmatic dependence).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------------------ misc
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }

constexpr float kHadScale = 0.08838834764831845f;   // 1/sqrt(128)

// Error bits written to a caller-visible status word when a bounded wait gives up.
enum : uint32_t { kStatusPipeTimeout = 1u, kStatusArrivalTimeout = 2u };

// ------------------------------------------------------------------------------ row sums of squares
// Sum over the row of T(x + d)^2 (d may be null: T(x)^2), fp32, this thread's share; 16-byte loads,
// several in flight, when both rows are 16-byte aligned (the usual case), else element by element.
template <typename T>
__device__ __forceinline__ float row_sumsq(const T* __restrict__ xr, const T* __restrict__ dr, int kd, int tid,
                                           int nthr)
{
    float ss = 0.f;
    const bool vec = ((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(dr)) & 15) == 0 && kd % 8 == 0;
    if (vec) {
        const uint4* x4 = reinterpret_cast<const uint4*>(xr);
        const uint4* d4 = reinterpret_cast<const uint4*>(dr);
#pragma unroll 4
        for (int v = tid; v < kd / 8; v += nthr) {
            const uint4 a = x4[v];
            const uint4 b = dr ? d4[v] : make_uint4(0, 0, 0, 0);
            const T* ae = reinterpret_cast<const T*>(&a);
            const T* be = reinterpret_cast<const T*>(&b);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float h = dr ? to_f32(from_f32<T>(to_f32(ae[i]) + to_f32(be[i]))) : to_f32(ae[i]);
                ss = fmaf(h, h, ss);
            }
        }
    } else {
        for (int i = tid; i < kd; i += nthr) {
            const float h = dr ? to_f32(from_f32<T>(to_f32(xr[i]) + to_f32(dr[i]))) : to_f32(xr[i]);
            ss = fmaf(h, h, ss);
        }
    }
    return ss;
}

// ------------------------------------------------------------------------------ per-head q/k post-processing
// (shared by exl3_qkv_post and the q/k/v GEMV epilogue) one warp holds a 128-vector as
// v[i] = element lane + 32 i.
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int h = 16; h >= 1; h >>= 1) v += __shfl_xor_sync(0xffffffffu, v, h);
    return v;
}

// x (4 values of a 128-vector in this lane) -> MLX-rounded RMSNorm with weight w
template <typename T>
__device__ __forceinline__ void head_rms(float (&v)[4], const T* __restrict__ w, float eps, int lane)
{
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) ss = fmaf(v[i], v[i], ss);
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / 128.0f + eps);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const T t = from_f32<T>(v[i] * inv);
        v[i] = to_f32(from_f32<T>(to_f32(w[lane + 32 * i]) * to_f32(t)));
    }
}

__device__ __forceinline__ void rope_half(float (&v)[4], const float* __restrict__ cs, const float* __restrict__ sn,
                                          int lane)
{
    // elements c = lane + 32 i; pairs (c, c + 64) for c < 64: (v[0], v[2]) and (v[1], v[3]).
    // Products and sums rounded separately (no contraction), as an elementwise framework op computes them.
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int c = lane + 32 * i;
        const float x1 = v[i], x2 = v[i + 2];
        const float co = cs[c], si = sn[c];
        v[i] = __fsub_rn(__fmul_rn(x1, co), __fmul_rn(x2, si));
        v[i + 2] = __fadd_rn(__fmul_rn(x2, co), __fmul_rn(x1, si));
    }
}

}  // namespace exl3
