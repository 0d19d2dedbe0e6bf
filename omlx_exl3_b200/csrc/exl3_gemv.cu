// EXL3 decode GEMV: grid planner and C entry points (exl3_gemv, exl3_gemv_noalloc, exl3_gemv_qkv_post,
// exl3_gemv_peer). The kernel and its design notes are in exl3_gemv_kernel.cuh.
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <tuple>

#include "exl3_gemv_kernel.cuh"

namespace exl3 {

template int launch_gemv_epi<0>(int, int, const GemvParams&, int, cudaStream_t);

// ---------------------------------------------------------------------------------------- host

struct GemvLaunch {
    int grid, J, blocks, KT, gran;
    long long units;
    bool mixed;                      // members of different bitrates: one CTA segment each
    int seg_cta[4], seg_bits[3], smem;
};

// Grid choice. A CTA's time is about its unit count plus a fixed cost per block segment it ends
// (the CTA-wide reduction; more when the block is split over CTAs: publish, fence, arrival ticket,
// the last arriver's sum). Measured on B200 at the 27B-class shapes, one segment end costs about
// as much as decoding 15 units, a split one about 45. Candidates: one CTA per SM, and grids that
// split every block evenly (s CTAs per block) or give every CTA d whole blocks. (Splitting a block
// over a thread-block cluster and summing in distributed shared memory was measured too: a few
// percent faster on some shapes, slower overall, since clusters must be co-scheduled in one GPC.)
static long long grid_cost(int blocks, int KT, int gran, long long G)
{
    constexpr long long kWholeEnd = 15, kSplitEnd = 45;
    const long long U = (long long)blocks * KT / gran;
    long long worst = 0;
    for (long long c = 0; c < G; ++c) {
        const long long u0 = c * U / G * gran, u1 = (c + 1) * U / G * gran;
        if (u1 <= u0) continue;
        long long cost = u1 - u0;
        for (long long b = u0 / KT; b * KT < u1; ++b) {
            const bool whole = b * KT >= u0 && (b + 1) * KT <= u1;
            cost += whole ? kWholeEnd : kSplitEnd;
        }
        worst = cost > worst ? cost : worst;
    }
    return worst;
}

static int pick_grid_uncached(int blocks, int KT, int gran, int sms)
{
    long long best_g = sms, best = grid_cost(blocks, KT, gran, sms);
    auto consider = [&](long long g) {
        if (g < 1 || g > sms || g == best_g) return;
        const long long c = grid_cost(blocks, KT, gran, g);
        if (c < best) { best = c; best_g = g; }
    };
    if (blocks <= sms) {
        for (int sp = sms / blocks; sp >= 1; --sp) consider((long long)sp * blocks);
    } else {
        for (int dd = 2; dd <= 8; ++dd)
            if (blocks % dd == 0) consider(blocks / dd);
    }
    return (int)best_g;
}

// The choice is cached per (blocks, KT, gran, SMs): exl3_gemv plans on every call.
static int pick_grid(int blocks, int KT, int gran, int sms)
{
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, int>, int> cache;
    const auto key = std::make_tuple(blocks, KT, gran, sms);
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    const int g = pick_grid_uncached(blocks, KT, gran, sms);
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = g;
    return g;
}

static int plan_gemv(const exl3_gemv_desc* d, GemvLaunch* L)
{
    if (!d) return EXL3_E_NULL;
    if (d->k <= 0 || d->k % 16 || d->n_members < 1 || d->n_members > 3 || d->rows < 1 || d->rows > 8)
        return EXL3_E_SHAPE;
    if (d->bits < 1 || d->bits > 8) return EXL3_E_BITS;
    if (d->codebook < 0 || d->codebook > 2) return EXL3_E_CODEBOOK;
    if (d->out_dtype != EXL3_F16 && d->out_dtype != EXL3_BF16) return EXL3_E_DTYPE;
    int blocks = 0, mb[3] = {d->bits, d->bits, d->bits};
    L->mixed = false;
    for (int m = 0; m < d->n_members; ++m) {
        if (d->n[m] <= 0 || d->n[m] % 128) return EXL3_E_SHAPE;
        blocks += d->n[m] / 128;
        mb[m] = d->member_bits[m] ? d->member_bits[m] : d->bits;
        if (mb[m] < 1 || mb[m] > 8) return EXL3_E_BITS;
        if (mb[m] != mb[0]) L->mixed = true;
    }
    L->blocks = blocks;
    L->KT = d->k / 16;
    L->units = (long long)blocks * L->KT;
    L->gran = L->KT % kNCW == 0 ? kNCW : 1;
    L->smem = 0;
    if (!L->mixed) {
        const long long granules = L->units / L->gran;
        long long G = d->grid > 0 ? d->grid : pick_grid(blocks, L->KT, L->gran, device_sm_count());
        if (G > granules) G = granules;
        L->grid = (int)G;
        if ((unsigned long long)L->units * (unsigned long long)(G + 1) >= (1ull << 32)) return EXL3_E_SHAPE;
        const long long per = (granules + G - 1) / G * L->gran;
        L->J = (int)((per + L->KT - 1) / L->KT + 1);
        return EXL3_OK;
    }
    // Mixed bitrates: each member gets a CTA segment in proportion to its units (the decode costs about
    // the same per weight at every bitrate), planned inside that share as a launch of its own would be.
    const int total = d->grid > 0 ? d->grid : device_sm_count();
    int seg = 0, J = 1;
    for (int m = 0; m < d->n_members; ++m) {
        const int bm = d->n[m] / 128;
        const long long um = (long long)bm * L->KT, gm = um / L->gran;
        long long cap = (long long)total * um / L->units;
        cap = cap < 1 ? 1 : cap;
        long long G = pick_grid(bm, L->KT, L->gran, (int)cap);
        G = G > gm ? gm : (G < 1 ? 1 : G);
        if ((unsigned long long)um * (unsigned long long)(G + 1) >= (1ull << 32)) return EXL3_E_SHAPE;
        const long long per = (gm + G - 1) / G * L->gran;
        const int Jm = (int)((per + L->KT - 1) / L->KT + 1);
        J = Jm > J ? Jm : J;
        L->seg_cta[m] = seg;
        L->seg_bits[m] = mb[m];
        seg += (int)G;
        const int sm = gemv_smem_bytes(mb[m]);
        L->smem = sm > L->smem ? sm : L->smem;
    }
    for (int m = d->n_members; m < 3; ++m) L->seg_bits[m] = mb[0];
    for (int m = d->n_members; m <= 3; ++m) L->seg_cta[m] = seg;
    L->grid = seg;
    L->J = J;
    return EXL3_OK;
}

}  // namespace exl3

extern "C" int exl3_gemv_workspace(const exl3_gemv_desc* desc, size_t* partial_bytes, size_t* counter_bytes)
{
    using namespace exl3;
    GemvLaunch L;
    if (int e = plan_gemv(desc, &L)) return e;
    if (partial_bytes) *partial_bytes = (size_t)L.grid * L.J * kRedStride * sizeof(float);
    if (counter_bytes) *counter_bytes = (size_t)L.blocks * sizeof(uint32_t);
    return EXL3_OK;
}

extern "C" int exl3_gemv_reset(uint32_t* counters, size_t counter_bytes, void* stream)
{
    if (!counters) return EXL3_E_NULL;
    return cudaMemsetAsync(counters, 0, counter_bytes, static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? EXL3_OK
               : EXL3_E_CUDA;
}

// Input computed inside the GEMV instead of a given xh (exl3_gemv_rot / exl3_gemv_swiglu*).
struct GemvPrologue {
    int kind;                // exl3::kProRot or exl3::kProSwiglu
    const void* src;
    int src_dtype;
    const void* suh;
    void* xs;
    size_t xs_bytes;
};

static size_t prologue_bytes(const exl3_gemv_desc* d, const exl3::GemvLaunch& L)
{
    return (size_t)L.grid * d->n_members * d->rows * d->k * sizeof(__half);
}

static int gemv_common(const exl3_gemv_desc* desc, const void* xh, const uint32_t* const* trellis, const void* svh,
                       void* y, float* partials, uint32_t* counters, const exl3_qkv_post_args* post,
                       const exl3_peer_group* peer, int slot, const GemvPrologue* pro, void* stream)
{
    using namespace exl3;
    GemvLaunch L;
    if (int e = plan_gemv(desc, &L)) return e;
    if ((!xh && !pro) || !trellis || !svh || (!y && !post && !peer) || !partials || !counters) return EXL3_E_NULL;
    if (pro) {
        if (!pro->src || !pro->suh || !pro->xs) return EXL3_E_NULL;
        if (desc->k % 128 || L.mixed || post) return EXL3_E_SHAPE;
        if (pro->src_dtype != EXL3_F16 && pro->src_dtype != EXL3_BF16 && pro->src_dtype != EXL3_F32)
            return EXL3_E_DTYPE;
        if (!aligned(pro->xs, 16) || !aligned(pro->suh, 2) || !aligned(pro->src, pro->src_dtype == EXL3_F32 ? 4 : 2))
            return EXL3_E_ALIGN;
        if (pro->xs_bytes < prologue_bytes(desc, L)) return EXL3_E_WORKSPACE;
    }
    for (int m = 0; m < desc->n_members; ++m) {
        if (!trellis[m]) return EXL3_E_NULL;
        if (!aligned(trellis[m], 16)) return EXL3_E_ALIGN;
    }
    if ((!pro && !aligned(xh, 4)) || !aligned(svh, 2) || !aligned(y, 2) || !aligned(partials, 16) || !aligned(counters, 4))
        return EXL3_E_ALIGN;
    if (int e = check_device()) return e;

    GemvParams prm{};
    int off = 0;
    for (int m = 0; m < 3; ++m) {
        const int mm = m < desc->n_members ? m : 0;
        prm.trellis[m] = trellis[mm];
        prm.nt_member[m] = desc->n[mm] / 16;
        prm.blk_off[m] = off;
        if (m < desc->n_members) off += desc->n[m] / 128;
    }
    prm.blk_off[3] = off;
    for (int m = desc->n_members; m < 3; ++m) prm.blk_off[m] = off + 1;   // never matched
    prm.nm = desc->n_members;
    prm.xh = static_cast<const __half*>(xh);
    prm.svh = static_cast<const __half*>(svh);
    prm.y = y;
    prm.partials = partials;
    prm.counters = counters;
    prm.k = desc->k;
    prm.KT = L.KT;
    prm.rows = desc->rows;
    prm.n_total = off * 128;
    prm.blocks = L.blocks;
    prm.out_bf16 = desc->out_dtype == EXL3_BF16;
    prm.J = L.J;
    prm.units = L.units;
    prm.gran = L.gran;
    if (post) prm.post = *post;
    if (peer) {
        if (int e = check_peer_group(peer, slot)) return e;
        if ((size_t)desc->rows * prm.n_total * 4 > peer->inbox_bytes) return EXL3_E_WORKSPACE;
        prm.ll_world = peer->world;
        for (int d = 0; d < 8; ++d)
            prm.ll[d] = d < peer->world ? peer_inbox(peer->base[d], *peer, slot, peer->rank) : nullptr;
        prm.epoch = peer_flags(peer->base[peer->rank], *peer) + kFlagEpoch;
    }

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (L.mixed) {
        if (peer) return EXL3_E_BITS;                        // row-parallel projections are single linears
        for (int m = 0; m < 4; ++m) prm.seg_cta[m] = L.seg_cta[m];
        for (int m = 0; m < 3; ++m) prm.seg_bits[m] = L.seg_bits[m];
        return post ? launch_gemv_seg<1>(desc->codebook, prm, L.grid, L.smem, s)
                    : launch_gemv_seg<0>(desc->codebook, prm, L.grid, L.smem, s);
    }
    if (pro) {
        prm.src = pro->src;
        prm.src_dtype = pro->src_dtype;
        prm.suh = static_cast<const __half*>(pro->suh);
        prm.xs = static_cast<__half*>(pro->xs);
        prm.xs_stride = (long long)desc->n_members * desc->rows * desc->k;
        if (pro->kind == kProRot)
            return peer ? EXL3_E_SHAPE : launch_gemv_epi<0, kProRot>(desc->bits, desc->codebook, prm, L.grid, s);
        return peer ? launch_gemv_epi<2, kProSwiglu>(desc->bits, desc->codebook, prm, L.grid, s)
                    : launch_gemv_epi<0, kProSwiglu>(desc->bits, desc->codebook, prm, L.grid, s);
    }
    if (post) return launch_gemv_epi<1>(desc->bits, desc->codebook, prm, L.grid, s);
    if (peer) return launch_gemv_epi<2>(desc->bits, desc->codebook, prm, L.grid, s);
    return launch_gemv_epi<0>(desc->bits, desc->codebook, prm, L.grid, s);
}

extern "C" int exl3_gemv_prologue_workspace(const exl3_gemv_desc* desc, size_t* xs_bytes)
{
    exl3::GemvLaunch L;
    if (int e = exl3::plan_gemv(desc, &L)) return e;
    if (xs_bytes) *xs_bytes = prologue_bytes(desc, L);
    return EXL3_OK;
}

extern "C" int exl3_gemv_rot(const exl3_gemv_desc* desc, const void* x, int x_dtype, const void* suh,
                             const uint32_t* const* trellis, const void* svh, void* y, float* partials,
                             uint32_t* counters, void* xs, size_t xs_bytes, void* stream)
{
    const GemvPrologue pro{exl3::kProRot, x, x_dtype, suh, xs, xs_bytes};
    return gemv_common(desc, nullptr, trellis, svh, y, partials, counters, nullptr, nullptr, 0, &pro, stream);
}

extern "C" int exl3_gemv_swiglu(const exl3_gemv_desc* desc, const void* gu, int gu_dtype, const void* suh,
                                const uint32_t* const* trellis, const void* svh, void* y, float* partials,
                                uint32_t* counters, void* xs, size_t xs_bytes, void* stream)
{
    if (!desc) return EXL3_E_NULL;
    if (desc->n_members != 1) return EXL3_E_SHAPE;
    const GemvPrologue pro{exl3::kProSwiglu, gu, gu_dtype, suh, xs, xs_bytes};
    return gemv_common(desc, nullptr, trellis, svh, y, partials, counters, nullptr, nullptr, 0, &pro, stream);
}

extern "C" int exl3_gemv_swiglu_peer(const exl3_gemv_desc* desc, const void* gu, int gu_dtype, const void* suh,
                                     const uint32_t* const* trellis, const void* svh, float* partials,
                                     uint32_t* counters, void* xs, size_t xs_bytes, const exl3_peer_group* g,
                                     int slot, void* stream)
{
    if (!desc || !g) return EXL3_E_NULL;
    if (desc->n_members != 1) return EXL3_E_SHAPE;
    const GemvPrologue pro{exl3::kProSwiglu, gu, gu_dtype, suh, xs, xs_bytes};
    return gemv_common(desc, nullptr, trellis, svh, nullptr, partials, counters, nullptr, g, slot, &pro, stream);
}

// ---------------------------------------------------------------------------------------- no-alloc
//
// exl3_gemv_noalloc: the same GEMV for callers that cannot allocate device memory. Such callers
// exist: code that runs while a CUDA graph is being captured (a cudaMalloc there breaks or
// invalidates the capture), hosts that have handed all device memory to their own pool allocator and
// forbid other allocations, and thin foreign-language bindings that only ever receive the input and
// output pointers and have no way to own a scratch buffer. Instead of caller-provided scratch, this
// entry point uses one fixed array in the library's device memory, sized below.

namespace exl3 {

// Scratch of the allocation-free entry point: arrival counters first, then split-k partials.
constexpr size_t kNoAllocScratchBytes = 4u << 20;                 // 4 MiB per device
constexpr size_t kNoAllocCounterBytes = 16u << 10;                // arrival counters of up to 4096 blocks
static __device__ __align__(256) uint8_t g_gemv_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_gemv_noalloc_scratch for the current device. In host code the array's name is
// only a host-side stand-in, so the address comes from the runtime: looked up on the first call on a
// device, and again whenever that device's current context is a different one (after a
// cudaDeviceReset the module is loaded afresh and the old address is stale). The context is read
// through the driver's cuCtxGetCurrent, fetched from the runtime so the library needs no libcuda link.
static void* current_context()
{
    using CtxGetCurrent = int (*)(void**);
    static CtxGetCurrent fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<CtxGetCurrent>(f);
    }();
    void* ctx = nullptr;
    if (fn && fn(&ctx) != 0) ctx = nullptr;
    return ctx;
}

static int noalloc_scratch(void** out)
{
    static std::mutex mu;
    static void* addr[64] = {nullptr};
    static const void* ctx_of[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return EXL3_E_CUDA;
    const void* ctx = current_context();
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev] || ctx != ctx_of[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_gemv_noalloc_scratch) != cudaSuccess || !p) return EXL3_E_CUDA;
        addr[dev] = p;
        ctx_of[dev] = current_context();   // the lookup made the device's context current if none was
    }
    *out = addr[dev];
    return EXL3_OK;
}

}  // namespace exl3

extern "C" int exl3_gemv_noalloc(const exl3_gemv_desc* desc, const void* xh, const uint32_t* const* trellis,
                                 const void* svh, void* y, void* stream)
{
    using namespace exl3;
    GemvLaunch L;
    if (int e = plan_gemv(desc, &L)) return e;
    const size_t counter_bytes = (size_t)L.blocks * sizeof(uint32_t);
    const size_t partial_bytes = (size_t)L.grid * L.J * kRedStride * sizeof(float);
    if (counter_bytes > kNoAllocCounterBytes || partial_bytes > kNoAllocScratchBytes - kNoAllocCounterBytes)
        return EXL3_E_WORKSPACE;
    if (int e = check_device()) return e;
    void* base = nullptr;
    if (int e = noalloc_scratch(&base)) return e;
    uint32_t* counters = static_cast<uint32_t*>(base);
    float* partials = reinterpret_cast<float*>(static_cast<uint8_t*>(base) + kNoAllocCounterBytes);
    // The array keeps whatever the previous call left; the arrival counters must start at zero.
    if (cudaMemsetAsync(counters, 0, counter_bytes, static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return EXL3_E_CUDA;
    return exl3_gemv(desc, xh, trellis, svh, y, partials, counters, stream);
}

extern "C" int exl3_gemv(const exl3_gemv_desc* desc, const void* xh, const uint32_t* const* trellis, const void* svh,
                         void* y, float* partials, uint32_t* counters, void* stream)
{
    return gemv_common(desc, xh, trellis, svh, y, partials, counters, nullptr, nullptr, 0, nullptr, stream);
}

extern "C" int exl3_gemv_qkv_post(const exl3_gemv_desc* desc, const void* xh, const uint32_t* const* trellis,
                                  const void* svh, float* partials, uint32_t* counters,
                                  const exl3_qkv_post_args* post, void* stream)
{
    if (!desc || !post) return EXL3_E_NULL;
    if (!post->q_norm_w || !post->k_norm_w || !post->cos_table || !post->sin_table || !post->pos || !post->k_cache ||
        !post->v_cache || !post->q_out)
        return EXL3_E_NULL;
    if (desc->n_members != 3 || post->hq < 1 || post->hkv < 1 || post->max_len < 1 || desc->n[0] != post->hq * 128 ||
        desc->n[1] != post->hkv * 128 || desc->n[2] != post->hkv * 128)
        return EXL3_E_SHAPE;
    return gemv_common(desc, xh, trellis, svh, nullptr, partials, counters, post, nullptr, 0, nullptr, stream);
}

extern "C" int exl3_gemv_peer(const exl3_gemv_desc* desc, const void* xh, const uint32_t* const* trellis,
                              const void* svh, float* partials, uint32_t* counters, const exl3_peer_group* g, int slot,
                              void* stream)
{
    if (!desc || !g) return EXL3_E_NULL;
    return gemv_common(desc, xh, trellis, svh, nullptr, partials, counters, nullptr, g, slot, nullptr, stream);
}
