// Peer-buffer protocol shared by the producers (exl3_gemv_peer, exl3_peer_put) and the consumer
// (exl3_ar_add_norm_rot) of the tensor-parallel all-reduce.
//
// A producer pushes its partial into the inbox (slot, its rank) of every rank as "LL" words: one
// 8-byte store per pair of 16-bit values, the low 32 bits the data, the high 32 bits the epoch of
// the all-reduce call the data belongs to. An aligned 64-bit store is single-copy atomic, so a reader
// that sees the epoch also sees the data: no fence, no separate flag and no second trip over NVLink.
// The epoch of the next call is the own flag block's "last completed" word + 1; producers read it
// after their dependency wait, i.e. after the previous all-reduce on this rank has completed.
#pragma once

#include <cstddef>
#include <cstdint>

#include "exl3_b200.h"

namespace exl3 {

// flag block (uint32 words): [8] epoch of the last completed call, [9] CTAs finished in the current
// call, [10] status bits
constexpr int kFlagEpoch = 8, kFlagDone = 9, kFlagStatus = 10;
enum : uint32_t { kStatusPeerTimeout = 4u };

__device__ __forceinline__ void st_ll(uint64_t* p, uint32_t data, uint32_t epoch)
{
    const uint64_t v = ((uint64_t)epoch << 32) | data;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_ll(const uint64_t* p)
{
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__host__ __device__ __forceinline__ uint32_t* peer_flags(void* base, const exl3_peer_group& g)
{
    return reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(base) + g.flag_off);
}

// Inbox (slot, src) inside the buffer at `base` (any rank's, as mapped in this process).
__host__ __device__ __forceinline__ uint64_t* peer_inbox(void* base, const exl3_peer_group& g, int slot, int src)
{
    return reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(base) + g.data_off +
                                       ((size_t)slot * g.world + src) * g.inbox_bytes);
}

// Host-side checks shared by every entry point that takes a group.
inline int check_peer_group(const exl3_peer_group* g, int slot)
{
    if (!g) return EXL3_E_NULL;
    if (g->world < 1 || g->world > 8 || g->rank < 0 || g->rank >= g->world || slot < 0 || slot > 1)
        return EXL3_E_SHAPE;
    for (int p = 0; p < g->world; ++p)
        if (!g->base[p]) return EXL3_E_NULL;
    if (g->flag_off % 64 || g->data_off % 16 || g->inbox_bytes % 16) return EXL3_E_ALIGN;
    return EXL3_OK;
}

}  // namespace exl3
