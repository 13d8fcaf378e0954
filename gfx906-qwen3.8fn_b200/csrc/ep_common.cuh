// ep_common.cuh -- types shared by the expert-parallel kernels and the
// routing kernel that feeds them: the layout of each rank's exported arena,
// the control words peers write into it, the peer table, and the release /
// acquire helpers that publish a rank's slots to a destination.
#pragma once
#include "common.cuh"
#include "ptx.cuh"

namespace qmoe {

constexpr int kEpMaxRanks = 8;
constexpr int kEpSlotIds = kTopK;   // (local expert, weight) entries per received slot

// Control words written by peers (one set per rank, in the exported arena).
struct EpCtl {
    uint64_t recv[kEpMaxRanks];         // by source: (slots written << 32) | epoch, one release store
    uint32_t done_epoch[kEpMaxRanks];   // by destination: partial rows of this epoch final
    uint32_t pad[8];
};

// Byte offsets inside a rank's exported arena (identical on every rank).
struct EpLayout {
    size_t codes, scales, ids, w, partial, ctl, bytes;
};
inline EpLayout make_ep_layout(int H, int slots) {
    EpLayout L;
    size_t o = 0;
    auto take = [&](size_t n) { const size_t r = o; o = (o + n + 255) & ~size_t(255); return r; };
    L.ctl = take(sizeof(EpCtl));
    L.codes = take(static_cast<size_t>(slots) * H);
    L.scales = take(static_cast<size_t>(slots) * (H / 32) * 8);
    L.ids = take(static_cast<size_t>(slots) * kEpSlotIds * 4);
    L.w = take(static_cast<size_t>(slots) * kEpSlotIds * 4);
    L.partial = take(static_cast<size_t>(slots) * H * 4);
    L.bytes = o;
    return L;
}

struct EpPeers {
    uint8_t *base[kEpMaxRanks];   // every rank's exported arena, mapped here
};

struct EpParams {
    EpPeers peers;
    EpLayout L;
    int rank, world, ecount, t_max, tokens, hidden;
    const int32_t *ids;           // [T][10] global expert ids of this rank's tokens
    const float *weights;         // [T][10]
    const int8_t *xcodes;         // [T][H]
    const float2 *xscales;        // [T][H/32]
    int32_t *pos;                 // [T][kEpMaxRanks] slot index in each destination
    uint8_t *dmask;               // [T] destination ranks
    int32_t *counts;              // [kEpMaxRanks] slots sent to each destination
    uint32_t *epoch;              // device epoch counter (local)
    uint32_t *blocks_done;        // dispatch completion counter (local)
    float *out;                   // [T][H] residual (combine)
    int *error;
};

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys64(uint64_t *p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Publish to destination d that this rank's `count` slots of `epoch` are in
// place (one lane per destination, after the CTA's stores are ordered before it).
__device__ __forceinline__ void ep_publish(const EpParams &p, int d, uint32_t count, uint32_t epoch) {
    EpCtl *c = reinterpret_cast<EpCtl *>(p.peers.base[d] + p.L.ctl);
    st_release_sys64(&c->recv[p.rank], (static_cast<uint64_t>(count) << 32) | epoch);
}


}  // namespace qmoe
