// tc_kernels.cuh -- tcgen05 / TMEM / shared-memory descriptor PTX wrappers for
// sm_100a and the tensor-core path's workspace (pre-arranged operand slots and
// tile list).  The kernels themselves are in tcr_kernels.cuh.
#pragma once
#include "common.cuh"
#include "expert_kernels.cuh"
#include "ptx.cuh"

namespace qmoe {

// ---- TMEM and MMA ------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, kind::i8, issued by one thread.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on `bar` once every previously issued tcgen05 op of this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core
// matrices, the two 16-byte K halves `lbo` bytes apart, successive 8-row
// groups `sbo` bytes apart.  Version 1 (Blackwell) in bits 46-47.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((addr >> 4) & 0x3fffu) | (static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}

// Byte offset of (row, k-half) in a K-major no-swizzle tile of 32-byte rows:
// 8-row groups of 256 bytes, the two 16-byte K halves 128 bytes apart.
__host__ __device__ __forceinline__ uint32_t tile_off(int row, int half) {
    return static_cast<uint32_t>((row >> 3) * 256 + half * 128 + (row & 7) * 16);
}

// ---- workspace ---------------------------------------------------------------
constexpr int kTcTile = 16;   // pairs per tensor-core tile (gate/up MMA N = 2 x 16 fragment rows)

// Arranged operand slots of one tile (filled by the gather kernel for gate/up
// and by the gate/up epilogue for down), K = H or I:
//   gate/up codes: per block, 2 * kTcTile rows of 32 bytes (one per pair and
//     16-element fragment, the other fragment's bytes zero; row order
//     tc_gu_brow in tcr_kernels.cuh) in the K-major core-matrix layout, blocks
//     in the kernel's stage order (tc_gu_pos);
//   down codes: per block, kTcTile rows of 32 bytes, blocks in order;
//   gate/up constants: per block, d8[kTcTile] then m4[kTcTile] fp32 with
//     m4 = -4*s8 (per fragment);
//   down constants: per block, d8[kTcTile] then m8[kTcTile], m8 = -8*s8.
__host__ __device__ constexpr size_t tc_gu_slot(int K) { return static_cast<size_t>(K / 32) * 2 * kTcTile * 32; }
__host__ __device__ constexpr size_t tc_dn_slot(int K) { return static_cast<size_t>(K / 32) * kTcTile * 32; }
__host__ __device__ constexpr size_t tc_gu_sc_slot(int K) { return static_cast<size_t>(K / 32) * 2 * kTcTile; }
__host__ __device__ constexpr size_t tc_dn_sc_slot(int K) { return static_cast<size_t>(K / 32) * 2 * kTcTile; }
// Position of gate/up block b (of 64) in the stage order: stage k holds blocks
// 4k..4k+3, then 4k+32..4k+35.
__host__ __device__ constexpr int tc_gu_pos(int b) { return 8 * ((b & 31) >> 2) + 4 * (b >> 5) + (b & 3); }

// Tensor-core path of one layer workspace: the tile list ({expert, first pair,
// count, 0}: each group in tiles of kTcTile pairs, the last one partial) and
// the arranged operand slots of every tile.
struct TcWorkspace {
    int4 *tiles;
    int *num_tiles;
    int max_tiles;
    uint8_t *b_gu, *b_dn;     // null when the workspace never runs the tensor-core path
    float *sc_gu, *sc_dn;
};

// Tiles of `pairs` (routed + shared) split per expert into tiles of at most
// kTcTile: at most ceil(n / kTcTile) <= n / kTcTile + 1 per group.
inline int tc_tiles_bound(int pairs) { return (pairs + kTcTile - 1) / kTcTile + kRouterExperts + 2; }

template <class ArenaT>
inline void tc_workspace_take(TcWorkspace &w, ArenaT &a, int pairs, int H, int I, bool tc_used) {
    w.max_tiles = tc_tiles_bound(pairs);
    w.tiles = a.template take<int4>(w.max_tiles);
    w.num_tiles = a.template take<int>(1);
    w.b_gu = w.b_dn = nullptr;
    w.sc_gu = w.sc_dn = nullptr;
    if (tc_used) {
        const size_t t = static_cast<size_t>(w.max_tiles);
        w.b_gu = a.template take<uint8_t>(t * tc_gu_slot(H));
        w.sc_gu = a.template take<float>(t * tc_gu_sc_slot(H));
        w.b_dn = a.template take<uint8_t>(t * tc_dn_slot(I));
        w.sc_dn = a.template take<float>(t * tc_dn_sc_slot(I));
    }
}

}  // namespace qmoe
