// tcr_kernels.cuh -- tcgen05 (kind::i8) grouped expert GEMMs with the weight
// rows on the TMEM lanes (every batch above decode size).
//
// One work item = (tile of <= 16 pairs of one expert's group, slab of 128
// weight rows).  The MMA is D[128 rows][N] = A . B^T, K = 32 per instruction
// = one quantisation block:
//   A = the slab's Q4_0 codes unpacked to unsigned bytes (0..15, u8),
//   B = the tile's Q8_1 activation codes (s8).
// A u8 x s8 product is the reference's uncentred dot sum(q * x)
// (src/quant.cpp:48-55) with |dot| < 2^16.
//
// Exact conversion: each TMEM column range is written by one MMA (no
// accumulation), so it holds the int32 dot; adding it to the bit pattern of
// 1.5 * 2^23 and subtracting 1.5 * 2^23 in fp32 gives the dot as an exact
// float (|dot| < 2^22) -- an integer add and half an f32x2 subtraction per
// value instead of the quarter-rate int-to-float conversion.
//
// Gate/up (the values the middle Q8_1 is quantised from) follow the
// reference's MMVQ order bit for bit (common.cuh: mmvq_term2 / mmvq_leaf), so
// the middle equals the reference CPU expert's: B holds two rows per pair,
// one per 16-element fragment (the other fragment's bytes zero): rows 0..15
// fragment 0 of pairs 0..15, rows 16..31 fragment 1, so the MMA (N = 32) gives
// both fragment dots with adjacent columns = adjacent pairs, and the fp32
// arithmetic runs as f32x2 over pairs; blocks b and b + 32 land in one TMEM
// region and form the tree's leaves; a pipeline stage carries blocks 2k,
// 2k+1, 2k+32, 2k+33 (one level-2 node of the tree), and the 16 nodes of an
// item are summed as a binary tree with a four-slot stack in registers.  Each
// epilogue thread owns one weight row (its TMEM lane) of gate and of up for
// 4 pairs; the item end runs SiLU(gate) * up and the Q8_1 of each 32-row
// middle block (one warp = one block per pair: lane = element, the
// reference's butterfly order) and writes the down pass's operand.
//
// Down (its output is never requantised) uses whole-block dots and
// acc += d4 * (dot * d8 - 8 * s8) per block in fp32, then a router-weighted
// red.add into the residual (lane = output row: coalesced).
//
// Warp roles (12 warps):
//   warp 0      TMEM allocation; lane 0 issues the TMA copies: raw weight
//               codes and scales through tensor maps, the tile's pre-arranged
//               activation operand as 1-D bulk copies;
//   warp 1      lane 0 issues the MMAs;
//   warps 2-3   unpack raw Q4_0 codes shared -> shared into the MMA layout;
//   warps 4-19  epilogue: four per TMEM lane quarter, 4 pairs each.
// Every barrier wait is bounded (ptx.cuh); a wait that gives up sets the
// timeout flag and the role leaves its loop.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "expert_kernels.cuh"
#include "ptx.cuh"
#include "tc_kernels.cuh"

namespace qmoe {

constexpr int kRowsM = 128;            // weight rows per MMA (TMEM lanes)
constexpr int kRowsKB = 4;             // quantisation blocks per pipeline stage
constexpr int kRowsCW = kTcTile / 4;   // pairs per epilogue warp (four warps per TMEM lane quarter)
constexpr int kRowsUnpackWarps = 2;
constexpr int kRowsEpiWarps = 16;
constexpr int kRowsWarps = 2 + kRowsUnpackWarps + kRowsEpiWarps;
constexpr int kRowsThreads = 32 * kRowsWarps;
constexpr int kRowsMinGroup = 1;       // batches above decode size: every group on this path
constexpr int kRowsHidden = 2048;      // the gate/up stage order pairs blocks b and b + 32 of 64
constexpr int kMagicBits = 0x4b400000;  // bit pattern of 1.5 * 2^23
constexpr float kMagicF = 12582912.0f; // 1.5 * 2^23

// Tensor maps over one weights object (all experts), built on the host.
struct alignas(64) TcrMaps {
    CUtensorMap codes[3];    // gate, up, down code bytes
    CUtensorMap scales[3];   // gate, up, down half scales
};

struct TcrParams {
    TcrMaps maps;
    int hidden, inter;
    int raw_rowmajor;          // codes staged [row][block] (3-D maps) instead of [block][row]
    const uint8_t *b_arr;      // arranged activation operand (tc_gu_slot / tc_dn_slot per tile)
    const float *bsc_arr;      // arranged per-pair constants (tc_gu_sc_slot / tc_dn_sc_slot per tile)
    const int4 *tiles;         // {expert, first pair, count, 0}
    const int *num_tiles;
    const int32_t *pair_token;
    const float *pair_weight;
    uint8_t *mid_arr;          // gate/up output = the down pass's b_arr
    float *mid_sc_arr;         // gate/up output = the down pass's bsc_arr
    float *out;                // down output [T][H]
    int *error;
    TapSink tap;
};

template <bool Down>
struct RowsStage {
    static constexpr int M = Down ? 1 : 2;                                    // matrices per item
    static constexpr int wins = Down ? 1 : 2;                                 // 8-block scale windows per stage
    static constexpr int brows = Down ? kTcTile : 2 * kTcTile;                // B rows per block
    static constexpr int bpc = Down ? 4 : 2;                                  // blocks per code copy
    static constexpr uint32_t codes = 0;                                      // M x 4 blocks x 128 rows x 16 B
    static constexpr uint32_t scales = codes + M * kRowsKB * kRowsM * 16;     // M x wins x [128][8] half
    static constexpr uint32_t b = scales + M * wins * kRowsM * 16;            // [4][brows][32]
    static constexpr uint32_t bsc = b + kRowsKB * brows * 32;                 // [4][cwords][kTcTile] fp32
    static constexpr int cwords = 2;                                          // constants per pair and block
    static constexpr uint32_t raw_bytes = (bsc + kRowsKB * cwords * kTcTile * 4 + 1023) / 1024 * 1024;
    static constexpr uint32_t a_bytes = M * kRowsKB * kRowsM * 32;            // unpacked A tiles
    static constexpr int raw_stages = Down ? 8 : 4;
    static constexpr int a_stages = Down ? 4 : 3;
    static constexpr uint32_t raw_off = 1024;
    static constexpr uint32_t a_off = raw_off + raw_stages * raw_bytes;
    static constexpr uint32_t smem = a_off + a_stages * a_bytes;
    // TMEM columns per region: down 4 blocks x 16 pairs (one stage), gate/up
    // 2 blocks x 2 matrices x 32 fragment columns (half a stage)
    static constexpr int reg_cols = Down ? 64 : 128;
    static constexpr int regions = 512 / reg_cols;
    static constexpr int regions_per_stage = Down ? 1 : 2;
};
static_assert(RowsStage<false>::smem <= 227 * 1024 && RowsStage<true>::smem <= 227 * 1024, "fits one CTA");
static_assert(RowsStage<false>::regions <= 8 && RowsStage<true>::regions <= 8, "barrier arrays hold 8");

// ---- PTX -------------------------------------------------------------------
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 8 consecutive TMEM columns of this warp's lane quarter (one 32-bit value each).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
// 4 consecutive TMEM columns of this warp's lane quarter.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}
__device__ __forceinline__ void tie4(uint32_t *r) {
    asm volatile("" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]) : : "memory");
}
// Two int32 dots as an exact f32x2 (|dot| < 2^22).
__device__ __forceinline__ uint64_t dots2(uint32_t a, uint32_t b) {
    return add2(pk2(a + static_cast<uint32_t>(kMagicBits), b + static_cast<uint32_t>(kMagicBits)),
                pkf2(-kMagicF, -kMagicF));
}
// Release a TMEM region read by this warp (its loads have completed).
__device__ __forceinline__ void region_release(uint64_t *empty_bar, int lane) {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar);
}

// Tie 8 registers to a point after the TMEM load wait, so no use of them is
// scheduled before it.
__device__ __forceinline__ void tie8(uint32_t *r) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
                 :
                 : "memory");
}

// Instruction descriptor: kind::i8, A unsigned 8-bit (weight codes), B signed
// 8-bit (activation codes), D s32, both operands K-major.
__host__ __device__ constexpr uint32_t rows_idesc(int m, int n) {
    return (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

// Sequence counters of the epilogue across items.
struct RowsSeq {
    int g = 0;          // pipeline stage sequence (raw and A rings advance together)
    uint32_t k = 0;     // TMEM region sequence
};

// 4 packed code bytes of lanes 4w..4w+3 in lane 4w (other lanes: don't care).
__device__ __forceinline__ uint32_t pack_lane_bytes(int8_t code) {
    uint32_t v = static_cast<uint8_t>(code);
    v |= __shfl_down_sync(0xffffffffu, v, 1) << 8;
    v |= __shfl_down_sync(0xffffffffu, v, 2) << 16;
    return v;
}

// SiLU(gate) * up of one middle value (the reference's sanitisation,
// src/hip/session_ops.hip:250-262) and the Q8_1 of the 32-value block the
// warp holds (lane = element).
struct MidQ {
    Q8Lane q;
    int flags;
};
__device__ __forceinline__ MidQ silu_q8(float g, float u) {
    int f = 0;
    const float gv = operand(g, f), uv = operand(u, f);
    const float act = arithmetic(__fdiv_rn(gv, __fadd_rn(1.0f, expf_ref(-gv))), f);
    const float val = arithmetic(__fmul_rn(act, uv), f);
    MidQ r;
    r.q = quantize_lane(f ? 0.0f : val);
    r.flags = f | r.q.flags;
    return r;
}

// ---- gate/up epilogue of one item (exact MMVQ order) -----------------------
// Pairs are handled two at a time (unit u = pairs pc0 + 2u, pc0 + 2u + 1) as
// packed f32x2 values; units without a real pair are skipped.
template <bool Tap>
__device__ __forceinline__ bool gu_epilogue_item(const TcrParams &p, uint8_t *smem, uint64_t *raw_full,
                                                 uint64_t *raw_empty, uint64_t *tm_full, uint64_t *tm_empty,
                                                 uint32_t tq, RowsSeq &sq, int item, int4 td, int lane, int quarter,
                                                 int chunk) {
    using St = RowsStage<false>;
    constexpr int R = St::regions, CW = kRowsCW, NP = kTcTile, U = CW / 2;
    const int I = p.inter;
    const int nb = kRowsHidden / 32, slabs = I / kRowsM;
    const int slab = item % slabs, tile = item / slabs;
    const int e = td.x, p0 = td.y, n = td.z;
    const int pc0 = chunk * CW;                               // this warp's first pair
    const int units = min(U, max(0, (n - pc0 + 1) / 2));      // units holding a real pair
    const int lrow = quarter * 32 + lane;                     // row within the slab
    const int row = slab * kRowsM + lrow;                     // middle row of this lane
    const uint64_t zero2 = 0ull;
    // binary-tree stack over the 16 level-2 nodes, per matrix and unit (s3 ends as the total)
    uint64_t s0[2][U], s1[2][U], s2[2][U], s3[2][U];
    int tap_base = 0;
    if constexpr (Tap) tap_base = (e == p.tap.expert) ? *p.tap.pair0 : 0;

    for (int ks = 0; ks < nb / kRowsKB; ++ks, ++sq.g) {
        const int s = sq.g % St::raw_stages;
        const uint8_t *st = smem + St::raw_off + s * St::raw_bytes;
        if (!mbar_wait(&raw_full[s], (sq.g / St::raw_stages) & 1, p.error)) return false;
        uint64_t la[2][U], node[2][U];
#pragma unroll 1
        for (int h = 0; h < 2; ++h, ++sq.k) {   // region h: blocks 2k+h (columns +0) and 2k+32+h (+32)
            const int r = static_cast<int>(sq.k % R);
            if (!mbar_wait(&tm_full[r], (sq.k / R) & 1, p.error)) return false;
            tc_fence_after();
            const uint32_t tr = tq + r * St::reg_cols + pc0;
            // pair constants d8 and -4 s8 of block 2k+h (slot h) and 2k+32+h (slot 2+h)
            const uint64_t *ka = reinterpret_cast<const uint64_t *>(
                reinterpret_cast<const float *>(st + St::bsc) + h * 2 * NP + pc0);
            const uint64_t *kb = reinterpret_cast<const uint64_t *>(
                reinterpret_cast<const float *>(st + St::bsc) + (2 + h) * 2 * NP + pc0);
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                // [block a / b][fragment] x this warp's CW pairs
                static_assert(CW == 4, "one x4 load per matrix, block and fragment");
                uint32_t v[2][2][CW];
#pragma unroll
                for (int q = 0; q < 2; ++q)
#pragma unroll
                    for (int f = 0; f < 2; ++f) tmem_ld4(tr + m * 64 + q * 32 + f * NP, v[q][f]);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 2; ++q)
#pragma unroll
                    for (int f = 0; f < 2; ++f) tie4(v[q][f]);
                // scales: window 0 holds blocks 2k, 2k+1, window 1 blocks 2k+32, 2k+33
                const uint16_t *sc = reinterpret_cast<const uint16_t *>(st + St::scales + m * 2 * kRowsM * 16);
                const int col = (2 * ks) % 8 + h;
                const float d4a = h2f(sc[lrow * 8 + col]), d4b = h2f(sc[kRowsM * 8 + lrow * 8 + col]);
                const uint64_t d4ap = pkf2(d4a, d4a), d4bp = pkf2(d4b, d4b);
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (u >= units) break;
                    const uint64_t d8a = ka[u], m4a = ka[NP / 2 + u], d8b = kb[u], m4b = kb[NP / 2 + u];
                    // exact fragment dots of the unit's two pairs: block a (2k+h) and b (2k+32+h)
                    const uint64_t ta0 = dots2(v[0][0][2 * u], v[0][0][2 * u + 1]);
                    const uint64_t ta1 = dots2(v[0][1][2 * u], v[0][1][2 * u + 1]);
                    const uint64_t tb0 = dots2(v[1][0][2 * u], v[1][0][2 * u + 1]);
                    const uint64_t tb1 = dots2(v[1][1][2 * u], v[1][1][2 * u + 1]);
                    // MMVQ lanes 2b+f (terms of block a) and 2b+f+64 (block b), summed, then the fragments
                    const uint64_t leaf =
                        add2(add2(mmvq_term2(ta0, d4ap, d8a, m4a, zero2), mmvq_term2(tb0, d4bp, d8b, m4b, zero2)),
                             add2(mmvq_term2(ta1, d4ap, d8a, m4a, zero2), mmvq_term2(tb1, d4bp, d8b, m4b, zero2)));
                    if (h == 0) la[m][u] = leaf;
                    else node[m][u] = add2(la[m][u], leaf);   // node k = L(2k) + L(2k+1)
                    if constexpr (Tap) {
                        float a0, a1, c0, c1, b0, b1, e0, e1;
                        upk2(ta0, a0, a1);
                        upk2(ta1, c0, c1);
                        upk2(tb0, b0, b1);
                        upk2(tb1, e0, e1);
                        const float da[2] = {a0 + c0, a1 + c1}, db[2] = {b0 + e0, b1 + e1};
#pragma unroll
                        for (int jj = 0; jj < 2; ++jj) {
                            const int j = 2 * u + jj;
                            const int pl = p0 + pc0 + j - tap_base;
                            if (e == p.tap.expert && pc0 + j < n && pl >= 0 && pl < p.tap.max_pairs) {
                                int32_t *dst = m == 0 ? p.tap.gate : p.tap.up;
                                const size_t base = (static_cast<size_t>(pl) * I + row) * nb;
                                dst[base + 2 * ks + h] = static_cast<int32_t>(da[jj]);
                                dst[base + 2 * ks + 32 + h] = static_cast<int32_t>(db[jj]);
                            }
                        }
                    }
                }
            }
            region_release(&tm_empty[r], lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[s]);   // done with the stage's scales and constants
        // push node k into the binary tree over k = 0..15 (one warp-uniform branch nest)
        if (!(ks & 1)) {
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int u = 0; u < U; ++u) s0[m][u] = node[m][u];
        } else if (!(ks & 2)) {
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int u = 0; u < U; ++u) s1[m][u] = add2(s0[m][u], node[m][u]);
        } else if (!(ks & 4)) {
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int u = 0; u < U; ++u) s2[m][u] = add2(s1[m][u], add2(s0[m][u], node[m][u]));
        } else {
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const uint64_t x = add2(s2[m][u], add2(s1[m][u], add2(s0[m][u], node[m][u])));
                    s3[m][u] = (ks & 8) ? add2(s3[m][u], x) : x;
                }
        }
    }

    // SiLU(gate) * up, then Q8_1 of the 32-row middle block held by this warp
    int flags = 0;
    const int jb = slab * (kRowsM / 32) + quarter;   // middle block index
    const int nbI = I / 32;
    uint8_t *mslot = p.mid_arr + static_cast<size_t>(tile) * tc_dn_slot(I) + static_cast<size_t>(jb) * NP * 32;
    float *msc = p.mid_sc_arr + static_cast<size_t>(tile) * tc_dn_sc_slot(I) + static_cast<size_t>(jb) * 2 * NP;
#pragma unroll
    for (int j = 0; j < CW; ++j) {
        const int c = pc0 + j;
        MidQ r{{0, 0, 0, 0}, 0};
        if (c < n) {   // padded pairs get zero codes and constants
            float g0, g1, u0, u1;
            upk2(s3[0][j / 2], g0, g1);
            upk2(s3[1][j / 2], u0, u1);
            r = silu_q8((j & 1) ? g1 : g0, (j & 1) ? u1 : u0);
            flags |= r.flags;
        }
        const uint32_t word = pack_lane_bytes(r.q.code);
        if ((lane & 3) == 0) *reinterpret_cast<uint32_t *>(mslot + tile_off(c, lane >> 4) + (lane & 15)) = word;
        if (lane == 0) {
            msc[c] = h2f(r.q.d);
            msc[NP + c] = -(8.0f * h2f(r.q.s));
        }
        if constexpr (Tap) {
            const int pl = p0 + c - tap_base;
            if (e == p.tap.expert && c < n && pl >= 0 && pl < p.tap.max_pairs) {
                p.tap.mid_codes[static_cast<size_t>(pl) * I + row] = r.q.code;
                if (lane == 0) p.tap.mid_ds[static_cast<size_t>(pl) * nbI + jb] = r.q.d | (uint32_t(r.q.s) << 16);
            }
        }
    }
    flags = __reduce_or_sync(0xffffffffu, flags);
    if (lane == 0) report(flags, p.error);
    return true;
}

// ---- down epilogue of one item ---------------------------------------------
template <bool Tap>
__device__ __forceinline__ bool dn_epilogue_item(const TcrParams &p, uint8_t *smem, uint64_t *raw_full,
                                                 uint64_t *raw_empty, uint64_t *tm_full, uint64_t *tm_empty,
                                                 uint32_t tq, RowsSeq &sq, int item, int4 td, int lane, int quarter,
                                                 int chunk) {
    using St = RowsStage<true>;
    constexpr int R = St::regions, CW = kRowsCW, NP = kTcTile;
    const int H = p.hidden, I = p.inter;
    const int nb = I / 32, slabs = H / kRowsM;
    const int slab = item % slabs;
    const int e = td.x, p0 = td.y, n = td.z;
    const int pc0 = chunk * CW;
    const int lrow = quarter * 32 + lane;
    const int row = slab * kRowsM + lrow;                     // output row of this lane
    uint64_t acc[CW / 2];
#pragma unroll
    for (int j = 0; j < CW / 2; ++j) acc[j] = 0ull;
    int tap_base = 0;
    if constexpr (Tap) tap_base = (e == p.tap.expert) ? *p.tap.pair0 : 0;

    for (int ks = 0; ks < nb / kRowsKB; ++ks, ++sq.g) {
        const int s = sq.g % St::raw_stages;
        const uint8_t *st = smem + St::raw_off + s * St::raw_bytes;
        if (!mbar_wait(&raw_full[s], (sq.g / St::raw_stages) & 1, p.error)) return false;
        const int r = static_cast<int>(sq.k % R);
        ++sq.k;
        if (!mbar_wait(&tm_full[r], ((sq.k - 1) / R) & 1, p.error)) return false;
        tc_fence_after();
        static_assert(CW == 4, "one x4 load per block");
        uint32_t v[kRowsKB][CW];
#pragma unroll
        for (int kb = 0; kb < kRowsKB; ++kb) tmem_ld4(tq + r * St::reg_cols + kb * NP + pc0, v[kb]);
        tmem_wait_ld();
#pragma unroll
        for (int kb = 0; kb < kRowsKB; ++kb) tie4(v[kb]);
        region_release(&tm_empty[r], lane);
        const uint16_t *sc = reinterpret_cast<const uint16_t *>(st + St::scales);
#pragma unroll
        for (int kb = 0; kb < kRowsKB; ++kb) {
            const float d4 = h2f(sc[lrow * 8 + (ks & 1) * 4 + kb]);
            const uint64_t d4p = pkf2(d4, d4);
            const uint64_t *d8p = reinterpret_cast<const uint64_t *>(
                reinterpret_cast<const float *>(st + St::bsc) + kb * 2 * NP + pc0);
#pragma unroll
            for (int u = 0; u < CW / 2; ++u) {
                const uint64_t t = dots2(v[kb][2 * u], v[kb][2 * u + 1]);   // exact dots
                acc[u] = fma2(d4p, fma2(t, d8p[u], d8p[NP / 2 + u]), acc[u]);
            }
            if constexpr (Tap) {
                if (e == p.tap.expert) {
#pragma unroll
                    for (int j = 0; j < CW; ++j) {
                        const int pl = p0 + pc0 + j - tap_base;
                        if (pc0 + j < n && pl >= 0 && pl < p.tap.max_pairs)
                            p.tap.down[(static_cast<size_t>(pl) * H + row) * nb + ks * kRowsKB + kb] =
                                static_cast<int32_t>(v[kb][j]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[s]);
    }
    // router-weighted scatter-add of the 128-row slab into the residual
    float a[CW];
#pragma unroll
    for (int j = 0; j < CW / 2; ++j) upk2(acc[j], a[2 * j], a[2 * j + 1]);
    int flags = 0;
    int tok_l = 0;
    float w_l = 0.0f;
    if (lane < CW && pc0 + lane < n) {
        tok_l = __ldg(p.pair_token + p0 + pc0 + lane);
        w_l = __ldg(p.pair_weight + p0 + pc0 + lane);
    }
#pragma unroll
    for (int j = 0; j < CW; ++j) {
        const int tok = __shfl_sync(0xffffffffu, tok_l, j);
        const float w = __shfl_sync(0xffffffffu, w_l, j);
        if (pc0 + j >= n) break;
        const float y = arithmetic(a[j], flags);
        const float cv = arithmetic(__fmul_rn(w, y), flags);
        atomicAdd(p.out + static_cast<size_t>(tok) * H + row, cv);
    }
    flags = __reduce_or_sync(0xffffffffu, flags);
    if (lane == 0) report(flags, p.error);
    return true;
}

// ---- the kernel ------------------------------------------------------------
template <bool Down, bool Tap>
__global__ void __launch_bounds__(kRowsThreads, 1) tc_rows_kernel(const __grid_constant__ TcrParams p) {
    using St = RowsStage<Down>;
    constexpr int M = St::M;
    constexpr int RS = St::raw_stages, AS = St::a_stages, R = St::regions;
    extern __shared__ __align__(128) uint8_t smem[];
    const int H = p.hidden, I = p.inter;
    const int K = Down ? I : H, nb = K / 32, ksteps = nb / kRowsKB;
    const int slabs = (Down ? H : I) / kRowsM;
    uint64_t *raw_full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *raw_empty = raw_full + 8;
    uint64_t *a_full = raw_empty + 8;
    uint64_t *a_empty = a_full + 8;
    uint64_t *tm_full = a_empty + 8;
    uint64_t *tm_empty = tm_full + 8;
    uint64_t *fin = tm_empty + 8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + 512);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < RS; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kRowsUnpackWarps + kRowsEpiWarps + 1);
        }
        for (int s = 0; s < AS; ++s) {
            mbar_init(&a_full[s], kRowsUnpackWarps);
            mbar_init(&a_empty[s], 1);
        }
        for (int r = 0; r < R; ++r) {
            mbar_init(&tm_full[r], 1);
            mbar_init(&tm_empty[r], kRowsEpiWarps);
        }
        mbar_init(fin, 1);
        mbar_fence_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dependency_wait();     // tile list and operands of the preceding kernels
    grid_launch_dependents();
    const int total = *p.num_tiles * slabs;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            for (int m = 0; m < M; ++m) {
                tma_prefetch_map(&p.maps.codes[Down ? 2 : m]);
                tma_prefetch_map(&p.maps.scales[Down ? 2 : m]);
            }
            constexpr uint32_t bbytes = kRowsKB * St::brows * 32, sbytes = kRowsKB * St::cwords * kTcTile * 4;
            const size_t bslot = Down ? tc_dn_slot(K) : tc_gu_slot(K);
            const size_t sslot = Down ? tc_dn_sc_slot(K) : tc_gu_sc_slot(K);
            int g = 0;
            bool failed = false;
            for (int item = blockIdx.x; item < total && !failed; item += gridDim.x) {
                const int tile = item / slabs, slab = item % slabs;
                const int e = p.tiles[tile].x;
                for (int ks = 0; ks < ksteps; ++ks, ++g) {
                    const int s = g % RS;
                    if (g >= RS && !mbar_wait(&raw_empty[s], ((g / RS) & 1) ^ 1, p.error)) { failed = true; break; }
                    uint8_t *st = smem + St::raw_off + s * St::raw_bytes;
                    mbar_arrive_expect_tx(&raw_full[s],
                                          M * (kRowsKB * kRowsM * 16 + St::wins * kRowsM * 16) + bbytes + sbytes);
                    for (int m = 0; m < M; ++m) {
                        const int mat = Down ? 2 : m;
                        // code copies: down blocks 4ks..4ks+3 at once; gate/up blocks (2ks, 2ks+1), then (+32, +33)
                        for (int c = 0; c < kRowsKB / St::bpc; ++c) {
                            const int b0 = Down ? kRowsKB * ks : 2 * ks + 32 * c;
                            uint8_t *dst = st + St::codes + (m * kRowsKB + c * St::bpc) * kRowsM * 16;
                            if (p.raw_rowmajor)
                                tma_load_3d(dst, &p.maps.codes[mat], b0 * 16, slab * kRowsM, e, &raw_full[s]);
                            else
                                tma_load_4d(dst, &p.maps.codes[mat], 0, slab * kRowsM, b0, e, &raw_full[s]);
                        }
                        for (int w = 0; w < St::wins; ++w) {
                            const int b0 = Down ? kRowsKB * ks : 2 * ks + 32 * w;
                            tma_load_3d(st + St::scales + (m * St::wins + w) * kRowsM * 16, &p.maps.scales[mat],
                                        b0 & ~7, slab * kRowsM, e, &raw_full[s]);
                        }
                    }
                    bulk_g2s(st + St::b, p.b_arr + static_cast<size_t>(tile) * bslot + static_cast<size_t>(ks) * bbytes,
                             bbytes, &raw_full[s]);
                    bulk_g2s(st + St::bsc,
                             p.bsc_arr + static_cast<size_t>(tile) * sslot +
                                 static_cast<size_t>(ks) * kRowsKB * St::cwords * kTcTile,
                             sbytes, &raw_full[s]);
                }
            }
            // keep the CTA alive until every issued copy has landed
            for (int k = g - RS > 0 ? g - RS : 0; k < g; ++k) mbar_wait(&raw_full[k % RS], (k / RS) & 1, p.error);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = rows_idesc(kRowsM, St::brows);
            int g = 0;
            uint32_t kseq = 0;
            bool failed = false;
            for (int item = blockIdx.x; item < total && !failed; item += gridDim.x) {
                for (int ks = 0; ks < ksteps && !failed; ++ks, ++g) {
                    const int sr = g % RS, sa = g % AS;
                    if (!mbar_wait(&a_full[sa], (g / AS) & 1, p.error) ||
                        !mbar_wait(&raw_full[sr], (g / RS) & 1, p.error)) {
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_st = smem_u32(smem + St::a_off + sa * St::a_bytes);
                    const uint32_t b_st = smem_u32(smem + St::raw_off + sr * St::raw_bytes + St::b);
                    for (int h = 0; h < St::regions_per_stage; ++h, ++kseq) {
                        const int r = static_cast<int>(kseq % R);
                        if (!mbar_wait(&tm_empty[r], (kseq / R) & 1, p.error)) { failed = true; break; }
                        tc_fence_after();
                        if (Down) {
                            // the stage's 4 blocks into the region's columns [16 kb, 16 kb + 16)
#pragma unroll
                            for (int kb = 0; kb < kRowsKB; ++kb) {
                                const uint64_t ad = smem_desc(a_st + kb * kRowsM * 32, 128, 256);
                                const uint64_t bd = smem_desc(b_st + kb * St::brows * 32, 128, 256);
                                mma_i8(tmem + r * St::reg_cols + kb * kTcTile, ad, bd, idesc, 0u);
                            }
                        } else {
                            // stage slots h (block 2k+h) and 2+h (block 2k+32+h): columns [0,32) and [32,64)
                            // of gate, +64 for up
#pragma unroll
                            for (int m = 0; m < 2; ++m)
#pragma unroll
                                for (int q = 0; q < 2; ++q) {
                                    const int slot = h + 2 * q;
                                    const uint64_t ad = smem_desc(a_st + (m * kRowsKB + slot) * kRowsM * 32, 128, 256);
                                    const uint64_t bd = smem_desc(b_st + slot * St::brows * 32, 128, 256);
                                    mma_i8(tmem + r * St::reg_cols + m * 64 + q * 32, ad, bd, idesc, 0u);
                                }
                        }
                        mma_commit(&tm_full[r]);
                    }
                    mma_commit(&a_empty[sa]);
                    mma_commit(&raw_empty[sr]);
                }
            }
            // every MMA of this CTA has completed before teardown
            mma_commit(fin);
            mbar_wait(fin, 0, p.error);
        }
    } else if (warp < 2 + kRowsUnpackWarps) {
        // ---------------- unpack: raw nibbles -> u8 K-major core matrices ----------------
        const int ut = threadIdx.x - 64;
        constexpr int kUnits = M * kRowsKB * kRowsM;
        constexpr int copies = kRowsKB / St::bpc;
        static_assert(kUnits % (32 * kRowsUnpackWarps) == 0, "whole unpack rounds");
        const bool rowmajor = p.raw_rowmajor != 0;
        int g = 0;
        bool failed = false;
        for (int item = blockIdx.x; item < total && !failed; item += gridDim.x) {
            for (int ks = 0; ks < ksteps; ++ks, ++g) {
                const int sr = g % RS, sa = g % AS;
                if (!mbar_wait(&raw_full[sr], (g / RS) & 1, p.error) ||
                    (g >= AS && !mbar_wait(&a_empty[sa], ((g / AS) & 1) ^ 1, p.error))) {
                    failed = true;
                    break;
                }
                const uint8_t *raw = smem + St::raw_off + sr * St::raw_bytes + St::codes;
                uint8_t *a = smem + St::a_off + sa * St::a_bytes;
#pragma unroll
                for (int i = 0; i < kUnits / (32 * kRowsUnpackWarps); ++i) {
                    const int u = ut + i * 32 * kRowsUnpackWarps;
                    const int m = u / (kRowsKB * kRowsM), kb = (u / kRowsM) % kRowsKB, row = u % kRowsM;
                    const int src = rowmajor ? ((m * copies + kb / St::bpc) * kRowsM + row) * St::bpc + kb % St::bpc
                                             : (m * kRowsKB + kb) * kRowsM + row;
                    const uint4 w = reinterpret_cast<const uint4 *>(raw)[src];
                    const uint4 lo = make_uint4(w.x & 0x0f0f0f0fu, w.y & 0x0f0f0f0fu, w.z & 0x0f0f0f0fu,
                                                w.w & 0x0f0f0f0fu);
                    const uint4 hi = make_uint4((w.x >> 4) & 0x0f0f0f0fu, (w.y >> 4) & 0x0f0f0f0fu,
                                                (w.z >> 4) & 0x0f0f0f0fu, (w.w >> 4) & 0x0f0f0f0fu);
                    uint8_t *dst = a + (m * kRowsKB + kb) * kRowsM * 32;
                    *reinterpret_cast<uint4 *>(dst + tile_off(row, 0)) = lo;
                    *reinterpret_cast<uint4 *>(dst + tile_off(row, 1)) = hi;
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&a_full[sa]);
                    mbar_arrive(&raw_empty[sr]);
                }
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int ew = warp - 2 - kRowsUnpackWarps;   // 0..15
        const int quarter = warp & 3, chunk = ew >> 2;    // TMEM lane quarter, pair chunk of kRowsCW
        const uint32_t tq = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        if (lane == 0)   // every region starts free
            for (int r = 0; r < R; ++r) mbar_arrive(&tm_empty[r]);
        RowsSeq sq;
        for (int item = blockIdx.x; item < total; item += gridDim.x) {
            const int4 td = p.tiles[item / slabs];
            const bool ok = Down ? dn_epilogue_item<Tap>(p, smem, raw_full, raw_empty, tm_full, tm_empty, tq, sq, item,
                                                         td, lane, quarter, chunk)
                                 : gu_epilogue_item<Tap>(p, smem, raw_full, raw_empty, tm_full, tm_empty, tq, sq, item,
                                                         td, lane, quarter, chunk);
            if (!ok) break;
        }
    }
    // teardown: every role is done with TMEM before warp 0 frees it
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// Gate/up B operand of every tile: for pair r < n of tile t (token
// pair_token[p0 + r]), row r = its Q8_1 codes of fragment 0 (elements 0..7
// and 16..23, the rest zero) and row 16 + r those of fragment 1, blocks in
// stage order, and the constants d8[16] then -4*s8[16]; pairs n..15 are zero.
// CTA (t, g): 32 threads (fragment rows) x blocks 8g..8g+7.
__global__ void __launch_bounds__(2 * kTcTile) tc_rows_gather_kernel(const int4 *tiles, const int *num_tiles,
                                                                     const int32_t *pair_token, Q8Planar xq, int H,
                                                                     uint8_t *b_arr, float *bsc_arr) {
    const int nb = H / 32, frow = threadIdx.x, pr = frow >> 1, frag = frow & 1, b0 = blockIdx.y * 8;
    for (int t = blockIdx.x; t < *num_tiles; t += gridDim.x) {
        const int4 td = tiles[t];
        uint4 v[16];
        float2 c[8];
        if (pr < td.z) {
            const int token = pair_token[td.y + pr];
            const uint4 *src = reinterpret_cast<const uint4 *>(xq.codes + static_cast<size_t>(token) * H) + 2 * b0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                v[i] = src[i];
                // keep this row's fragment: bytes 0..7 of each 16-byte half (fragment 0) or 8..15 (fragment 1)
                if (frag) v[i].x = v[i].y = 0u;
                else v[i].z = v[i].w = 0u;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = xq.scales[static_cast<size_t>(token) * nb + b0 + i];
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = make_float2(0.0f, 0.0f);
        }
        uint8_t *slot = b_arr + static_cast<size_t>(t) * tc_gu_slot(H);
        float *ss = bsc_arr + static_cast<size_t>(t) * tc_gu_sc_slot(H);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int pos = tc_gu_pos(b0 + i);
            uint8_t *dst = slot + static_cast<size_t>(pos) * 2 * kTcTile * 32;
            *reinterpret_cast<uint4 *>(dst + tile_off(frag * kTcTile + pr, 0)) = v[2 * i];
            *reinterpret_cast<uint4 *>(dst + tile_off(frag * kTcTile + pr, 1)) = v[2 * i + 1];
            if (!frag) {
                ss[pos * 2 * kTcTile + pr] = c[i].x;
                ss[pos * 2 * kTcTile + kTcTile + pr] = -(4.0f * c[i].y);
            }
        }
    }
}

inline int tc_rows_configure() {
    const int gu = static_cast<int>(RowsStage<false>::smem), dn = static_cast<int>(RowsStage<true>::smem);
    if (cudaFuncSetAttribute(tc_rows_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, gu) !=
            cudaSuccess ||
        cudaFuncSetAttribute(tc_rows_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, gu) !=
            cudaSuccess ||
        cudaFuncSetAttribute(tc_rows_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, dn) !=
            cudaSuccess ||
        cudaFuncSetAttribute(tc_rows_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, dn) !=
            cudaSuccess)
        return MOE_CUDA_ERROR;
    return MOE_OK;
}

}  // namespace qmoe
