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
// Exact conversion: before the integer MMAs of a TMEM region, one bf16 MMA
// (kind::f16, A = 1 at k = 0, B = 1.5 * 2^23 at k = 0, f32 accumulator)
// writes the bit pattern of 1.5 * 2^23 into every column of the region; the
// integer MMAs then accumulate (s32) onto it, so each column holds
// 0x4B400000 + dot, i.e. the float 1.5 * 2^23 + dot exactly (|dot| < 2^22),
// and one f32x2 subtraction per two values gives the dots as exact floats --
// no integer instruction and no quarter-rate conversion on the CUDA cores.
//
// Gate/up (the values the middle Q8_1 is quantised from) follow the
// reference's MMVQ order bit for bit (common.cuh: mmvq_term2), so the middle
// equals the reference CPU expert's: B holds two rows per pair, one per
// 16-element fragment (the other fragment's bytes zero), chunk-major
// (tc_gu_brow: the 8 rows of pairs 4c..4c+3 adjacent), so the MMA (N = 32)
// gives every epilogue warp its 4 pairs x 2 fragments as 8 adjacent columns
// and the fp32 arithmetic runs as f32x2 over pairs; blocks b and b + 32 land
// in one TMEM region and form the tree's leaves; a pipeline stage carries
// blocks 4k..4k+3 and 4k+32..4k+35 (four leaves: one node two levels above
// them), and the 8 nodes of a matrix are summed as a binary tree with a
// four-slot stack in registers.  Each epilogue thread owns one weight row (its TMEM lane) of gate
// and of up for 4 pairs; the item end runs SiLU(gate) * up and the Q8_1 of
// each 32-row middle block (one warp = one block per pair: lane = element,
// the reference's butterfly order) and writes the down pass's operand.
//
// Down (its output is never requantised) uses whole-block dots and
// acc += d4 * (dot * d8 - 8 * s8) per block in fp32 -- for Q4_1 down matrices
// the reference's block term acc + fma(dot, half(d4 d8), half(m4 s8)) -- then
// a router-weighted red.add into the residual (lane = output row: coalesced).
//
// Warp roles (gate/up and Q4_1 down 20 warps, Q4_0 down 12):
//   warp 0      TMEM allocation; lane 0 issues the TMA copies: raw weight
//               codes and scales through tensor maps, the tile's pre-arranged
//               activation operand as 1-D bulk copies;
//   warp 1      lane 0 issues the MMAs;
//   warps 2-3   unpack raw 4-bit codes shared -> shared into the MMA layout;
//   warps 4-    epilogue: gate/up and Q4_1 down four per TMEM lane quarter
//               with 4 pairs each, Q4_0 down two per quarter with 8 pairs each.
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
constexpr int kRowsKB = 8;             // quantisation blocks per pipeline stage
constexpr int kRowsBlocksPerCopy = 4;  // blocks per TMA code copy (gate/up: two copies per stage)
constexpr int kRowsUnpackWarps = 2;
constexpr int kRowsMinGroup = 1;       // batches above decode size: every group on this path
constexpr int kRowsHidden = 2048;      // the gate/up stage order pairs blocks b and b + 32 of 64
constexpr float kMagicF = 12582912.0f; // 1.5 * 2^23 (bits 0x4B400000)
constexpr uint32_t kBf16One = 0x3f80u, kBf16Magic = 0x4b40u;   // bf16 1.0 and 1.5 * 2^23

// B row of (pair p, fragment f) in a gate/up block: chunk-major, the 8 rows
// of pairs 4c..4c+3 adjacent (fragment 0 then 1).
__host__ __device__ constexpr int tc_gu_brow(int p, int f) { return (p >> 2) * 8 + f * 4 + (p & 3); }

// Tensor maps over one weights object (all experts), built on the host.
struct alignas(64) TcrMaps {
    CUtensorMap codes[3];    // gate, up, down code bytes
    CUtensorMap scales[3];   // gate, up, down half scales
    CUtensorMap down_mins;   // Q4_1 down matrices: half minima (layout of the down scales)
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

constexpr int kRowsBarSlots = 16;   // entries per barrier array

// Shared-memory rings of one CTA.  Each feeds its own consumers, so every
// ring is released as soon as they are done with it:
//   codes  the slab's raw Q4_0 codes of one stage (8 blocks x 128 rows x
//          16 B of one matrix), read by the unpack warps;
//   side   the tile's arranged activation operand (B, read by the MMAs) and
//          per-pair constants (read by the epilogue) of one stage;
//   scale  the weight rows' half scales of a stage group (gate/up: blocks
//          8j..8j+7 and 32+8j..32+8j+7 of one matrix = 2 stages; down: blocks
//          8j..8j+7 = 1 stage, and their minima for Q4_1), read by the epilogue;
//   A      the unpacked A operand of one stage (u8, K-major core matrices).
// Q41: the down kernel of Q4_1 matrices (same layout, more epilogue warps).
template <bool Down, bool Q41 = false>
struct RowsStage {
    static constexpr int M = Down ? 1 : 2;                                    // matrices per item (one per stage)
    // epilogue warps (per TMEM lane quarter: epi_warps / 4) and pairs per warp: gate/up and the
    // Q4_1 down term run longer dependent fp32 chains per pair and need the warps to hide their
    // latency, the Q4_0 down term the fewer per-warp fixed costs of wider warps
    static constexpr int epi_warps = Down && !Q41 ? 8 : 16;
    static constexpr int cw = kTcTile * 4 / epi_warps;
    static constexpr int threads = 32 * (2 + kRowsUnpackWarps + epi_warps);
    static constexpr int kb = kRowsKB;                                        // quantisation blocks per stage
    static constexpr int wins = 2;   // 8-block windows per group (gate/up: blocks 8j.., 32+8j..; down: scales, Q4_1 minima)
    static constexpr int spw = Down ? 1 : 2;                                  // stages per scale group
    static constexpr int brows = Down ? kTcTile : 2 * kTcTile;                // B rows per block
    static constexpr int bpc = kRowsBlocksPerCopy;                            // blocks per code copy
    static constexpr int cwords = 2;                                          // constants per pair and block
    static constexpr uint32_t codes_bytes = kb * kRowsM * 16;
    static constexpr uint32_t b = 0;                                          // side: [kb][brows][32]
    static constexpr uint32_t bsc = b + kb * brows * 32;                      // side: [kb][cwords][kTcTile] fp32
    static constexpr uint32_t side_bytes = bsc + kb * cwords * kTcTile * 4;
    static constexpr uint32_t sc_win = kRowsM * 16;                           // [128][8] half
    static constexpr uint32_t sc_bytes = wins * sc_win;
    static constexpr uint32_t a_bytes = kb * kRowsM * 32;                     // unpacked A tiles
    static constexpr int code_stages = 4;                // powers of two: cheap slot and phase arithmetic
    static constexpr int side_stages = Down ? 8 : 4;
    static constexpr int sc_stages = 4;
    static constexpr int a_stages = 3;
    static constexpr uint32_t codes_off = 2048;
    static constexpr uint32_t side_off = codes_off + code_stages * codes_bytes;
    static constexpr uint32_t sc_off = (side_off + side_stages * side_bytes + 1023) / 1024 * 1024;
    static constexpr uint32_t a_off = sc_off + sc_stages * sc_bytes;
    static constexpr uint32_t magic_off = a_off + a_stages * a_bytes;        // bf16 A [128][16], B [128][16]
    static constexpr uint32_t smem = magic_off + 2 * kRowsM * 32;
    // TMEM columns per region = one stage: kb blocks x brows (down 8 x 16
    // pairs = 4 regions, gate/up 8 x 16 pairs x 2 fragments = 2 regions)
    static constexpr int reg_cols = kb * brows;
    static constexpr int regions = 512 / reg_cols;
    static_assert(side_bytes % 128 == 0 && sc_bytes % 1024 == 0 && codes_bytes % 1024 == 0, "ring alignment");
    static_assert((side_off % 1024) == 0 && (sc_off % 1024) == 0 && (a_off % 1024) == 0, "ring alignment");
};
// Polls of the TMA producer without progress (each followed by a ~64 ns
// sleep) before it declares the consumers stopped: well above any real stall.
constexpr uint32_t kProducerIdleLimit = 1u << 25;
static_assert(RowsStage<false>::smem <= 227 * 1024 && RowsStage<true>::smem <= 227 * 1024, "fits one CTA");
static_assert(RowsStage<true>::code_stages <= kRowsBarSlots && RowsStage<true>::side_stages <= kRowsBarSlots &&
                  RowsStage<true>::regions <= kRowsBarSlots && RowsStage<false>::regions <= kRowsBarSlots,
              "barrier arrays");

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
// 16 consecutive TMEM columns of this warp's lane quarter.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tie16(uint32_t *r) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}
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
// Two TMEM words 0x4B400000 + dot as the exact f32x2 of the dots (|dot| < 2^22).
__device__ __forceinline__ uint64_t from_magic2(uint32_t a, uint32_t b) {
    return add2(pk2(a, b), pkf2(-kMagicF, -kMagicF));
}
__device__ __forceinline__ float lo_half(uint32_t w) { return h2f(static_cast<uint16_t>(w & 0xffffu)); }
__device__ __forceinline__ float hi_half(uint32_t w) { return h2f(static_cast<uint16_t>(w >> 16)); }
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

// CW consecutive TMEM columns of this warp's lane quarter (CW = 4 or 8), and their tie.
template <int CW>
__device__ __forceinline__ void tmem_ld_cw(uint32_t taddr, uint32_t *r) {
    if constexpr (CW == 8) tmem_ld8(taddr, r);
    else tmem_ld4(taddr, r);
}
template <int CW>
__device__ __forceinline__ void tie_cw(uint32_t *r) {
    if constexpr (CW == 8) tie8(r);
    else tie4(r);
}

// Instruction descriptor: kind::i8, A unsigned 8-bit (weight codes), B signed
// 8-bit (activation codes), D s32, both operands K-major.
__host__ __device__ constexpr uint32_t rows_idesc(int m, int n) {
    return (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}
// Instruction descriptor: kind::f16, A and B bf16, D f32, both K-major.
__host__ __device__ constexpr uint32_t magic_idesc(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}
// D[tmem] = A[smem] . B[smem]^T, kind::f16 (bf16 operands, f32 accumulator), issued by one thread.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(0u)
        : "memory");
}

// Sequence counters of the epilogue across items.
struct RowsSeq {
    int g = 0;          // pipeline stage sequence (raw and A rings advance together)
    uint32_t k = 0;     // TMEM region sequence
};

// Barriers of one CTA (shared memory), one full/empty pair per ring slot, as
// fixed offsets from one base (one register, not one per array).
struct RowsBars {
    uint64_t *base;
    __device__ uint64_t *code_full(int i) const { return base + 0 * kRowsBarSlots + i; }
    __device__ uint64_t *code_empty(int i) const { return base + 1 * kRowsBarSlots + i; }
    __device__ uint64_t *side_full(int i) const { return base + 2 * kRowsBarSlots + i; }
    __device__ uint64_t *side_empty(int i) const { return base + 3 * kRowsBarSlots + i; }
    __device__ uint64_t *sc_full(int i) const { return base + 4 * kRowsBarSlots + i; }
    __device__ uint64_t *sc_empty(int i) const { return base + 5 * kRowsBarSlots + i; }
    __device__ uint64_t *a_full(int i) const { return base + 6 * kRowsBarSlots + i; }
    __device__ uint64_t *a_empty(int i) const { return base + 7 * kRowsBarSlots + i; }
    __device__ uint64_t *tm_full(int i) const { return base + 8 * kRowsBarSlots + i; }
    __device__ uint64_t *tm_empty(int i) const { return base + 9 * kRowsBarSlots + i; }
    __device__ uint64_t *fin() const { return base + 10 * kRowsBarSlots; }
};

// Unpack stage g's raw Q4_0 codes (shared) into unsigned bytes in the K-major
// core-matrix layout of its A slot (shared), split over the unpack warps'
// threads (ut = 0 .. 32 * kRowsUnpackWarps - 1); each warp then arrives on
// the A slot's full barrier and the code slot's empty barrier.  False when a
// wait gave up.
template <bool Down>
__device__ __forceinline__ bool rows_unpack(uint8_t *smem, const RowsBars &b, int g, int ut, bool rowmajor, int lane,
                                            int *error) {
    using St = RowsStage<Down>;
    constexpr int kThreads = 32 * kRowsUnpackWarps;
    const int sr = g % St::code_stages, sa = g % St::a_stages;
    if (!mbar_wait(b.code_full(sr), (g / St::code_stages) & 1, error)) return false;
    if (g >= St::a_stages && !mbar_wait(b.a_empty(sa), ((g / St::a_stages) & 1) ^ 1, error)) return false;
    const uint8_t *raw = smem + St::codes_off + sr * St::codes_bytes;
    uint8_t *a = smem + St::a_off + sa * St::a_bytes;
    constexpr int kUnits = St::kb * kRowsM;
    static_assert(kUnits % kThreads == 0, "whole unpack rounds");
#pragma unroll
    for (int i = 0; i < kUnits / kThreads; ++i) {
        const int u = ut + i * kThreads;
        const int kb = u / kRowsM, row = u % kRowsM;
        const int src = rowmajor ? ((kb / St::bpc) * kRowsM + row) * St::bpc + kb % St::bpc : kb * kRowsM + row;
        const uint4 w = reinterpret_cast<const uint4 *>(raw)[src];
        const uint4 lo = make_uint4(w.x & 0x0f0f0f0fu, w.y & 0x0f0f0f0fu, w.z & 0x0f0f0f0fu, w.w & 0x0f0f0f0fu);
        const uint4 hi = make_uint4((w.x >> 4) & 0x0f0f0f0fu, (w.y >> 4) & 0x0f0f0f0fu, (w.z >> 4) & 0x0f0f0f0fu,
                                    (w.w >> 4) & 0x0f0f0f0fu);
        uint8_t *dst = a + kb * kRowsM * 32;
        *reinterpret_cast<uint4 *>(dst + tile_off(row, 0)) = lo;
        *reinterpret_cast<uint4 *>(dst + tile_off(row, 1)) = hi;
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
        mbar_arrive(b.a_full(sa));
        mbar_arrive(b.code_empty(sr));
    }
    return true;
}

// 4 packed code bytes of lanes 4w..4w+3 in lane 4w (other lanes: don't care).
__device__ __forceinline__ uint32_t pack_lane_bytes(int8_t code) {
    uint32_t v = static_cast<uint8_t>(code);
    v |= __shfl_down_sync(0xffffffffu, v, 1) << 8;
    v |= __shfl_down_sync(0xffffffffu, v, 2) << 16;
    return v;
}

// Q8_1 lane of one middle value and the sticky flags raised for it.
struct MidQ {
    Q8Lane q;
    int flags;
};

// ---- gate/up epilogue of one item (exact MMVQ order) -----------------------
// Pairs are handled two at a time (unit u = pairs pc0 + 2u, pc0 + 2u + 1) as
// packed f32x2 values.  Units without a real pair run the same arithmetic on
// the tile's zero padding (zero B rows and constants: every term is 0), which
// costs less than a branch per unit and leaf.
template <bool Tap>
__device__ __forceinline__ bool gu_epilogue_item(const TcrParams &p, uint8_t *smem, const RowsBars &bars,
                                                 uint32_t tq, RowsSeq &sq, int item, int4 td,
                                                 int lane, int quarter, int chunk) {
    using St = RowsStage<false>;
    constexpr int R = St::regions, CW = St::cw, NP = kTcTile, U = CW / 2;
    constexpr int kNodes = kRowsHidden / 32 / St::kb;        // 8 stages per matrix
    constexpr int kLeaves = St::kb / 2;                      // leaves per stage: blocks b and b + 32
    static_assert(kLeaves == 4, "a stage is one node two levels above the leaves");
    static_assert(CW == 4 || CW == 8, "one x8 / x16 load per block: 1 or 2 chunks x (4 pairs x 2 fragments)");
    const int I = p.inter;
    const int nb = kRowsHidden / 32, slabs = I / kRowsM;
    const int slab = item % slabs, tile = item / slabs;
    const int e = td.x, p0 = td.y, n = td.z;
    const int pc0 = chunk * CW;                               // this warp's first pair
    const int lrow = quarter * 32 + lane;                     // row within the slab
    const int row = slab * kRowsM + lrow;                     // middle row of this lane
    const uint64_t zero2 = 0ull;
    // binary-tree stack over the 8 stage nodes of the current matrix, per unit (s3 ends as the
    // total); the gate totals wait in gt while the up pass runs
    uint64_t s0[U], s1[U], s2[U], s3[U], gt[U];
#pragma unroll
    for (int u = 0; u < U; ++u) s3[u] = gt[u] = 0ull;
    int tap_base = 0;
    if constexpr (Tap) tap_base = (e == p.tap.expert) ? *p.tap.pair0 : 0;

    for (int ks = 0; ks < 2 * kNodes; ++ks, ++sq.g, ++sq.k) {
        const int m = ks / kNodes, kk = ks % kNodes;          // matrix (gate, up), node within it
        const int s = sq.g % St::side_stages;
        const uint8_t *st = smem + St::side_off + s * St::side_bytes;
        if (!mbar_wait(bars.side_full(s), (sq.g / St::side_stages) & 1, p.error)) return false;
        const int q = sq.g / St::spw, qs = q % St::sc_stages;   // scale group (its windows stay for spw stages)
        if (kk % St::spw == 0 && !mbar_wait(bars.sc_full(qs), (q / St::sc_stages) & 1, p.error)) return false;
        // d4 of this row: window 0 holds blocks 4kk..4kk+3 at columns 4 (kk % 2) .., window 1 blocks 4kk+32..
        const uint8_t *d4row = smem + St::sc_off + qs * St::sc_bytes + lrow * 16 + (kk & 1) * 8;
        const uint2 d4w0 = *reinterpret_cast<const uint2 *>(d4row);
        const uint2 d4w1 = *reinterpret_cast<const uint2 *>(d4row + kRowsM * 16);
        const int r = static_cast<int>(sq.k % R);
        if (!mbar_wait(bars.tm_full(r), (sq.k / R) & 1, p.error)) return false;
        tc_fence_after();
        const uint32_t tr = tq + r * St::reg_cols + chunk * 2 * CW;
        uint64_t node[U], la[U], lc[U];
#pragma unroll
        for (int h = 0; h < kLeaves; ++h) {   // leaf h: block 4kk+h (slot h) and 4kk+32+h (slot 4+h)
            // columns: per chunk of 4 pairs, fragment 0 of the pairs, then fragment 1
            uint32_t va[2 * CW], vb[2 * CW];
            if constexpr (CW == 8) {
                tmem_ld16(tr + h * 32, va);
                tmem_ld16(tr + (kLeaves + h) * 32, vb);
                tmem_wait_ld();
                tie16(va);
                tie16(vb);
            } else {
                tmem_ld8(tr + h * 32, va);
                tmem_ld8(tr + (kLeaves + h) * 32, vb);
                tmem_wait_ld();
                tie8(va);
                tie8(vb);
            }
            if (h == kLeaves - 1) region_release(bars.tm_empty(r), lane);
            // pair constants d8 and m4 = -4 s8 of block 4kk+h (slot h) and 4kk+32+h (slot 4+h), as pair units
            const uint4 *ka = reinterpret_cast<const uint4 *>(reinterpret_cast<const float *>(st + St::bsc) +
                                                              h * 2 * NP + pc0);
            const uint4 *kb = reinterpret_cast<const uint4 *>(reinterpret_cast<const float *>(st + St::bsc) +
                                                              (kLeaves + h) * 2 * NP + pc0);
            uint64_t d8a[U], m4a[U], d8b[U], m4b[U];
#pragma unroll
            for (int v = 0; v < U / 2; ++v) {
                const uint4 xa = ka[v], ya = ka[NP / 4 + v], xb = kb[v], yb = kb[NP / 4 + v];
                d8a[2 * v] = pk2(xa.x, xa.y), d8a[2 * v + 1] = pk2(xa.z, xa.w);
                m4a[2 * v] = pk2(ya.x, ya.y), m4a[2 * v + 1] = pk2(ya.z, ya.w);
                d8b[2 * v] = pk2(xb.x, xb.y), d8b[2 * v + 1] = pk2(xb.z, xb.w);
                m4b[2 * v] = pk2(yb.x, yb.y), m4b[2 * v + 1] = pk2(yb.z, yb.w);
            }
            const uint32_t wa = (h < 2) ? d4w0.x : d4w0.y, wb = (h < 2) ? d4w1.x : d4w1.y;
            const float d4a = (h & 1) ? hi_half(wa) : lo_half(wa);
            const float d4b = (h & 1) ? hi_half(wb) : lo_half(wb);
            const uint64_t d4ap = pkf2(d4a, d4a), d4bp = pkf2(d4b, d4b);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                // exact fragment dots of the unit's two pairs: block a (4kk+h) and b (4kk+32+h)
                const int c0 = (u >> 1) * 8 + (u & 1) * 2;   // fragment 0 of the unit's pairs; fragment 1 at +4
                const uint64_t ta0 = from_magic2(va[c0], va[c0 + 1]);
                const uint64_t ta1 = from_magic2(va[c0 + 4], va[c0 + 5]);
                const uint64_t tb0 = from_magic2(vb[c0], vb[c0 + 1]);
                const uint64_t tb1 = from_magic2(vb[c0 + 4], vb[c0 + 5]);
                // MMVQ lanes 2b+f (terms of block a) and 2b+f+64 (block b), summed, then the fragments
                const uint64_t leaf = add2(add2(mmvq_term2(ta0, d4ap, d8a[u], m4a[u], zero2),
                                                mmvq_term2(tb0, d4bp, d8b[u], m4b[u], zero2)),
                                           add2(mmvq_term2(ta1, d4ap, d8a[u], m4a[u], zero2),
                                                mmvq_term2(tb1, d4bp, d8b[u], m4b[u], zero2)));
                // node kk = (L(4kk) + L(4kk+1)) + (L(4kk+2) + L(4kk+3))
                if (h == 0) la[u] = leaf;
                else if (h == 1) la[u] = add2(la[u], leaf);
                else if (h == 2) lc[u] = leaf;
                else node[u] = add2(la[u], add2(lc[u], leaf));
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
                            dst[base + 4 * kk + h] = static_cast<int32_t>(da[jj]);
                            dst[base + 4 * kk + 32 + h] = static_cast<int32_t>(db[jj]);
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) {   // done with the stage's constants (and, at a group's end, its scale windows)
            mbar_arrive(bars.side_empty(s));
            if (kk % St::spw == St::spw - 1) mbar_arrive(bars.sc_empty(qs));
        }
        // push node kk into the binary tree over kk = 0..7 (one warp-uniform branch nest)
        if (!(kk & 1)) {
#pragma unroll
            for (int u = 0; u < U; ++u) s0[u] = node[u];
        } else if (!(kk & 2)) {
#pragma unroll
            for (int u = 0; u < U; ++u) s1[u] = add2(s0[u], node[u]);
        } else if (!(kk & 4)) {
#pragma unroll
            for (int u = 0; u < U; ++u) s2[u] = add2(s1[u], add2(s0[u], node[u]));
        } else {
#pragma unroll
            for (int u = 0; u < U; ++u) s3[u] = add2(s2[u], add2(s1[u], add2(s0[u], node[u])));
            if (ks == kNodes - 1) {
#pragma unroll
                for (int u = 0; u < U; ++u) gt[u] = s3[u];
            }
        }
    }

    // SiLU(gate) * up, then Q8_1 of the 32-row middle block held by this warp
    int flags = 0;
    const int jb = slab * (kRowsM / 32) + quarter;   // middle block index
    const int nbI = I / 32;
    uint8_t *mslot = p.mid_arr + static_cast<size_t>(tile) * tc_dn_slot(I) + static_cast<size_t>(jb) * NP * 32;
    float *msc = p.mid_sc_arr + static_cast<size_t>(tile) * tc_dn_sc_slot(I) + static_cast<size_t>(jb) * 2 * NP;
    // the reference's sanitisation (src/hip/session_ops.hip:250-262); the 4 exponentials together
    float gv[CW], uv[CW], ng[CW], ex[CW];
    int fj[CW];
#pragma unroll
    for (int j = 0; j < CW; ++j) {
        float g0, g1, u0, u1;
        upk2(gt[j / 2], g0, g1);
        upk2(s3[j / 2], u0, u1);
        fj[j] = 0;
        gv[j] = operand((j & 1) ? g1 : g0, fj[j]);
        uv[j] = operand((j & 1) ? u1 : u0, fj[j]);
        ng[j] = -gv[j];
    }
#pragma unroll
    for (int j = 0; j < CW; j += 2) {   // two at a time: the lookups overlap, the register peak stays low
        const float nj[2] = {ng[j], ng[j + 1]};
        float xj[2];
        expf_ref_n<2>(nj, xj);
        ex[j] = xj[0];
        ex[j + 1] = xj[1];
    }
#pragma unroll
    for (int j = 0; j < CW; ++j) {
        const int c = pc0 + j;
        MidQ r{{0, 0, 0, 0}, 0};
        if (c < n) {   // padded pairs get zero codes and constants
            int f = fj[j];
            const float act = arithmetic(__fdiv_rn(gv[j], __fadd_rn(1.0f, ex[j])), f);
            const float val = arithmetic(__fmul_rn(act, uv[j]), f);
            r.q = quantize_lane(f ? 0.0f : val);
            r.flags = f | r.q.flags;
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
// Q41: Q4_1 down matrices (minima in the stage group's second window).
template <bool Tap, bool Q41>
__device__ __forceinline__ bool dn_epilogue_item(const TcrParams &p, uint8_t *smem, const RowsBars &bars,
                                                 uint32_t tq, RowsSeq &sq, int item, int4 td,
                                                 int lane, int quarter, int chunk) {
    using St = RowsStage<true, Q41>;
    constexpr int R = St::regions, CW = St::cw, NP = kTcTile;
    static_assert(CW == 4 || CW == 8, "one x4 / x8 load per block");
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

    for (int ks = 0; ks < nb / St::kb; ++ks, ++sq.g) {
        const int s = sq.g % St::side_stages;
        const uint8_t *st = smem + St::side_off + s * St::side_bytes;
        if (!mbar_wait(bars.side_full(s), (sq.g / St::side_stages) & 1, p.error)) return false;
        const int q = sq.g / St::spw, qs = q % St::sc_stages;
        if (ks % St::spw == 0 && !mbar_wait(bars.sc_full(qs), (q / St::sc_stages) & 1, p.error)) return false;
        // d4 of the stage's blocks 8ks..8ks+7: the whole 8-block window of this row
        static_assert(St::kb == 8 && St::spw == 1, "one scale window per stage");
        const uint4 d4q = *reinterpret_cast<const uint4 *>(smem + St::sc_off + qs * St::sc_bytes + lrow * 16);
        uint4 m4q = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (Q41)
            m4q = *reinterpret_cast<const uint4 *>(smem + St::sc_off + qs * St::sc_bytes + St::sc_win + lrow * 16);
        const int r = static_cast<int>(sq.k % R);
        ++sq.k;
        if (!mbar_wait(bars.tm_full(r), ((sq.k - 1) / R) & 1, p.error)) return false;
        tc_fence_after();
        // the first half's loads, then the second half's in flight while the first half computes
        uint32_t v[St::kb][CW];
        constexpr int KH = St::kb / 2;
#pragma unroll
        for (int kb = 0; kb < KH; ++kb) tmem_ld_cw<CW>(tq + r * St::reg_cols + kb * NP + pc0, v[kb]);
        tmem_wait_ld();
#pragma unroll
        for (int kb = 0; kb < KH; ++kb) tie_cw<CW>(v[kb]);
#pragma unroll
        for (int kb = KH; kb < St::kb; ++kb) tmem_ld_cw<CW>(tq + r * St::reg_cols + kb * NP + pc0, v[kb]);
        const float *cb = reinterpret_cast<const float *>(st + St::bsc);
#pragma unroll
        for (int kb = 0; kb < St::kb; ++kb) {
            if (kb == KH) {
                tmem_wait_ld();
#pragma unroll
                for (int k2 = KH; k2 < St::kb; ++k2) tie_cw<CW>(v[k2]);
                region_release(bars.tm_empty(r), lane);
            }
            const uint32_t hw = kb < 2 ? d4q.x : kb < 4 ? d4q.y : kb < 6 ? d4q.z : d4q.w;
            const float d4 = (kb & 1) ? hi_half(hw) : lo_half(hw);
            const uint64_t d4p = pkf2(d4, d4);
            uint64_t d8p[CW / 2], m8p[CW / 2];
#pragma unroll
            for (int c = 0; c < CW / 4; ++c) {
                const uint4 d8 = *reinterpret_cast<const uint4 *>(cb + kb * 2 * NP + pc0 + 4 * c);
                const uint4 m8 = *reinterpret_cast<const uint4 *>(cb + kb * 2 * NP + NP + pc0 + 4 * c);
                d8p[2 * c] = pk2(d8.x, d8.y);
                d8p[2 * c + 1] = pk2(d8.z, d8.w);
                m8p[2 * c] = pk2(m8.x, m8.y);
                m8p[2 * c + 1] = pk2(m8.z, m8.w);
            }
            uint64_t m4p = 0ull;
            if constexpr (Q41) {
                const uint32_t mw = kb < 2 ? m4q.x : kb < 4 ? m4q.y : kb < 6 ? m4q.z : m4q.w;
                const float m4 = (kb & 1) ? hi_half(mw) : lo_half(mw);
                m4p = pkf2(m4, m4);
            }
#pragma unroll
            for (int u = 0; u < CW / 2; ++u) {
                const uint64_t t = from_magic2(v[kb][2 * u], v[kb][2 * u + 1]);   // exact dots
                if constexpr (Q41) {
                    // s8 = -m8 / 8 exactly; half(d4 d8) and half(m4 s8) of exact fp32 products
                    const uint64_t s8 = mul2(m8p[u], pkf2(-0.125f, -0.125f));
                    const uint64_t dd = round_half2(mul2(d4p, d8p[u]));
                    const uint64_t ms = round_half2(mul2(m4p, s8));
                    acc[u] = add2(acc[u], fma2(t, dd, ms));
                } else {
                    acc[u] = fma2(d4p, fma2(t, d8p[u], m8p[u]), acc[u]);
                }
                if constexpr (Tap) {
                    float t0, t1;
                    upk2(t, t0, t1);
                    const float tt[2] = {t0, t1};
#pragma unroll
                    for (int jj = 0; jj < 2; ++jj) {
                        const int j = 2 * u + jj;
                        const int pl = p0 + pc0 + j - tap_base;
                        if (e == p.tap.expert && pc0 + j < n && pl >= 0 && pl < p.tap.max_pairs)
                            p.tap.down[(static_cast<size_t>(pl) * H + row) * nb + ks * St::kb + kb] =
                                static_cast<int32_t>(tt[jj]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(bars.side_empty(s));
            if (ks % St::spw == St::spw - 1) mbar_arrive(bars.sc_empty(qs));
        }
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
template <bool Down, bool Tap, bool Q41 = false>
__global__ void __launch_bounds__(RowsStage<Down, Q41>::threads, 1) tc_rows_kernel(const __grid_constant__ TcrParams p) {
    using St = RowsStage<Down, Q41>;
    constexpr int CS = St::code_stages, SS = St::side_stages, QS = St::sc_stages, AS = St::a_stages;
    constexpr int R = St::regions;
    extern __shared__ __align__(128) uint8_t smem[];
    const int H = p.hidden, I = p.inter;
    const int K = Down ? I : H, nb = K / 32, nodes = nb / St::kb;
    const int ksteps = Down ? nodes : 2 * nodes;     // gate/up: the gate pass, then the up pass
    const int slabs = (Down ? H : I) / kRowsM;
    RowsBars bars{reinterpret_cast<uint64_t *>(smem)};
    uint64_t *fin = bars.fin();
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + 1536);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < CS; ++s) {
            mbar_init(bars.code_full(s), 1);
            mbar_init(bars.code_empty(s), kRowsUnpackWarps);
        }
        for (int s = 0; s < SS; ++s) {
            mbar_init(bars.side_full(s), 1);
            mbar_init(bars.side_empty(s), St::epi_warps + 1);   // + the MMAs' commit (B operand)
        }
        for (int s = 0; s < QS; ++s) {
            mbar_init(bars.sc_full(s), 1);
            mbar_init(bars.sc_empty(s), St::epi_warps);
        }
        for (int s = 0; s < AS; ++s) {
            mbar_init(bars.a_full(s), kRowsUnpackWarps);
            mbar_init(bars.a_empty(s), 1);
        }
        for (int r = 0; r < R; ++r) {
            mbar_init(bars.tm_full(r), 1);
            mbar_init(bars.tm_empty(r), St::epi_warps);
        }
        mbar_init(fin, 1);
        mbar_fence_init();
    }
    // bf16 operands of the conversion-offset MMA: A row r = (1, 0, ..., 0), B row n = (1.5 * 2^23, 0, ..., 0)
    for (int c = threadIdx.x; c < 4 * kRowsM; c += blockDim.x) {
        const int which = c / (2 * kRowsM), rest = c % (2 * kRowsM), row = rest >> 1, half = rest & 1;
        const uint4 v = make_uint4(half ? 0u : (which ? kBf16Magic : kBf16One), 0u, 0u, 0u);
        *reinterpret_cast<uint4 *>(smem + St::magic_off + which * kRowsM * 32 + tile_off(row, half)) = v;
    }
    fence_proxy_async();
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
        // One thread feeds the code ring and the side/scale rings
        // independently: it polls (without blocking) for the next free slot of
        // each and issues whichever copy can go, so the codes (released by the
        // unpack) run ahead of the side data (released by the epilogue) and
        // neither ring's consumers hold the other back.  Side copies never pass
        // the code copies of the same stage.
        if (lane == 0) {
            for (int m = 0; m < St::M; ++m) {
                tma_prefetch_map(&p.maps.codes[Down ? 2 : m]);
                tma_prefetch_map(&p.maps.scales[Down ? 2 : m]);
                if (Down && Q41) tma_prefetch_map(&p.maps.down_mins);
            }
            constexpr uint32_t bbytes = St::kb * St::brows * 32, sbytes = St::kb * St::cwords * kTcTile * 4;
            const size_t bslot = Down ? tc_dn_slot(K) : tc_gu_slot(K);
            const size_t sslot = Down ? tc_dn_sc_slot(K) : tc_gu_sc_slot(K);
            const int total_g = blockIdx.x < total ? (total - blockIdx.x + gridDim.x - 1) / gridDim.x * ksteps : 0;
            // per-ring cursors, advanced stage by stage (the tile record is read once per item)
            struct Cursor {
                int item, ks, tile, slab, e;
            };
            auto start = [&](Cursor &c, int item) {
                c.item = item;
                c.ks = 0;
                c.tile = item / slabs;
                c.slab = item - c.tile * slabs;
                c.e = item < total ? p.tiles[c.tile].x : 0;
            };
            auto advance = [&](Cursor &c) {
                if (++c.ks == ksteps) start(c, c.item + gridDim.x);
            };
            Cursor cc_, cs_;
            start(cc_, blockIdx.x);
            cs_ = cc_;
            int gc = 0, gs = 0;          // next stage of the code ring, of the side ring
            uint32_t idle = 0;
            while (gs < total_g) {
                bool progress = false;
                if (gc < total_g && (gc < CS || mbar_test(bars.code_empty(gc % CS), ((gc / CS) & 1) ^ 1))) {
                    const int mat = Down ? 2 : cc_.ks / nodes, kk = cc_.ks % nodes, c = gc % CS;
                    uint8_t *dst0 = smem + St::codes_off + c * St::codes_bytes;
                    mbar_arrive_expect_tx(bars.code_full(c), St::codes_bytes);
                    // down blocks 8kk..8kk+3, 8kk+4..8kk+7; gate/up blocks 4kk..4kk+3, then 4kk+32..4kk+35
                    for (int cp = 0; cp < St::kb / St::bpc; ++cp) {
                        const int b0 = Down ? St::kb * kk + St::bpc * cp : St::bpc * kk + 32 * cp;
                        uint8_t *dst = dst0 + cp * St::bpc * kRowsM * 16;
                        if (p.raw_rowmajor)
                            tma_load_3d(dst, &p.maps.codes[mat], b0 * 16, cc_.slab * kRowsM, cc_.e, bars.code_full(c));
                        else
                            tma_load_4d(dst, &p.maps.codes[mat], 0, cc_.slab * kRowsM, b0, cc_.e, bars.code_full(c));
                    }
                    ++gc;
                    advance(cc_);
                    progress = true;
                }
                if (gs < gc) {
                    const int mat = Down ? 2 : cs_.ks / nodes, ks = cs_.ks % nodes, sd = gs % SS;
                    const int q = gs / St::spw, qs = q % QS;
                    const bool group = ks % St::spw == 0;   // also the scale windows of this stage group
                    if ((gs < SS || mbar_test(bars.side_empty(sd), ((gs / SS) & 1) ^ 1)) &&
                        (!group || q < QS || mbar_test(bars.sc_empty(qs), ((q / QS) & 1) ^ 1))) {
                        uint8_t *st = smem + St::side_off + sd * St::side_bytes;
                        mbar_arrive_expect_tx(bars.side_full(sd), bbytes + sbytes);
                        bulk_g2s(st + St::b,
                                 p.b_arr + static_cast<size_t>(cs_.tile) * bslot + static_cast<size_t>(ks) * bbytes,
                                 bbytes, bars.side_full(sd));
                        bulk_g2s(st + St::bsc,
                                 p.bsc_arr + static_cast<size_t>(cs_.tile) * sslot +
                                     static_cast<size_t>(ks) * St::kb * St::cwords * kTcTile,
                                 sbytes, bars.side_full(sd));
                        if (group) {
                            // gate/up blocks 8j and 32 + 8j of the stage's matrix; down blocks 8j (and
                            // their minima for Q4_1)
                            constexpr int wins = Down && !Q41 ? 1 : St::wins;
                            mbar_arrive_expect_tx(bars.sc_full(qs), wins * St::sc_win);
#pragma unroll
                            for (int w = 0; w < wins; ++w) {
                                const int b0 = Down ? St::kb * ks : St::bpc * ks + 32 * w;
                                const CUtensorMap *map = Down && w == 1 ? &p.maps.down_mins : &p.maps.scales[mat];
                                tma_load_3d(smem + St::sc_off + qs * St::sc_bytes + w * St::sc_win, map, b0 & ~7,
                                            cs_.slab * kRowsM, cs_.e, bars.sc_full(qs));
                            }
                        }
                        ++gs;
                        advance(cs_);
                        progress = true;
                    }
                }
                if (progress) {
                    idle = 0;
                } else {
                    if (++idle > kProducerIdleLimit) {   // the consumers stopped (a bounded wait gave up)
                        atomicOr(p.error, kFlagTimeout);
                        break;
                    }
                    __nanosleep(64);
                }
            }
            // keep the CTA alive until every issued copy has landed
            for (int g = gc - CS > 0 ? gc - CS : 0; g < gc; ++g)
                mbar_wait(bars.code_full(g % CS), (g / CS) & 1, p.error);
            for (int g = gs - SS > 0 ? gs - SS : 0; g < gs; ++g)
                mbar_wait(bars.side_full(g % SS), (g / SS) & 1, p.error);
            const int nq = (gs + St::spw - 1) / St::spw;
            for (int q = nq - QS > 0 ? nq - QS : 0; q < nq; ++q)
                mbar_wait(bars.sc_full(q % QS), (q / QS) & 1, p.error);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = rows_idesc(kRowsM, St::brows);
            const uint32_t idesc_mg = magic_idesc(kRowsM, kRowsM);   // the offset MMA: 128 columns at a time
            const uint64_t amg = smem_desc(smem_u32(smem + St::magic_off), 128, 256);
            const uint64_t bmg = smem_desc(smem_u32(smem + St::magic_off + kRowsM * 32), 128, 256);
            int g = 0;
            uint32_t kseq = 0;
            bool failed = false;
            for (int item = blockIdx.x; item < total && !failed; item += gridDim.x) {
                for (int ks = 0; ks < ksteps && !failed; ++ks, ++g) {
                    const int sr = g % SS, sa = g % AS;
                    if (!mbar_wait(bars.a_full(sa), (g / AS) & 1, p.error) ||
                        !mbar_wait(bars.side_full(sr), (g / SS) & 1, p.error)) {
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_st = smem_u32(smem + St::a_off + sa * St::a_bytes);
                    const uint32_t b_st = smem_u32(smem + St::side_off + sr * St::side_bytes + St::b);
                    {
                        const int r = static_cast<int>(kseq % R);
                        if (!mbar_wait(bars.tm_empty(r), (kseq / R) & 1, p.error)) {
                            failed = true;
                            break;
                        }
                        ++kseq;
                        tc_fence_after();
                        // every column of the region = 1.5 * 2^23 (f32), then the integer dots added onto it:
                        // stage slot kb (gate/up blocks 4k..4k+3, 4k+32..4k+35; down 8k..8k+7) into columns
                        // [brows kb, brows (kb + 1))
                        static_assert(St::reg_cols % kRowsM == 0, "whole offset MMAs per region");
#pragma unroll
                        for (int c = 0; c < St::reg_cols; c += kRowsM) mma_bf16(tmem + r * St::reg_cols + c, amg, bmg, idesc_mg);
#pragma unroll
                        for (int kb = 0; kb < St::kb; ++kb) {
                            const uint64_t ad = smem_desc(a_st + kb * kRowsM * 32, 128, 256);
                            const uint64_t bd = smem_desc(b_st + kb * St::brows * 32, 128, 256);
                            mma_i8(tmem + r * St::reg_cols + kb * St::brows, ad, bd, idesc, 1u);
                        }
                        mma_commit(bars.tm_full(r));
                    }
                    mma_commit(bars.a_empty(sa));
                    mma_commit(bars.side_empty(sr));
                }
            }
            // every MMA of this CTA has completed before teardown
            mma_commit(fin);
            mbar_wait(fin, 0, p.error);
        }
    } else if (warp < 2 + kRowsUnpackWarps) {
        // ---------------- unpack: raw nibbles -> u8 K-major core matrices ----------------
        const bool rowmajor = p.raw_rowmajor != 0;
        int g = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < total && ok; item += gridDim.x)
            for (int ks = 0; ks < ksteps && ok; ++ks, ++g)
                ok = rows_unpack<Down>(smem, bars, g, threadIdx.x - 64, rowmajor, lane, p.error);
    } else {
        // ---------------- epilogue ----------------
        const int ew = warp - 2 - kRowsUnpackWarps;       // 0 .. epi_warps - 1
        const int quarter = warp & 3, chunk = ew >> 2;    // TMEM lane quarter, pair chunk of St::cw pairs
        const uint32_t tq = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        if (lane == 0)   // every region starts free
            for (int r = 0; r < R; ++r) mbar_arrive(bars.tm_empty(r));
        RowsSeq sq;
        bool ok = true;
        for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
            const int4 td = p.tiles[item / slabs];
            ok = Down ? dn_epilogue_item<Tap, Q41>(p, smem, bars, tq, sq, item, td, lane, quarter, chunk)
                      : gu_epilogue_item<Tap>(p, smem, bars, tq, sq, item, td, lane, quarter, chunk);
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
// pair_token[p0 + r]), row tc_gu_brow(r, 0) = its Q8_1 codes of fragment 0
// (elements 0..7 and 16..23, the rest zero) and row tc_gu_brow(r, 1) those of
// fragment 1, blocks in stage order, and the constants d8[16] then
// -4*s8[16]; pairs n..15 are zero.
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
            *reinterpret_cast<uint4 *>(dst + tile_off(tc_gu_brow(pr, frag), 0)) = v[2 * i];
            *reinterpret_cast<uint4 *>(dst + tile_off(tc_gu_brow(pr, frag), 1)) = v[2 * i + 1];
            if (!frag) {
                ss[pos * 2 * kTcTile + pr] = c[i].x;
                ss[pos * 2 * kTcTile + kTcTile + pr] = -(4.0f * c[i].y);
            }
        }
    }
}

inline int tc_rows_configure() {
    const int gu = static_cast<int>(RowsStage<false>::smem), dn = static_cast<int>(RowsStage<true>::smem);
    const cudaFuncAttribute a = cudaFuncAttributeMaxDynamicSharedMemorySize;
    if (cudaFuncSetAttribute(tc_rows_kernel<false, false>, a, gu) != cudaSuccess ||
        cudaFuncSetAttribute(tc_rows_kernel<false, true>, a, gu) != cudaSuccess ||
        cudaFuncSetAttribute(tc_rows_kernel<true, false>, a, dn) != cudaSuccess ||
        cudaFuncSetAttribute(tc_rows_kernel<true, true>, a, dn) != cudaSuccess ||
        cudaFuncSetAttribute(tc_rows_kernel<true, false, true>, a, dn) != cudaSuccess ||
        cudaFuncSetAttribute(tc_rows_kernel<true, true, true>, a, dn) != cudaSuccess)
        return MOE_CUDA_ERROR;
    return MOE_OK;
}

}  // namespace qmoe
