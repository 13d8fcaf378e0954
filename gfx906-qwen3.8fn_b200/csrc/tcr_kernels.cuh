// tcr_kernels.cuh -- tcgen05 (kind::i8) grouped expert GEMMs with the weight
// rows on the TMEM lanes (prefill and every batch above decode size).
//
// One work item = (expert group tile of <= 64 pairs, slab of 128 weight rows).
// The MMA is D[128 rows][Np pairs] = A . B^T, K = 32 per instruction = one
// quantisation block, so every MMA result is one per-block integer dot:
//   A = the slab's Q4_0 codes unpacked to unsigned bytes (0..15, u8),
//   B = the tile's Q8_1 activation codes (s8), Np = 16 * ceil(n / 16).
// A u8 x s8 product gives the reference's uncentred dot sum(q * x) directly
// (src/quant.cpp:48-55), |dot| <= 15 * 127 * 32 < 2^16.
//
// Exact conversion: every TMEM accumulator is preloaded with the bit pattern
// of 1.5 * 2^23 (0x4b400000) and each MMA accumulates onto it, so the int32
// result bits are 0x4b400000 + dot, which read as fp32 is exactly
// 1.5 * 2^23 + dot (|dot| < 2^22 keeps the exponent).  One f32x2 subtraction
// per two columns recovers the dot as an exact fp32; the reader then stores
// the pattern back.  Per element the epilogue is
//   acc += d4 * (dot * d8 - 8 * s8)
// as two packed FMAs (d4 per lane = weight row, d8 and -8*s8 per column).
//
// Gate/up items hold 128 middle rows: two MMAs per block, gate into columns
// [0, Np) and up into [64, 64 + Np) of the block's TMEM region, so the thread
// of lane r owns gate row r and up row r of every pair.  The item end runs
// SiLU(gate) * up and the Q8_1 requantisation of each 32-row middle block --
// one warp holds exactly one block per pair column (lane = element), which is
// the reference's XOR-butterfly sum order -- and writes the middle codes in
// the down pass's operand layout.  Down items hold 128 output rows and end in
// a router-weighted red.add into the residual (lane = row: coalesced).
//
// Warp roles (12 warps):
//   warp 0      TMEM allocation; lane 0 issues the TMA copies: raw weight
//               codes and scales through 4-D/3-D tensor maps, the tile's
//               pre-arranged activation operand as 1-D bulk copies;
//   warp 1      lane 0 issues the MMAs (one elected thread);
//   warps 2-3   unpack raw Q4_0 codes shared -> shared into the MMA layout;
//   warps 4-11  epilogue: two per TMEM lane quarter, each owning half of the
//               tile's columns.
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
constexpr int kRowsNP = kTcTile;       // pairs per tile at most (MMA N)
constexpr int kRowsKB = 4;             // quantisation blocks per pipeline stage
constexpr int kRowsUnpackWarps = 2;
constexpr int kRowsEpiWarps = 8;
constexpr int kRowsWarps = 2 + kRowsUnpackWarps + kRowsEpiWarps;
constexpr int kRowsThreads = 32 * kRowsWarps;
constexpr int kRowsMinGroup = 1;       // batches above decode size: every group on this path
constexpr uint32_t kMagicBits = 0x4b400000u;
constexpr float kMagicF = 12582912.0f; // 1.5 * 2^23

// Tensor maps over one weights object (all experts), built on the host.
struct alignas(64) TcrMaps {
    CUtensorMap codes[3];    // gate, up, down code bytes
    CUtensorMap scales[3];   // gate, up, down half scales
};

struct TcrParams {
    TcrMaps maps;
    int hidden, inter;
    int raw_rowmajor;          // codes staged [row][block] (3-D map) instead of [block][row]
    const uint8_t *b_arr;      // arranged activation operand, one slot per tile
    const float *bsc_arr;      // arranged (d8, -8*s8) per (tile, block, pair)
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

// Arranged operand slots: tile t, block b holds Np rows of 32 code bytes in
// the K-major core-matrix layout at t * slot + b * Np * 32, and the per-pair
// constants d8[Np] then m8[Np] at t * sc_slot + b * 2 * Np floats.
__host__ __device__ constexpr size_t rows_b_slot(int K) { return static_cast<size_t>(kRowsNP) * 32 * (K / 32); }
__host__ __device__ constexpr size_t rows_sc_slot(int K) { return static_cast<size_t>(kRowsNP) * 2 * (K / 32); }

template <bool Down>
struct RowsStage {
    static constexpr int M = Down ? 1 : 2;                                   // matrices per item
    static constexpr uint32_t codes = 0;                                     // M x 4 blocks x 128 rows x 16 B
    static constexpr uint32_t scales = codes + M * kRowsKB * kRowsM * 16;    // M x [128][8] half
    static constexpr uint32_t b = scales + M * kRowsM * 8 * 2;               // [4][Np][32]
    static constexpr uint32_t bsc = b + kRowsKB * kRowsNP * 32;              // [4][2][Np] fp32
    static constexpr uint32_t raw_bytes = bsc + kRowsKB * 2 * kRowsNP * 4;
    static constexpr uint32_t a_bytes = M * kRowsKB * kRowsM * 32;           // unpacked A tiles
    static constexpr int raw_stages = Down ? 6 : 4;
    static constexpr int a_stages = Down ? 4 : 3;
    static constexpr uint32_t raw_off = 1024;
    static constexpr uint32_t a_off = raw_off + raw_stages * raw_bytes;
    static constexpr uint32_t smem = a_off + a_stages * a_bytes;
    static constexpr int reg_cols = Down ? 64 : 128;                         // TMEM columns per block
    static constexpr int regions = 512 / reg_cols;
};
static_assert(RowsStage<false>::smem <= 227 * 1024 && RowsStage<true>::smem <= 227 * 1024, "fits one CTA");
static_assert(RowsStage<false>::raw_bytes % 1024 == 0 && RowsStage<true>::raw_bytes % 1024 == 0, "aligned");

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
// Store the preload pattern into 8 consecutive columns.
__device__ __forceinline__ void tmem_st8_magic(uint32_t taddr) {
    const uint32_t m = kMagicBits;
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(m)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
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
    uint32_t k = 0;     // block sequence (TMEM regions)
};

// 4 packed code bytes of lanes 4w..4w+3 in lane 4w (other lanes: don't care).
__device__ __forceinline__ uint32_t pack_lane_bytes(int8_t code) {
    uint32_t v = static_cast<uint8_t>(code);
    v |= __shfl_down_sync(0xffffffffu, v, 1) << 8;
    v |= __shfl_down_sync(0xffffffffu, v, 2) << 16;
    return v;
}

// ---- epilogue of one item, CW columns per warp and matrix -----------------
template <bool Down, bool Tap, int CW>
__device__ __forceinline__ bool rows_epilogue_item(const TcrParams &p, uint8_t *smem, uint64_t *raw_full,
                                                   uint64_t *raw_empty, uint64_t *tm_full, uint64_t *tm_empty,
                                                   uint32_t tq, RowsSeq &sq, int item, int4 td, int lane, int quarter,
                                                   int chunk) {
    using St = RowsStage<Down>;
    constexpr int M = St::M;
    constexpr int R = St::regions;
    const int H = p.hidden, I = p.inter;
    const int K = Down ? I : H, nb = K / 32, ksteps = nb / kRowsKB;
    const int rows_total = Down ? H : I, slabs = rows_total / kRowsM;
    const int slab = item % slabs, tile = item / slabs;
    const int e = td.x, p0 = td.y, n = td.z, np = 2 * CW;
    const int col0 = chunk * CW;
    const int row = slab * kRowsM + quarter * 32 + lane;   // weight row (gate/up: middle row) of this lane
    uint64_t acc[M][CW / 2];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int j = 0; j < CW / 2; ++j) acc[m][j] = 0ull;
    const uint64_t unbias = pkf2(-kMagicF, -kMagicF);
    int tap_base = 0;
    if constexpr (Tap) tap_base = (e == p.tap.expert) ? *p.tap.pair0 : 0;

    for (int ks = 0; ks < ksteps; ++ks, ++sq.g) {
        const int s = sq.g % St::raw_stages;
        const uint8_t *st = smem + St::raw_off + s * St::raw_bytes;
        // acquire the TMA writes of this stage's scales (the phase is complete or about to be)
        if (!mbar_wait(&raw_full[s], (sq.g / St::raw_stages) & 1, p.error)) return false;
#pragma unroll 1
        for (int kb = 0; kb < kRowsKB; ++kb, ++sq.k) {
            const int r = static_cast<int>(sq.k % R);
            if (!mbar_wait(&tm_full[r], (sq.k / R) & 1, p.error)) return false;
            tc_fence_after();
            uint32_t v[M][CW];
#pragma unroll
            for (int m = 0; m < M; ++m)
#pragma unroll
                for (int j = 0; j < CW; j += 8) tmem_ld8(tq + r * St::reg_cols + m * 64 + col0 + j, &v[m][j]);
            tmem_wait_ld();
#pragma unroll
            for (int m = 0; m < M; ++m)
#pragma unroll
                for (int j = 0; j < CW; j += 8) tie8(&v[m][j]);
            // give the region back: preload pattern into the columns just read
#pragma unroll
            for (int m = 0; m < M; ++m)
#pragma unroll
                for (int j = 0; j < CW; j += 8) tmem_st8_magic(tq + r * St::reg_cols + m * 64 + col0 + j);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tm_empty[r]);
            // weight scale of this lane's row (both matrices), pair constants per column
            uint64_t d4p[M];
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const uint16_t *sc = reinterpret_cast<const uint16_t *>(st + St::scales + m * kRowsM * 16);
                const float d4 = h2f(sc[(quarter * 32 + lane) * 8 + (ks & 1) * 4 + kb]);
                d4p[m] = pkf2(d4, d4);
            }
            const float *d8p = reinterpret_cast<const float *>(st + St::bsc) + kb * 2 * np + col0;
            const float *m8p = d8p + np;
#pragma unroll
            for (int j4 = 0; j4 < CW / 4; ++j4) {
                const float4 d8q = *reinterpret_cast<const float4 *>(d8p + 4 * j4);
                const float4 m8q = *reinterpret_cast<const float4 *>(m8p + 4 * j4);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint64_t d8 = h ? pkf2(d8q.z, d8q.w) : pkf2(d8q.x, d8q.y);
                    const uint64_t m8 = h ? pkf2(m8q.z, m8q.w) : pkf2(m8q.x, m8q.y);
                    const int j = 4 * j4 + 2 * h;
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        const uint64_t t = add2(pk2(v[m][j], v[m][j + 1]), unbias);   // exact dots
                        acc[m][j / 2] = fma2(d4p[m], fma2(t, d8, m8), acc[m][j / 2]);
                    }
                }
            }
            if constexpr (Tap) {
                if (e == p.tap.expert) {
                    const int b = ks * kRowsKB + kb;
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        int32_t *dst = Down ? p.tap.down : (m == 0 ? p.tap.gate : p.tap.up);
#pragma unroll
                        for (int j = 0; j < CW; ++j) {
                            const int pl = p0 + col0 + j - tap_base;
                            if (col0 + j < n && pl >= 0 && pl < p.tap.max_pairs)
                                dst[(static_cast<size_t>(pl) * rows_total + row) * nb + b] =
                                    static_cast<int32_t>(__uint_as_float(v[m][j]) - kMagicF);
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[s]);   // done with the stage's scales
    }

    float a[M][CW];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int j = 0; j < CW / 2; ++j) upk2(acc[m][j], a[m][2 * j], a[m][2 * j + 1]);
    int flags = 0;
    if constexpr (!Down) {
        // SiLU(gate) * up, then Q8_1 of the 32-row middle block held by this warp
        const int jb = slab * (kRowsM / 32) + quarter;   // middle block index
        const int nbI = I / 32;
        uint8_t *mslot = p.mid_arr + static_cast<size_t>(tile) * rows_b_slot(I) + static_cast<size_t>(jb) * np * 32;
        float *msc = p.mid_sc_arr + static_cast<size_t>(tile) * rows_sc_slot(I) + static_cast<size_t>(jb) * 2 * np;
#pragma unroll
        for (int j = 0; j < CW; ++j) {
            const int c = col0 + j;
            Q8Lane q{0, 0, 0, 0};
            if (c < n) {
                int f = 0;
                const float gv = operand(a[0][j], f), uv = operand(a[1][j], f);
                const float act = arithmetic(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), f);
                const float val = arithmetic(__fmul_rn(act, uv), f);
                q = quantize_lane(f ? 0.0f : val);
                flags |= f | q.flags;
            }
            // padded columns (c >= n) get zero codes and constants
            const uint32_t word = pack_lane_bytes(q.code);
            if ((lane & 3) == 0)
                *reinterpret_cast<uint32_t *>(mslot + tile_off(c, lane >> 4) + (lane & 15)) = word;
            if (lane == 0) {
                msc[c] = h2f(q.d);
                msc[np + c] = -(8.0f * h2f(q.s));
            }
            if constexpr (Tap) {
                const int pl = p0 + c - tap_base;
                if (e == p.tap.expert && c < n && pl >= 0 && pl < p.tap.max_pairs) {
                    p.tap.mid_codes[static_cast<size_t>(pl) * I + row] = q.code;
                    if (lane == 0) p.tap.mid_ds[static_cast<size_t>(pl) * nbI + jb] = q.d | (uint32_t(q.s) << 16);
                }
            }
        }
    } else {
        // router-weighted scatter-add of the 128-row slab into the residual
        int tok_l = 0;
        float w_l = 0.0f;
        if (lane < CW && col0 + lane < n) {
            tok_l = __ldg(p.pair_token + p0 + col0 + lane);
            w_l = __ldg(p.pair_weight + p0 + col0 + lane);
        }
#pragma unroll
        for (int j = 0; j < CW; ++j) {
            const int tok = __shfl_sync(0xffffffffu, tok_l, j);
            const float w = __shfl_sync(0xffffffffu, w_l, j);
            if (col0 + j >= n) break;
            const float y = arithmetic(a[0][j], flags);
            const float cv = arithmetic(__fmul_rn(w, y), flags);
            atomicAdd(p.out + static_cast<size_t>(tok) * H + row, cv);
        }
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
            int g = 0;
            bool failed = false;
            for (int item = blockIdx.x; item < total && !failed; item += gridDim.x) {
                const int tile = item / slabs, slab = item % slabs;
                const int4 td = p.tiles[tile];
                const int np = (td.z + 15) & ~15;
                const uint32_t bbytes = kRowsKB * np * 32, sbytes = kRowsKB * np * 8;
                for (int ks = 0; ks < ksteps; ++ks, ++g) {
                    const int s = g % RS;
                    if (g >= RS && !mbar_wait(&raw_empty[s], ((g / RS) & 1) ^ 1, p.error)) { failed = true; break; }
                    uint8_t *st = smem + St::raw_off + s * St::raw_bytes;
                    mbar_arrive_expect_tx(&raw_full[s], M * (kRowsKB * kRowsM * 16 + kRowsM * 16) + bbytes + sbytes);
                    for (int m = 0; m < M; ++m) {
                        const int mat = Down ? 2 : m;
                        if (p.raw_rowmajor)
                            tma_load_3d(st + St::codes + m * kRowsKB * kRowsM * 16, &p.maps.codes[mat],
                                        ks * kRowsKB * 16, slab * kRowsM, td.x, &raw_full[s]);
                        else
                            tma_load_4d(st + St::codes + m * kRowsKB * kRowsM * 16, &p.maps.codes[mat], 0,
                                        slab * kRowsM, ks * kRowsKB, td.x, &raw_full[s]);
                        tma_load_3d(st + St::scales + m * kRowsM * 16, &p.maps.scales[mat], (ks * kRowsKB) & ~7,
                                    slab * kRowsM, td.x, &raw_full[s]);
                    }
                    bulk_g2s(st + St::b,
                             p.b_arr + static_cast<size_t>(tile) * rows_b_slot(K) + static_cast<size_t>(ks) * bbytes,
                             bbytes, &raw_full[s]);
                    bulk_g2s(st + St::bsc,
                             p.bsc_arr + static_cast<size_t>(tile) * rows_sc_slot(K) +
                                 static_cast<size_t>(ks) * kRowsKB * 2 * np,
                             sbytes, &raw_full[s]);
                }
            }
            // keep the CTA alive until every issued copy has landed
            for (int k = g - RS > 0 ? g - RS : 0; k < g; ++k) mbar_wait(&raw_full[k % RS], (k / RS) & 1, p.error);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int g = 0;
            uint32_t kseq = 0;
            bool failed = false;
            for (int item = blockIdx.x; item < total && !failed; item += gridDim.x) {
                const int4 td = p.tiles[item / slabs];
                const int np = (td.z + 15) & ~15;
                const uint32_t idesc = rows_idesc(kRowsM, np);
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
                    for (int kb = 0; kb < kRowsKB; ++kb, ++kseq) {
                        const int r = static_cast<int>(kseq % R);
                        if (!mbar_wait(&tm_empty[r], (kseq / R) & 1, p.error)) { failed = true; break; }
                        tc_fence_after();
                        const uint64_t bd = smem_desc(b_st + kb * np * 32, 128, 256);
#pragma unroll
                        for (int m = 0; m < M; ++m) {
                            const uint64_t ad = smem_desc(a_st + (m * kRowsKB + kb) * kRowsM * 32, 128, 256);
                            mma_i8(tmem + r * St::reg_cols + m * 64, ad, bd, idesc, 1u);
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
#pragma unroll 4
                for (int u = ut; u < kUnits; u += 32 * kRowsUnpackWarps) {
                    const int m = u / (kRowsKB * kRowsM), kb = (u / kRowsM) % kRowsKB, row = u % kRowsM;
                    const int src =
                        p.raw_rowmajor ? (m * kRowsM + row) * kRowsKB + kb : (m * kRowsKB + kb) * kRowsM + row;
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
        const int ew = warp - 2 - kRowsUnpackWarps;   // 0..7
        const int quarter = warp & 3, chunk = ew >> 2;
        const uint32_t tq = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        // preload every column of this warp's half of its lane quarter
        for (int c = chunk * 256; c < chunk * 256 + 256; c += 8) tmem_st8_magic(tq + c);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int r = 0; r < R; ++r) mbar_arrive(&tm_empty[r]);
        RowsSeq sq;
        for (int item = blockIdx.x; item < total; item += gridDim.x) {
            const int4 td = p.tiles[item / slabs];
            const int cw = ((td.z + 15) & ~15) / 2;
            bool ok;
            switch (cw) {
            case 8:
                ok = rows_epilogue_item<Down, Tap, 8>(p, smem, raw_full, raw_empty, tm_full, tm_empty, tq, sq, item, td,
                                                      lane, quarter, chunk);
                break;
            case 16:
                ok = rows_epilogue_item<Down, Tap, 16>(p, smem, raw_full, raw_empty, tm_full, tm_empty, tq, sq, item,
                                                       td, lane, quarter, chunk);
                break;
            case 24:
                ok = rows_epilogue_item<Down, Tap, 24>(p, smem, raw_full, raw_empty, tm_full, tm_empty, tq, sq, item,
                                                       td, lane, quarter, chunk);
                break;
            default:
                ok = rows_epilogue_item<Down, Tap, 32>(p, smem, raw_full, raw_empty, tm_full, tm_empty, tq, sq, item,
                                                       td, lane, quarter, chunk);
                break;
            }
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

// Gate/up B operand of every tile: row r < n of tile t is the Q8_1 codes of
// token pair_token[p0 + r] and its constants (d8, -8*s8); rows n..Np-1 are
// zero.  CTA (t, g): 64 threads (rows) x blocks 8g..8g+7.
__global__ void __launch_bounds__(kRowsNP) tc_rows_gather_kernel(const int4 *tiles, const int *num_tiles,
                                                                 const int32_t *pair_token, Q8Planar xq, int H,
                                                                 uint8_t *b_arr, float *bsc_arr) {
    const int nb = H / 32, row = threadIdx.x, b0 = blockIdx.y * 8;
    for (int t = blockIdx.x; t < *num_tiles; t += gridDim.x) {
        const int4 td = tiles[t];
        const int np = (td.z + 15) & ~15;
        if (row >= np) continue;
        uint4 v[16];
        float2 c[8];
        if (row < td.z) {
            const int token = pair_token[td.y + row];
            const uint4 *src = reinterpret_cast<const uint4 *>(xq.codes + static_cast<size_t>(token) * H) + 2 * b0;
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = src[i];
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = xq.scales[static_cast<size_t>(token) * nb + b0 + i];
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = make_float2(0.0f, 0.0f);
        }
        uint8_t *slot = b_arr + static_cast<size_t>(t) * rows_b_slot(H);
        float *ss = bsc_arr + static_cast<size_t>(t) * rows_sc_slot(H);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int b = b0 + i;
            uint8_t *dst = slot + static_cast<size_t>(b) * np * 32;
            *reinterpret_cast<uint4 *>(dst + tile_off(row, 0)) = v[2 * i];
            *reinterpret_cast<uint4 *>(dst + tile_off(row, 1)) = v[2 * i + 1];
            ss[b * 2 * np + row] = c[i].x;
            ss[b * 2 * np + np + row] = -(8.0f * c[i].y);
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
