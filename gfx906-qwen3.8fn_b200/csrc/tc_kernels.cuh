// tc_kernels.cuh -- tcgen05 (kind::i8) grouped GEMMs for large expert groups.
//
// One work item = (expert e, up to 128 consecutive pairs of e's group, one
// slab of 64 weight rows).  The MMA is D[128 pairs][64 rows] = A . B^T with
//   A = the pairs' Q8_1 activation codes (s8, gathered by pair -> token),
//   B = the slab's Q4_0 codes unpacked to centred s8 (q - 8),
// K = 32 per instruction = one quantisation block, so every MMA result is one
// per-block integer dot.  TMEM lanes are pairs and TMEM columns are weight
// rows: the per-pair block scales stay in registers and the per-row scale is
// one shared-memory broadcast.
//
// Exactness: with centred weights the MMA returns dot_c = sum (q-8)*x; the
// reference's uncentred dot is dot_c + 8*sum(x codes) (an integer identity),
// and d4*(dot*d8 - 8*s8) = d4*(dot_c*d8 + c8) with the per-(pair, block)
// constant c8 = 8*(sum(x codes)*d8 - s8) computed once by the quantiser.
// |dot_c| <= 32*8*127 < 2^15, so each result is read from TMEM as a 16-bit
// value (two columns per register) and turned into an exact fp32 by placing
// it, offset by 2^15, in the mantissa of 1.5*2^23 (two logic operations and
// one subtraction per pair of columns).
//
// Warp roles (12 warps, three per SM sub-partition):
//   warp 0      TMEM allocation, then one lane issues the MMAs, two blocks
//               per TMEM region (4 regions of 128 columns);
//   warps 1..3  producers: gather activation rows with cp.async, load and
//               unpack weight codes, stage per-block scales (software-
//               pipelined one stage ahead);
//   warps 4..11 epilogue: two per TMEM lane quarter, 32 columns each; per
//               region they load both blocks, release the region, and scale
//               and accumulate in fp32 registers with packed f32x2 arithmetic
//               while the next region's loads are in flight; at the end of an
//               item they run SiLU*up + Q8_1 requantisation (gate/up, split
//               over both threads of a pair row) or the router-weighted bulk
//               reduce-add into the residual (down).
// All barrier waits are bounded (ptx.cuh).
#pragma once
#include "common.cuh"
#include "expert_kernels.cuh"
#include "ptx.cuh"

namespace qmoe {

constexpr int kTcM = 128;          // pairs per tile (MMA M, TMEM lanes)
constexpr int kTcN = 64;           // weight rows per item (MMA N, TMEM columns per block)
constexpr int kTcKB = 4;           // quantisation blocks per pipeline stage
constexpr int kTcStages = 6;       // shared-memory ring depth
constexpr int kTcRegions = 4;      // TMEM regions of two block results (4 x 128 = 512 columns)
constexpr int kTcColumns = kTcRegions * 2 * kTcN;
constexpr int kTcProducerWarps = 3;
constexpr int kTcEpilogueWarps = 8;   // two per TMEM lane quarter, 32 columns each
constexpr int kTcWarps = 1 + kTcProducerWarps + kTcEpilogueWarps;
constexpr int kTcThreads = 32 * kTcWarps;
constexpr int kTcXchStride = 68;   // floats per exchange row (16-byte accesses by 8 lanes hit 32 banks)
constexpr int kTcMinGroup = 16;    // groups with at least this many pairs use the tensor-core path
constexpr float kTcUnbias = 12615680.0f;   // 1.5 * 2^23 + 2^15
static_assert(kTcWarps % 4 == 0, "whole warps per SM sub-partition keep the register budget");

// ---- PTX wrappers ------------------------------------------------------------
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
// 32 columns of this warp's lane quarter as 16-bit values, two adjacent columns
// per register (the lower column in the low half).
__device__ __forceinline__ void tmem_ld16p(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.pack::16b.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// Both blocks of a region: columns [0, 32) of block 0 and of block 1 (64 columns on).
__device__ __forceinline__ void tmem_ld_pair(uint32_t taddr, uint32_t (&r)[32]) {
    tmem_ld16p(taddr, r);
    tmem_ld16p(taddr + kTcN, r + 16);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Wait for outstanding TMEM loads, tying the destination registers to the wait
// so that no use of them is scheduled before it.
__device__ __forceinline__ void tmem_wait_ld32(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                   "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

__device__ __forceinline__ void cp_async16(void *dst_smem, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void *dst_smem, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_group1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Bulk reduce-add of `bytes` (multiple of 16) of fp32 from shared to global.
__device__ __forceinline__ void bulk_reduce_add_f32(float *dst, const float *src_smem, uint32_t bytes) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(dst),
                 "r"(smem_u32(src_smem)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core
// matrices, the two 16-byte K halves `lbo` bytes apart, successive 8-row
// groups `sbo` bytes apart.  Version 1 (Blackwell) in bits 46-47.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((addr >> 4) & 0x3fffu) | (static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}

// Instruction descriptor: kind::i8, A and B signed 8-bit, D s32, both K-major.
constexpr uint32_t tc_idesc(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

// Byte offset of (row, k-half) in a K-major no-swizzle tile: 8-row groups of
// 256 bytes, the two 16-byte K halves 128 bytes apart.
__device__ __forceinline__ uint32_t tile_off(int row, int half) {
    return static_cast<uint32_t>((row >> 3) * 256 + half * 128 + (row & 7) * 16);
}

// Unpack 16 Q4_0 code bytes to 32 centred signed bytes: low nibbles -> K 0..15,
// high nibbles -> K 16..31 (the element order of the block).
__device__ __forceinline__ void unpack_centred(const uint4 w, uint4 &lo, uint4 &hi) {
    // per byte: q + 120 stays in 120..135 (no carry between bytes); flipping
    // bit 7 subtracts 128, giving q - 8 in two's complement.
    auto c = [](uint32_t v) { return ((v & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u; };
    lo = make_uint4(c(w.x), c(w.y), c(w.z), c(w.w));
    hi = make_uint4(c(w.x >> 4), c(w.y >> 4), c(w.z >> 4), c(w.w >> 4));
}

// Two 16-bit two's-complement dots (low half first) -> the fp32 pair
// (kTcUnbias + v): the bit pattern 0x4b400000 + (v + 2^15) is the float
// 1.5*2^23 + 2^15 + v exactly for |v| < 2^15.
__device__ __forceinline__ uint64_t dot16x2(uint32_t r) {
    return pk2((r & 0xffffu) ^ 0x4b408000u, (r >> 16) ^ 0x4b408000u);
}

// Q8_1 of one 32-value block held as two halves of 16 by two threads, with
// the reference's rules (quant.cpp:275-325).  The maximum does not depend on
// order and the raw sum's pairwise tree (XOR butterfly 1,2,4,8,16) is
// (tree of values 0..15) + (tree of values 16..31), so the split block is
// identical to one quantised by a single thread.
struct Q8Half {
    float amax, sum;   // over this half, non-finite values taken as 0
    int bad;           // a value was non-finite
};
__device__ __forceinline__ Q8Half q8_half_stats(float (&x)[16]) {
    Q8Half q{0.0f, 0.0f, 0};
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        if (!isfinite(x[i])) { q.bad = 1; x[i] = 0.0f; }
        q.amax = fmaxf(q.amax, fabsf(x[i]));
        t[i] = x[i];
    }
#pragma unroll
    for (int m = 1; m < 16; m <<= 1)
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if ((i & (2 * m - 1)) == 0) t[i] = __fadd_rn(t[i], t[i + m]);
    q.sum = t[0];
    return q;
}
struct Q8Codes {
    uint16_t d, s;        // half scale and raw sum of the whole block
    int representable;    // the scale and the sum fit a half
    int bad_code;         // a code of this half fell outside [-127, 127]
    int csum;             // sum of this half's codes
};
// Codes of one half given the whole block's maximum, raw sum and non-finite flag.
__device__ __forceinline__ Q8Codes q8_half_codes(const float (&x)[16], float amax, float sum, int bad,
                                                 int8_t (&code)[16]) {
    Q8Codes q;
    const float d = __fdiv_rn(amax, 127.0f);
    q.d = f2h(d);
    q.s = f2h(sum);
    q.representable = isfinite(sum) && (q.s & 0x7c00u) != 0x7c00u && (q.d & 0x7c00u) != 0x7c00u &&
                      (amax == 0.0f || d > 0.0f);
    q.bad_code = 0;
    q.csum = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float c = (!bad && q.representable && amax != 0.0f) ? roundf(__fdiv_rn(x[i], d)) : 0.0f;
        const bool ok = isfinite(c) && c >= -127.0f && c <= 127.0f;
        q.bad_code |= ok ? 0 : 1;
        code[i] = static_cast<int8_t>(ok ? c : 0.0f);
        q.csum += code[i];
    }
    return q;
}

// ---- shared parameters ---------------------------------------------------------
struct TcParams {
    const uint8_t *weights;
    ExpertLayout layout;
    // A operand and its per-(row, block) constants (d8, c8), pre-arranged per
    // tile so that each stage is one contiguous run: block b of tile t at
    // a_arr + (t*nb + b)*4096 in the K-major core-matrix layout of TcStage::a,
    // constants at sc_arr + (t*nb + b)*128.
    const uint8_t *a_arr;
    const float2 *sc_arr;
    const int4 *tiles;          // {expert, first pair, count, 0}
    const int *num_tiles;
    const int32_t *pair_token;
    const float *pair_weight;
    uint8_t *mid_arr;           // gate/up output: the down kernel's a_arr
    float2 *mid_sc_arr;         // gate/up output: the down kernel's sc_arr
    float *out;                 // down output [T][H]
    int *error;
};

// Stage layout inside the ring.
struct TcStage {
    static constexpr uint32_t a = 0;                                   // kTcKB x [128 x 32] s8
    static constexpr uint32_t b = a + kTcKB * kTcM * 32;               // kTcKB x [64 x 32] s8
    static constexpr uint32_t d4 = b + kTcKB * kTcN * 32;              // [kTcKB][64] fp32 weight scales
    static constexpr uint32_t sc = d4 + kTcKB * kTcN * 4;              // [kTcKB][128] float2 (d8, c8)
    static constexpr uint32_t bytes = sc + kTcKB * kTcM * 8;
};
static_assert(TcStage::bytes % 128 == 0, "stage size keeps 128-byte alignment");

struct TcSmem {
    static constexpr uint32_t bars = 0;                                 // 4 barrier arrays of 8
    static constexpr uint32_t tmem_slot = 256;
    static constexpr uint32_t ring = 1024;
    static constexpr uint32_t xch = ring + kTcStages * TcStage::bytes;  // [128][68] fp32 rows
    static constexpr uint32_t part = xch + kTcM * kTcXchStride * 4;     // [128][2][4] half-block statistics
    static constexpr uint32_t bytes = part + kTcM * 2 * 4 * 4;
};
static_assert(TcSmem::bytes <= 227 * 1024, "fits the opt-in shared memory of one CTA");

// Persistent loop shared by both kernels.  `Down` selects the down projection
// (K = I, weight slabs of the down matrix, reduce-add epilogue) versus
// gate/up (K = H, 32 gate rows + 32 up rows, SiLU*up + Q8_1 epilogue).
template <bool Down>
__global__ void __launch_bounds__(kTcThreads, 1) tc_expert_kernel(TcParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int H = p.layout.hidden, I = p.layout.inter;
    const int K = Down ? I : H, nb = K / 32, ksteps = nb / kTcKB;
    const int slabs = Down ? H / kTcN : I / (kTcN / 2);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + TcSmem::bars);
    uint64_t *empty = full + 8;
    uint64_t *tm_full = empty + 8;
    uint64_t *tm_empty = tm_full + 8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + TcSmem::tmem_slot);
    uint8_t *ring = smem + TcSmem::ring;
    float *xch = reinterpret_cast<float *>(smem + TcSmem::xch);
    float *part = reinterpret_cast<float *>(smem + TcSmem::part);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full[s], kTcProducerWarps);
            mbar_init(&empty[s], 1 + kTcEpilogueWarps);
        }
        for (int r = 0; r < kTcRegions; ++r) {
            mbar_init(&tm_full[r], 1);
            mbar_init(&tm_empty[r], kTcEpilogueWarps);
        }
        mbar_fence_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kTcColumns);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int total = *p.num_tiles * slabs;
    bool failed = false;

    if (warp == 0) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = tc_idesc(kTcM, kTcN);
            int q = 0, kseq = 0;   // stage sequence, block sequence
            for (int item = blockIdx.x; item < total && !failed; item += gridDim.x) {
                for (int ks = 0; ks < ksteps && !failed; ++ks, ++q) {
                    const int s = q % kTcStages;
                    if (!mbar_wait(&full[s], (q / kTcStages) & 1, p.error)) { failed = true; break; }
                    tc_fence_after();
                    const uint32_t st = smem_u32(ring + s * TcStage::bytes);
                    for (int kb = 0; kb < kTcKB; ++kb, ++kseq) {
                        // blocks 2h and 2h+1 of the sequence share region h % kTcRegions
                        const int h = kseq >> 1, r = h % kTcRegions;
                        if ((kseq & 1) == 0) {
                            if (!mbar_wait(&tm_empty[r], (h / kTcRegions) & 1, p.error)) { failed = true; break; }
                            tc_fence_after();
                        }
                        const uint64_t ad = smem_desc(st + TcStage::a + kb * kTcM * 32, 128, 256);
                        const uint64_t bd = smem_desc(st + TcStage::b + kb * kTcN * 32, 128, 256);
                        mma_i8(tmem + (2 * r + (kseq & 1)) * kTcN, ad, bd, idesc, 0u);
                        if (kseq & 1) mma_commit(&tm_full[r]);
                    }
                    mma_commit(&empty[s]);   // stage s may be refilled once these MMAs are done
                }
            }
        }
    } else if (warp <= kTcProducerWarps) {
        // ---------------- producers ----------------
        // A and its block constants are one contiguous 16 KB + 4 KB run per stage
        // in the pre-arranged buffers: one thread issues them as bulk copies
        // counted on the stage's full barrier.  The producer warps load (one
        // stage ahead, into registers), unpack and store the weight codes.
        constexpr int kProducerThreads = 32 * kTcProducerWarps;
        constexpr int kBPer = (kTcN * kTcKB + kProducerThreads - 1) / kProducerThreads;
        const int pt = threadIdx.x - 32;
        const int my_items = static_cast<int>(blockIdx.x) < total ? (total - 1 - blockIdx.x) / gridDim.x + 1 : 0;
        const int nstages = my_items * ksteps;
        int4 td_next = make_int4(0, 0, 0, 0);
        uint4 wn[kBPer];
        uint16_t dn[kBPer];
        // global loads of stage g's weight codes and scales into wn/dn
        auto prefetch = [&](int g) {
            const int item = blockIdx.x + (g / ksteps) * gridDim.x, ks = g % ksteps;
            if (ks == 0) td_next = p.tiles[item / slabs];
            const int slab = item % slabs;
            const uint8_t *ex = p.weights + static_cast<size_t>(td_next.x) * p.layout.bytes;
#pragma unroll
            for (int j = 0; j < kBPer; ++j) {
                const int idx = pt + j * kProducerThreads;
                if (idx < kTcN * kTcKB) {
                    const int col = idx & (kTcN - 1), kb = idx / kTcN;
                    size_t code_off, sc_off;
                    int row;
                    if (Down) {
                        row = slab * kTcN + col;
                        code_off = p.layout.down_codes;
                        sc_off = p.layout.down_scales;
                    } else {
                        row = slab * (kTcN / 2) + (col & 31);
                        code_off = col < 32 ? p.layout.gate_codes : p.layout.up_codes;
                        sc_off = col < 32 ? p.layout.gate_scales : p.layout.up_scales;
                    }
                    const size_t blk = static_cast<size_t>(row) * nb + ks * kTcKB + kb;
                    wn[j] = __ldg(reinterpret_cast<const uint4 *>(ex + code_off) + blk);
                    dn[j] = __ldg(reinterpret_cast<const uint16_t *>(ex + sc_off) + blk);
                }
            }
        };
        if (nstages > 0) prefetch(0);
        for (int g = 0; g < nstages; ++g) {
            const int ks = g % ksteps, s = g % kTcStages;
            const int tile = (blockIdx.x + (g / ksteps) * gridDim.x) / slabs;
            uint4 wc[kBPer];
            uint16_t dc[kBPer];
#pragma unroll
            for (int j = 0; j < kBPer; ++j) {
                wc[j] = wn[j];
                dc[j] = dn[j];
            }
            if (g + 1 < nstages) prefetch(g + 1);
            if (g >= kTcStages && !mbar_wait(&empty[s], ((g / kTcStages) & 1) ^ 1, p.error)) { failed = true; break; }
            uint8_t *st = ring + s * TcStage::bytes;
            if (pt == 0) {
                const size_t blk0 = static_cast<size_t>(tile) * nb + static_cast<size_t>(ks) * kTcKB;
                mbar_expect_tx(&full[s], kTcKB * kTcM * 32 + kTcKB * kTcM * 8);
                bulk_g2s(st + TcStage::a, p.a_arr + blk0 * (kTcM * 32), kTcKB * kTcM * 32, &full[s]);
                bulk_g2s(st + TcStage::sc, p.sc_arr + blk0 * kTcM, kTcKB * kTcM * 8, &full[s]);
            }
            // B: 64 weight rows x kTcKB blocks of codes, unpacked to centred s8
#pragma unroll
            for (int j = 0; j < kBPer; ++j) {
                const int idx = pt + j * kProducerThreads;
                if (idx < kTcN * kTcKB) {
                    const int col = idx & (kTcN - 1), kb = idx / kTcN;
                    uint4 lo, hi;
                    unpack_centred(wc[j], lo, hi);
                    *reinterpret_cast<uint4 *>(st + TcStage::b + kb * kTcN * 32 + tile_off(col, 0)) = lo;
                    *reinterpret_cast<uint4 *>(st + TcStage::b + kb * kTcN * 32 + tile_off(col, 1)) = hi;
                    reinterpret_cast<float *>(st + TcStage::d4)[kb * kTcN + col] = h2f(dc[j]);
                }
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
        }
    } else {
        // ---------------- epilogue ----------------
        const int ew = warp - 1 - kTcProducerWarps;        // 0..7
        const int quarter = warp & 3;                      // TMEM lane quarter this warp may access
        const int chunk = ew >> 2;                         // 32-column chunk 0..1
        const int m = quarter * 32 + lane;                 // pair row of this thread
        const uint32_t tq = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + chunk * 32;
        float *xrow = xch + m * kTcXchStride;
        float *mine = part + (m * 2 + chunk) * 4;
        const float *other = part + (m * 2 + (chunk ^ 1)) * 4;
        if (lane == 0)
            for (int r = 0; r < kTcRegions; ++r) mbar_arrive(&tm_empty[r]);   // every region starts free
        const uint64_t unbias = pkf2(-kTcUnbias, -kTcUnbias);
        int q0 = 0, h0 = 0;   // stage and block-pair sequence numbers at the start of the item
        for (int item = blockIdx.x; item < total; item += gridDim.x, q0 += ksteps, h0 += nb / 2) {
            const int4 td = p.tiles[item / slabs];
            const int p0 = td.y, n = td.z, slab = item % slabs;
            const bool live = quarter * 32 < n;   // this warp's lanes hold at least one real pair
            uint64_t acc[16];                      // 32 fp32 accumulators as packed pairs
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = 0ull;
            // Issue the TMEM loads of block pair h (once the MMA has committed it).
            auto fetch = [&](int h, uint32_t(&v)[32]) -> bool {
                const int hh = h0 + h, r = hh % kTcRegions;
                if (!mbar_wait(&tm_full[r], (hh / kTcRegions) & 1, p.error)) return false;
                tc_fence_after();
                if (live) tmem_ld_pair(tq + r * 2 * kTcN, v);
                return true;
            };
            // Block pair h: its loads (issued one pair earlier) land and the region
            // is released at once; the next pair's loads are issued and run while
            // this pair is scaled and accumulated.
            auto step = [&](int h, uint32_t(&cur)[32], uint32_t(&nxt)[32]) -> bool {
                const int hh = h0 + h, r = hh % kTcRegions;
                const int q = q0 + (2 * h) / kTcKB, s = q % kTcStages, kb = (2 * h) % kTcKB;
                tmem_wait_ld32(cur);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tm_empty[r]);
                if (h + 1 < nb / 2 && !fetch(h + 1, nxt)) return false;
                const uint8_t *st = ring + s * TcStage::bytes;
                // Acquire the producers' writes of this stage's scales directly.  The
                // phase cannot have moved on: refilling needs this warp's release below.
                if (kb == 0 && !mbar_wait(&full[s], (q / kTcStages) & 1, p.error)) return false;
                if (live) {
#pragma unroll
                    for (int b = 0; b < 2; ++b) {
                        const float2 sc = reinterpret_cast<const float2 *>(st + TcStage::sc)[(kb + b) * kTcM + m];
                        const uint64_t d8 = pkf2(sc.x, sc.x), c8 = pkf2(sc.y, sc.y);
                        const ulonglong2 *d4v = reinterpret_cast<const ulonglong2 *>(
                            st + TcStage::d4 + ((kb + b) * kTcN + chunk * 32) * 4);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const ulonglong2 dd = d4v[j];   // weight scales of 4 columns (broadcast)
                            // exact dot_c of 2 columns, then acc += d4 * (dot_c * d8 + c8)
                            const uint64_t t0 = add2(dot16x2(cur[b * 16 + 2 * j]), unbias);
                            const uint64_t t1 = add2(dot16x2(cur[b * 16 + 2 * j + 1]), unbias);
                            acc[2 * j] = fma2(dd.x, fma2(t0, d8, c8), acc[2 * j]);
                            acc[2 * j + 1] = fma2(dd.y, fma2(t1, d8, c8), acc[2 * j + 1]);
                        }
                    }
                }
                if (kb + 2 == kTcKB) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[s]);   // done with the stage's scales
                }
                return true;
            };
            uint32_t va[32], vb[32];
            bool ok = fetch(0, va);
            for (int h = 0; h < nb / 2 && ok; h += 2) ok = step(h, va, vb) && step(h + 1, vb, va);
            if (!ok) tmem_wait_ld();
            if (!Down) {
                // Gate (chunk 0) and up (chunk 1) accumulators meet in row m of the
                // exchange; thread (m, chunk) then produces middle values
                // chunk*16 .. chunk*16+15 of the slab's Q8_1 block.  The first
                // barrier also tells every epilogue warp whether one gave up.
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float a0, a1, a2, a3;
                    upk2(acc[2 * j], a0, a1);
                    upk2(acc[2 * j + 1], a2, a3);
                    *reinterpret_cast<float4 *>(xrow + chunk * 32 + 4 * j) = make_float4(a0, a1, a2, a3);
                }
                if (named_barrier_or(2, 32 * kTcEpilogueWarps, !ok)) { failed = true; break; }
                const bool real = m < n;
                float mid[16];
                int flags = 0;
#pragma unroll
                for (int c = 0; c < 16; c += 4) {
                    const float4 g4 = *reinterpret_cast<const float4 *>(xrow + chunk * 16 + c);
                    const float4 u4 = *reinterpret_cast<const float4 *>(xrow + 32 + chunk * 16 + c);
                    const float gs[4] = {g4.x, g4.y, g4.z, g4.w}, us[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        int f = 0;
                        const float g = operand(gs[k], f), u = operand(us[k], f);
                        // fast exponential and division: a few ulp from the decode kernels'
                        // expf/IEEE form, far inside the layer tolerance
                        const float act = arithmetic(__fdividef(g, 1.0f + __expf(-g)), f);
                        const float val = arithmetic(__fmul_rn(act, u), f);
                        mid[c + k] = (f || !real) ? 0.0f : val;
                        flags |= real ? f : 0;
                    }
                }
                const Q8Half hq = q8_half_stats(mid);
                mine[0] = __int_as_float(__float_as_int(hq.amax) | (hq.bad << 31));   // sign bit: non-finite seen
                mine[1] = hq.sum;
                named_barrier(2, 32 * kTcEpilogueWarps);
                const float oa = other[0], os = other[1];
                const int bad = hq.bad | (__float_as_int(oa) < 0 ? 1 : 0);
                const float amax = fmaxf(hq.amax, fabsf(oa));
                const float sum = chunk == 0 ? __fadd_rn(hq.sum, os) : __fadd_rn(os, hq.sum);
                int8_t code[16];
                const Q8Codes qc = q8_half_codes(mid, amax, sum, bad, code);
                reinterpret_cast<int *>(mine)[2] = qc.csum;
                reinterpret_cast<int *>(mine)[3] = qc.bad_code;
                named_barrier(2, 32 * kTcEpilogueWarps);
                const int bad_code = qc.bad_code | reinterpret_cast<const int *>(other)[3];
                const bool valid = !bad && qc.representable && !bad_code;
                if (real) {
                    // middle block `slab` of this tile in the down kernel's A layout
                    const size_t mblk = static_cast<size_t>(item / slabs) * (I / 32) + slab;
                    int4 cv = *reinterpret_cast<const int4 *>(code);
                    if (!valid) cv = make_int4(0, 0, 0, 0);
                    *reinterpret_cast<int4 *>(p.mid_arr + mblk * (kTcM * 32) + tile_off(m, chunk)) = cv;
                    if (chunk == 0) {
                        const uint16_t hd = (valid && amax != 0.0f) ? qc.d : uint16_t(0);
                        const uint16_t hs = (valid && amax != 0.0f) ? qc.s : uint16_t(0);
                        const int csum = valid ? qc.csum + reinterpret_cast<const int *>(other)[2] : 0;
                        p.mid_sc_arr[mblk * kTcM + m] =
                            make_float2(h2f(hd), 8.0f * (static_cast<float>(csum) * h2f(hd) - h2f(hs)));
                    }
                    report(flags | (bad ? kFlagInvalid : 0) | ((qc.representable && !bad_code) ? 0 : kFlagArithmetic),
                           p.error);
                }
                // Row m's exchange words are read only by the two threads of row
                // m before the second barrier and its statistics only after the
                // third, so the next item may rewrite them without another barrier.
            } else {
                if (!ok) { failed = true; break; }
                // The thread's 32 columns become router-weighted contributions in
                // its own part of row m and are reduce-added by the bulk engine;
                // the part is rewritten only after the engine has read it.
                if (m < n) {
                    const float w = p.pair_weight[p0 + m];
                    int flags = 0;
                    bulk_wait_read0();
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        float y[4];
                        upk2(acc[2 * j], y[0], y[1]);
                        upk2(acc[2 * j + 1], y[2], y[3]);
#pragma unroll
                        for (int k = 0; k < 4; ++k) y[k] = arithmetic(__fmul_rn(w, arithmetic(y[k], flags)), flags);
                        *reinterpret_cast<float4 *>(xrow + chunk * 32 + 4 * j) = make_float4(y[0], y[1], y[2], y[3]);
                    }
                    fence_proxy_async();
                    bulk_reduce_add_f32(
                        p.out + static_cast<size_t>(p.pair_token[p0 + m]) * H + slab * kTcN + chunk * 32,
                        xrow + chunk * 32, 32 * 4);
                    bulk_commit();
                    report(flags, p.error);
                }
            }
        }
        if (Down) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");   // reduce-adds fully done
    }
    // teardown: every role is done with TMEM before warp 0 frees it
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTcColumns);
    }
}

struct TcWorkspace {
    float2 *x_tc;       // (d8, c8) of the quantised input [T][H/32]
    int4 *tiles;        // tensor-core tile list
    int *num_tiles;
    int max_tiles;
    // pre-arranged A operands (see TcParams): gate/up from x, down from the
    // gate/up epilogue; null when the workspace never runs the tensor-core path
    uint8_t *a_gu, *a_dn;
    float2 *sc_gu, *sc_dn;
};

template <class ArenaT>
inline void tc_workspace_take(TcWorkspace &w, ArenaT &a, int T, int H, int I, bool tc_used) {
    const int pairs = T * (kTopK + 1);
    w.x_tc = a.template take<float2>(static_cast<size_t>(T) * (H / 32));
    w.max_tiles = (pairs + kTcM - 1) / kTcM + kRouterExperts + 1;
    w.tiles = a.template take<int4>(w.max_tiles);
    w.num_tiles = a.template take<int>(1);
    w.a_gu = w.a_dn = nullptr;
    w.sc_gu = w.sc_dn = nullptr;
    if (tc_used) {
        const size_t bg = static_cast<size_t>(w.max_tiles) * (H / 32), bd = static_cast<size_t>(w.max_tiles) * (I / 32);
        w.a_gu = a.template take<uint8_t>(bg * kTcM * 32);
        w.sc_gu = a.template take<float2>(bg * kTcM);
        w.a_dn = a.template take<uint8_t>(bd * kTcM * 32);
        w.sc_dn = a.template take<float2>(bd * kTcM);
    }
}

// Gate/up A operand of every tensor-core tile: row r of tile t is the Q8_1
// codes (and constants) of token pair_token[p0 + r], written block by block
// into the arranged layout.  CTA (t, g): 128 threads (rows) x blocks 8g..8g+7.
__global__ void __launch_bounds__(kTcM) tc_gather_kernel(const int4 *tiles, const int *num_tiles,
                                                         const int32_t *pair_token, const int8_t *xcodes,
                                                         const float2 *xtc, int H, uint8_t *a_arr, float2 *sc_arr) {
    const int nb = H / 32, row = threadIdx.x, b0 = blockIdx.y * 8;
    for (int t = blockIdx.x; t < *num_tiles; t += gridDim.x) {
        const int4 td = tiles[t];
        if (row >= td.z) continue;
        const int token = pair_token[td.y + row];
        const uint4 *src = reinterpret_cast<const uint4 *>(xcodes + static_cast<size_t>(token) * H) + 2 * b0;
        const float2 *ssrc = xtc + static_cast<size_t>(token) * nb + b0;
        uint4 v[16];
        float2 c[8];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = src[i];
#pragma unroll
        for (int i = 0; i < 8; ++i) c[i] = ssrc[i];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const size_t blk = static_cast<size_t>(t) * nb + b0 + i;
            uint8_t *dst = a_arr + blk * (kTcM * 32);
            *reinterpret_cast<uint4 *>(dst + tile_off(row, 0)) = v[2 * i];
            *reinterpret_cast<uint4 *>(dst + tile_off(row, 1)) = v[2 * i + 1];
            sc_arr[blk * kTcM + row] = c[i];
        }
    }
}

inline int tc_configure() {
    if (cudaFuncSetAttribute(tc_expert_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(TcSmem::bytes)) != cudaSuccess ||
        cudaFuncSetAttribute(tc_expert_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(TcSmem::bytes)) != cudaSuccess)
        return MOE_CUDA_ERROR;
    return MOE_OK;
}

}  // namespace qmoe
