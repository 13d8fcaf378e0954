// tc_kernels.cuh -- tcgen05 (kind::i8) grouped GEMMs for large expert groups.
//
// One work item = (expert e, up to 128 consecutive pairs of e's group, one
// slab of 64 weight rows).  The MMA is D[128 pairs][64 rows] += A . B^T with
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
// Each block's TMEM columns are pre-loaded with the bit pattern of 1.5*2^23,
// so after the integer MMA accumulates dot_c (|dot_c| <= 32*8*127 < 2^22) the
// column holds the float 1.5*2^23 + dot_c exactly: the epilogue subtracts the
// constant (exact) instead of converting int -> float.
//
// Warp roles (21 warps):
//   warp 0      TMEM allocation, then one lane issues the MMAs;
//   warps 1..4  producers: gather activation rows with cp.async, load and
//               unpack weight codes, stage per-block scales;
//   warps 5..20 epilogue: four per TMEM lane quarter, 16 columns each; they
//               read each block's result, re-bias its TMEM columns, scale and
//               accumulate in fp32 registers; at the end of an item they run
//               SiLU*up + Q8_1 requantisation (gate/up) or the router-weighted
//               bulk reduce-add into the residual (down).
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
constexpr int kTcRegions = 8;      // TMEM block-result regions (8 x 64 = 512 columns)
constexpr int kTcProducerWarps = 4;
constexpr int kTcEpilogueWarps = 16;
constexpr int kTcWarps = 1 + kTcProducerWarps + kTcEpilogueWarps;
constexpr int kTcThreads = 32 * kTcWarps;
constexpr int kTcMinGroup = 16;    // groups with at least this many pairs use the tensor-core path
constexpr uint32_t kTcBias = 0x4b400000u;   // bit pattern of 1.5 * 2^23

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
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16_const(uint32_t taddr, uint32_t v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
        "r"(v)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(void *dst_smem, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
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

// Quantise 32 values held by one thread with the reference's rules
// (quant.cpp:275-325): the raw sum uses the same pairwise tree as the XOR
// butterfly 1,2,4,8,16.
struct Q8Block {
    uint16_t d, s;
    int flags;
    float c8;          // 8 * (sum(codes) * d - s) with the stored half values
};
__device__ __forceinline__ Q8Block quantize_thread32(float (&x)[32], int8_t (&code)[32]) {
    int bad = 0;
    float amax = 0.0f;
    float t[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        if (!isfinite(x[i])) { bad = 1; x[i] = 0.0f; }
        amax = fmaxf(amax, fabsf(x[i]));
        t[i] = x[i];
    }
#pragma unroll
    for (int m = 1; m < 32; m <<= 1)
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if ((i & m) == 0 && (i & (2 * m - 1)) == 0) t[i] = __fadd_rn(t[i], t[i + m]);
    const float sum = t[0];
    const float d = __fdiv_rn(amax, 127.0f);
    const uint16_t hd = f2h(d), hs = f2h(sum);
    const bool representable = isfinite(sum) && (hs & 0x7c00u) != 0x7c00u && (hd & 0x7c00u) != 0x7c00u &&
                               (amax == 0.0f || d > 0.0f);
    int bad_code = 0, csum = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float c = (!bad && representable && amax != 0.0f) ? roundf(__fdiv_rn(x[i], d)) : 0.0f;
        if (!isfinite(c) || c < -127.0f || c > 127.0f) bad_code = 1;
        code[i] = static_cast<int8_t>(isfinite(c) && c >= -127.0f && c <= 127.0f ? c : 0.0f);
    }
    const bool valid = !bad && representable && !bad_code;
    Q8Block q;
    q.d = (valid && amax != 0.0f) ? hd : uint16_t(0);
    q.s = (valid && amax != 0.0f) ? hs : uint16_t(0);
    q.flags = (bad ? kFlagInvalid : 0) | ((representable && !bad_code) ? 0 : kFlagArithmetic);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        if (!valid) code[i] = 0;
        csum += code[i];
    }
    q.c8 = 8.0f * (static_cast<float>(csum) * h2f(q.d) - h2f(q.s));
    return q;
}

// ---- shared parameters ---------------------------------------------------------
struct TcParams {
    const uint8_t *weights;
    ExpertLayout layout;
    const int8_t *act;          // gate/up: x codes [T][H];  down: middle codes [pairs][I]
    const float2 *act_tc;       // per (row of act, block): (d8, c8)
    int act_by_token;           // 1: A row = pair_token[pair] (gate/up), 0: A row = pair (down)
    const int4 *tiles;          // {expert, first pair, count, 0}
    const int *num_tiles;
    const int32_t *pair_token;
    const float *pair_weight;
    Q8Planar mid;               // gate/up output
    float2 *mid_tc;             // gate/up output (d8, c8) per (pair, block)
    float *out;                 // down output [T][H]
    int *error;
};

// Stage layout inside the ring.
struct TcStage {
    static constexpr uint32_t a = 0;                                   // kTcKB x [128 x 32] s8
    static constexpr uint32_t b = a + kTcKB * kTcM * 32;               // kTcKB x [64 x 32] s8
    static constexpr uint32_t d4 = b + kTcKB * kTcN * 32;              // [kTcKB][64] half
    static constexpr uint32_t sc = d4 + kTcKB * kTcN * 2;              // [128][kTcKB] float2
    static constexpr uint32_t bytes = sc + kTcM * kTcKB * 8;
};
static_assert(TcStage::bytes % 128 == 0, "stage size keeps 128-byte alignment");

struct TcSmem {
    static constexpr uint32_t bars = 0;                                 // 4 barrier arrays of 8
    static constexpr uint32_t tmem_slot = 256;
    static constexpr uint32_t ring = 1024;
    static constexpr uint32_t xch = ring + kTcStages * TcStage::bytes;  // [128][64] fp32 exchange
    static constexpr uint32_t bytes = xch + kTcM * kTcN * 4;
};

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
        tmem_alloc(tmem_slot, kTcRegions * kTcN);
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
                        const int r = kseq % kTcRegions;
                        if (!mbar_wait(&tm_empty[r], (kseq / kTcRegions) & 1, p.error)) { failed = true; break; }
                        tc_fence_after();
                        const uint64_t ad = smem_desc(st + TcStage::a + kb * kTcM * 32, 128, 256);
                        const uint64_t bd = smem_desc(st + TcStage::b + kb * kTcN * 32, 128, 256);
                        mma_i8(tmem + r * kTcN, ad, bd, idesc, 1u);
                        mma_commit(&tm_full[r]);
                    }
                    mma_commit(&empty[s]);   // stage s may be refilled once these MMAs are done
                }
            }
        }
    } else if (warp <= kTcProducerWarps) {
        // ---------------- producers ----------------
        const int pt = threadIdx.x - 32;   // 0..127: one pair row of A each
        int q = 0;
        for (int item = blockIdx.x; item < total && !failed; item += gridDim.x) {
            const int4 td = p.tiles[item / slabs];
            const int e = td.x, p0 = td.y, n = td.z, slab = item % slabs;
            const uint8_t *ex = p.weights + static_cast<size_t>(e) * p.layout.bytes;
            const int arow = pt < n ? (p.act_by_token ? p.pair_token[p0 + pt] : p0 + pt) : -1;
            for (int ks = 0; ks < ksteps; ++ks, ++q) {
                const int s = q % kTcStages;
                if (q >= kTcStages && !mbar_wait(&empty[s], ((q / kTcStages) & 1) ^ 1, p.error)) { failed = true; break; }
                uint8_t *st = ring + s * TcStage::bytes;
                const int b0 = ks * kTcKB;
                // A: this thread's pair row, kTcKB blocks x 2 halves, plus its block scales
                if (arow >= 0) {
                    const int8_t *src = p.act + static_cast<size_t>(arow) * K + b0 * 32;
#pragma unroll
                    for (int kb = 0; kb < kTcKB; ++kb)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            cp_async16(st + TcStage::a + kb * kTcM * 32 + tile_off(pt, h), src + kb * 32 + h * 16);
                    const float2 *ss = p.act_tc + static_cast<size_t>(arow) * nb + b0;
                    cp_async16(st + TcStage::sc + pt * kTcKB * 8, ss);
                    cp_async16(st + TcStage::sc + pt * kTcKB * 8 + 16, ss + 2);
                }
                // B: 64 weight rows x kTcKB blocks of codes, unpacked; two (row, block) per thread
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int idx = pt + u * 128;          // 0..255
                    const int col = idx & 63, kb = idx >> 6;
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
                    const size_t blk = static_cast<size_t>(row) * nb + b0 + kb;
                    const uint4 w = __ldg(reinterpret_cast<const uint4 *>(ex + code_off) + blk);
                    uint4 lo, hi;
                    unpack_centred(w, lo, hi);
                    *reinterpret_cast<uint4 *>(st + TcStage::b + kb * kTcN * 32 + tile_off(col, 0)) = lo;
                    *reinterpret_cast<uint4 *>(st + TcStage::b + kb * kTcN * 32 + tile_off(col, 1)) = hi;
                    reinterpret_cast<uint16_t *>(st + TcStage::d4)[kb * kTcN + col] =
                        __ldg(reinterpret_cast<const uint16_t *>(ex + sc_off) + blk);
                }
                cp_async_wait_all();
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int ew = warp - 1 - kTcProducerWarps;        // 0..15
        const int quarter = warp & 3;                      // TMEM lane quarter this warp may access
        const int chunk = ew >> 2;                         // 16-column chunk 0..3
        const int m = quarter * 32 + lane;                 // pair row of this thread
        const uint32_t tq = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + chunk * 16;
        // initial bias of every region, then release all regions once
        for (int r = 0; r < kTcRegions; ++r) tmem_st16_const(tq + r * kTcN, kTcBias);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int r = 0; r < kTcRegions; ++r) mbar_arrive(&tm_empty[r]);
        int q = 0, kseq = 0, it = 0;
        for (int item = blockIdx.x; item < total && !failed; item += gridDim.x, ++it) {
            const int4 td = p.tiles[item / slabs];
            const int p0 = td.y, n = td.z, slab = item % slabs;
            float acc[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
            for (int ks = 0; ks < ksteps && !failed; ++ks, ++q) {
                const int s = q % kTcStages;
                const uint8_t *st = ring + s * TcStage::bytes;
                // Acquire the producers' writes of this stage's scales directly.  The
                // phase cannot have moved on: refilling needs this warp's release below.
                if (!mbar_wait(&full[s], (q / kTcStages) & 1, p.error)) { failed = true; break; }
                for (int kb = 0; kb < kTcKB; ++kb, ++kseq) {
                    const int r = kseq % kTcRegions;
                    if (!mbar_wait(&tm_full[r], (kseq / kTcRegions) & 1, p.error)) { failed = true; break; }
                    tc_fence_after();
                    uint32_t v[16];
                    tmem_ld16(tq + r * kTcN, v);
                    tmem_wait_ld();
                    tmem_st16_const(tq + r * kTcN, kTcBias);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tm_empty[r]);
                    const float2 sc = reinterpret_cast<const float2 *>(st + TcStage::sc)[m * kTcKB + kb];
                    const uint4 *d4v = reinterpret_cast<const uint4 *>(st + TcStage::d4 + (kb * kTcN + chunk * 16) * 2);
                    const uint4 dA = d4v[0], dB = d4v[1];
                    const uint32_t dw[8] = {dA.x, dA.y, dA.z, dA.w, dB.x, dB.y, dB.z, dB.w};
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float d4 = h2f(static_cast<uint16_t>(dw[j >> 1] >> (16 * (j & 1))));
                        const float t = __int_as_float(v[j]) - 12582912.0f;   // exact: the centred dot
                        acc[j] = fmaf(d4, fmaf(t, sc.x, sc.y), acc[j]);
                    }
                }
                if (failed) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);   // this warp is done with the stage's scales
            }
            if (failed) break;
            // ---- item epilogue: exchange accumulators through shared memory ----
#pragma unroll
            for (int j = 0; j < 16; ++j) xch[m * kTcN + chunk * 16 + j] = acc[j];
            named_barrier(2, 32 * kTcEpilogueWarps);
            if (!Down) {
                if (chunk == 0 && m < n) {
                    float mid[32];
                    int flags = 0;
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        int f = 0;
                        const float g = operand(xch[m * kTcN + c], f), u = operand(xch[m * kTcN + 32 + c], f);
                        const float act = arithmetic(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), f);
                        const float val = arithmetic(__fmul_rn(act, u), f);
                        mid[c] = f ? 0.0f : val;
                        flags |= f;
                    }
                    int8_t code[32];
                    const Q8Block qb = quantize_thread32(mid, code);
                    const size_t pair = static_cast<size_t>(p0 + m);
                    int4 *dst = reinterpret_cast<int4 *>(p.mid.codes + pair * I + slab * 32);
                    const int4 *srcv = reinterpret_cast<const int4 *>(code);
                    dst[0] = srcv[0];
                    dst[1] = srcv[1];
                    const int mslabs = I / 32;
                    p.mid.scales[pair * mslabs + slab] = make_float2(h2f(qb.d), h2f(qb.s));
                    p.mid_tc[pair * mslabs + slab] = make_float2(h2f(qb.d), qb.c8);
                    report(flags | qb.flags, p.error);
                }
            } else {
                if (chunk == 0 && m < n) {
                    const float w = p.pair_weight[p0 + m];
                    int flags = 0;
#pragma unroll
                    for (int c = 0; c < kTcN; ++c) {
                        const float y = arithmetic(xch[m * kTcN + c], flags);
                        xch[m * kTcN + c] = arithmetic(__fmul_rn(w, y), flags);
                    }
                    fence_proxy_async();
                    bulk_reduce_add_f32(p.out + static_cast<size_t>(p.pair_token[p0 + m]) * H + slab * kTcN,
                                        xch + m * kTcN, kTcN * 4);
                    bulk_commit();
                    bulk_wait_read0();
                    report(flags, p.error);
                }
            }
            named_barrier(2, 32 * kTcEpilogueWarps);   // xch free for the next item
        }
        if (Down) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");   // reduce-adds fully done
    }
    // teardown: every role is done with TMEM before warp 0 frees it
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTcRegions * kTcN);
    }
}

struct TcWorkspace {
    float2 *x_tc;       // (d8, c8) of the quantised input [T][H/32]
    float2 *mid_tc;     // (d8, c8) of the middle [pairs][I/32]
    int4 *tiles;        // tensor-core tile list
    int *num_tiles;
    int max_tiles;
};

template <class ArenaT>
inline void tc_workspace_take(TcWorkspace &w, ArenaT &a, int T, int H, int I) {
    const int pairs = T * (kTopK + 1);
    w.x_tc = a.template take<float2>(static_cast<size_t>(T) * (H / 32));
    w.mid_tc = a.template take<float2>(static_cast<size_t>(pairs) * (I / 32));
    w.max_tiles = (pairs + kTcM - 1) / kTcM + kRouterExperts + 1;
    w.tiles = a.template take<int4>(w.max_tiles);
    w.num_tiles = a.template take<int>(1);
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
