// expert_kernels.cuh -- Q8_1 quantisation and the weight-streaming grouped
// expert kernels (decode-size groups), plus the synthetic generator and
// layout repacks.
//
// Weight layout (one expert, planar; same byte count as the canonical blocks):
//   gate codes [I][H/32][16] | up codes [I][H/32][16] | down codes [H][I/32][16]
//   | gate scales [I][H/32] half | up scales | down scales [H][I/32] half
//   [| down minima [H][I/32] half, when the down matrix is Q4_1]
// Block (r, b) of a matrix is canonical block r*(K/32)+b: its 16 code bytes
// and its half scale (and minimum), split so code rows load as aligned
// 16-byte vectors (the reference's optional planar layout,
// src/hip/expert.hip:147-159).  Gate and up are Q4_0; down is Q4_0 or Q4_1
// (the reference's layers 0-5 carry Q4_1 down matrices,
// src/memory_main.hip:41-42).
#pragma once
#include "common.cuh"

namespace qmoe {

constexpr int kDownQ4_0 = 0;
constexpr int kDownQ4_1 = 1;

struct ExpertLayout {
    size_t gate_codes, up_codes, down_codes, gate_scales, up_scales, down_scales, down_mins, bytes;
    int hidden, inter;
    int down_type;   // kDownQ4_0 or kDownQ4_1
};

inline ExpertLayout make_layout(int H, int I, int down_type = kDownQ4_0) {
    ExpertLayout L;
    const size_t codes = static_cast<size_t>(H) * I / 2, scales = static_cast<size_t>(H) * I / 16;
    L.gate_codes = 0;
    L.up_codes = codes;
    L.down_codes = 2 * codes;
    L.gate_scales = 3 * codes;
    L.up_scales = 3 * codes + scales;
    L.down_scales = 3 * codes + 2 * scales;
    L.down_mins = 3 * codes + 3 * scales;
    L.bytes = 3 * codes + 3 * scales + (down_type == kDownQ4_1 ? scales : 0);
    L.hidden = H;
    L.inter = I;
    L.down_type = down_type;
    return L;
}

// One Q4_1 block's contribution with the reference's contract
// (src/quant.cpp:88-102, src/cpu_expert.cpp:194-205): the products d4*d8 and
// m4*s8 (exact in fp32 for half operands) are rounded to half (RNE), then
// acc + fma(dot, half(d4*d8), half(m4*s8)) -- inner FMA, separate add.
__device__ __forceinline__ float block_term_q4_1(int dot, float d4, float m4, float d8, float s8, float acc) {
    const float dd = __half2float(__float2half_rn(__fmul_rn(d4, d8)));
    const float ms = __half2float(__float2half_rn(__fmul_rn(m4, s8)));
    return __fadd_rn(acc, fmaf(small_int_to_float(dot), dd, ms));
}

// ---------------------------------------------------------------------------
// fp32 [rows][K] -> Q8_1.  One warp per 32-value block, lane = element.
// Writes the planar form (codes/scales) and/or canonical 36-byte blocks.
__global__ void __launch_bounds__(256)
quantize_kernel(const float *x, size_t blocks, Q8Planar out, uint8_t *canonical, int *error) {
    const size_t warp_global = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const size_t stride = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
    for (size_t b = warp_global; b < blocks; b += stride) {
        const Q8Lane q = quantize_lane(x[b * 32 + lane]);
        if (out.codes) {
            out.codes[b * 32 + lane] = q.code;
            if (lane == 0) out.scales[b] = make_float2(h2f(q.d), h2f(q.s));
        }
        if (canonical) {
            uint8_t *blk = canonical + b * 36;
            blk[4 + lane] = static_cast<uint8_t>(q.code);
            if (lane == 0) {
                blk[0] = q.d & 0xff; blk[1] = q.d >> 8;
                blk[2] = q.s & 0xff; blk[3] = q.s >> 8;
            }
        }
        if (lane == 0) report(q.flags, error);
    }
}

// ---------------------------------------------------------------------------
// Seeded synthetic Q4_0 weights, bit-identical to the oracle's generator.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t synth_base(uint64_t seed, uint32_t layer, uint32_t expert,
                                               uint32_t matrix) {
    const uint64_t stream = (static_cast<uint64_t>(layer) << 32) |
                            (static_cast<uint64_t>(expert) << 8) | matrix;
    return mix64(seed ^ mix64(stream + 0x9e3779b97f4a7c15ull));
}

// Grid-stride over (expert, matrix, block); writes the planar layout.
__global__ void __launch_bounds__(256)
synth_kernel(uint8_t *base, ExpertLayout L, int experts_total, uint64_t seed, uint32_t layer, int e_first,
             int e_count) {
    const size_t gate_blocks = static_cast<size_t>(L.inter) * (L.hidden / 32);
    const size_t per_expert = 3 * gate_blocks;  // gate, up, down have equal block counts
    const size_t total = per_expert * experts_total;
    for (size_t g = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
         g += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint32_t e = static_cast<uint32_t>(g / per_expert);
        const size_t rem = g % per_expert;
        const uint32_t m = static_cast<uint32_t>(rem / gate_blocks);
        const size_t i = rem % gate_blocks;
        // local expert e < e_count is global expert e_first + e; the one after is the shared expert
        const uint32_t ge = e < static_cast<uint32_t>(e_count) ? static_cast<uint32_t>(e_first) + e : 512u;
        const uint64_t b = synth_base(seed, layer, ge, m);
        const uint64_t c0 = mix64(b + (i << 6) + 0), c1 = mix64(b + (i << 6) + 1);
        uint32_t mx = 0;
#pragma unroll 4
        for (int j = 2; j < 34; ++j) {
            const uint64_t r = mix64(b + (i << 6) + static_cast<uint64_t>(j));
            const uint32_t s = static_cast<uint32_t>(r & 0xffffu) + static_cast<uint32_t>((r >> 16) & 0xffffu) +
                               static_cast<uint32_t>((r >> 32) & 0xffffu) + static_cast<uint32_t>(r >> 48);
            const uint32_t dev = s >= 131070u ? s - 131070u : 131070u - s;
            mx = dev > mx ? dev : mx;
        }
        const uint16_t d = f2h(__fmul_rn(static_cast<float>(mx), 6.6073582e-08f));
        uint8_t *ex = base + static_cast<size_t>(e) * L.bytes;
        if (m == 2 && L.down_type == kDownQ4_1) {
            // Q4_1 down: minimum -8 d (0.5 + u/65536), u a 16-bit draw
            const uint64_t r = mix64(b + (i << 6) + 34);
            const float f = 0.5f + static_cast<float>(r & 0xffffu) * (1.0f / 65536.0f);
            reinterpret_cast<uint16_t *>(ex + L.down_mins)[i] = f2h(__fmul_rn(-8.0f * h2f(d), f));
        }
        const size_t code_off = m == 0 ? L.gate_codes : m == 1 ? L.up_codes : L.down_codes;
        const size_t scale_off = m == 0 ? L.gate_scales : m == 1 ? L.up_scales : L.down_scales;
        reinterpret_cast<uint4 *>(ex + code_off)[i] =
            make_uint4(static_cast<uint32_t>(c0), static_cast<uint32_t>(c0 >> 32),
                       static_cast<uint32_t>(c1), static_cast<uint32_t>(c1 >> 32));
        reinterpret_cast<uint16_t *>(ex + scale_off)[i] = d;
    }
}

// canonical 18-byte blocks <-> planar (codes, scales).  dir 0: canonical ->
// planar, dir 1: planar -> canonical.
__global__ void __launch_bounds__(256)
repack_kernel(uint8_t *canonical, uint8_t *codes, uint16_t *scales, size_t blocks, int dir) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < blocks;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        uint8_t *c = canonical + i * 18;
        if (dir == 0) {
            scales[i] = static_cast<uint16_t>(c[0] | (c[1] << 8));
            for (int j = 0; j < 16; ++j) codes[i * 16 + j] = c[2 + j];
        } else {
            c[0] = scales[i] & 0xff;
            c[1] = scales[i] >> 8;
            for (int j = 0; j < 16; ++j) c[2 + j] = codes[i * 16 + j];
        }
    }
}

// canonical 20-byte Q4_1 blocks (half d, half m, 16 code bytes) <-> planar
// (codes, scales, minima).  dir 0: canonical -> planar, dir 1: back.
__global__ void __launch_bounds__(256)
repack_q4_1_kernel(uint8_t *canonical, uint8_t *codes, uint16_t *scales, uint16_t *mins, size_t blocks, int dir) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < blocks;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        uint8_t *c = canonical + i * 20;
        if (dir == 0) {
            scales[i] = static_cast<uint16_t>(c[0] | (c[1] << 8));
            mins[i] = static_cast<uint16_t>(c[2] | (c[3] << 8));
            for (int j = 0; j < 16; ++j) codes[i * 16 + j] = c[4 + j];
        } else {
            c[0] = scales[i] & 0xff;
            c[1] = scales[i] >> 8;
            c[2] = mins[i] & 0xff;
            c[3] = mins[i] >> 8;
            for (int j = 0; j < 16; ++j) c[4 + j] = codes[i * 16 + j];
        }
    }
}

// Where the rows of a down projection go.  Normally the router-weighted
// scatter-add into the residual (red.global.add, sanitised).  In trace mode
// (put<true>, a separate kernel instantiation so the normal epilogue carries
// no branch) the raw, unweighted row of pair (token, rank) is stored
// at contrib[token][rank][H] -- the reference's moe_scatter layout
// (src/hip/session_ops.hip:358-373) -- and the shared expert's row at
// shared[token][H]; the fold kernel then applies the reference's rank-order
// fold and sigmoid-gated shared add.
struct DownSink {
    float *out;
    float *contrib = nullptr;
    float *shared = nullptr;
    const int32_t *pair_rank = nullptr;   // rank of each routed pair
    int shared_expert = 0;                // expert index of the shared expert's tiles
    template <bool Trace>
    __device__ __forceinline__ void put(int e, int p0, int tok, int j, int row, int H, float v, float w,
                                        int *error) const {
        if constexpr (Trace) {
            float *dst = e == shared_expert ? shared + static_cast<size_t>(tok) * H
                                            : contrib + (static_cast<size_t>(tok) * kTopK + pair_rank[p0 + j]) * H;
            dst[row] = v;
            return;
        }
        int flags = 0;
        const float y = arithmetic(v, flags);
        const float c = arithmetic(__fmul_rn(w, y), flags);
        atomicAdd(out + static_cast<size_t>(tok) * H + row, c);
        report(flags, error);
    }
};

// Records the per-block integer dots (and the middle Q8_1) of one expert's
// pairs for bit-exact parity checks.  Only the Tap instantiations of the
// streaming and tensor-core kernels write it (moe_debug_block_dots).
struct TapSink {
    int expert = -1;                 // expert index whose pairs are recorded
    const int32_t *pair0 = nullptr;  // device: index of that expert's first pair
    int max_pairs = 0;
    int32_t *gate = nullptr, *up = nullptr, *down = nullptr;   // [pair][row][block]
    int8_t *mid_codes = nullptr;     // [pair][I]
    uint32_t *mid_ds = nullptr;      // [pair][I/32]: half d | half s << 16
};

// ---------------------------------------------------------------------------
// Shared parameters of the grouped expert kernels.
struct GroupParams {
    const uint8_t *weights;     // expert 0 region; expert e at weights + e * layout.bytes
    ExpertLayout layout;
    Q8Planar x;                 // quantised tokens [T][H]
    Q8Planar mid;               // middle per pair [P][I]
    const TileRec *tiles;
    const int *num_tiles;
    const int32_t *pair_token;
    const float *pair_weight;
    DownSink sink;              // out [T][H] (or the trace-mode buffers)
    int *error;
};

constexpr int kGemvThreads = 256;

// Gate/up for one (tile, 32-row slab): warp w owns gate rows and up rows
// slab*32 + 4w .. +3; lane l owns blocks l, l+32, ...  Results feed SiLU*up
// and the slab's Q8_1 middle block (32 consecutive channels = one block),
// the fused silu_up_q8_1 of the reference (src/hip/linear.hip:99-150,509-525).
template <int NT>
__global__ void __launch_bounds__(kGemvThreads)
gate_up_kernel(GroupParams p) {
    const int H = p.layout.hidden, I = p.layout.inter;
    const int nb = H / 32, slabs = I / 32;
    extern __shared__ __align__(128) uint8_t smem[];
    int4 *sx = reinterpret_cast<int4 *>(smem);                          // [NT][H/16]
    float2 *ss = reinterpret_cast<float2 *>(smem + NT * H);             // [NT][nb]
    float *smid = reinterpret_cast<float *>(smem + NT * H + NT * nb * 8);  // [NT][32]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int total = *p.num_tiles * slabs;
    for (int item = blockIdx.x; item < total; item += gridDim.x) {
        const int tile = item / slabs, slab = item % slabs;
        const TileRec &td = p.tiles[tile];
        const int e = td.e, p0 = td.p0, n = td.n;
        __syncthreads();
        for (int idx = threadIdx.x; idx < n * (H / 16); idx += kGemvThreads) {
            const int j = idx / (H / 16), v = idx % (H / 16);
            const int tok = p.pair_token[p0 + j];
            sx[j * (H / 16) + v] = reinterpret_cast<const int4 *>(p.x.codes + static_cast<size_t>(tok) * H)[v];
        }
        for (int idx = threadIdx.x; idx < n * nb; idx += kGemvThreads) {
            const int j = idx / nb, b = idx % nb;
            const int tok = p.pair_token[p0 + j];
            ss[j * nb + b] = p.x.scales[static_cast<size_t>(tok) * nb + b];
        }
        __syncthreads();
        const uint8_t *ex = p.weights + static_cast<size_t>(e) * p.layout.bytes;
        const uint4 *gcodes = reinterpret_cast<const uint4 *>(ex + p.layout.gate_codes);
        const uint4 *ucodes = reinterpret_cast<const uint4 *>(ex + p.layout.up_codes);
        const uint16_t *gsc = reinterpret_cast<const uint16_t *>(ex + p.layout.gate_scales);
        const uint16_t *usc = reinterpret_cast<const uint16_t *>(ex + p.layout.up_scales);
        const int row0 = slab * 32 + warp * 4;
        float acc[8][NT];
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int j = 0; j < NT; ++j) acc[r][j] = 0.0f;
        for (int b = lane; b < nb; b += 32) {
            uint4 wc[8];
            float d4[8];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const size_t blk = static_cast<size_t>(row0 + r) * nb + b;
                wc[r] = __ldg(gcodes + blk);
                wc[4 + r] = __ldg(ucodes + blk);
                d4[r] = h2f(__ldg(gsc + blk));
                d4[4 + r] = h2f(__ldg(usc + blk));
            }
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                if (j < n) {
                    const int4 xlo = sx[j * (H / 16) + 2 * b], xhi = sx[j * (H / 16) + 2 * b + 1];
                    const float2 sc = ss[j * nb + b];
                    const float s8x8 = 8.0f * sc.y;
#pragma unroll
                    for (int r = 0; r < 8; ++r)
                        acc[r][j] = block_term(block_dot(wc[r], xlo, xhi), d4[r], sc.x, s8x8, acc[r][j]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int j = 0; j < NT; ++j) acc[r][j] = warp_sum(acc[r][j]);
        // SiLU(gate) * up with the reference's sanitisation (session_ops.hip:250-262).
        if (lane < 4) {
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                if (j < n) {
                    float g = acc[0][j], u = acc[4][j];
#pragma unroll
                    for (int r = 1; r < 4; ++r)
                        if (lane == r) { g = acc[r][j]; u = acc[4 + r][j]; }
                    int flags = 0;
                    g = operand(g, flags);
                    u = operand(u, flags);
                    const float act = arithmetic(__fdiv_rn(g, __fadd_rn(1.0f, expf_ref(-g))), flags);
                    const float v = arithmetic(__fmul_rn(act, u), flags);
                    smid[j * 32 + warp * 4 + lane] = flags ? 0.0f : v;
                    report(flags, p.error);
                }
            }
        }
        __syncthreads();
        for (int j = warp; j < n; j += kGemvThreads / 32) {
            const Q8Lane q = quantize_lane(smid[j * 32 + lane]);
            const size_t pair = static_cast<size_t>(p0 + j);
            p.mid.codes[pair * I + slab * 32 + lane] = q.code;
            if (lane == 0) {
                p.mid.scales[pair * slabs + slab] = make_float2(h2f(q.d), h2f(q.s));
                report(q.flags, p.error);
            }
        }
    }
}

// Down projection for one (tile, 64-row slab) with the router-weighted
// scatter-add into out: thread t owns row slab*64 + t/4 and blocks t%4,
// t%4+4, ...; the four partial sums meet in two shuffles, then
// out[token][row] += weight * y (red.global.add).  Replaces the reference's
// scatter + rank fold (src/hip/session_ops.hip:292-324,358-373).
template <int NT, bool Trace = false>
__global__ void __launch_bounds__(kGemvThreads)
down_kernel(GroupParams p) {
    const int H = p.layout.hidden, I = p.layout.inter;
    const int nbd = I / 32, dslabs = H / 64;
    extern __shared__ __align__(128) uint8_t smem[];
    int4 *sm = reinterpret_cast<int4 *>(smem);                           // [NT][I/16]
    float2 *ss = reinterpret_cast<float2 *>(smem + NT * I);              // [NT][nbd]
    int *stok = reinterpret_cast<int *>(smem + NT * I + NT * nbd * 8);   // [NT]
    float *swt = reinterpret_cast<float *>(stok + NT);                   // [NT]
    const int q = threadIdx.x & 3;
    const int total = *p.num_tiles * dslabs;
    for (int item = blockIdx.x; item < total; item += gridDim.x) {
        const int tile = item / dslabs, ds = item % dslabs;
        const TileRec &td = p.tiles[tile];
        const int e = td.e, p0 = td.p0, n = td.n;
        __syncthreads();
        for (int idx = threadIdx.x; idx < n * (I / 16); idx += kGemvThreads) {
            const int j = idx / (I / 16), v = idx % (I / 16);
            sm[j * (I / 16) + v] = reinterpret_cast<const int4 *>(p.mid.codes + static_cast<size_t>(p0 + j) * I)[v];
        }
        for (int idx = threadIdx.x; idx < n * nbd; idx += kGemvThreads) {
            const int j = idx / nbd, b = idx % nbd;
            ss[j * nbd + b] = p.mid.scales[static_cast<size_t>(p0 + j) * nbd + b];
        }
        if (threadIdx.x < n) {
            stok[threadIdx.x] = p.pair_token[p0 + threadIdx.x];
            swt[threadIdx.x] = p.pair_weight[p0 + threadIdx.x];
        }
        __syncthreads();
        const uint8_t *ex = p.weights + static_cast<size_t>(e) * p.layout.bytes;
        const uint4 *dcodes = reinterpret_cast<const uint4 *>(ex + p.layout.down_codes);
        const uint16_t *dsc = reinterpret_cast<const uint16_t *>(ex + p.layout.down_scales);
        const uint16_t *dmn = reinterpret_cast<const uint16_t *>(ex + p.layout.down_mins);
        const bool q41 = p.layout.down_type == kDownQ4_1;
        const int row = ds * 64 + (threadIdx.x >> 2);
        float acc[NT];
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[j] = 0.0f;
        for (int b = q; b < nbd; b += 4) {
            const size_t blk = static_cast<size_t>(row) * nbd + b;
            const uint4 wc = __ldg(dcodes + blk);
            const float d4 = h2f(__ldg(dsc + blk));
            const float m4 = q41 ? h2f(__ldg(dmn + blk)) : 0.0f;
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                if (j < n) {
                    const int4 xlo = sm[j * (I / 16) + 2 * b], xhi = sm[j * (I / 16) + 2 * b + 1];
                    const float2 sc = ss[j * nbd + b];
                    const int dot = block_dot(wc, xlo, xhi);
                    acc[j] = q41 ? block_term_q4_1(dot, d4, m4, sc.x, sc.y, acc[j])
                                 : block_term(dot, d4, sc.x, 8.0f * sc.y, acc[j]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], 1);
            acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], 2);
        }
#pragma unroll
        for (int j = 0; j < NT; ++j)
            if (j < n && (j & 3) == q) p.sink.put<Trace>(e, p0, stok[j], j, row, H, acc[j], swt[j], p.error);
    }
}

// Trace-mode fold over the stored contributions, element (t, c) per thread,
// in the reference's order: routed_fold (src/hip/session_ops.hip:305-324,
// ten separately rounded multiply/adds over ranks 0..9 from 0, zero on any
// flag), then shared_sigmoid_add (:376-391, scale * shared added to that,
// zero on any flag; the scale is the shared gate's sigmoid computed by the
// routing kernel with the same operations), then out = value (overwrite)
// or out + value.
__global__ void __launch_bounds__(256)
fold_kernel(const float *contrib, const float *weights, const float *shared, const float *shared_scale, int T, int H,
            float *out, int overwrite, int *error) {
    const size_t total = static_cast<size_t>(T) * H;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t t = i / H, c = i % H;
        int flags = 0;
        float value = 0.0f;
#pragma unroll
        for (int r = 0; r < kTopK; ++r) {
            const float x = operand(contrib[(t * kTopK + r) * H + c], flags);
            const float scale = operand(weights[t * kTopK + r], flags);
            const float contribution = arithmetic(__fmul_rn(scale, x), flags);
            value = arithmetic(__fadd_rn(value, contribution), flags);
        }
        value = flags ? 0.0f : value;
        report(flags, error);
        if (shared) {
            int f2 = 0;
            const float x = operand(shared[i], f2);
            const float original = operand(value, f2);
            const float scale = operand(shared_scale[t], f2);
            const float contribution = arithmetic(__fmul_rn(scale, x), f2);
            const float v = arithmetic(__fadd_rn(original, contribution), f2);
            value = f2 ? 0.0f : v;
            report(f2, error);
        }
        out[i] = overwrite ? value : __fadd_rn(out[i], value);
    }
}

// Parity tap / fixture linear: canonical or planar Q4_0 weights [rows][K/32]
// against canonical Q8_1 [columns][K/32]; thread per (row, column) walking
// the blocks serially.  Writes fp32 results and optionally every per-block
// int32 dot computed by block_dot() -- the routine the production kernels use.
__global__ void __launch_bounds__(256)
q4_linear_kernel(const uint8_t *canonical_w, const uint8_t *codes, const uint16_t *scales, int rows,
                 int nb, const uint8_t *xq, int columns, float *out, int32_t *dots) {
    const size_t total = static_cast<size_t>(rows) * columns;
    for (size_t g = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
         g += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(g / rows), r = static_cast<int>(g % rows);
        float acc = 0.0f;
        for (int b = 0; b < nb; ++b) {
            const size_t blk = static_cast<size_t>(r) * nb + b;
            uint4 wc;
            uint16_t hd;
            if (canonical_w) {
                const uint8_t *s = canonical_w + blk * 18;
                hd = static_cast<uint16_t>(s[0] | (s[1] << 8));
                uint32_t wv[4];
                for (int k = 0; k < 4; ++k)
                    wv[k] = s[2 + 4 * k] | (s[3 + 4 * k] << 8) | (s[4 + 4 * k] << 16) | (static_cast<uint32_t>(s[5 + 4 * k]) << 24);
                wc = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            } else {
                wc = reinterpret_cast<const uint4 *>(codes)[blk];
                hd = scales[blk];
            }
            const uint8_t *a = xq + (static_cast<size_t>(c) * nb + b) * 36;
            int xv[8];
            for (int k = 0; k < 8; ++k)
                xv[k] = a[4 + 4 * k] | (a[5 + 4 * k] << 8) | (a[6 + 4 * k] << 16) | (static_cast<int>(a[7 + 4 * k]) << 24);
            const int dot = block_dot(wc, make_int4(xv[0], xv[1], xv[2], xv[3]), make_int4(xv[4], xv[5], xv[6], xv[7]));
            const float d8 = h2f(static_cast<uint16_t>(a[0] | (a[1] << 8)));
            const float s8 = h2f(static_cast<uint16_t>(a[2] | (a[3] << 8)));
            acc = block_term(dot, h2f(hd), d8, 8.0f * s8, acc);
            if (dots) dots[(static_cast<size_t>(c) * rows + r) * nb + b] = dot;
        }
        out[static_cast<size_t>(c) * rows + r] = acc;
    }
}

// Parity tap for Q4_1 weights: canonical 20-byte blocks [rows][K/32] against
// canonical Q8_1 [columns][K/32]; the block terms of block_term_q4_1 summed
// in ascending block order, optional per-block int32 dots.
// Canonical weights when w is non-null, else the planar (codes, scales, mins).
__global__ void __launch_bounds__(256)
q4_1_linear_kernel(const uint8_t *w, const uint8_t *codes, const uint16_t *scales, const uint16_t *mins, int rows,
                   int nb, const uint8_t *xq, int columns, float *out, int32_t *dots) {
    const size_t total = static_cast<size_t>(rows) * columns;
    for (size_t g = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
         g += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(g / rows), r = static_cast<int>(g % rows);
        float acc = 0.0f;
        for (int b = 0; b < nb; ++b) {
            const size_t blk = static_cast<size_t>(r) * nb + b;
            uint16_t hd, hm;
            uint32_t wv[4];
            if (w) {
                const uint8_t *s = w + blk * 20;
                hd = static_cast<uint16_t>(s[0] | (s[1] << 8));
                hm = static_cast<uint16_t>(s[2] | (s[3] << 8));
                for (int k = 0; k < 4; ++k)
                    wv[k] = s[4 + 4 * k] | (s[5 + 4 * k] << 8) | (s[6 + 4 * k] << 16) |
                            (static_cast<uint32_t>(s[7 + 4 * k]) << 24);
            } else {
                const uint4 c = reinterpret_cast<const uint4 *>(codes)[blk];
                wv[0] = c.x; wv[1] = c.y; wv[2] = c.z; wv[3] = c.w;
                hd = scales[blk];
                hm = mins[blk];
            }
            const uint8_t *a = xq + (static_cast<size_t>(c) * nb + b) * 36;
            int xv[8];
            for (int k = 0; k < 8; ++k)
                xv[k] = a[4 + 4 * k] | (a[5 + 4 * k] << 8) | (a[6 + 4 * k] << 16) | (static_cast<int>(a[7 + 4 * k]) << 24);
            const int dot = block_dot(make_uint4(wv[0], wv[1], wv[2], wv[3]), make_int4(xv[0], xv[1], xv[2], xv[3]),
                                      make_int4(xv[4], xv[5], xv[6], xv[7]));
            const float d8 = h2f(static_cast<uint16_t>(a[0] | (a[1] << 8)));
            const float s8 = h2f(static_cast<uint16_t>(a[2] | (a[3] << 8)));
            acc = block_term_q4_1(dot, h2f(hd), h2f(hm), d8, s8, acc);
            if (dots) dots[(static_cast<size_t>(c) * rows + r) * nb + b] = dot;
        }
        out[static_cast<size_t>(c) * rows + r] = acc;
    }
}

}  // namespace qmoe
