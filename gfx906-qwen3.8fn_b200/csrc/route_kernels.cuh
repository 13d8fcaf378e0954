// route_kernels.cuh -- router softmax, top-10 selection and stable grouping.
//
// Replaces three reference stages with device work and no host round trip:
//  * router_softmax (src/hip/session_ops.hip:401-434),
//  * select_routes (src/session.hip:666-687, a host partial_sort),
//  * RouteGroups::prepare (src/routes.cpp:59-115, a host counting sort) plus
//    the per-layer pinned upload of the {token, rank} list (src/session.hip:393-410).
// Index results are bit-exact with the reference algorithms: every float
// operation is a separately rounded IEEE op in the reference's order.
#pragma once
#include "common.cuh"
#include "ep_common.cuh"
#include "ptx.cuh"

namespace qmoe {

constexpr int kChunk = 32;         // tokens per routing chunk (one bit each in a 32-bit mask)
constexpr int kRouteThreads = 1024; // 32 warps: one per token of a chunk

// Exponential used by the router softmax.  The same operation sequence is
// the specification in the CPU oracle: Cody-Waite reduction with ln2 split
// into an exact-product high part and a low part, degree-7 Taylor polynomial
// of e^r in Horner form, exact power-of-two scaling in two steps.
__device__ __forceinline__ float route_exp(float x) {
    if (!(x == x)) return x;
    if (x < -104.0f) return 0.0f;
    if (x > 88.8f) return __int_as_float(0x7f800000);
    const float n = rintf(__fmul_rn(x, 1.44269502f));
    float r = fmaf(-n, 0.693145751953125f, x);
    r = fmaf(-n, 1.42860677e-06f, r);
    float p = 1.98412701e-04f;
    p = fmaf(p, r, 1.38888892e-03f);
    p = fmaf(p, r, 8.33333377e-03f);
    p = fmaf(p, r, 4.16666679e-02f);
    p = fmaf(p, r, 1.66666672e-01f);
    p = fmaf(p, r, 5.00000000e-01f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int k = static_cast<int>(n);
    const int k1 = k / 2, k2 = k - k1;
    const float s1 = __int_as_float((127 + k1) << 23), s2 = __int_as_float((127 + k2) << 23);
    return __fmul_rn(__fmul_rn(p, s1), s2);
}

struct RouteParams {
    const float *logits;    // [T][512]
    const float *x;         // [T][H] (shared-expert gate input); may be null without shared
    const float *gate_vec;  // [H] or null (no shared expert)
    int tokens, hidden;
    float *probs;           // optional [T][512]
    int32_t *ids;           // [T][10]
    float *weights;         // [T][10]
    uint32_t *masks;        // [chunks][512]: bit j set when token chunk*32+j routes to expert e
    int32_t *pair_token;    // shared-expert pairs are written at [T*10 + t]
    float *pair_weight;
    int32_t *pair_rank;
    int *error;
};

// Route token t with one warp: softmax, top-10, renormalised weights and the
// chunk mask bit j in smask[expert]; ids/weights also go to shared-memory
// copies when ids_s is given.
__device__ __forceinline__ void route_topk_token(const RouteParams &p, int t, int j, uint32_t *smask, int lane,
                                                 int32_t *ids_s = nullptr, float *w_s = nullptr) {
    {
        const float *row = p.logits + static_cast<size_t>(t) * kRouterExperts;
        int flags = 0;
        float w[16];
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            w[k] = operand(row[lane + 32 * k], flags);
            mx = fmaxf(mx, w[k]);
        }
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
        float total = 0.0f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float shifted = arithmetic(__fsub_rn(w[k], mx), flags);
            w[k] = arithmetic(route_exp(shifted), flags);
            total = arithmetic(__fadd_rn(total, w[k]), flags);
        }
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) total = __fadd_rn(total, __shfl_xor_sync(0xffffffffu, total, m));
        total = arithmetic(total, flags);
        if (!(total > 0.0f)) flags |= kFlagArithmetic;
        const float inv = total > 0.0f ? arithmetic(__fdiv_rn(1.0f, total), flags) : 0.0f;
#pragma unroll
        for (int k = 0; k < 16; ++k) w[k] = arithmetic(__fmul_rn(w[k], inv), flags);
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) flags |= __shfl_xor_sync(0xffffffffu, flags, m);
        if (flags) {
#pragma unroll
            for (int k = 0; k < 16; ++k) w[k] = 0.0f;
        }
        if (p.probs) {
            float *prow = p.probs + static_cast<size_t>(t) * kRouterExperts;
#pragma unroll
            for (int k = 0; k < 16; ++k) prow[lane + 32 * k] = w[k];
        }
        if (lane == 0) report(flags, p.error);

        // top-10 by (probability desc, id asc): ten warp-wide arg-max rounds.
        // Probabilities are non-negative, so their bit patterns (+1, 0 =
        // taken) order like the values: one warp max picks the value, one
        // warp min the lowest id holding it.
        uint32_t taken = 0u;
        int sel_id[kTopK];
        float sel_p[kTopK];
        uint32_t key[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) key[k] = __float_as_uint(w[k]) + 1u;
#pragma unroll
        for (int r = 0; r < kTopK; ++r) {
            // the lane's best untaken key by a 4-level tree; at every node the
            // left operand has the lower id, so ties keep it
            uint32_t kv[16];
            int ki[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                kv[k] = ((taken >> k) & 1u) ? 0u : key[k];
                ki[k] = k;
            }
#pragma unroll
            for (int w2 = 8; w2 > 0; w2 >>= 1)
#pragma unroll
                for (int k = 0; k < w2; ++k) {
                    const bool right = kv[2 * k + 1] > kv[2 * k];
                    kv[k] = right ? kv[2 * k + 1] : kv[2 * k];
                    ki[k] = right ? ki[2 * k + 1] : ki[2 * k];
                }
            const uint32_t best = kv[0];
            const int bk = ki[0];
            const uint32_t mk = __reduce_max_sync(0xffffffffu, best);
            const uint32_t bi = __reduce_min_sync(0xffffffffu, best == mk ? static_cast<uint32_t>(lane + 32 * bk)
                                                                           : 0xffffffffu);
            if (static_cast<int>(bi & 31u) == lane) taken |= 1u << (bi >> 5);
            sel_id[r] = static_cast<int>(bi);
            sel_p[r] = __uint_as_float(mk - 1u);
        }
        // Renormalisation: buckets[id % 32] accumulate in rank order, then an
        // XOR butterfly 1..16, floor 1/16384, reciprocal, separate multiply.
        float bucket = 0.0f;
#pragma unroll
        for (int r = 0; r < kTopK; ++r)
            if ((sel_id[r] & 31) == lane) bucket = __fadd_rn(bucket, sel_p[r]);
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) bucket = __fadd_rn(bucket, __shfl_xor_sync(0xffffffffu, bucket, m));
        const float den = fmaxf(bucket, 1.0f / 16384.0f);
        const float inv_den = __fdiv_rn(1.0f, den);
#pragma unroll
        for (int r = 0; r < kTopK; ++r) {
            if (lane == r) {
                const float wr = __fmul_rn(sel_p[r], inv_den);
                p.ids[t * kTopK + r] = sel_id[r];
                p.weights[t * kTopK + r] = wr;
                if (ids_s) {
                    ids_s[j * kTopK + r] = sel_id[r];
                    w_s[j * kTopK + r] = wr;
                }
                atomicOr(&smask[sel_id[r]], 1u << j);
            }
        }
    }
}

// Shared expert of token t with one warp: raw gate = x . gate_vec, weight =
// 1/(1+exp(-raw)) (src/hip/session_ops.hip:376-391), written as pair T*10 + t.
__device__ __forceinline__ void route_shared_gate(const RouteParams &p, int t, int lane) {
    {
        if (p.gate_vec) {
            const float4 *xr = reinterpret_cast<const float4 *>(p.x + static_cast<size_t>(t) * p.hidden);
            const float4 *gv = reinterpret_cast<const float4 *>(p.gate_vec);
            float acc = 0.0f;
            for (int h = lane; h < p.hidden / 4; h += 32) {
                const float4 a = xr[h], b = gv[h];
                acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
                acc = fmaf(a.z, b.z, acc); acc = fmaf(a.w, b.w, acc);
            }
            acc = warp_sum(acc);
            if (lane == 0) {
                int f = 0;
                const float raw = operand(acc, f);
                const float scale = arithmetic(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-raw))), f);
                const int pair = p.tokens * kTopK + t;
                p.pair_token[pair] = t;
                p.pair_weight[pair] = scale;
                if (p.pair_rank) p.pair_rank[pair] = kTopK;
                report(f, p.error);
            }
        }
    }
}

__device__ __forceinline__ void route_one_token(const RouteParams &p, int t, int j, uint32_t *smask, int lane) {
    route_topk_token(p, t, j, smask, lane);
    route_shared_gate(p, t, lane);
}

// One CTA per chunk of 32 tokens; one warp per token.
__global__ void __launch_bounds__(kRouteThreads)
route_topk_kernel(RouteParams p) {
    __shared__ uint32_t smask[kRouterExperts];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int e = threadIdx.x; e < kRouterExperts; e += kRouteThreads) smask[e] = 0u;
    __syncthreads();
    const int chunk = blockIdx.x;
    for (int j = warp; j < kChunk; j += kRouteThreads / 32) {
        const int t = chunk * kChunk + j;
        if (t >= p.tokens) break;
        route_one_token(p, t, j, smask, lane);
    }
    __syncthreads();
    uint32_t *out = p.masks + static_cast<size_t>(chunk) * kRouterExperts;
    for (int e = threadIdx.x; e < kRouterExperts; e += kRouteThreads) out[e] = smask[e];
}

// Block-wide exclusive scan of one int per thread (blockDim.x == 512).
__device__ __forceinline__ int block_exclusive_scan_512(int v, int *total_out) {
    __shared__ int warp_tot[16];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, inc, d);
        if (lane >= d) inc += o;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int w = lane < 16 ? warp_tot[lane] : 0;
#pragma unroll
        for (int d = 1; d < 16; d <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, w, d);
            if (lane >= d) w += o;
        }
        if (lane < 16) warp_tot[lane] = w;   // inclusive warp totals
    }
    __syncthreads();
    const int before = warp > 0 ? warp_tot[warp - 1] : 0;
    if (total_out) *total_out = warp_tot[15];
    __syncthreads();
    return before + inc - v;
}

// Per-expert prefix over chunks.  Grid: 16 CTAs x 1024 threads; CTA b owns
// experts 32b..32b+31 (lane = expert), warp w owns a contiguous range of
// chunks.  base[c][e] = entries of expert e in chunks before c; counts[e] =
// group size.
__global__ void __launch_bounds__(1024)
route_chunk_prefix_kernel(const uint32_t *masks, int chunks, int32_t *base, int32_t *counts) {
    __shared__ int part[32][33];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e = blockIdx.x * 32 + lane;
    const int per = (chunks + 31) / 32;
    const int c0 = min(chunks, warp * per), c1 = min(chunks, c0 + per);
    int s = 0;
    for (int c = c0; c < c1; ++c) s += __popc(masks[static_cast<size_t>(c) * kRouterExperts + e]);
    part[warp][lane] = s;
    __syncthreads();
    int run = 0;
    for (int w = 0; w < warp; ++w) run += part[w][lane];
    for (int c = c0; c < c1; ++c) {
        const size_t idx = static_cast<size_t>(c) * kRouterExperts + e;
        base[idx] = run;
        run += __popc(masks[idx]);
    }
    if (warp == 31) counts[e] = run;
}

struct ScanParams {
    const int32_t *counts;  // [512]
    int tokens, tile;       // tile = tokens per work tile
    int has_shared;
    int32_t *offsets;       // [514]: 512 routed groups, shared group, end
    TileRec *tiles;
    int32_t *tile_off;      // [512]: first tile of each routed expert
    int32_t *pair_token;    // shared-expert pairs (written by route_topk at tokens*10 + t,
    float *pair_weight;     // or here at offsets[512] + t when shared_w is given)
    int *num_tiles;         // [0] tiles, [1] how many of them (at the end) are shared-expert tiles
    int max_tiles;
    int *error;
    // Groups of at least tc_min pairs (0: never) go to the tensor-core path,
    // split evenly into ceil(n / tc_tile) tiles: {expert, first pair, count, 0}.
    int tc_min = 0, tc_tile = 128, tc_max = 0;
    int4 *tc_tiles = nullptr;
    int *tc_num = nullptr;
    // Shared-expert pairs supplied directly (expert parallelism): pair
    // offsets[512] + i is token shared_token0 + i with weight shared_w[i], and
    // the shared expert's weights sit at index shared_expert.
    const float *shared_w = nullptr;
    int shared_token0 = 0;
    int shared_expert = kRouterExperts;
};

// One CTA of 512 threads (thread = expert): exclusive scan over experts and
// the work-tile list (tiles of at most `tile` pairs of one expert).
__global__ void __launch_bounds__(512) route_scan_kernel(ScanParams p) {
    const int e = threadIdx.x;
    const int run = p.counts[e];
    int total = 0;
    const int off = block_exclusive_scan_512(run, &total);
    p.offsets[e] = off;
    if (e == kRouterExperts - 1) {
        p.offsets[kRouterExperts] = total;
        p.offsets[kRouterExperts + 1] = total + (p.has_shared ? p.tokens : 0);
    }
    const bool big = p.tc_min > 0 && run >= p.tc_min;
    const int ntiles = big ? 0 : (run + p.tile - 1) / p.tile;
    const int ntc = big ? (run + p.tc_tile - 1) / p.tc_tile : 0;
    int tiles_total = 0, tc_total = 0;
    const int toff = block_exclusive_scan_512(ntiles, &tiles_total);
    const int tcoff = block_exclusive_scan_512(ntc, &tc_total);
    p.tile_off[e] = big ? -1 : toff;
    for (int i = 0; i < ntiles; ++i) {
        const int idx = toff + i;
        if (idx < p.max_tiles) {
            TileRec &t = p.tiles[idx];
            t.e = e;
            t.p0 = off + i * p.tile;
            t.n = min(p.tile, run - i * p.tile);
            t.pad = 0;
        }
    }
    for (int i = 0; i < ntc; ++i)
        if (tcoff + i < p.tc_max) {
            const int a = i * run / ntc, b = (i + 1) * run / ntc;
            p.tc_tiles[tcoff + i] = make_int4(e, off + a, b - a, 0);
        }
    int shared_tiles = 0, shared_tc = 0;
    // shared pair i: from route_topk at tokens*10 + i, or given directly
    const int shared_src = p.shared_w ? total : p.tokens * kTopK;
    if (p.has_shared && p.shared_w)
        for (int i = e; i < p.tokens; i += 512) {
            p.pair_token[total + i] = p.shared_token0 + i;
            p.pair_weight[total + i] = p.shared_w[i];
        }
    if (p.has_shared && p.tc_min > 0 && p.tokens >= p.tc_min) {
        shared_tc = (p.tokens + p.tc_tile - 1) / p.tc_tile;
        for (int i = e; i < shared_tc; i += 512)
            if (tc_total + i < p.tc_max) {
                const int a = i * p.tokens / shared_tc, b = (i + 1) * p.tokens / shared_tc;
                p.tc_tiles[tc_total + i] = make_int4(p.shared_expert, total + a, b - a, 0);
            }
    } else if (p.has_shared) {
        shared_tiles = (p.tokens + p.tile - 1) / p.tile;
        for (int i = e; i < shared_tiles; i += 512) {
            const int idx = tiles_total + i;
            if (idx < p.max_tiles) {
                TileRec &t = p.tiles[idx];
                t.e = p.shared_expert;
                t.p0 = total + i * p.tile;
                t.n = min(p.tile, p.tokens - i * p.tile);
                t.pad = 0;
                for (int j = 0; j < kGemvTile; ++j) {
                    const bool live = j < t.n;
                    const int k = i * p.tile + j;
                    t.tok[j] = live ? (p.shared_w ? p.shared_token0 + k : p.pair_token[shared_src + k]) : 0;
                    t.w[j] = live ? (p.shared_w ? p.shared_w[k] : p.pair_weight[shared_src + k]) : 0.0f;
                }
            }
        }
    }
    if (e == 0) {
        int n = tiles_total + shared_tiles;
        if (n > p.max_tiles) { atomicOr(p.error, kFlagArithmetic); n = p.max_tiles; }
        p.num_tiles[0] = n;
        p.num_tiles[1] = max(0, n - tiles_total);
        if (p.tc_num) {
            int m = tc_total + shared_tc;
            if (m > p.tc_max) { atomicOr(p.error, kFlagArithmetic); m = p.tc_max; }
            *p.tc_num = m;
        }
    }
}

struct ScatterParams {
    const uint32_t *masks;
    const int32_t *base;
    const int32_t *offsets;
    const int32_t *ids;
    const float *weights;
    int32_t *pair_token;
    int32_t *pair_rank;
    float *pair_weight;
    TileRec *tiles;
    const int32_t *tile_off;
    int max_tiles;
};

// Thread per (chunk, expert): stable placement by token order within the chunk.
__global__ void __launch_bounds__(256) route_scatter_kernel(ScatterParams p) {
    const int chunk = blockIdx.x, e = blockIdx.y * 256 + threadIdx.x;
    const size_t idx = static_cast<size_t>(chunk) * kRouterExperts + e;
    uint32_t m = p.masks[idx];
    if (!m) return;
    int pos = p.offsets[e] + p.base[idx];
    while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1u;
        const int t = chunk * kChunk + j;
        int r = 0;
#pragma unroll
        for (int k = 0; k < kTopK; ++k)
            if (p.ids[t * kTopK + k] == e) r = k;
        const float w = p.weights[t * kTopK + r];
        p.pair_token[pos] = t;
        if (p.pair_rank) p.pair_rank[pos] = r;
        p.pair_weight[pos] = w;
        if (p.tiles && p.tile_off[e] >= 0) {   // tensor-core groups have no small tiles
            const int local = pos - p.offsets[e];
            const int tile = p.tile_off[e] + local / kGemvTile;
            if (tile < p.max_tiles) {
                p.tiles[tile].tok[local % kGemvTile] = t;
                p.tiles[tile].w[local % kGemvTile] = w;
            }
        }
        ++pos;
    }
}

// Single-expert fixture routing: pair t = token t of expert 0 with weight 1.
__global__ void identity_route_kernel(int tokens, int tile, TileRec *tiles, int *num_tiles,
                                      int32_t *pair_token, float *pair_weight) {
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < tokens; t += gridDim.x * blockDim.x) {
        pair_token[t] = t;
        pair_weight[t] = 1.0f;
        TileRec &r = tiles[t / tile];
        r.tok[t % tile] = t;
        r.w[t % tile] = 1.0f;
        if (t % tile == 0) {
            r.e = 0;
            r.p0 = t;
            r.n = min(tile, tokens - t);
            r.pad = 0;
            for (int j = r.n; j < tile; ++j) { r.tok[j] = 0; r.w[j] = 0.0f; }
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        num_tiles[0] = (tokens + tile - 1) / tile;
        num_tiles[1] = 0;
    }
}

// ---------------------------------------------------------------------------
// Decode-size batches (T <= 32, one routing chunk): Q8_1 quantisation of x,
// routing, grouping and the tile list in ONE CTA of 512 threads, replacing the
// six launches of the general path.  Same arithmetic, same outputs.
struct SmallRouteParams {
    RouteParams r;
    // Expert parallelism (ep_on): the quantising CTAs also store every row into
    // every rank's receive buffer at slot rank*t_max + token, and the routing
    // CTA writes each destination's (local expert, weight) lists and publishes
    // the epoch once all rows are in place -- dispatch without its own launch.
    int ep_on = 0;
    EpParams ep;
    uint32_t *quant_done = nullptr;   // quantising CTAs finished (rewound by the routing CTA)
    Q8Planar xq;            // quantised x output
    int32_t *offsets;       // [514]
    TileRec *tiles;
    int32_t *tile_off;
    int *num_tiles;         // [0] tiles, [1] how many of them (at the end) are shared-expert tiles
    int max_tiles;
};

__global__ void __launch_bounds__(512) route_small_kernel(SmallRouteParams sp) {
    const RouteParams &p = sp.r;
    __shared__ uint32_t smask[kRouterExperts];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, e = threadIdx.x;
    const int T = p.tokens, H = p.hidden;
    // Launched with programmatic serialisation: the CTAs may be resident
    // before the preceding kernel (which may still read this layer's tile list
    // and activation buffers) has finished; wait for it.  No early trigger: expert
    // CTAs made resident while routing runs measured slower than a launch at
    // its end.
    grid_dependency_wait();
    if (blockIdx.x > 0) {
        // blocks 1.. quantise x, one warp per 32-value block, alongside the routing block
        const int stride = (gridDim.x - 1) * 16, nb = H / 32;
        for (int b = (blockIdx.x - 1) * 16 + warp; b < T * nb; b += stride) {
            const Q8Lane q = quantize_lane(p.x[static_cast<size_t>(b) * 32 + lane]);
            sp.xq.codes[static_cast<size_t>(b) * 32 + lane] = q.code;
            if (lane == 0) {
                sp.xq.scales[b] = make_float2(h2f(q.d), h2f(q.s));
                report(q.flags, p.error);
            }
            if (sp.ep_on) {   // the row block into every rank's receive buffer (fixed slot)
                const int t = b / nb, j = b % nb;
                const size_t slot = static_cast<size_t>(sp.ep.rank) * sp.ep.t_max + t;
                for (int d = 0; d < sp.ep.world; ++d) {
                    uint8_t *base = sp.ep.peers.base[d];
                    reinterpret_cast<int8_t *>(base + sp.ep.L.codes)[slot * H + j * 32 + lane] = q.code;
                    if (lane == 0)
                        reinterpret_cast<float2 *>(base + sp.ep.L.scales)[slot * nb + j] =
                            make_float2(h2f(q.d), h2f(q.s));
                }
            }
        }
        if (sp.ep_on) {
            __syncthreads();
            if (threadIdx.x == 0) {
                __threadfence_system();
                atomicAdd(sp.quant_done, 1u);
            }
        }
        return;
    }
    __shared__ int32_t ids_s[kChunk * kTopK];
    __shared__ float w_s[kChunk * kTopK];
    smask[e] = 0u;
    __syncthreads();
    if (sp.ep_on && e == 0) *sp.ep.epoch += 1u;
    // warps 0..T-1 route token = warp (and 16 + warp); the shared gates run on
    // the idle warps T..2T-1 in parallel when T <= 8, else after the routing
    for (int t = warp; t < T; t += 16) route_topk_token(p, t, t, smask, lane, ids_s, w_s);
    for (int t = T <= 8 ? warp - T : warp; t >= 0 && t < T; t += 16) route_shared_gate(p, t, lane);
    __syncthreads();   // ids/weights (global and shared) and smask complete
    if (sp.ep_on) {
        const EpParams &ep = sp.ep;
        // each destination's (local expert, weight) lists of this rank's tokens
        for (int i = e; i < T * ep.world * kTopK; i += blockDim.x) {
            const int k = i % kTopK, d = (i / kTopK) % ep.world, t = i / (kTopK * ep.world);
            const int gid = ids_s[t * kTopK + k];
            const bool own = gid >= 0 && gid / ep.ecount == d;
            const size_t slot = static_cast<size_t>(ep.rank) * ep.t_max + t;
            reinterpret_cast<int32_t *>(ep.peers.base[d] + ep.L.ids)[slot * kEpSlotIds + k] = own ? gid - d * ep.ecount : -1;
            reinterpret_cast<float *>(ep.peers.base[d] + ep.L.w)[slot * kEpSlotIds + k] = own ? w_s[t * kTopK + k] : 0.0f;
        }
        // destinations and slots for the combine: token t sits at index t in every region
        if (e < T) {
            uint32_t mask = 1u << ep.rank;
            for (int k = 0; k < kTopK; ++k) {
                const int gid = ids_s[e * kTopK + k];
                if (gid >= 0 && gid < ep.ecount * ep.world) mask |= 1u << (gid / ep.ecount);
            }
            ep.dmask[e] = static_cast<uint8_t>(mask);
            for (int d = 0; d < kEpMaxRanks; ++d) ep.pos[e * kEpMaxRanks + d] = e;
        }
        // every quantising CTA has stored its rows (and fenced them system-wide)
        if (e == 0) {
            const long long t0 = clock64();
            bool all_in = true;
            while (ld_acquire_gpu_u32(sp.quant_done) != gridDim.x - 1) {
                if (clock64() - t0 > (1ll << 31)) { atomicOr(p.error, kFlagTimeout); all_in = false; break; }
                __nanosleep(32);
            }
            // Rewind for the next call only after a complete count: after a
            // timeout late CTAs may still add to it, so it is left for the host
            // to clear once the stream is idle (moe_ep_read_flags).
            if (all_in) *sp.quant_done = 0u;
        }
        __syncthreads();
        if (e < ep.world) ep_publish(ep, e, static_cast<uint32_t>(T), *ep.epoch);
        return;
    }
    const uint32_t mask = smask[e];
    const int count = __popc(mask);
    int total = 0;
    const int off = block_exclusive_scan_512(count, &total);
    sp.offsets[e] = off;
    if (e == kRouterExperts - 1) {
        sp.offsets[kRouterExperts] = total;
        sp.offsets[kRouterExperts + 1] = total + (p.gate_vec ? T : 0);
    }
    const int ntiles = (count + kGemvTile - 1) / kGemvTile;
    int tiles_total = 0;
    const int toff = block_exclusive_scan_512(ntiles, &tiles_total);
    sp.tile_off[e] = toff;
    int pos = 0;
    for (uint32_t m = mask; m; m &= m - 1u, ++pos) {
        const int t = __ffs(m) - 1;
        int r = 0;
#pragma unroll
        for (int k = 0; k < kTopK; ++k)
            if (ids_s[t * kTopK + k] == e) r = k;
        const float w = w_s[t * kTopK + r];
        const int pair = off + pos;
        p.pair_token[pair] = t;
        if (p.pair_rank) p.pair_rank[pair] = r;
        p.pair_weight[pair] = w;
        const int tile = toff + pos / kGemvTile, slot = pos % kGemvTile;
        if (tile < sp.max_tiles) {
            TileRec &rec = sp.tiles[tile];
            if (slot == 0) {
                rec.e = e;
                rec.p0 = pair;
                rec.n = min(kGemvTile, count - pos);
                rec.pad = 0;
            }
            rec.tok[slot] = t;
            rec.w[slot] = w;
        }
    }
    int shared_tiles = 0;
    if (p.gate_vec) {
        shared_tiles = (T + kGemvTile - 1) / kGemvTile;
        if (e < shared_tiles && tiles_total + e < sp.max_tiles) {
            TileRec &rec = sp.tiles[tiles_total + e];
            rec.e = kRouterExperts;
            rec.p0 = total + e * kGemvTile;
            rec.n = min(kGemvTile, T - e * kGemvTile);
            rec.pad = 0;
            for (int j = 0; j < kGemvTile; ++j) {
                const bool live = j < rec.n;
                rec.tok[j] = live ? p.pair_token[T * kTopK + e * kGemvTile + j] : 0;
                rec.w[j] = live ? p.pair_weight[T * kTopK + e * kGemvTile + j] : 0.0f;
            }
        }
    }
    if (e == 0) {
        int n = tiles_total + shared_tiles;
        if (n > sp.max_tiles) { atomicOr(p.error, kFlagArithmetic); n = sp.max_tiles; }
        sp.num_tiles[0] = n;
        sp.num_tiles[1] = max(0, n - tiles_total);
    }
}

}  // namespace qmoe
