// stream_kernels.cuh -- persistent weight-streaming expert kernels (decode and
// small groups).  One CTA per SM: warp 0 is the producer, which streams each
// work item's weights into a ring of shared-memory stages with cp.async.bulk
// (completion counted on an mbarrier); warps 1..8 are consumers that run the
// u4 x s8 dp4a dots out of shared memory and release each stage on an
// "empty" mbarrier.  Three gate/up stages (72 KB each) or five down stages
// (43 KB each, minima slice included) make the ring, so HBM latency is
// covered by bytes in flight rather than by resident warps.
//
// Work is coarse per warp on purpose: a consumer lane handles 16 (gate/up)
// or 8 (down) block-rows per stage, so the fixed per-stage work (reductions,
// SiLU, barriers) stays small next to the dot products.  Activation rows are
// read through L1 (prefetched before the weights arrive).  The per-item body
// is compiled once per tile size n = 1..4.
#pragma once
#include "common.cuh"
#include "expert_kernels.cuh"
#include "ptx.cuh"

namespace qmoe {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kStreamThreads = 32 + kConsumerThreads;
constexpr int kGuRows = 32;    // gate rows and up rows per item: one Q8_1 middle block
constexpr int kDnRows = 128;   // down rows per item
constexpr int kGuGroupsMax = 2;   // gate/up items in flight per CTA: 1 or 2 (stream_gate_up_kernel<G>)
constexpr int kDnLaneRows = kDnRows / (8 * kConsumerWarps);   // down rows per consumer lane
static_assert(kDnLaneRows >= 1 && kDnRows % (8 * kConsumerWarps) == 0, "down rows split evenly over lanes");
constexpr int kMaxStages = 8;  // ring slots (two mbarriers each in the first 128 bytes)

struct StreamParams {
    const uint8_t *weights;
    ExpertLayout layout;
    Q8Planar x, mid;
    const TileRec *tiles;
    const int *num_tiles;   // [0] tiles, [1] shared-expert tiles at the end of the list
    DownSink sink;          // down rows: weighted scatter-add into out, or trace-mode stores
    int *error;
    int stages;
    uint32_t stage_bytes;
    TapSink tap;            // per-block dot tap (Tap instantiations only)
};

// Where a Tap instantiation stores the dots of one item of the tapped expert.
struct ItemTap {
    int32_t *dst0 = nullptr, *dst1 = nullptr;   // gate and up (or down) dot arrays, null when not tapped
    int pl = 0;                                 // pair-local index of the item's first pair
    int rows = 0, nb = 0, row0 = 0, max_pairs = 0;
    __device__ __forceinline__ void put(int32_t *dst, int j, int row, int b, int dot) const {
        const int q = pl + j;
        if (q >= 0 && q < max_pairs) dst[(static_cast<size_t>(q) * rows + row0 + row) * nb + b] = dot;
    }
};

// ---- stage layouts (meta, then codes, then half scales) --------------------
struct GuStage {
    uint32_t meta, gcodes, ucodes, gsc, usc, bytes;
    __host__ __device__ GuStage(int H) {
        const uint32_t nb = H / 32;
        meta = 0;
        gcodes = 128;
        ucodes = gcodes + kGuRows * nb * 16;
        gsc = ucodes + kGuRows * nb * 16;
        usc = gsc + kGuRows * nb * 2;
        bytes = usc + kGuRows * nb * 2;
        bytes = (bytes + 127) & ~127u;
    }
};

// The minima slice (Q4_1 down matrices) is reserved in every stage, so one
// ring layout serves both down types.
struct DnStage {
    uint32_t meta, dcodes, dsc, dmin, mcodes, msc, bytes;
    __host__ __device__ DnStage(int I) {
        const uint32_t nb = I / 32;
        meta = 0;
        dcodes = 128;
        dsc = dcodes + kDnRows * nb * 16;
        dmin = dsc + kDnRows * nb * 2;
        mcodes = dmin + kDnRows * nb * 2;
        msc = mcodes + kGemvTile * I;
        bytes = msc + kGemvTile * nb * 8;
        bytes = (bytes + 127) & ~127u;
    }
};

// Order of the work items.  CTA c takes positions c, c + G, c + 2G, ... (G =
// gridDim.x), so with r = total % G the CTAs c >= r get one item fewer.  The
// shared-expert items (the list's last S items, all tokens: the most dot
// products per weight byte) are placed at positions r .. r+S-1, i.e. on those
// CTAs, instead of on the CTAs that already have the extra item.  The map is a
// bijection of [0, total) for any S.
struct ItemOrder {
    int total, heavy_at, heavy_n;
    __device__ __forceinline__ int operator()(int pos) const {
        if (pos < heavy_at) return pos;
        if (pos < heavy_at + heavy_n) return total - heavy_n + (pos - heavy_at);
        return pos - heavy_n;
    }
};

__device__ __forceinline__ ItemOrder item_order(const int *num_tiles, int slabs) {
    const int2 nt = *reinterpret_cast<const int2 *>(num_tiles);
    ItemOrder o;
    o.total = nt.x * slabs;
    o.heavy_n = min(max(nt.y, 0), nt.x) * slabs;
    o.heavy_at = min(o.total % static_cast<int>(gridDim.x), o.total - o.heavy_n);
    return o;
}

__device__ __forceinline__ TileRec load_tile(const TileRec *t) {
    TileRec r;
    const int4 *s = reinterpret_cast<const int4 *>(t);
    int4 *d = reinterpret_cast<int4 *>(&r);
#pragma unroll
    for (int i = 0; i < static_cast<int>(sizeof(TileRec) / 16); ++i) d[i] = __ldg(s + i);
    return r;
}

// Producer loop (one thread).  `issue(item, stage, bar, rec)` arms `bar` with
// the byte count and enqueues the bulk copies of one item.
template <class Issue>
__device__ __forceinline__ void stream_producer(const StreamParams &p, uint8_t *stages, uint64_t *full,
                                                uint64_t *empty, const ItemOrder &order, int slabs, Issue issue) {
    const int total = order.total;
    int i = 0;
    int pos = blockIdx.x;
    TileRec next;
    if (pos < total) next = load_tile(p.tiles + order(pos) / slabs);
    for (; pos < total; pos += gridDim.x, ++i) {
        const int item = order(pos);
        const TileRec rec = next;
        const int following = pos + gridDim.x;
        if (following < total) next = load_tile(p.tiles + order(following) / slabs);
        const int s = i % p.stages;
        if (i >= p.stages && !mbar_wait(&empty[s], ((i / p.stages) & 1) ^ 1, p.error)) break;
        uint8_t *st = stages + static_cast<size_t>(s) * p.stage_bytes;
        *reinterpret_cast<TileRec *>(st) = rec;        // meta, published by the arrive in issue()
        issue(item, st, &full[s], rec);
    }
    // Keep the CTA alive until every issued copy has landed.
    for (int k = i - p.stages > 0 ? i - p.stages : 0; k < i; ++k)
        mbar_wait(&full[k % p.stages], (k / p.stages) & 1, p.error);
}

__device__ __forceinline__ void init_ring(uint64_t *full, uint64_t *empty, int stages, int consumers) {
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], consumers); }
        mbar_fence_init();
    }
    __syncthreads();
}

// ---- gate/up + SiLU*up + Q8_1 middle ---------------------------------------
// The consumer warps form G groups that take the CTA's items in turn (item i
// goes to group i % G), so that G items are in flight; with two, one item's
// latencies (activation loads, butterflies, the SiLU's exp lookups, the Q8_1
// reductions) overlap the other's, which pays when a CTA has about one item
// (decode of one or two tokens) and costs when it has many.  Warp cw of a
// group owns gate rows and up rows R*cw .. R*cw+R-1 of the slab (R = 4 G);
// lane l owns blocks l, l+32, ...
template <int N, int R, bool Tap>
__device__ __forceinline__ void gate_up_item(const StreamParams &p, const uint8_t *st, const GuStage &L,
                                             const int4 *const *xr, const float2 *const *sr, int cw, int lane,
                                             uint64_t *empty_bar, float *mid, const ItemTap &tap) {
    const int nb = p.layout.hidden / 32;
    const uint4 *gc = reinterpret_cast<const uint4 *>(st + L.gcodes);
    const uint4 *uc = reinterpret_cast<const uint4 *>(st + L.ucodes);
    const uint16_t *gs = reinterpret_cast<const uint16_t *>(st + L.gsc);
    const uint16_t *us = reinterpret_cast<const uint16_t *>(st + L.usc);
    // Every (row, pair) value in the reference's MMVQ reduction order, so the
    // middle Q8_1 is bit-identical to the reference CPU expert's.  Lane l takes
    // the blocks b % 64 in {l, l + 32}: a0 accumulates b % 64 == l, a1 b % 64 ==
    // l + 32, each as (fragment 0, fragment 1); rows 0..R-1 gate, R..2R-1 up.
    // After each pair's butterflies lane r < R holds gate and up of row R*cw + r.
    static_assert(R <= 32, "a matrix's rows fit one reduce-scatter");
    float gsel[N], usel[N];
#pragma unroll
    for (int j = 0; j < N; ++j) {
#pragma unroll
        for (int mtx = 0; mtx < 2; ++mtx) {   // gate rows, then up rows
            const uint4 *cd = mtx ? uc : gc;
            const uint16_t *sd = mtx ? us : gs;
            uint64_t a0[R], a1[R];
#pragma unroll
            for (int r = 0; r < R; ++r) a0[r] = a1[r] = 0ull;
            for (int b0 = lane; b0 < nb; b0 += 64) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int b = b0 + 32 * half;
                    if (b >= nb) break;
                    const int4 lo = __ldg(xr[j] + 2 * b), hi = __ldg(xr[j] + 2 * b + 1);
                    const float2 sc = __ldg(sr[j] + b);
                    const float m4 = -(4.0f * sc.y);
                    const uint64_t d8 = pkf2(sc.x, sc.x), m4p = pkf2(m4, m4);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int blk = (cw * R + r) * nb + b;
                        const uint4 w = cd[blk];
                        const float d4 = h2f(sd[blk]);
                        int f0, f1;
                        frag_dots(w, lo, hi, f0, f1);
                        const uint64_t dots = pkf2(small_int_to_float(f0), small_int_to_float(f1));
                        if (half) a1[r] = mmvq_term2(dots, pkf2(d4, d4), d8, m4p, a1[r]);
                        else a0[r] = mmvq_term2(dots, pkf2(d4, d4), d8, m4p, a0[r]);
                        if constexpr (Tap) {
                            if (tap.dst0) tap.put(mtx ? tap.dst1 : tap.dst0, j, cw * R + r, b, f0 + f1);
                        }
                    }
                }
            }
            float leaf[R];
#pragma unroll
            for (int r = 0; r < R; ++r) leaf[r] = mmvq_leaf(a0[r], a1[r]);
            const float tot = warp_tree_sum_n<R>(leaf, lane);   // lane l: row l % R
            if (mtx) usel[j] = tot;
            else gsel[j] = tot;
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar);   // slab fully read by this warp
    // SiLU(gate) * up with the reference's sanitisation (session_ops.hip:250-262):
    // lane r < R finishes row R*cw + r, the exponentials of the item's pairs together.
    if (lane < R) {
        int fl[N];
        float gv[N], uv[N], ng[N], ex[N];
#pragma unroll
        for (int j = 0; j < N; ++j) {
            fl[j] = 0;
            gv[j] = operand(gsel[j], fl[j]);
            uv[j] = operand(usel[j], fl[j]);
            ng[j] = -gv[j];
        }
        expf_ref_n<N>(ng, ex);
#pragma unroll
        for (int j = 0; j < N; ++j) {
            int flags = fl[j];
            const float act = arithmetic(__fdiv_rn(gv[j], __fadd_rn(1.0f, ex[j])), flags);
            const float v = arithmetic(__fmul_rn(act, uv[j]), flags);
            mid[j * 32 + cw * R + lane] = flags ? 0.0f : v;
            report(flags, p.error);
        }
    }
}

template <int G, bool Tap>
__global__ void __launch_bounds__(kStreamThreads, 1)
stream_gate_up_kernel(StreamParams p) {
    static_assert(G >= 1 && G <= kGuGroupsMax && kConsumerWarps % G == 0, "consumer groups");
    constexpr int kGroupWarps = kConsumerWarps / G, R = kGuRows / kGroupWarps;
    extern __shared__ __align__(128) uint8_t smem[];
    const int H = p.layout.hidden, I = p.layout.inter, nb = H / 32, slabs = I / kGuRows;
    const GuStage L(H);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMaxStages;
    float *smid = reinterpret_cast<float *>(smem + 128);                 // [groups][2][kGemvTile][32]
    uint8_t *stages = smem + 128 + kGuGroupsMax * 2 * kGemvTile * 32 * 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    init_ring(full, empty, p.stages, kGroupWarps);
    grid_dependency_wait();     // tile list and x codes of the routing kernels
    grid_launch_dependents();   // the down kernel may take SMs as this grid's CTAs finish
    const ItemOrder order = item_order(p.num_tiles, slabs);

    if (warp == 0) {
        if (lane != 0) return;
        stream_producer(p, stages, full, empty, order, slabs,
                        [&](int item, uint8_t *st, uint64_t *bar, const TileRec &rec) {
            const int slab = item % slabs;
            const uint8_t *ex = p.weights + static_cast<size_t>(rec.e) * p.layout.bytes;
            const uint32_t code_bytes = kGuRows * nb * 16, sc_bytes = kGuRows * nb * 2;
            mbar_arrive_expect_tx(bar, 2 * code_bytes + 2 * sc_bytes);
            bulk_g2s(st + L.gcodes, ex + p.layout.gate_codes + static_cast<size_t>(slab) * code_bytes, code_bytes, bar);
            bulk_g2s(st + L.ucodes, ex + p.layout.up_codes + static_cast<size_t>(slab) * code_bytes, code_bytes, bar);
            bulk_g2s(st + L.gsc, ex + p.layout.gate_scales + static_cast<size_t>(slab) * sc_bytes, sc_bytes, bar);
            bulk_g2s(st + L.usc, ex + p.layout.up_scales + static_cast<size_t>(slab) * sc_bytes, sc_bytes, bar);
        });
        return;
    }

    const int grp = (warp - 1) / kGroupWarps, cw = (warp - 1) % kGroupWarps;
    bool failed = false;
    int i = 0;
    const int tap_base = (Tap && p.tap.expert >= 0) ? *p.tap.pair0 : 0;
    for (int pos = blockIdx.x; pos < order.total; pos += gridDim.x, ++i) {
        if (i % G != grp) continue;   // the other group's item
        const int item = order(pos);
        const TileRec rec = load_tile(p.tiles + item / slabs);
        const int n = rec.n < kGemvTile ? rec.n : kGemvTile;
        const int4 *xr[kGemvTile];
        const float2 *sr[kGemvTile];
#pragma unroll
        for (int j = 0; j < kGemvTile; ++j) {
            const int t = j < n ? rec.tok[j] : rec.tok[0];
            xr[j] = reinterpret_cast<const int4 *>(p.x.codes + static_cast<size_t>(t) * H);
            sr[j] = p.x.scales + static_cast<size_t>(t) * nb;
            if (j < n) {   // pull the tile's activation lines into L1 while the weights stream in
                for (int b = lane; b < nb; b += 32) prefetch_l1(xr[j] + 2 * b);
                if (lane * 16 < nb) prefetch_l1(sr[j] + lane * 16);
            }
        }
        const int s = i % p.stages;
        if (!failed && !mbar_wait(&full[s], (i / p.stages) & 1, p.error)) failed = true;
        float *mid = smid + (grp * 2 + ((i / G) & 1)) * kGemvTile * 32;
        ItemTap tap;
        if (Tap && rec.e == p.tap.expert) {
            tap.dst0 = p.tap.gate;
            tap.dst1 = p.tap.up;
            tap.pl = rec.p0 - tap_base;
            tap.rows = I;
            tap.nb = nb;
            tap.row0 = (item % slabs) * kGuRows;
            tap.max_pairs = p.tap.max_pairs;
        }
        if (!failed) {
            const uint8_t *st = stages + static_cast<size_t>(s) * p.stage_bytes;
            switch (n) {
            case 1: gate_up_item<1, R, Tap>(p, st, L, xr, sr, cw, lane, &empty[s], mid, tap); break;
            case 2: gate_up_item<2, R, Tap>(p, st, L, xr, sr, cw, lane, &empty[s], mid, tap); break;
            case 3: gate_up_item<3, R, Tap>(p, st, L, xr, sr, cw, lane, &empty[s], mid, tap); break;
            default: gate_up_item<4, R, Tap>(p, st, L, xr, sr, cw, lane, &empty[s], mid, tap); break;
            }
        }
        named_barrier(1 + grp, kGroupWarps * 32);   // every warp of the group, even after a failed wait
        if (failed) continue;
        const int slab = item % slabs;
        for (int j = cw; j < n; j += kGroupWarps) {
            const Q8Lane q = quantize_lane(mid[j * 32 + lane]);
            const size_t pair = static_cast<size_t>(rec.p0 + j);
            p.mid.codes[pair * I + slab * 32 + lane] = q.code;
            if (lane == 0) {
                p.mid.scales[pair * slabs + slab] = make_float2(h2f(q.d), h2f(q.s));
                report(q.flags, p.error);
            }
            if constexpr (Tap) {
                const int pl = rec.p0 + j - tap_base;
                if (rec.e == p.tap.expert && pl >= 0 && pl < p.tap.max_pairs) {
                    p.tap.mid_codes[static_cast<size_t>(pl) * I + slab * 32 + lane] = q.code;
                    if (lane == 0) p.tap.mid_ds[static_cast<size_t>(pl) * slabs + slab] = q.d | (uint32_t(q.s) << 16);
                }
            }
        }
    }
}

// ---- down + router-weighted scatter-add -------------------------------------
// Consumer warp cw owns rows 8R*cw .. 8R*cw+8R-1 of the 128-row slab (R =
// kDnLaneRows): lane l takes rows 8R*cw + l/4 + 8k (k < R) and blocks l%4,
// l%4+4, ...; two shuffles finish each row, then out[token][row] += weight * y
// (red.global.add).
template <int N, bool Q41, bool Trace, bool Tap>
__device__ __forceinline__ void down_item(const uint8_t *st, const DnStage &L, int I, int H, int row0,
                                          int lr0, int q, uint64_t *empty_bar, int lane, const DownSink &sink,
                                          int *error, const TapSink &tsink, int tap_base) {
    const int nb = I / 32;
    const TileRec &meta = *reinterpret_cast<const TileRec *>(st);
    const int me = meta.e, mp0 = meta.p0;   // read before the stage is released
    ItemTap tap;
    if (Tap && me == tsink.expert) {
        tap.dst0 = tsink.down;
        tap.pl = mp0 - tap_base;
        tap.rows = H;
        tap.nb = I / 32;
        tap.row0 = row0 - lr0;
        tap.max_pairs = tsink.max_pairs;
    }
    const uint4 *dc = reinterpret_cast<const uint4 *>(st + L.dcodes);
    const uint16_t *ds = reinterpret_cast<const uint16_t *>(st + L.dsc);
    const uint16_t *dm = reinterpret_cast<const uint16_t *>(st + L.dmin);
    const int4 *mc = reinterpret_cast<const int4 *>(st + L.mcodes);
    const float2 *ms = reinterpret_cast<const float2 *>(st + L.msc);
    constexpr int R = kDnLaneRows;
    static_assert(R % 2 == 0, "down rows are accumulated in f32x2 pairs");
    int tok[N];
    float w[N];
    uint64_t acc2[R / 2][N];   // rows (lr0 + 16p, lr0 + 16p + 8) packed as f32x2
#pragma unroll
    for (int j = 0; j < N; ++j) {
        tok[j] = meta.tok[j];
        w[j] = meta.w[j];
#pragma unroll
        for (int k = 0; k < R / 2; ++k) acc2[k][j] = 0ull;
    }
    float acc[R][N];
    if constexpr (Q41) {
        // Q4_1: every (row, block) needs its own half-rounded products, so
        // the terms stay scalar.
#pragma unroll
        for (int k = 0; k < R; ++k)
#pragma unroll
            for (int j = 0; j < N; ++j) acc[k][j] = 0.0f;
        for (int b = q; b < nb; b += 4) {
            uint4 wk[R];
            float d4[R], m4[R];
#pragma unroll
            for (int k = 0; k < R; ++k) {
                wk[k] = dc[(lr0 + 8 * k) * nb + b];
                d4[k] = h2f(ds[(lr0 + 8 * k) * nb + b]);
                m4[k] = h2f(dm[(lr0 + 8 * k) * nb + b]);
            }
#pragma unroll
            for (int j = 0; j < N; ++j) {
                const int4 xlo = mc[j * (I / 16) + 2 * b], xhi = mc[j * (I / 16) + 2 * b + 1];
                const float2 sc = ms[j * nb + b];
#pragma unroll
                for (int k = 0; k < R; ++k)
                    acc[k][j] = block_term_q4_1(block_dot2(wk[k], xlo, xhi), d4[k], m4[k], sc.x, sc.y, acc[k][j]);
                if constexpr (Tap) {
                    if (tap.dst0)
#pragma unroll
                        for (int k = 0; k < R; ++k) tap.put(tap.dst0, j, lr0 + 8 * k, b, block_dot(wk[k], xlo, xhi));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar);   // stage fully read by this warp
    } else {
        for (int b = q; b < nb; b += 4) {
            uint4 wk[R];
            uint64_t dk[R / 2];
#pragma unroll
            for (int k = 0; k < R; ++k) wk[k] = dc[(lr0 + 8 * k) * nb + b];
#pragma unroll
            for (int k = 0; k < R / 2; ++k)
                dk[k] = pkf2(h2f(ds[(lr0 + 16 * k) * nb + b]), h2f(ds[(lr0 + 16 * k + 8) * nb + b]));
#pragma unroll
            for (int j = 0; j < N; ++j) {
                const int4 xlo = mc[j * (I / 16) + 2 * b], xhi = mc[j * (I / 16) + 2 * b + 1];
                const float2 sc = ms[j * nb + b];
                const float ns = -(8.0f * sc.y);
                const uint64_t d8 = pkf2(sc.x, sc.x), nsp = pkf2(ns, ns);
#pragma unroll
                for (int k = 0; k < R / 2; ++k)
                    acc2[k][j] = block_term2(block_dot2(wk[2 * k], xlo, xhi), block_dot2(wk[2 * k + 1], xlo, xhi),
                                             dk[k], d8, nsp, acc2[k][j]);
                if constexpr (Tap) {
                    if (tap.dst0)
#pragma unroll
                        for (int k = 0; k < R; ++k) tap.put(tap.dst0, j, lr0 + 8 * k, b, block_dot(wk[k], xlo, xhi));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar);   // stage fully read by this warp
#pragma unroll
        for (int k = 0; k < R / 2; ++k)
#pragma unroll
            for (int j = 0; j < N; ++j) upk2(acc2[k][j], acc[2 * k][j], acc[2 * k + 1][j]);
    }
#pragma unroll
    for (int k = 0; k < R; ++k)
#pragma unroll
        for (int j = 0; j < N; ++j) {
            float v = acc[k][j];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            if ((j & 3) == q) sink.put<Trace>(me, mp0, tok[j], j, row0 + 8 * k, H, v, w[j], error);
        }
}

template <bool Trace, bool Tap>
__global__ void __launch_bounds__(kStreamThreads, 1)
stream_down_kernel(StreamParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int H = p.layout.hidden, I = p.layout.inter, nb = I / 32, slabs = H / kDnRows;
    const DnStage L(I);
    const bool q41 = p.layout.down_type == kDownQ4_1;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMaxStages;
    uint8_t *stages = smem + 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    init_ring(full, empty, p.stages, kConsumerWarps);
    grid_launch_dependents();   // the next layer's routing CTAs may take the SMs' spare room and wait
    const ItemOrder order = item_order(p.num_tiles, slabs);

    if (warp == 0) {
        // Producer.  The tile list comes from the routing kernels, which
        // completed before the gate/up grid started, so the weights of the
        // first ring stages stream while gate/up finishes; the middle
        // activations of those stages are fetched after grid_dependency_wait.
        if (lane != 0) return;
        const uint32_t code_bytes = kDnRows * nb * 16, sc_bytes = kDnRows * nb * 2;
        auto issue_mid = [&](uint8_t *st, uint64_t *bar, const TileRec &rec) {
            // the tile's pairs are consecutive: one copy each for codes and scales
            bulk_g2s(st + L.mcodes, p.mid.codes + static_cast<size_t>(rec.p0) * I, rec.n * I, bar);
            bulk_g2s(st + L.msc, p.mid.scales + static_cast<size_t>(rec.p0) * nb, rec.n * nb * 8, bar);
        };
        bool dep = false;
        int i = 0;
        auto resolve = [&]() {   // wait for gate/up, then the middle rows of the stages already armed
            grid_dependency_wait();
            dep = true;
            for (int k = 0; k < i; ++k) {
                uint8_t *st = stages + static_cast<size_t>(k % p.stages) * p.stage_bytes;
                issue_mid(st, &full[k % p.stages], *reinterpret_cast<const TileRec *>(st));
            }
        };
        for (int pos = blockIdx.x; pos < order.total; pos += gridDim.x, ++i) {
            const int item = order(pos);
            const TileRec rec = load_tile(p.tiles + item / slabs);
            const int s = i % p.stages;
            if (i >= p.stages) {
                if (!dep) resolve();
                if (!mbar_wait(&empty[s], ((i / p.stages) & 1) ^ 1, p.error)) break;
            }
            uint8_t *st = stages + static_cast<size_t>(s) * p.stage_bytes;
            *reinterpret_cast<TileRec *>(st) = rec;
            const int slab = item % slabs;
            const uint8_t *ex = p.weights + static_cast<size_t>(rec.e) * p.layout.bytes;
            mbar_arrive_expect_tx(&full[s], code_bytes + (q41 ? 2 : 1) * sc_bytes + rec.n * (I + nb * 8));
            bulk_g2s(st + L.dcodes, ex + p.layout.down_codes + static_cast<size_t>(slab) * code_bytes, code_bytes,
                     &full[s]);
            bulk_g2s(st + L.dsc, ex + p.layout.down_scales + static_cast<size_t>(slab) * sc_bytes, sc_bytes,
                     &full[s]);
            if (q41)
                bulk_g2s(st + L.dmin, ex + p.layout.down_mins + static_cast<size_t>(slab) * sc_bytes, sc_bytes,
                         &full[s]);
            if (dep) issue_mid(st, &full[s], rec);
        }
        if (!dep) resolve();
        // keep the CTA alive until every issued copy has landed
        for (int k = i - p.stages > 0 ? i - p.stages : 0; k < i; ++k)
            mbar_wait(&full[k % p.stages], (k / p.stages) & 1, p.error);
        return;
    }

    const int cw = warp - 1, q = lane & 3;
    const int lr0 = cw * 8 * kDnLaneRows + (lane >> 2);
    const int tap_base = (Tap && p.tap.expert >= 0) ? *p.tap.pair0 : 0;
    int i = 0;
    for (int pos = blockIdx.x; pos < order.total; pos += gridDim.x, ++i) {
        const int item = order(pos);
        const int s = i % p.stages;
        if (!mbar_wait(&full[s], (i / p.stages) & 1, p.error)) break;
        const uint8_t *st = stages + static_cast<size_t>(s) * p.stage_bytes;
        const int n = reinterpret_cast<const TileRec *>(st)->n;
        const int row0 = (item % slabs) * kDnRows + lr0;
        if (q41) {
            switch (n) {
            case 1:
                down_item<1, true, Trace, Tap>(st, L, I, H, row0, lr0, q, &empty[s], lane, p.sink, p.error,
                                                            p.tap, tap_base);
                break;
            case 2:
                down_item<2, true, Trace, Tap>(st, L, I, H, row0, lr0, q, &empty[s], lane, p.sink, p.error,
                                                            p.tap, tap_base);
                break;
            case 3:
                down_item<3, true, Trace, Tap>(st, L, I, H, row0, lr0, q, &empty[s], lane, p.sink, p.error,
                                                            p.tap, tap_base);
                break;
            default:
                down_item<4, true, Trace, Tap>(st, L, I, H, row0, lr0, q, &empty[s], lane, p.sink, p.error,
                                                            p.tap, tap_base);
                break;
            }
        } else {
            switch (n) {
            case 1:
                down_item<1, false, Trace, Tap>(st, L, I, H, row0, lr0, q, &empty[s], lane, p.sink, p.error,
                                                            p.tap, tap_base);
                break;
            case 2:
                down_item<2, false, Trace, Tap>(st, L, I, H, row0, lr0, q, &empty[s], lane, p.sink, p.error,
                                                            p.tap, tap_base);
                break;
            case 3:
                down_item<3, false, Trace, Tap>(st, L, I, H, row0, lr0, q, &empty[s], lane, p.sink, p.error,
                                                            p.tap, tap_base);
                break;
            default:
                down_item<4, false, Trace, Tap>(st, L, I, H, row0, lr0, q, &empty[s], lane, p.sink, p.error,
                                                            p.tap, tap_base);
                break;
            }
        }
    }
}

inline int stream_stages(uint32_t stage_bytes, int limit) {
    const uint32_t budget = 227 * 1024 - 1024;
    int s = static_cast<int>(budget / stage_bytes);
    return s < limit ? s : limit;
}

}  // namespace qmoe
