// stream_kernels.cuh -- persistent weight-streaming expert kernels (decode and
// small groups).  One CTA per SM: warp 0 is the producer, which streams each
// work item's weight slab, activation rows and scales into a ring of
// shared-memory stages with cp.async.bulk (completion counted on an mbarrier);
// warps 1..8 are consumers that run the u4 x s8 dp4a dots out of shared
// memory and release the stage on an "empty" mbarrier.  Every SM keeps one to
// two ~90 KB stages in flight, so HBM latency is covered by bytes in flight
// rather than by resident warps.
#pragma once
#include "common.cuh"
#include "expert_kernels.cuh"
#include "ptx.cuh"

namespace qmoe {

constexpr int kConsumerWarps = 8;
constexpr int kStreamThreads = 32 * (kConsumerWarps + 1);
constexpr int kGuRows = 32;    // gate rows and up rows per item: one Q8_1 middle block
constexpr int kDnRows = 128;   // down rows per item
constexpr int kMaxStages = 4;

struct StreamParams {
    const uint8_t *weights;
    ExpertLayout layout;
    Q8Planar x, mid;
    const TileRec *tiles;
    const int *num_tiles;
    float *out;
    int *error;
    int stages;
    uint32_t stage_bytes;
};

// ---- stage layouts -------------------------------------------------------
struct GuStage {
    uint32_t meta, gcodes, ucodes, gsc, usc, xcodes, xsc, bytes;
    __host__ __device__ GuStage(int H) {
        const uint32_t nb = H / 32;
        meta = 0;
        gcodes = 128;
        ucodes = gcodes + kGuRows * nb * 16;
        gsc = ucodes + kGuRows * nb * 16;
        usc = gsc + kGuRows * nb * 2;
        xcodes = usc + kGuRows * nb * 2;
        xsc = xcodes + kGemvTile * H;
        bytes = xsc + kGemvTile * nb * 8;
        bytes = (bytes + 127) & ~127u;
    }
};

struct DnStage {
    uint32_t meta, dcodes, dsc, mcodes, msc, bytes;
    __host__ __device__ DnStage(int I) {
        const uint32_t nb = I / 32;
        meta = 0;
        dcodes = 128;
        dsc = dcodes + kDnRows * nb * 16;
        mcodes = dsc + kDnRows * nb * 2;
        msc = mcodes + kGemvTile * I;
        bytes = msc + kGemvTile * nb * 8;
        bytes = (bytes + 127) & ~127u;
    }
};

__device__ __forceinline__ TileRec load_tile(const TileRec *t) {
    TileRec r;
    const int4 *s = reinterpret_cast<const int4 *>(t);
    int4 *d = reinterpret_cast<int4 *>(&r);
#pragma unroll
    for (int i = 0; i < 5; ++i) d[i] = __ldg(s + i);
    return r;
}

// Common producer loop: `issue(item, stage_ptr, bar, rec)` enqueues the bulk
// copies of one item and returns their byte count.
template <class Issue>
__device__ __forceinline__ void stream_producer(const StreamParams &p, uint8_t *stages, uint64_t *full,
                                                uint64_t *empty, int total, int slabs, Issue issue) {
    int i = 0;
    int item = blockIdx.x;
    TileRec next;
    if (item < total) next = load_tile(p.tiles + item / slabs);
    for (; item < total; item += gridDim.x, ++i) {
        const TileRec rec = next;
        const int following = item + gridDim.x;
        if (following < total) next = load_tile(p.tiles + following / slabs);
        const int s = i % p.stages;
        if (i >= p.stages && !mbar_wait(&empty[s], ((i / p.stages) & 1) ^ 1, p.error)) break;
        uint8_t *st = stages + static_cast<size_t>(s) * p.stage_bytes;
        *reinterpret_cast<TileRec *>(st) = rec;        // meta, published by the arrive below
        issue(item, st, &full[s], rec);
    }
    // Keep the CTA alive until every issued copy has landed.
    const int issued = i;
    for (int k = issued - p.stages > 0 ? issued - p.stages : 0; k < issued; ++k)
        mbar_wait(&full[k % p.stages], (k / p.stages) & 1, p.error);
}

// ---- gate/up + SiLU*up + Q8_1 middle ---------------------------------------
__global__ void __launch_bounds__(kStreamThreads, 1)
stream_gate_up_kernel(StreamParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int H = p.layout.hidden, I = p.layout.inter, nb = H / 32, slabs = I / kGuRows;
    const GuStage L(H);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMaxStages;
    float *smid = reinterpret_cast<float *>(smem + 128);                 // [2][kGemvTile][32]
    uint8_t *stages = smem + 128 + 2 * kGemvTile * 32 * 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], kConsumerWarps); }
        mbar_fence_init();
    }
    __syncthreads();
    const int total = *p.num_tiles * slabs;

    if (warp == 0) {
        if (lane != 0) return;
        stream_producer(p, stages, full, empty, total, slabs,
                        [&](int item, uint8_t *st, uint64_t *bar, const TileRec &rec) {
            const int slab = item % slabs;
            const uint8_t *ex = p.weights + static_cast<size_t>(rec.e) * p.layout.bytes;
            const uint32_t code_bytes = kGuRows * nb * 16, sc_bytes = kGuRows * nb * 2;
            const uint32_t bytes = 2 * code_bytes + 2 * sc_bytes + rec.n * (H + nb * 8);
            mbar_arrive_expect_tx(bar, bytes);
            bulk_g2s(st + L.gcodes, ex + p.layout.gate_codes + static_cast<size_t>(slab) * code_bytes, code_bytes, bar);
            bulk_g2s(st + L.ucodes, ex + p.layout.up_codes + static_cast<size_t>(slab) * code_bytes, code_bytes, bar);
            bulk_g2s(st + L.gsc, ex + p.layout.gate_scales + static_cast<size_t>(slab) * sc_bytes, sc_bytes, bar);
            bulk_g2s(st + L.usc, ex + p.layout.up_scales + static_cast<size_t>(slab) * sc_bytes, sc_bytes, bar);
            for (int j = 0; j < rec.n; ++j) {
                bulk_g2s(st + L.xcodes + j * H, p.x.codes + static_cast<size_t>(rec.tok[j]) * H, H, bar);
                bulk_g2s(st + L.xsc + j * nb * 8, p.x.scales + static_cast<size_t>(rec.tok[j]) * nb, nb * 8, bar);
            }
        });
        return;
    }

    const int cw = warp - 1;
    int i = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x, ++i) {
        const int s = i % p.stages;
        if (!mbar_wait(&full[s], (i / p.stages) & 1, p.error)) break;
        const uint8_t *st = stages + static_cast<size_t>(s) * p.stage_bytes;
        const TileRec &meta = *reinterpret_cast<const TileRec *>(st);
        const int n = meta.n, p0 = meta.p0, slab = item % slabs;
        const uint4 *gc = reinterpret_cast<const uint4 *>(st + L.gcodes);
        const uint4 *uc = reinterpret_cast<const uint4 *>(st + L.ucodes);
        const uint16_t *gs = reinterpret_cast<const uint16_t *>(st + L.gsc);
        const uint16_t *us = reinterpret_cast<const uint16_t *>(st + L.usc);
        const int4 *xc = reinterpret_cast<const int4 *>(st + L.xcodes);
        const float2 *xs = reinterpret_cast<const float2 *>(st + L.xsc);
        float acc[8][kGemvTile];
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int j = 0; j < kGemvTile; ++j) acc[r][j] = 0.0f;
        for (int b = lane; b < nb; b += 32) {
            uint4 wc[8];
            float d4[8];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int blk = (cw * 4 + r) * nb + b;
                wc[r] = gc[blk];
                wc[4 + r] = uc[blk];
                d4[r] = h2f(gs[blk]);
                d4[4 + r] = h2f(us[blk]);
            }
#pragma unroll
            for (int j = 0; j < kGemvTile; ++j) {
                if (j < n) {
                    const int4 xlo = xc[j * (H / 16) + 2 * b], xhi = xc[j * (H / 16) + 2 * b + 1];
                    const float2 sc = xs[j * nb + b];
                    const float s8x8 = 8.0f * sc.y;
#pragma unroll
                    for (int r = 0; r < 8; ++r)
                        acc[r][j] = block_term(block_dot(wc[r], xlo, xhi), d4[r], sc.x, s8x8, acc[r][j]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);   // stage fully read by this warp
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int j = 0; j < kGemvTile; ++j)
                if (j < n) acc[r][j] = warp_sum(acc[r][j]);
        float *mid = smid + (i & 1) * kGemvTile * 32;
        if (lane < 4) {
#pragma unroll
            for (int j = 0; j < kGemvTile; ++j) {
                if (j < n) {
                    float g = acc[0][j], u = acc[4][j];
#pragma unroll
                    for (int r = 1; r < 4; ++r)
                        if (lane == r) { g = acc[r][j]; u = acc[4 + r][j]; }
                    int flags = 0;
                    g = operand(g, flags);
                    u = operand(u, flags);
                    const float act = arithmetic(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), flags);
                    const float v = arithmetic(__fmul_rn(act, u), flags);
                    mid[j * 32 + cw * 4 + lane] = flags ? 0.0f : v;
                    report(flags, p.error);
                }
            }
        }
        named_barrier(1, 32 * kConsumerWarps);
        for (int j = cw; j < n; j += kConsumerWarps) {
            const Q8Lane q = quantize_lane(mid[j * 32 + lane]);
            const size_t pair = static_cast<size_t>(p0 + j);
            p.mid.codes[pair * I + slab * 32 + lane] = q.code;
            if (lane == 0) {
                p.mid.scales[pair * slabs + slab] = make_float2(h2f(q.d), h2f(q.s));
                report(q.flags, p.error);
            }
        }
    }
}

// ---- down + router-weighted scatter-add -------------------------------------
__global__ void __launch_bounds__(kStreamThreads, 1)
stream_down_kernel(StreamParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int H = p.layout.hidden, I = p.layout.inter, nb = I / 32, slabs = H / kDnRows;
    const DnStage L(I);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMaxStages;
    uint8_t *stages = smem + 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], kConsumerWarps); }
        mbar_fence_init();
    }
    __syncthreads();
    const int total = *p.num_tiles * slabs;

    if (warp == 0) {
        if (lane != 0) return;
        stream_producer(p, stages, full, empty, total, slabs,
                        [&](int item, uint8_t *st, uint64_t *bar, const TileRec &rec) {
            const int slab = item % slabs;
            const uint8_t *ex = p.weights + static_cast<size_t>(rec.e) * p.layout.bytes;
            const uint32_t code_bytes = kDnRows * nb * 16, sc_bytes = kDnRows * nb * 2;
            const uint32_t bytes = code_bytes + sc_bytes + rec.n * (I + nb * 8);
            mbar_arrive_expect_tx(bar, bytes);
            bulk_g2s(st + L.dcodes, ex + p.layout.down_codes + static_cast<size_t>(slab) * code_bytes, code_bytes, bar);
            bulk_g2s(st + L.dsc, ex + p.layout.down_scales + static_cast<size_t>(slab) * sc_bytes, sc_bytes, bar);
            // the tile's pairs are consecutive: one copy each for codes and scales
            bulk_g2s(st + L.mcodes, p.mid.codes + static_cast<size_t>(rec.p0) * I, rec.n * I, bar);
            bulk_g2s(st + L.msc, p.mid.scales + static_cast<size_t>(rec.p0) * nb, rec.n * nb * 8, bar);
        });
        return;
    }

    const int cw = warp - 1, half = lane >> 4, hl = lane & 15;
    int i = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x, ++i) {
        const int s = i % p.stages;
        if (!mbar_wait(&full[s], (i / p.stages) & 1, p.error)) break;
        const uint8_t *st = stages + static_cast<size_t>(s) * p.stage_bytes;
        const TileRec meta = *reinterpret_cast<const TileRec *>(st);
        const int n = meta.n, slab = item % slabs;
        const uint4 *dc = reinterpret_cast<const uint4 *>(st + L.dcodes);
        const uint16_t *ds = reinterpret_cast<const uint16_t *>(st + L.dsc);
        const int4 *mc = reinterpret_cast<const int4 *>(st + L.mcodes);
        const float2 *ms = reinterpret_cast<const float2 *>(st + L.msc);
        float res[kDnRows / kConsumerWarps / 2][kGemvTile];
#pragma unroll
        for (int pass = 0; pass < kDnRows / kConsumerWarps / 2; ++pass) {
            const int lr = cw * (kDnRows / kConsumerWarps) + pass * 2 + half;
            float acc[kGemvTile];
#pragma unroll
            for (int j = 0; j < kGemvTile; ++j) acc[j] = 0.0f;
            for (int b = hl; b < nb; b += 16) {
                const uint4 wc = dc[lr * nb + b];
                const float d4 = h2f(ds[lr * nb + b]);
#pragma unroll
                for (int j = 0; j < kGemvTile; ++j) {
                    if (j < n) {
                        const int4 xlo = mc[j * (I / 16) + 2 * b], xhi = mc[j * (I / 16) + 2 * b + 1];
                        const float2 sc = ms[j * nb + b];
                        acc[j] = block_term(block_dot(wc, xlo, xhi), d4, sc.x, 8.0f * sc.y, acc[j]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kGemvTile; ++j) res[pass][j] = acc[j];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
        for (int pass = 0; pass < kDnRows / kConsumerWarps / 2; ++pass) {
            const int row = slab * kDnRows + cw * (kDnRows / kConsumerWarps) + pass * 2 + half;
#pragma unroll
            for (int j = 0; j < kGemvTile; ++j) {
                if (j < n) {
                    float v = res[pass][j];
                    v += __shfl_xor_sync(0xffffffffu, v, 8);
                    v += __shfl_xor_sync(0xffffffffu, v, 4);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    if (hl == j) {
                        int flags = 0;
                        const float y = arithmetic(v, flags);
                        const float c = arithmetic(__fmul_rn(meta.w[j], y), flags);
                        atomicAdd(p.out + static_cast<size_t>(meta.tok[j]) * H + row, c);
                        report(flags, p.error);
                    }
                }
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
