// ep_kernels.cuh -- expert parallelism over peer memory (NVLink / NVSwitch).
//
// Rank r of P owns routed experts [r*E/P, (r+1)*E/P) plus a replica of the
// shared expert, and its own shard of the tokens.  One forward:
//   1. quantise + route the rank's tokens (top-10 over all 512 experts);
//   2. plan: for every token the set of destination ranks (ranks owning one
//      of its experts, plus the rank itself, which runs the shared expert, so
//      own token t is own slot t) and its slot in each destination's receive
//      region (stable, in token order);
//   3. dispatch: one warp per (token, destination) stores the token's Q8_1
//      row, tensor-core block constants and its (local expert, weight) list
//      straight into the destination's receive buffer (peer stores); the
//      last CTA publishes, per destination, the slot count and the epoch
//      (for T <= 32 the routing launch does steps 2-3 itself: its quantising
//      CTAs store every row into every rank at slot source * T_max + t);
//   4. every rank waits for all P epochs, groups its received slots by local
//      expert (the single-GPU grouping kernels over slot masks) and runs the
//      expert kernels, accumulating each slot's weighted expert outputs into
//      its local partial buffer;
//   5. the combine launch publishes "done" to every peer; after all peers are
//      done, each rank pulls, for each of its tokens, the partial rows from the destinations
//      it used (peer loads, destinations in ascending order) and adds them
//      into its residual.
// Receive regions are fixed per source (slot = source * T_max + index), so no
// global exchange of counts is needed.  Epochs live in device memory and
// advance once per forward on every rank, so a captured CUDA graph replays
// correctly.  Every wait on a peer is bounded (kFlagTimeout on expiry).
#pragma once
#include "common.cuh"
#include "ep_common.cuh"
#include "ptx.cuh"
#include "route_kernels.cuh"

namespace qmoe {

// Plan (one CTA of 1024 threads): destination masks and per-destination
// exclusive positions in token order; also advances the epoch.
__global__ void __launch_bounds__(1024) ep_plan_kernel(EpParams p) {
    __shared__ unsigned long long wsum[2][32];
    __shared__ int running[kEpMaxRanks];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < kEpMaxRanks) running[tid] = 0;
    if (tid == 0) *p.epoch += 1u;
    __syncthreads();
    for (int c = 0; c < p.tokens; c += 1024) {
        const int t = c + tid;
        uint32_t mask = 0u;
        if (t < p.tokens) {
            mask = 1u << p.rank;
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                const int e = p.ids[t * kTopK + k];
                if (e >= 0 && e < p.ecount * p.world) mask |= 1u << (e / p.ecount);
            }
            p.dmask[t] = static_cast<uint8_t>(mask);
        }
        // 16-bit counters per destination packed in two 64-bit words
        unsigned long long lo = 0ull, hi = 0ull;
#pragma unroll
        for (int d = 0; d < 4; ++d) lo |= static_cast<unsigned long long>((mask >> d) & 1u) << (16 * d);
#pragma unroll
        for (int d = 0; d < 4; ++d) hi |= static_cast<unsigned long long>((mask >> (d + 4)) & 1u) << (16 * d);
        unsigned long long ilo = lo, ihi = hi;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long a = __shfl_up_sync(0xffffffffu, ilo, o), b = __shfl_up_sync(0xffffffffu, ihi, o);
            if (lane >= o) { ilo += a; ihi += b; }
        }
        if (lane == 31) { wsum[0][warp] = ilo; wsum[1][warp] = ihi; }
        __syncthreads();
        if (warp == 0) {
            unsigned long long a = wsum[0][lane], b = wsum[1][lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b, o);
                if (lane >= o) { a += x; b += y; }
            }
            wsum[0][lane] = a;   // inclusive warp totals
            wsum[1][lane] = b;
        }
        __syncthreads();
        const unsigned long long plo = (warp ? wsum[0][warp - 1] : 0ull) + ilo - lo;
        const unsigned long long phi = (warp ? wsum[1][warp - 1] : 0ull) + ihi - hi;
        if (t < p.tokens) {
#pragma unroll
            for (int d = 0; d < kEpMaxRanks; ++d) {
                const unsigned long long v = d < 4 ? plo >> (16 * d) : phi >> (16 * (d - 4));
                p.pos[t * kEpMaxRanks + d] = running[d] + static_cast<int>(v & 0xffffu);
            }
        }
        __syncthreads();
        if (tid < kEpMaxRanks) {
            const unsigned long long v = tid < 4 ? wsum[0][31] >> (16 * tid) : wsum[1][31] >> (16 * (tid - 4));
            running[tid] += static_cast<int>(v & 0xffffu);
        }
        __syncthreads();
    }
    if (tid < kEpMaxRanks) p.counts[tid] = running[tid];
}

// Dispatch: one warp per (token, destination).  Peer stores of the row, then
// the last CTA publishes counts and the epoch to every destination.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpParams p) {
    const int lane = threadIdx.x & 31;
    const int H = p.hidden, nb = H / 32;
    const int items = p.tokens * p.world;
    for (int it = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; it < items; it += (gridDim.x * blockDim.x) >> 5) {
        const int t = it / p.world, d = it % p.world;
        if (!((p.dmask[t] >> d) & 1u)) continue;
        const size_t slot = static_cast<size_t>(p.rank) * p.t_max + p.pos[t * kEpMaxRanks + d];
        uint8_t *dst = p.peers.base[d];
        // codes: H bytes as 16-byte vectors
        const uint4 *sc = reinterpret_cast<const uint4 *>(p.xcodes + static_cast<size_t>(t) * H);
        uint4 *dc = reinterpret_cast<uint4 *>(dst + p.L.codes + slot * H);
        for (int i = lane; i < H / 16; i += 32) dc[i] = sc[i];
        // block scales: nb float2
        const uint4 *ss = reinterpret_cast<const uint4 *>(p.xscales + static_cast<size_t>(t) * nb);
        uint4 *ds = reinterpret_cast<uint4 *>(dst + p.L.scales + slot * nb * 8);
        for (int i = lane; i < nb / 2; i += 32) ds[i] = ss[i];
        // (local expert, weight) list: the routed experts d owns (the shared
        // expert of the own tokens is added by the receiver's grouping)
        if (lane < kEpSlotIds) {
            int id = -1;
            float w = 0.0f;
            const int e = p.ids[t * kTopK + lane];
            if (e >= 0 && e / p.ecount == d) {
                id = e - d * p.ecount;
                w = p.weights[t * kTopK + lane];
            }
            reinterpret_cast<int32_t *>(dst + p.L.ids)[slot * kEpSlotIds + lane] = id;
            reinterpret_cast<float *>(dst + p.L.w)[slot * kEpSlotIds + lane] = w;
        }
    }
    // completion: every CTA fences its peer stores before counting itself
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const uint32_t ticket = atomicAdd(p.blocks_done, 1u);
        if (ticket == gridDim.x - 1) {
            __threadfence_system();
            const uint32_t epoch = *p.epoch;
            for (int d = 0; d < p.world; ++d) ep_publish(p, d, static_cast<uint32_t>(p.counts[d]), epoch);
            *p.blocks_done = 0u;
        }
    }
}

// Decode sizes (T <= 32): plan and dispatch in one CTA of 1024 threads.  Warp
// 0 plans with ballots (lane = token), every warp then copies (token,
// destination) rows, and after a CTA barrier lane d of warp 0 publishes to
// destination d -- the release is cumulative over the barrier, so no grid
// ticket and no serial loop over destinations.
__global__ void __launch_bounds__(1024) ep_plan_dispatch_small_kernel(EpParams p) {
    __shared__ uint32_t sm_mask[32];
    __shared__ int sm_pos[32][kEpMaxRanks];
    __shared__ int sm_count[kEpMaxRanks];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int H = p.hidden, nb = H / 32;
    if (warp == 0) {
        const int t = lane;
        uint32_t mask = 0u;
        if (t < p.tokens) {
            mask = 1u << p.rank;
#pragma unroll
            for (int k = 0; k < kTopK; ++k) {
                const int e = p.ids[t * kTopK + k];
                if (e >= 0 && e < p.ecount * p.world) mask |= 1u << (e / p.ecount);
            }
            p.dmask[t] = static_cast<uint8_t>(mask);
        }
        sm_mask[lane] = mask;
#pragma unroll
        for (int d = 0; d < kEpMaxRanks; ++d) {
            const uint32_t b = __ballot_sync(0xffffffffu, (mask >> d) & 1u);
            const int pos = __popc(b & ((1u << lane) - 1u));
            sm_pos[lane][d] = pos;
            if (t < p.tokens) p.pos[t * kEpMaxRanks + d] = pos;
            if (lane == 0) sm_count[d] = __popc(b);
        }
        if (lane == 0) *p.epoch += 1u;
    }
    __syncthreads();
    for (int it = warp; it < p.tokens * p.world; it += 32) {
        const int t = it / p.world, d = it % p.world;
        if (!((sm_mask[t] >> d) & 1u)) continue;
        const size_t slot = static_cast<size_t>(p.rank) * p.t_max + sm_pos[t][d];
        uint8_t *dst = p.peers.base[d];
        const uint4 *sc = reinterpret_cast<const uint4 *>(p.xcodes + static_cast<size_t>(t) * H);
        uint4 *dc = reinterpret_cast<uint4 *>(dst + p.L.codes + slot * H);
        for (int i = lane; i < H / 16; i += 32) dc[i] = sc[i];
        const uint4 *ss = reinterpret_cast<const uint4 *>(p.xscales + static_cast<size_t>(t) * nb);
        uint4 *ds = reinterpret_cast<uint4 *>(dst + p.L.scales + slot * nb * 8);
        for (int i = lane; i < nb / 2; i += 32) ds[i] = ss[i];
        if (lane < kEpSlotIds) {
            int id = -1;
            float w = 0.0f;
            const int e = p.ids[t * kTopK + lane];
            if (e >= 0 && e / p.ecount == d) {
                id = e - d * p.ecount;
                w = p.weights[t * kTopK + lane];
            }
            reinterpret_cast<int32_t *>(dst + p.L.ids)[slot * kEpSlotIds + lane] = id;
            reinterpret_cast<float *>(dst + p.L.w)[slot * kEpSlotIds + lane] = w;
        }
    }
    __syncthreads();
    if (warp == 0 && lane < p.world)   // the system-scope release orders the whole CTA's stores (barrier above)
        ep_publish(p, lane, static_cast<uint32_t>(sm_count[lane]), *p.epoch);
    if (threadIdx.x < kEpMaxRanks) p.counts[threadIdx.x] = sm_count[threadIdx.x];
}

// Wait until every source has published the current epoch in its receive
// word (one lane per peer, bounded by ~2^31 cycles).
__global__ void ep_wait_kernel(const uint64_t *recv, const uint32_t *epoch, int world, int *error) {
    const int d = threadIdx.x;
    if (d >= world) return;
    const uint32_t want = *epoch;
    const long long t0 = clock64();
    while (static_cast<uint32_t>(ld_acquire_sys64(&recv[d])) != want) {
        if (clock64() - t0 > (1ll << 31)) {
            atomicOr(error, kFlagTimeout);
            return;
        }
        __nanosleep(64);
    }
}

// Received slots -> chunk masks over local experts (32 slots per CTA).  The
// partial rows of the slots start at zero: the combine of the previous epoch
// cleared every row it consumed.
struct EpGroupParams {
    const uint8_t *arena;   // own exported arena
    EpLayout L;
    int t_max, slots, hidden;
    uint32_t *masks;        // [slots/32][512]
    float *partial;
};
__device__ __forceinline__ bool ep_slot_valid(const EpCtl *c, int slot, int t_max) {
    return static_cast<uint32_t>(slot % t_max) < static_cast<uint32_t>(c->recv[slot / t_max] >> 32);
}
__global__ void __launch_bounds__(256) ep_masks_kernel(EpGroupParams g) {
    __shared__ uint32_t smask[kRouterExperts];
    const EpCtl *c = reinterpret_cast<const EpCtl *>(g.arena + g.L.ctl);
    const int32_t *ids = reinterpret_cast<const int32_t *>(g.arena + g.L.ids);
    for (int e = threadIdx.x; e < kRouterExperts; e += blockDim.x) smask[e] = 0u;
    __syncthreads();
    const int s0 = blockIdx.x * kChunk;
    for (int i = threadIdx.x; i < kChunk * kEpSlotIds; i += blockDim.x) {
        const int j = i / kEpSlotIds, k = i % kEpSlotIds, slot = s0 + j;
        if (slot < g.slots && ep_slot_valid(c, slot, g.t_max)) {
            const int id = ids[static_cast<size_t>(slot) * kEpSlotIds + k];
            if (id >= 0 && id < kRouterExperts) atomicOr(&smask[id], 1u << j);
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kRouterExperts; e += blockDim.x)
        g.masks[static_cast<size_t>(blockIdx.x) * kRouterExperts + e] = smask[e];
}

// Decode-size receive side (slots <= 512, one CTA of 512 threads, thread =
// local expert): wait for every source's dispatch, chunk masks in shared
// memory, counts, scan, stable placement of the pairs, the own tokens'
// shared-expert pairs and the work-tile list -- the work of ep_wait, ep_masks,
// route_chunk_prefix, route_scan and ep_scatter in one launch.
struct EpSmallGroupParams {
    const uint8_t *arena;
    EpLayout L;
    int t_max, slots, world, tokens, has_shared, shared_token0, shared_expert;
    const uint32_t *epoch;
    const float *shared_w;    // [tokens] own tokens' shared-expert gate weights
    int32_t *offsets;         // [514]
    int32_t *pair_token;
    int32_t *pair_rank;
    float *pair_weight;
    TileRec *tiles;
    int *num_tiles;           // [0] tiles, [1] shared-expert tiles at the end of the list
    int max_tiles;
    int *error;
};
constexpr int kEpSmallSlots = 256;   // world <= 8 ranks x T_max <= 32
__global__ void __launch_bounds__(512) ep_group_small_kernel(EpSmallGroupParams g) {
    __shared__ uint32_t smask[kEpSmallSlots / kChunk][kRouterExperts];
    __shared__ int16_t sid[kEpSmallSlots * kEpSlotIds];   // received (local expert) lists, -1 = none
    __shared__ float sw[kEpSmallSlots * kEpSlotIds];
    __shared__ int scount[kEpMaxRanks];
    __shared__ int failed;
    const int e = threadIdx.x, lane = e & 31;
    const EpCtl *c = reinterpret_cast<const EpCtl *>(g.arena + g.L.ctl);
    if (e < 32) {
        bool ok = true;
        if (e < g.world) {
            const uint32_t want = *g.epoch;
            const long long t0 = clock64();
            uint64_t v;
            while (static_cast<uint32_t>(v = ld_acquire_sys64(&c->recv[e])) != want) {
                if (clock64() - t0 > (1ll << 31)) {
                    atomicOr(g.error, kFlagTimeout);
                    ok = false;
                    break;
                }
                __nanosleep(64);
            }
            scount[e] = static_cast<int>(v >> 32);
        }
        ok = __all_sync(0xffffffffu, ok);
        if (e == 0) failed = !ok;
    }
    const int chunks = g.slots / kChunk;
    for (int k = 0; k < chunks; ++k) smask[k][e] = 0u;
    __syncthreads();
    if (failed) {
        if (e == 0) { g.num_tiles[0] = 0; g.num_tiles[1] = 0; }
        return;
    }
    // one pass over the received lists (independent loads), into shared memory
    const int32_t *ids = reinterpret_cast<const int32_t *>(g.arena + g.L.ids);
    const float *ws = reinterpret_cast<const float *>(g.arena + g.L.w);
    for (int i = e; i < g.slots * kEpSlotIds; i += blockDim.x) {
        const int slot = i / kEpSlotIds;
        const bool valid = slot % g.t_max < scount[slot / g.t_max];
        const int id = valid ? ids[i] : -1;
        const bool live = id >= 0 && id < kRouterExperts;
        sid[i] = static_cast<int16_t>(live ? id : -1);
        sw[i] = live ? ws[i] : 0.0f;
        if (live) atomicOr(&smask[slot / kChunk][id], 1u << (slot % kChunk));
    }
    __syncthreads();
    int count = 0;
    for (int k = 0; k < chunks; ++k) count += __popc(smask[k][e]);
    int total = 0;
    const int off = block_exclusive_scan_512(count, &total);
    g.offsets[e] = off;
    if (e == kRouterExperts - 1) {
        g.offsets[kRouterExperts] = total;
        g.offsets[kRouterExperts + 1] = total + (g.has_shared ? g.tokens : 0);
    }
    const int ntiles = (count + kGemvTile - 1) / kGemvTile;
    int tiles_total = 0;
    const int toff = block_exclusive_scan_512(ntiles, &tiles_total);
    int pos = 0;
    for (int k = 0; k < chunks; ++k)
        for (uint32_t m = smask[k][e]; m; m &= m - 1u, ++pos) {
            const int slot = k * kChunk + __ffs(m) - 1;
            int r = 0;
#pragma unroll
            for (int q = 0; q < kEpSlotIds; ++q)
                if (sid[slot * kEpSlotIds + q] == e) r = q;
            const float w = sw[slot * kEpSlotIds + r];
            const int pair = off + pos;
            g.pair_token[pair] = slot;
            if (g.pair_rank) g.pair_rank[pair] = r;
            g.pair_weight[pair] = w;
            const int tile = toff + pos / kGemvTile, j = pos % kGemvTile;
            if (tile < g.max_tiles) {
                TileRec &rec = g.tiles[tile];
                if (j == 0) {
                    rec.e = e;
                    rec.p0 = pair;
                    rec.n = min(kGemvTile, count - pos);
                    rec.pad = 0;
                }
                rec.tok[j] = slot;
                rec.w[j] = w;
            }
        }
    int shared_tiles = 0;
    if (g.has_shared) {
        for (int i = e; i < g.tokens; i += blockDim.x) {
            g.pair_token[total + i] = g.shared_token0 + i;
            g.pair_weight[total + i] = g.shared_w[i];
        }
        shared_tiles = (g.tokens + kGemvTile - 1) / kGemvTile;
        for (int i = e; i < shared_tiles; i += blockDim.x) {
            if (tiles_total + i >= g.max_tiles) continue;
            TileRec &rec = g.tiles[tiles_total + i];
            rec.e = g.shared_expert;
            rec.p0 = total + i * kGemvTile;
            rec.n = min(kGemvTile, g.tokens - i * kGemvTile);
            rec.pad = 0;
            for (int j = 0; j < kGemvTile; ++j) {
                const bool live = j < rec.n;
                rec.tok[j] = live ? g.shared_token0 + i * kGemvTile + j : 0;
                rec.w[j] = live ? g.shared_w[i * kGemvTile + j] : 0.0f;
            }
        }
    }
    if (e == 0) {
        int n = tiles_total + shared_tiles;
        if (n > g.max_tiles) { atomicOr(g.error, kFlagArithmetic); n = g.max_tiles; }
        g.num_tiles[0] = n;
        g.num_tiles[1] = max(0, n - tiles_total);
    }
    (void)lane;
}

// Stable placement of received (slot, local expert) pairs, as
// route_scatter_kernel but over slot lists of kEpSlotIds entries.
struct EpScatterParams {
    const uint8_t *arena;
    EpLayout L;
    const uint32_t *masks;
    const int32_t *base;
    const int32_t *offsets;
    int32_t *pair_token;
    int32_t *pair_rank;
    float *pair_weight;
    TileRec *tiles;
    const int32_t *tile_off;
    int max_tiles;
};
__global__ void __launch_bounds__(256) ep_scatter_kernel(EpScatterParams p) {
    const int chunk = blockIdx.x, e = blockIdx.y * 256 + threadIdx.x;
    const size_t idx = static_cast<size_t>(chunk) * kRouterExperts + e;
    uint32_t m = p.masks[idx];
    if (!m) return;
    const int32_t *ids = reinterpret_cast<const int32_t *>(p.arena + p.L.ids);
    const float *ws = reinterpret_cast<const float *>(p.arena + p.L.w);
    int pos = p.offsets[e] + p.base[idx];
    while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1u;
        const int slot = chunk * kChunk + j;
        int r = 0;
#pragma unroll
        for (int k = 0; k < kEpSlotIds; ++k)
            if (ids[static_cast<size_t>(slot) * kEpSlotIds + k] == e) r = k;
        const float w = ws[static_cast<size_t>(slot) * kEpSlotIds + r];
        p.pair_token[pos] = slot;
        if (p.pair_rank) p.pair_rank[pos] = r;
        p.pair_weight[pos] = w;
        if (p.tiles && p.tile_off[e] >= 0) {
            const int local = pos - p.offsets[e];
            const int tile = p.tile_off[e] + local / kGemvTile;
            if (tile < p.max_tiles) {
                p.tiles[tile].tok[local % kGemvTile] = slot;
                p.tiles[tile].w[local % kGemvTile] = w;
            }
        }
        ++pos;
    }
}

// Combine: publish this rank's "partials final", wait until every peer has
// published its own (bounded), then out[t] += sum over the token's destinations d (ascending) of the
// partial row d holds for it, clearing that row for the next epoch.  One CTA
// per token, one float4 column per thread for H <= 4 * kEpCombineThreads, so
// every peer load of the token is in flight at once (one NVLink round trip).
constexpr int kEpCombineThreads = 512;
__global__ void __launch_bounds__(kEpCombineThreads) ep_combine_kernel(EpParams p) {
    __shared__ int ready;
    const int t = blockIdx.x;
    grid_launch_dependents();   // the next layer's routing CTAs may become resident and wait
    // This rank's partial rows are final (the expert kernels before this launch
    // completed): CTA 0 publishes that to every peer first.
    if (t == 0 && threadIdx.x < p.world) {
        __threadfence_system();
        EpCtl *c = reinterpret_cast<EpCtl *>(p.peers.base[threadIdx.x] + p.L.ctl);
        st_release_sys(&c->done_epoch[p.rank], *p.epoch);
    }
    if (t >= p.tokens) return;
    if (threadIdx.x < 32) {
        const EpCtl *c = reinterpret_cast<const EpCtl *>(p.peers.base[p.rank] + p.L.ctl);
        bool ok = true;
        if (threadIdx.x < p.world) {
            const uint32_t want = *p.epoch;
            const long long t0 = clock64();
            while (ld_acquire_sys(&c->done_epoch[threadIdx.x]) != want) {
                if (clock64() - t0 > (1ll << 31)) {
                    atomicOr(p.error, kFlagTimeout);
                    ok = false;
                    break;
                }
                __nanosleep(64);
            }
        }
        ok = __all_sync(0xffffffffu, ok);
        if (threadIdx.x == 0) ready = ok;
    }
    __syncthreads();
    if (!ready) return;
    const uint32_t mask = p.dmask[t];
    const int H = p.hidden;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 *rows[kEpMaxRanks];   // this token's partial row on every destination (null: not used)
#pragma unroll
    for (int d = 0; d < kEpMaxRanks; ++d) {
        const bool use = d < p.world && ((mask >> d) & 1u);
        const size_t slot = static_cast<size_t>(p.rank) * p.t_max + (use ? p.pos[t * kEpMaxRanks + d] : 0);
        rows[d] = use ? reinterpret_cast<float4 *>(p.peers.base[d] + p.L.partial) + slot * (H / 4) : nullptr;
    }
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        // all remote loads first (one NVLink round trip), then the in-order sum
        float4 v[kEpMaxRanks];
#pragma unroll
        for (int d = 0; d < kEpMaxRanks; ++d) v[d] = rows[d] ? rows[d][i] : zero;
#pragma unroll
        for (int d = 0; d < kEpMaxRanks; ++d)
            if (rows[d]) rows[d][i] = zero;
        float4 acc = zero;
#pragma unroll
        for (int d = 0; d < kEpMaxRanks; ++d) {
            if (!rows[d]) continue;
            acc.x = __fadd_rn(acc.x, v[d].x);
            acc.y = __fadd_rn(acc.y, v[d].y);
            acc.z = __fadd_rn(acc.z, v[d].z);
            acc.w = __fadd_rn(acc.w, v[d].w);
        }
        float4 *o = reinterpret_cast<float4 *>(p.out + static_cast<size_t>(t) * H) + i;
        float4 r = *o;
        r.x = __fadd_rn(r.x, acc.x);
        r.y = __fadd_rn(r.y, acc.y);
        r.z = __fadd_rn(r.z, acc.z);
        r.w = __fadd_rn(r.w, acc.w);
        *o = r;
    }
}

}  // namespace qmoe
