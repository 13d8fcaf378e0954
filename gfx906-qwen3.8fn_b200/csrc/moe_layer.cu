// moe_layer.cu -- C ABI of the routed-MoE expert FFN (see include/qwen_moe_b200.h).
//
// Orchestration of one forward (all device work, no host synchronisation):
//   quantize x -> route top-k (softmax, top-10, weights, shared gate, chunk masks)
//   -> chunk prefix -> expert scan + tile list -> stable scatter of pairs
//   -> gate/up + SiLU*up + Q8_1 middle -> down + weighted scatter-add.
// Replaces the reference's Layer::ffn body (src/session.hip:1412-1556) and
// Experts::run/run_chunk/project (src/session.hip:976-1071).
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <vector>

#include "common.cuh"
#include "expert_kernels.cuh"
#include "route_kernels.cuh"
#include "stream_kernels.cuh"
#include "tc_kernels.cuh"
#include "tcr_kernels.cuh"
#include "ep_kernels.cuh"
#include "router_kernels.cuh"

using namespace qmoe;

namespace {

thread_local char g_message[256];

int fail(int status, const char *message) {
    std::snprintf(g_message, sizeof(g_message), "%s", message);
    return status;
}

int cuda_status(cudaError_t e, const char *where) {
    if (e == cudaSuccess) return MOE_OK;
    std::snprintf(g_message, sizeof(g_message), "%s: %s", where, cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? MOE_OUT_OF_MEMORY : MOE_CUDA_ERROR;
}

#define MOE_CUDA(call)                                        \
    do {                                                      \
        const cudaError_t _e = (call);                        \
        if (_e != cudaSuccess) return cuda_status(_e, #call); \
    } while (0)

struct DeviceGuard {
    int previous = -1;
    cudaError_t status = cudaSuccess;
    explicit DeviceGuard(int device) {
        status = cudaGetDevice(&previous);
        if (status == cudaSuccess && previous != device) status = cudaSetDevice(device);
        else if (status == cudaSuccess) previous = -1;
    }
    ~DeviceGuard() {
        if (previous >= 0) cudaSetDevice(previous);
    }
};

bool aligned(const void *p, size_t a) { return p && reinterpret_cast<uintptr_t>(p) % a == 0; }

bool overlap(const void *a, size_t an, const void *b, size_t bn) {
    const auto x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + bn && y < x + an;
}

int validate_desc(const moe_layer_desc *d) {
    if (!d) return fail(MOE_INVALID_ARGUMENT, "null layer description");
    if (d->hidden <= 0 || d->hidden > 16384 || d->hidden % 256 || d->inter <= 0 || d->inter > 16384 ||
        d->inter % 32)
        return fail(MOE_INVALID_ARGUMENT, "hidden must be a multiple of 256, inter of 32, both <= 16384");
    if (d->experts != kRouterExperts || d->top_k != kTopK)
        return fail(MOE_NOT_SUPPORTED, "only 512 experts with top-10 routing are supported");
    if (d->has_shared != 0 && d->has_shared != 1) return fail(MOE_INVALID_ARGUMENT, "has_shared must be 0 or 1");
    if (d->max_tokens < 1 || d->max_tokens > 65536)
        return fail(MOE_INVALID_ARGUMENT, "max_tokens must be 1..65536");
    return MOE_OK;
}

// Bump allocator over one device arena.
struct Arena {
    uint8_t *base = nullptr;
    size_t used = 0;
    template <class T> T *take(size_t count) {
        used = (used + 255) & ~size_t(255);
        T *p = reinterpret_cast<T *>(base + used);
        used += count * sizeof(T);
        return p;
    }
};

// The C library's expf corrections embedded by the build (csrc/expf_table.c):
// little-endian uint32 pairs (x bits, expf(x) bits).
extern "C" const unsigned char qmoe_expf_table_begin[], qmoe_expf_table_end[];

constexpr int kExpfDevices = 64;
std::mutex g_expf_mutex;
bool g_expf_loaded[kExpfDevices] = {};

// out[i] = expf_ref of the float with bits first + i (the SiLU's exponential).
__global__ void debug_expf_kernel(uint32_t first, uint32_t count, float *out) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
        out[i] = expf_ref(__uint_as_float(first + i));
}

// Fill the current device's g_expf_fix hash table (once per device).
int expf_table_upload() {
    int device = 0;
    MOE_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= kExpfDevices) return fail(MOE_NOT_SUPPORTED, "device ordinal above 63");
    std::lock_guard<std::mutex> lock(g_expf_mutex);
    if (g_expf_loaded[device]) return MOE_OK;
    static std::vector<uint4> table;   // kExpfBucket / 2 uint4 per bucket
    if (table.empty()) {
        const size_t n = static_cast<size_t>(qmoe_expf_table_end - qmoe_expf_table_begin) / 8;
        constexpr uint32_t nbk = 1u << kExpfBucketsLog2;
        std::vector<uint32_t> t(static_cast<size_t>(nbk) * kExpfBucket * 2, kExpfEmpty);   // (key, value) entries
        for (size_t i = 0; i < n; ++i) {
            uint32_t kv[2];
            std::memcpy(kv, qmoe_expf_table_begin + 8 * i, 8);
            uint32_t b = expf_fix_bucket(kv[0]);
            bool placed = false;
            for (int probe = 0; probe < kExpfMaxProbe && !placed; ++probe, b = (b + 1) & (nbk - 1))
                for (int j = 0; j < kExpfBucket && !placed; ++j) {
                    uint32_t *entry = &t[(static_cast<size_t>(b) * kExpfBucket + j) * 2];
                    if (entry[0] == kExpfEmpty) {
                        entry[0] = kv[0];
                        entry[1] = kv[1];
                        placed = true;
                    }
                }
            if (!placed) return fail(MOE_CUDA_ERROR, "expf correction table: probe chain too long");
        }
        std::vector<uint4> packed(t.size() / 4);
        std::memcpy(packed.data(), t.data(), t.size() * sizeof(uint32_t));
        table.swap(packed);
    }
    MOE_CUDA(cudaMemcpyToSymbol(g_expf_fix, table.data(), table.size() * sizeof(uint4)));
    g_expf_loaded[device] = true;
    return MOE_OK;
}

int sm_count(int device) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    return n > 0 ? n : 148;
}

}  // namespace

struct moe_weights_s {
    moe_layer_desc desc;
    ExpertLayout layout;
    int experts_total;       // routed + shared
    int expert_first = 0;    // global id of local expert 0 (expert-parallel shards)
    int expert_count = kRouterExperts;   // routed experts held; the shared expert follows
    uint8_t *base = nullptr; // experts_total * layout.bytes
    float *gate_vec = nullptr;
    float *router = nullptr;     // ffn_gate_inp as fp32 [512][H] (zero until uploaded)
    uint8_t *staging = nullptr;  // canonical bytes of one expert (3 matrices)
    cudaEvent_t staged = nullptr;  // recorded after the last repack that read `staging`
    TcrMaps maps;                // tensor maps of the codes and scales (tensor-core path)
    int raw_rowmajor = 0;        // codes maps are 3-D [expert][row][bytes] (4-D [expert][block][row][16] refused)
    bool tc_ok = false;          // the tensor-core kernels can run on these weights
};

struct moe_layer_s {
    moe_layer_desc desc;
    ExpertLayout layout;
    int chunks_max, pairs_max, tiles_max, sms;
    Arena arena;
    Q8Planar xq, mid;
    int32_t *ids, *base, *counts, *offsets, *pair_token, *pair_rank;
    float *weights, *pair_weight;
    uint32_t *masks;
    TileRec *tiles;
    int32_t *tile_off;
    int *num_tiles;
    int *error;
    int gu_stages, dn_stages;   // shared-memory ring depth of the streaming kernels (0: not used)
    float *logits = nullptr;    // [max_tokens][512] router logits of moe_forward_hidden
    TcWorkspace tc;
};

namespace {

int tiles_bound(int tokens, int has_shared) {
    const int pairs = tokens * kTopK;
    const int routed = (pairs + kGemvTile - 1) / kGemvTile + std::min(kRouterExperts, pairs);
    return routed + (has_shared ? (tokens + kGemvTile - 1) / kGemvTile : 0);
}

size_t gate_up_smem(int H) { return static_cast<size_t>(kGemvTile) * H + kGemvTile * (H / 32) * 8 + kGemvTile * 32 * 4; }
size_t down_smem(int I) { return static_cast<size_t>(kGemvTile) * I + kGemvTile * (I / 32) * 8 + 2 * kGemvTile * 4; }

size_t stream_gu_smem(int H, int stages) {
    return 128 + kGuGroupsMax * 2 * kGemvTile * 32 * 4 + size_t(stages) * GuStage(H).bytes;
}
constexpr int kGuStagesMax = 3;
size_t stream_dn_smem(int I, int stages) { return 128 + size_t(stages) * DnStage(I).bytes; }

int configure_kernels(moe_layer_s *h, int H, int I) {
    MOE_CUDA(cudaFuncSetAttribute(gate_up_kernel<kGemvTile>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(gate_up_smem(H))));
    MOE_CUDA(cudaFuncSetAttribute(down_kernel<kGemvTile, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(down_smem(I))));
    MOE_CUDA(cudaFuncSetAttribute(down_kernel<kGemvTile>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(down_smem(I))));
    // The streaming kernels need at least two stages in shared memory.
    h->gu_stages = stream_stages(GuStage(H).bytes + 1024, kGuStagesMax);   // + the middle buffers
    h->dn_stages = stream_stages(DnStage(I).bytes, 5);
    if (h->gu_stages < 2 || h->dn_stages < 2) h->gu_stages = h->dn_stages = 0;
    if (h->gu_stages) {
        const int gu = static_cast<int>(stream_gu_smem(H, h->gu_stages));
        const int dn = static_cast<int>(stream_dn_smem(I, h->dn_stages));
        MOE_CUDA(cudaFuncSetAttribute(stream_gate_up_kernel<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, gu));
        MOE_CUDA(cudaFuncSetAttribute(stream_gate_up_kernel<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, gu));
        MOE_CUDA(cudaFuncSetAttribute(stream_gate_up_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, gu));
        MOE_CUDA(cudaFuncSetAttribute(stream_gate_up_kernel<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, gu));
        MOE_CUDA(cudaFuncSetAttribute(stream_down_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, dn));
        MOE_CUDA(cudaFuncSetAttribute(stream_down_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, dn));
        MOE_CUDA(cudaFuncSetAttribute(stream_down_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, dn));
    }
    return MOE_OK;
}

// Launch with programmatic stream serialisation: the kernel may begin while
// the preceding kernel of the stream finishes, and orders itself after it
// with grid_dependency_wait().
template <class... Args>
cudaError_t launch_overlapped(void (*kernel)(Args...), int grid, int block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// Tensor maps over every expert of a weights object for the TMA loads of the
// tensor-core kernels: per matrix the code bytes as {16 bytes, row, block,
// expert} (box 16 x 128 rows x 4 blocks: a copy lands block-major, each
// block's 128 rows contiguous) -- or, where the driver refuses that stride
// order, as {row bytes, row, expert} (box 64 bytes x 128 rows) -- and the
// half scales (and the minima of Q4_1 down matrices) as {block, row, expert}
// (box 8 blocks x 128 rows).  Weights of other shapes (the gate/up stage order
// is that of 64 blocks, H = 2048; I a multiple of 256) run every group on the
// streaming kernels instead.
int build_maps(moe_weights_s *w) {
    const ExpertLayout &L = w->layout;
    w->tc_ok = false;
    if (L.hidden != kRowsHidden || L.inter % (2 * kRowsM)) return MOE_OK;
    const EncodeTiledFn enc = encode_tiled();
    if (!enc) return fail(MOE_CUDA_ERROR, "cuTensorMapEncodeTiled is not available from the driver");
    const size_t code_off[3] = {L.gate_codes, L.up_codes, L.down_codes};
    const size_t sc_off[3] = {L.gate_scales, L.up_scales, L.down_scales};
    const cuuint64_t rows[3] = {cuuint64_t(L.inter), cuuint64_t(L.inter), cuuint64_t(L.hidden)};
    const cuuint64_t nbm[3] = {cuuint64_t(L.hidden / 32), cuuint64_t(L.hidden / 32), cuuint64_t(L.inter / 32)};
    const cuuint64_t E = static_cast<cuuint64_t>(w->experts_total), EB = static_cast<cuuint64_t>(L.bytes);
    const cuuint32_t one[4] = {1, 1, 1, 1};
    int rowmajor = 0;
    for (; rowmajor < 2; ++rowmajor) {
        bool ok = true;
        for (int m = 0; m < 3 && ok; ++m) {
            CUresult r;
            if (!rowmajor) {
                const cuuint64_t dims[4] = {16, rows[m], nbm[m], E};
                const cuuint64_t strides[3] = {nbm[m] * 16, 16, EB};
                const cuuint32_t box[4] = {16, kRowsM, cuuint32_t(kRowsBlocksPerCopy), 1};
                r = enc(&w->maps.codes[m], CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, w->base + code_off[m], dims, strides, box,
                        one, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            } else {
                const cuuint64_t dims[3] = {nbm[m] * 16, rows[m], E};
                const cuuint64_t strides[2] = {nbm[m] * 16, EB};
                const cuuint32_t box[3] = {cuuint32_t(16 * kRowsBlocksPerCopy), kRowsM, 1};
                r = enc(&w->maps.codes[m], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, w->base + code_off[m], dims, strides, box,
                        one, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            }
            ok = r == CUDA_SUCCESS;
        }
        if (ok) break;
    }
    if (rowmajor == 2) return fail(MOE_CUDA_ERROR, "cuTensorMapEncodeTiled refused the weight code maps");
    for (int m = 0; m < 3; ++m) {
        const cuuint64_t dims[3] = {nbm[m], rows[m], E};
        const cuuint64_t strides[2] = {nbm[m] * 2, EB};
        const cuuint32_t box[3] = {8, kRowsM, 1};
        if (enc(&w->maps.scales[m], CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, w->base + sc_off[m], dims, strides, box, one,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return fail(MOE_CUDA_ERROR, "cuTensorMapEncodeTiled refused the weight scale maps");
    }
    if (L.down_type == kDownQ4_1) {
        const cuuint64_t dims[3] = {nbm[2], rows[2], E};
        const cuuint64_t strides[2] = {nbm[2] * 2, EB};
        const cuuint32_t box[3] = {8, kRowsM, 1};
        if (enc(&w->maps.down_mins, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, w->base + L.down_mins, dims, strides, box, one,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return fail(MOE_CUDA_ERROR, "cuTensorMapEncodeTiled refused the down minima map");
    }
    w->raw_rowmajor = rowmajor;
    w->tc_ok = true;
    return MOE_OK;
}

GroupParams group_params(moe_layer_s *h, const moe_weights_s *w, float *out) {
    GroupParams g;
    g.weights = w->base;
    g.layout = w->layout;
    g.x = h->xq;
    g.mid = h->mid;
    g.tiles = h->tiles;
    g.num_tiles = h->num_tiles;
    g.pair_token = h->pair_token;
    g.pair_weight = h->pair_weight;
    g.sink.out = out;
    g.error = h->error;
    return g;
}

TcrParams tcr_params(moe_layer_s *h, const moe_weights_s *w, float *out, bool down, const TapSink *tap) {
    TcrParams t;
    t.maps = w->maps;
    t.hidden = w->layout.hidden;
    t.inter = w->layout.inter;
    t.raw_rowmajor = w->raw_rowmajor;
    t.b_arr = down ? h->tc.b_dn : h->tc.b_gu;
    t.bsc_arr = down ? h->tc.sc_dn : h->tc.sc_gu;
    t.tiles = h->tc.tiles;
    t.num_tiles = h->tc.num_tiles;
    t.pair_token = h->pair_token;
    t.pair_weight = h->pair_weight;
    t.mid_arr = h->tc.b_dn;
    t.mid_sc_arr = h->tc.sc_dn;
    t.out = out;
    t.error = h->error;
    if (tap) t.tap = *tap;
    return t;
}

// Tensor-core expert kernel over the tile list already in the workspace:
// persistent, one CTA per SM at most.
int launch_tc(moe_layer_s *h, const moe_weights_s *w, float *out, int tc_tiles, bool down, cudaStream_t s,
              const TapSink *tap) {
    const ExpertLayout &L = w->layout;
    const int items = tc_tiles * ((down ? L.hidden : L.inter) / kRowsM);
    const int grid = std::max(1, std::min(items, h->sms));
    const TcrParams prm = tcr_params(h, w, out, down, tap);
    cudaError_t e;
    if (down && L.down_type == kDownQ4_1)
        e = launch_overlapped(tap ? tc_rows_kernel<true, true, true> : tc_rows_kernel<true, false, true>, grid,
                              RowsStage<true, true>::threads, RowsStage<true, true>::smem, s, prm);
    else if (down)
        e = launch_overlapped(tap ? tc_rows_kernel<true, true> : tc_rows_kernel<true, false>, grid, RowsStage<true>::threads,
                              RowsStage<true>::smem, s, prm);
    else
        e = launch_overlapped(tap ? tc_rows_kernel<false, true> : tc_rows_kernel<false, false>, grid, RowsStage<false>::threads,
                              RowsStage<false>::smem, s, prm);
    return cuda_status(e, "tc_rows_kernel");
}

// gate/up + down over the tile lists already in the workspace: the streaming
// dp4a kernels for the small tiles (`stream_groups`: decode sizes, trace
// mode) and the tensor-core kernels for `tc_tiles` (an upper
// bound on the device-written count).  `events` (optional, three entries) are
// recorded before the gate/up kernels, between gate/up and down, and after
// down.  `tap` records one expert's per-block dots (parity taps).
int launch_experts(moe_layer_s *h, const moe_weights_s *w, float *out, int max_tiles, cudaStream_t s,
                   void *const *events = nullptr, int tc_tiles = 0, const DownSink *trace = nullptr,
                   bool stream_groups = true, const TapSink *tap = nullptr) {
    const ExpertLayout &L = w->layout;
    DownSink sink;
    if (trace) sink = *trace;
    sink.out = out;
    if (h->gu_stages) {
        StreamParams sp;
        sp.weights = w->base;
        sp.layout = L;
        sp.x = h->xq;
        sp.mid = h->mid;
        sp.tiles = h->tiles;
        sp.num_tiles = h->num_tiles;
        sp.sink = sink;
        sp.error = h->error;
        if (tap) sp.tap = *tap;
        const int gu_items = max_tiles * (L.inter / kGuRows), dn_items = max_tiles * (L.hidden / kDnRows);
        if (tc_tiles) {
            tc_rows_gather_kernel<<<dim3(std::min(tc_tiles, h->sms * 8), L.hidden / 256), 2 * kTcTile, 0, s>>>(
                h->tc.tiles, h->tc.num_tiles, h->pair_token, h->xq, L.hidden, h->tc.b_gu, h->tc.sc_gu);
            MOE_CUDA(cudaGetLastError());
        }
        if (events) MOE_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[0]), s));
        if (stream_groups) {
            sp.stages = h->gu_stages;
            sp.stage_bytes = GuStage(L.hidden).bytes;
            // two items in flight per CTA when the CTAs have about one item each (decode of 1-2 tokens)
            const bool two = gu_items <= 2 * h->sms;
            auto gu_kernel = two ? (tap ? stream_gate_up_kernel<2, true> : stream_gate_up_kernel<2, false>)
                                 : (tap ? stream_gate_up_kernel<1, true> : stream_gate_up_kernel<1, false>);
            MOE_CUDA(launch_overlapped(gu_kernel, std::max(1, std::min(gu_items, h->sms)), kStreamThreads,
                                       stream_gu_smem(L.hidden, sp.stages), s, sp));
        }
        if (tc_tiles)
            if (const int st = launch_tc(h, w, out, tc_tiles, false, s, tap)) return st;
        if (events) MOE_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[1]), s));
        if (stream_groups) {
            sp.stages = h->dn_stages;
            sp.stage_bytes = DnStage(L.inter).bytes;
            auto kernel = trace ? stream_down_kernel<true, false>
                                : (tap ? stream_down_kernel<false, true> : stream_down_kernel<false, false>);
            MOE_CUDA(launch_overlapped(kernel, std::max(1, std::min(dn_items, h->sms)), kStreamThreads,
                                       stream_dn_smem(L.inter, sp.stages), s, sp));
        }
        if (tc_tiles)
            if (const int st = launch_tc(h, w, out, tc_tiles, true, s, tap)) return st;
        if (events) MOE_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[2]), s));
        return MOE_OK;
    }
    GroupParams g = group_params(h, w, out);
    g.sink = sink;
    const int slabs = L.inter / 32, dslabs = L.hidden / 64;
    const int gu_grid = std::max(1, std::min(max_tiles * slabs, h->sms * 8));
    const int dn_grid = std::max(1, std::min(max_tiles * dslabs, h->sms * 8));
    if (events) MOE_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[0]), s));
    gate_up_kernel<kGemvTile><<<gu_grid, kGemvThreads, gate_up_smem(L.hidden), s>>>(g);
    MOE_CUDA(cudaGetLastError());
    if (events) MOE_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[1]), s));
    if (trace) down_kernel<kGemvTile, true><<<dn_grid, kGemvThreads, down_smem(L.inter), s>>>(g);
    else down_kernel<kGemvTile><<<dn_grid, kGemvThreads, down_smem(L.inter), s>>>(g);
    MOE_CUDA(cudaGetLastError());
    if (events) MOE_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[2]), s));
    return MOE_OK;
}

int launch_quantize(const float *x, size_t blocks, Q8Planar out, uint8_t *canonical, int *error, int sms,
                    cudaStream_t s) {
    const size_t warps = blocks;
    const int grid = static_cast<int>(std::max<size_t>(1, std::min<size_t>((warps + 7) / 8, size_t(sms) * 16)));
    quantize_kernel<<<grid, 256, 0, s>>>(x, blocks, out, canonical, error);
    return cuda_status(cudaGetLastError(), "quantize_kernel");
}

int launch_route(moe_layer_s *h, const moe_weights_s *w, const float *x, const float *logits, int T,
                 float *probs, cudaStream_t s, const EpParams *ep = nullptr, uint32_t *quant_done = nullptr,
                 bool allow_tc = true) {
    const int chunks = (T + kChunk - 1) / kChunk;
    RouteParams rp;
    rp.logits = logits;
    rp.x = x;
    rp.gate_vec = (w && h->desc.has_shared) ? w->gate_vec : nullptr;
    rp.tokens = T;
    rp.hidden = h->desc.hidden;
    rp.probs = probs;
    rp.ids = h->ids;
    rp.weights = h->weights;
    rp.masks = h->masks;
    rp.pair_token = h->pair_token;
    rp.pair_weight = h->pair_weight;
    rp.pair_rank = h->pair_rank;
    rp.error = h->error;
    if (T <= kChunk) {   // one chunk: quantise + route + group + tiles in one launch
        SmallRouteParams sr;
        sr.r = rp;
        sr.xq = x ? h->xq : Q8Planar{nullptr, nullptr};
        sr.offsets = h->offsets;
        sr.tiles = h->tiles;
        sr.tile_off = h->tile_off;
        sr.num_tiles = h->num_tiles;
        sr.max_tiles = h->tiles_max;
        if (ep) {
            sr.ep_on = 1;
            sr.ep = *ep;
            sr.quant_done = quant_done;
        }
        // block 0 routes; the others quantise x (one warp per 32-value block)
        const int qblocks = sr.xq.codes ? (T * (h->desc.hidden / 32) + 15) / 16 : 0;
        return cuda_status(launch_overlapped(route_small_kernel, 1 + qblocks, 512, 0, s, sr), "route_small_kernel");
    }
    route_topk_kernel<<<chunks, kRouteThreads, 0, s>>>(rp);
    MOE_CUDA(cudaGetLastError());
    route_chunk_prefix_kernel<<<kRouterExperts / 32, 1024, 0, s>>>(h->masks, chunks, h->base, h->counts);
    MOE_CUDA(cudaGetLastError());
    ScanParams sp;
    sp.counts = h->counts;
    sp.tokens = T;
    sp.tile = kGemvTile;
    sp.has_shared = rp.gate_vec != nullptr;
    sp.offsets = h->offsets;
    sp.tiles = h->tiles;
    sp.tile_off = h->tile_off;
    sp.pair_token = h->pair_token;
    sp.pair_weight = h->pair_weight;
    sp.num_tiles = h->num_tiles;
    sp.max_tiles = h->tiles_max;
    sp.error = h->error;
    if (x && allow_tc && w && w->tc_ok) {   // forward above decode size: the groups go to the tensor-core kernels
        sp.tc_min = kRowsMinGroup;
        sp.tc_tile = kTcTile;
        sp.tc_max = h->tc.max_tiles;
        sp.tc_tiles = h->tc.tiles;
        sp.tc_num = h->tc.num_tiles;
    }
    route_scan_kernel<<<1, 512, 0, s>>>(sp);
    MOE_CUDA(cudaGetLastError());
    ScatterParams cp;
    cp.masks = h->masks;
    cp.base = h->base;
    cp.offsets = h->offsets;
    cp.ids = h->ids;
    cp.weights = h->weights;
    cp.pair_token = h->pair_token;
    cp.pair_rank = h->pair_rank;
    cp.pair_weight = h->pair_weight;
    cp.tiles = h->tiles;
    cp.tile_off = h->tile_off;
    cp.max_tiles = h->tiles_max;
    route_scatter_kernel<<<dim3(chunks, kRouterExperts / 256), 256, 0, s>>>(cp);
    MOE_CUDA(cudaGetLastError());
    return MOE_OK;
}

}  // namespace

extern "C" {

const char *moe_last_error_message(void) { return g_message; }

int moe_abi_version(void) { return (1 << 16) | 1; }

const char *moe_status_string(int status) {
    switch (status) {
    case MOE_OK: return "ok";
    case MOE_INVALID_ARGUMENT: return "invalid_argument";
    case MOE_NOT_SUPPORTED: return "not_supported";
    case MOE_CUDA_ERROR: return "cuda_error";
    case MOE_NUMERIC_ERROR: return "numeric_error";
    case MOE_TIMEOUT: return "timeout";
    case MOE_OUT_OF_MEMORY: return "out_of_memory";
    default: return "unknown";
    }
}

size_t moe_weights_expert_bytes(const moe_layer_desc *desc) {
    if (!desc) return 0;
    return make_layout(desc->hidden, desc->inter).bytes;
}

// ---------------------------------------------------------------- weights --
int moe_weights_create(const moe_layer_desc *desc, moe_weights_t *out) {
    return moe_weights_create_typed(desc, MOE_Q4_0, out);
}

int moe_weights_create_typed(const moe_layer_desc *desc, int down_type, moe_weights_t *out) {
    if (!out) return fail(MOE_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    if (const int st = validate_desc(desc)) return st;
    if (down_type != MOE_Q4_0 && down_type != MOE_Q4_1)
        return fail(MOE_NOT_SUPPORTED, "down matrices must be Q4_0 or Q4_1");
    DeviceGuard guard(desc->device);
    MOE_CUDA(guard.status);
    auto *w = new (std::nothrow) moe_weights_s();
    if (!w) return fail(MOE_OUT_OF_MEMORY, "host allocation");
    w->desc = *desc;
    w->layout = make_layout(desc->hidden, desc->inter, down_type == MOE_Q4_1 ? kDownQ4_1 : kDownQ4_0);
    w->experts_total = desc->experts + desc->has_shared;
    const size_t rbytes = sizeof(float) * kRouterExperts * desc->hidden;
    cudaError_t e = cudaMalloc(&w->base, w->layout.bytes * w->experts_total);
    if (e == cudaSuccess) e = cudaMalloc(&w->gate_vec, sizeof(float) * desc->hidden);
    if (e == cudaSuccess) e = cudaMalloc(&w->router, rbytes);
    if (e == cudaSuccess) e = cudaMalloc(&w->staging, w->layout.bytes / 16 * 18);
    if (e == cudaSuccess) e = cudaMemset(w->gate_vec, 0, sizeof(float) * desc->hidden);
    if (e == cudaSuccess) e = cudaMemset(w->router, 0, rbytes);
    const int st = e != cudaSuccess ? cuda_status(e, "moe_weights_create") : build_maps(w);
    if (st) {
        cudaFree(w->base); cudaFree(w->gate_vec); cudaFree(w->router); cudaFree(w->staging);
        delete w;
        return st;
    }
    *out = w;
    return MOE_OK;
}

int moe_weights_destroy(moe_weights_t w) {
    if (!w) return MOE_OK;
    DeviceGuard guard(w->desc.device);
    cudaFree(w->base);
    cudaFree(w->gate_vec);
    cudaFree(w->router);
    cudaFree(w->staging);
    if (w->staged) cudaEventDestroy(w->staged);
    delete w;
    return MOE_OK;
}

int moe_weights_upload_expert(moe_weights_t w, int expert, const void *gate, const void *up, const void *down,
                              void *stream) {
    if (!w || !gate || !up || !down) return fail(MOE_INVALID_ARGUMENT, "null weights argument");
    if (expert < 0 || expert >= w->experts_total) return fail(MOE_INVALID_ARGUMENT, "expert index out of range");
    DeviceGuard guard(w->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    const ExpertLayout &L = w->layout;
    const size_t blocks = static_cast<size_t>(L.hidden) * L.inter / 32;  // per matrix
    uint8_t *ex = w->base + static_cast<size_t>(expert) * L.bytes;
    const void *src[3] = {gate, up, down};
    const size_t codes[3] = {L.gate_codes, L.up_codes, L.down_codes};
    const size_t scales[3] = {L.gate_scales, L.up_scales, L.down_scales};
    // The staging buffer holds all three matrices; a previous upload (on any
    // stream) must have finished reading it before these copies overwrite it.
    if (!w->staged) MOE_CUDA(cudaEventCreateWithFlags(&w->staged, cudaEventDisableTiming));
    else MOE_CUDA(cudaStreamWaitEvent(s, w->staged, 0));
    size_t off = 0;
    for (int m = 0; m < 3; ++m) {
        const bool q41 = m == 2 && L.down_type == kDownQ4_1;
        const size_t bytes = blocks * (q41 ? 20 : 18);
        MOE_CUDA(cudaMemcpyAsync(w->staging + off, src[m], bytes, cudaMemcpyHostToDevice, s));
        if (q41)
            repack_q4_1_kernel<<<256, 256, 0, s>>>(w->staging + off, ex + codes[m],
                                                   reinterpret_cast<uint16_t *>(ex + scales[m]),
                                                   reinterpret_cast<uint16_t *>(ex + L.down_mins), blocks, 0);
        else
            repack_kernel<<<256, 256, 0, s>>>(w->staging + off, ex + codes[m],
                                              reinterpret_cast<uint16_t *>(ex + scales[m]), blocks, 0);
        MOE_CUDA(cudaGetLastError());
        off += bytes;
    }
    MOE_CUDA(cudaEventRecord(w->staged, s));
    return MOE_OK;
}

int moe_weights_download_expert(moe_weights_t w, int expert, void *gate, void *up, void *down, void *stream) {
    if (!w || !gate || !up || !down) return fail(MOE_INVALID_ARGUMENT, "null weights argument");
    if (expert < 0 || expert >= w->experts_total) return fail(MOE_INVALID_ARGUMENT, "expert index out of range");
    DeviceGuard guard(w->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    const ExpertLayout &L = w->layout;
    const size_t blocks = static_cast<size_t>(L.hidden) * L.inter / 32;
    uint8_t *ex = w->base + static_cast<size_t>(expert) * L.bytes;
    void *dst[3] = {gate, up, down};
    const size_t codes[3] = {L.gate_codes, L.up_codes, L.down_codes};
    const size_t scales[3] = {L.gate_scales, L.up_scales, L.down_scales};
    if (w->staged) MOE_CUDA(cudaStreamWaitEvent(s, w->staged, 0));   // uploads done with the staging buffer
    for (int m = 0; m < 3; ++m) {
        const bool q41 = m == 2 && L.down_type == kDownQ4_1;
        if (q41)
            repack_q4_1_kernel<<<256, 256, 0, s>>>(w->staging, ex + codes[m], reinterpret_cast<uint16_t *>(ex + scales[m]),
                                                   reinterpret_cast<uint16_t *>(ex + L.down_mins), blocks, 1);
        else
            repack_kernel<<<256, 256, 0, s>>>(w->staging, ex + codes[m], reinterpret_cast<uint16_t *>(ex + scales[m]),
                                              blocks, 1);
        MOE_CUDA(cudaGetLastError());
        MOE_CUDA(cudaMemcpyAsync(dst[m], w->staging, blocks * (q41 ? 20 : 18), cudaMemcpyDeviceToHost, s));
        MOE_CUDA(cudaStreamSynchronize(s));
    }
    return MOE_OK;
}

int moe_weights_upload_shared_gate(moe_weights_t w, const float *gate_vec, void *stream) {
    if (!w || !gate_vec) return fail(MOE_INVALID_ARGUMENT, "null shared gate argument");
    if (!w->desc.has_shared) return fail(MOE_INVALID_ARGUMENT, "layer has no shared expert");
    DeviceGuard guard(w->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    MOE_CUDA(cudaMemcpyAsync(w->gate_vec, gate_vec, sizeof(float) * w->desc.hidden, cudaMemcpyHostToDevice, s));
    MOE_CUDA(cudaStreamSynchronize(s));
    return MOE_OK;
}

int moe_weights_upload_router(moe_weights_t w, const float *router, void *stream) {
    if (!w || !router) return fail(MOE_INVALID_ARGUMENT, "null router argument");
    if (!w->router) return fail(MOE_NOT_SUPPORTED, "these weights hold no router matrix");
    DeviceGuard guard(w->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    MOE_CUDA(cudaMemcpyAsync(w->router, router, sizeof(float) * kRouterExperts * w->desc.hidden,
                             cudaMemcpyHostToDevice, s));
    MOE_CUDA(cudaStreamSynchronize(s));
    return MOE_OK;
}

int moe_weights_synthesize(moe_weights_t w, uint64_t seed, uint32_t layer, void *stream) {
    if (!w) return fail(MOE_INVALID_ARGUMENT, "null weights");
    DeviceGuard guard(w->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    synth_kernel<<<sm_count(w->desc.device) * 8, 256, 0, s>>>(w->base, w->layout, w->experts_total, seed, layer,
                                                              w->expert_first, w->expert_count);
    return cuda_status(cudaGetLastError(), "synth_kernel");
}

// ------------------------------------------------------------------ layer --
int moe_layer_create(const moe_layer_desc *desc, moe_layer_t *out) {
    if (!out) return fail(MOE_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    if (const int st = validate_desc(desc)) return st;
    DeviceGuard guard(desc->device);
    MOE_CUDA(guard.status);
    if (const int st = expf_table_upload()) return st;
    auto *h = new (std::nothrow) moe_layer_s();
    if (!h) return fail(MOE_OUT_OF_MEMORY, "host allocation");
    h->desc = *desc;
    h->layout = make_layout(desc->hidden, desc->inter);
    h->sms = sm_count(desc->device);
    const int T = desc->max_tokens, H = desc->hidden, I = desc->inter;
    h->chunks_max = (T + kChunk - 1) / kChunk;
    h->pairs_max = T * (kTopK + 1);
    h->tiles_max = tiles_bound(T, 1);
    // size the arena with a dry run
    for (int pass = 0; pass < 2; ++pass) {
        Arena &a = h->arena;
        a.used = 0;
        h->xq.codes = a.take<int8_t>(static_cast<size_t>(T) * H);
        h->xq.scales = a.take<float2>(static_cast<size_t>(T) * (H / 32));
        h->mid.codes = a.take<int8_t>(static_cast<size_t>(h->pairs_max) * I);
        h->mid.scales = a.take<float2>(static_cast<size_t>(h->pairs_max) * (I / 32));
        h->ids = a.take<int32_t>(static_cast<size_t>(T) * kTopK);
        h->weights = a.take<float>(static_cast<size_t>(T) * kTopK);
        h->logits = a.take<float>(static_cast<size_t>(T) * kRouterExperts);
        h->masks = a.take<uint32_t>(static_cast<size_t>(h->chunks_max) * kRouterExperts);
        h->base = a.take<int32_t>(static_cast<size_t>(h->chunks_max) * kRouterExperts);
        h->counts = a.take<int32_t>(kRouterExperts);
        h->offsets = a.take<int32_t>(kRouterExperts + 2);
        h->pair_token = a.take<int32_t>(h->pairs_max);
        h->pair_rank = a.take<int32_t>(h->pairs_max);
        h->pair_weight = a.take<float>(h->pairs_max);
        h->tiles = a.take<TileRec>(h->tiles_max);
        h->tile_off = a.take<int32_t>(kRouterExperts);
        h->num_tiles = a.take<int>(2);   // [0] work tiles, [1] shared-expert tiles at the end
        h->error = a.take<int>(1);
        tc_workspace_take(h->tc, a, h->pairs_max, H, I, T > kChunk);
        if (pass == 0) {
            const size_t bytes = a.used + 256;
            const cudaError_t e = cudaMalloc(&a.base, bytes);
            if (e != cudaSuccess) { delete h; return cuda_status(e, "moe_layer_create"); }
            cudaMemset(a.base, 0, bytes);
        }
    }
    if (const int st = configure_kernels(h, H, I)) { cudaFree(h->arena.base); delete h; return st; }
    if (const int st = tc_rows_configure()) { cudaFree(h->arena.base); delete h; return st; }
    *out = h;
    return MOE_OK;
}

int moe_layer_destroy(moe_layer_t h) {
    if (!h) return MOE_OK;
    DeviceGuard guard(h->desc.device);
    cudaFree(h->arena.base);
    delete h;
    return MOE_OK;
}

int moe_layer_read_flags(moe_layer_t h, int *flags, int clear, void *stream) {
    if (!h || !flags) return fail(MOE_INVALID_ARGUMENT, "null argument");
    DeviceGuard guard(h->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    MOE_CUDA(cudaMemcpyAsync(flags, h->error, sizeof(int), cudaMemcpyDeviceToHost, s));
    if (clear) MOE_CUDA(cudaMemsetAsync(h->error, 0, sizeof(int), s));
    MOE_CUDA(cudaStreamSynchronize(s));
    return MOE_OK;
}

int moe_route(moe_layer_t h, const float *logits, int tokens, float *probs, int32_t *ids, float *weights,
              int32_t *offsets, int32_t *token, int32_t *rank, void *stream) {
    if (!h || !aligned(logits, 4)) return fail(MOE_INVALID_ARGUMENT, "null or misaligned logits");
    if (tokens < 1 || tokens > h->desc.max_tokens) return fail(MOE_INVALID_ARGUMENT, "tokens outside 1..max_tokens");
    DeviceGuard guard(h->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    if (const int st = launch_route(h, nullptr, nullptr, logits, tokens, probs, s)) return st;
    const size_t n = static_cast<size_t>(tokens) * kTopK;
    if (ids) MOE_CUDA(cudaMemcpyAsync(ids, h->ids, n * 4, cudaMemcpyDeviceToDevice, s));
    if (weights) MOE_CUDA(cudaMemcpyAsync(weights, h->weights, n * 4, cudaMemcpyDeviceToDevice, s));
    if (offsets) MOE_CUDA(cudaMemcpyAsync(offsets, h->offsets, (kRouterExperts + 1) * 4, cudaMemcpyDeviceToDevice, s));
    if (token) MOE_CUDA(cudaMemcpyAsync(token, h->pair_token, n * 4, cudaMemcpyDeviceToDevice, s));
    if (rank) MOE_CUDA(cudaMemcpyAsync(rank, h->pair_rank, n * 4, cudaMemcpyDeviceToDevice, s));
    return MOE_OK;
}

int moe_forward(moe_layer_t h, moe_weights_t w, const float *x, const float *logits, int tokens, float *out,
                int flags, void *stream) {
    return moe_forward_profiled(h, w, x, logits, tokens, out, flags, stream, nullptr);
}

}  // extern "C"

namespace {
int forward_impl(moe_layer_t h, moe_weights_t w, const float *x, const float *logits, int tokens, float *out,
                 int flags, void *stream, void *const *events, const TapSink *tap) {
    if (!h || !w) return fail(MOE_INVALID_ARGUMENT, "null layer or weights");
    if (std::memcmp(&h->desc, &w->desc, offsetof(moe_layer_desc, device) + sizeof(int)) != 0)
        return fail(MOE_INVALID_ARGUMENT, "layer and weights describe different shapes or devices");
    if (tokens < 1 || tokens > h->desc.max_tokens) return fail(MOE_INVALID_ARGUMENT, "tokens outside 1..max_tokens");
    if (!aligned(x, 16) || !aligned(logits, 16) || !aligned(out, 16))
        return fail(MOE_INVALID_ARGUMENT, "x, logits and out must be 16-byte aligned device pointers");
    if (flags != MOE_OUT_ACCUMULATE && flags != MOE_OUT_OVERWRITE) return fail(MOE_INVALID_ARGUMENT, "bad flags");
    const int H = h->desc.hidden;
    const size_t xbytes = static_cast<size_t>(tokens) * H * 4, lbytes = static_cast<size_t>(tokens) * kRouterExperts * 4;
    if (overlap(out, xbytes, logits, lbytes)) return fail(MOE_INVALID_ARGUMENT, "out overlaps logits");
    if (flags == MOE_OUT_OVERWRITE && overlap(out, xbytes, x, xbytes))
        return fail(MOE_INVALID_ARGUMENT, "overwrite requires out disjoint from x (accumulate may alias exactly)");
    if (flags == MOE_OUT_ACCUMULATE && overlap(out, xbytes, x, xbytes) && out != x)
        return fail(MOE_INVALID_ARGUMENT, "out may alias x only exactly");
    DeviceGuard guard(h->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    if (flags == MOE_OUT_OVERWRITE) MOE_CUDA(cudaMemsetAsync(out, 0, xbytes, s));
    if (tokens > kChunk)   // small batches quantise inside the fused routing kernel
        if (const int st = launch_quantize(x, static_cast<size_t>(tokens) * H / 32, h->xq, nullptr, h->error, h->sms, s))
            return st;
    if (const int st = launch_route(h, w, x, logits, tokens, nullptr, s)) return st;
    // Above decode size every group runs on the tensor-core kernels (the
    // device writes the tile count; this is its upper bound).
    const bool tc = tokens > kChunk && w->tc_ok;
    const int tc_tiles = tc ? tc_tiles_bound(tokens * (kTopK + 1)) : 0;
    return launch_experts(h, w, out, tiles_bound(tokens, h->desc.has_shared), s, events, tc_tiles, nullptr, !tc, tap);
}
}  // namespace

extern "C" {

int moe_forward_profiled(moe_layer_t h, moe_weights_t w, const float *x, const float *logits, int tokens,
                         float *out, int flags, void *stream, void *const *events) {
    return forward_impl(h, w, x, logits, tokens, out, flags, stream, events, nullptr);
}

int moe_debug_expf(uint32_t first_bits, uint32_t count, float *out, void *stream) {
    if (!out) return fail(MOE_INVALID_ARGUMENT, "null output");
    if (count == 0) return MOE_OK;
    if (static_cast<uint64_t>(first_bits) + count - 1 > 0xffffffffull)
        return fail(MOE_INVALID_ARGUMENT, "the input range passes 0xffffffff");
    if (const int st = expf_table_upload()) return st;
    int device = 0;
    MOE_CUDA(cudaGetDevice(&device));
    debug_expf_kernel<<<sm_count(device) * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(first_bits, count, out);
    return cuda_status(cudaGetLastError(), "debug_expf_kernel");
}

int moe_debug_block_dots(moe_layer_t h, moe_weights_t w, const float *x, const float *logits, int tokens, int expert,
                         int max_pairs, int32_t *gate_dots, int32_t *up_dots, int32_t *down_dots, int8_t *mid_codes,
                         uint32_t *mid_ds, float *out, void *stream) {
    if (!h || !w) return fail(MOE_INVALID_ARGUMENT, "null layer or weights");
    if (expert < 0 || expert > w->expert_count || (expert == w->expert_count && !h->desc.has_shared))
        return fail(MOE_INVALID_ARGUMENT, "expert must be a routed expert index or the shared expert's");
    if (max_pairs < 1 || max_pairs > h->desc.max_tokens)
        return fail(MOE_INVALID_ARGUMENT, "max_pairs must be 1..max_tokens");
    const int H = h->desc.hidden, I = h->desc.inter;
    const size_t gbytes = static_cast<size_t>(max_pairs) * I * (H / 32) * 4;
    const size_t dbytes = static_cast<size_t>(max_pairs) * H * (I / 32) * 4;
    const void *outs[5] = {gate_dots, up_dots, down_dots, mid_codes, mid_ds};
    const size_t sizes[5] = {gbytes, gbytes, dbytes, static_cast<size_t>(max_pairs) * I,
                             static_cast<size_t>(max_pairs) * (I / 32) * 4};
    for (int i = 0; i < 5; ++i) {
        if (!aligned(outs[i], 4)) return fail(MOE_INVALID_ARGUMENT, "null or misaligned tap buffer");
        for (int j = 0; j < i; ++j)
            if (overlap(outs[i], sizes[i], outs[j], sizes[j])) return fail(MOE_INVALID_ARGUMENT, "tap buffers overlap");
    }
    TapSink tap;
    tap.expert = expert;
    tap.pair0 = h->offsets + expert;   // offsets[512] is the shared expert's first pair
    tap.max_pairs = max_pairs;
    tap.gate = gate_dots;
    tap.up = up_dots;
    tap.down = down_dots;
    tap.mid_codes = mid_codes;
    tap.mid_ds = mid_ds;
    return forward_impl(h, w, x, logits, tokens, out, MOE_OUT_OVERWRITE, stream, nullptr, &tap);
}

int moe_router_logits(moe_weights_t w, const float *x, int tokens, float *logits, void *stream) {
    if (!w || !w->router) return fail(MOE_INVALID_ARGUMENT, "null weights or no router matrix");
    if (tokens < 1 || tokens > 65536) return fail(MOE_INVALID_ARGUMENT, "tokens must be 1..65536");
    const int H = w->desc.hidden;
    if (!aligned(x, 16) || !aligned(logits, 16) ||
        overlap(logits, static_cast<size_t>(tokens) * kRouterExperts * 4, x, static_cast<size_t>(tokens) * H * 4))
        return fail(MOE_INVALID_ARGUMENT, "x and logits must be disjoint 16-byte aligned device buffers");
    DeviceGuard guard(w->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    if (tokens <= kRouterGemvTokens)
        router_gemv_kernel<<<kRouterExperts / kRouterGemvWarps, 32 * kRouterGemvWarps, 0, s>>>(x, w->router, logits,
                                                                                              tokens, H);
    else
        router_gemm_kernel<<<dim3(kRouterExperts / kRouterTile, (tokens + kRouterTile - 1) / kRouterTile), 256, 0, s>>>(
            x, w->router, logits, tokens, H);
    return cuda_status(cudaGetLastError(), "router kernel");
}

int moe_forward_hidden(moe_layer_t h, moe_weights_t w, const float *x, int tokens, float *out, int flags,
                       void *stream) {
    if (!h || !w) return fail(MOE_INVALID_ARGUMENT, "null layer or weights");
    if (tokens < 1 || tokens > h->desc.max_tokens) return fail(MOE_INVALID_ARGUMENT, "tokens outside 1..max_tokens");
    if (const int st = moe_router_logits(w, x, tokens, h->logits, stream)) return st;
    return moe_forward_profiled(h, w, x, h->logits, tokens, out, flags, stream, nullptr);
}

int moe_forward_contributions(moe_layer_t h, moe_weights_t w, const float *x, const float *logits, int tokens,
                              float *contrib, float *shared, float *out, int flags, void *stream) {
    if (!h || !w) return fail(MOE_INVALID_ARGUMENT, "null layer or weights");
    if (std::memcmp(&h->desc, &w->desc, offsetof(moe_layer_desc, device) + sizeof(int)) != 0)
        return fail(MOE_INVALID_ARGUMENT, "layer and weights describe different shapes or devices");
    if (tokens < 1 || tokens > h->desc.max_tokens) return fail(MOE_INVALID_ARGUMENT, "tokens outside 1..max_tokens");
    if (flags != MOE_OUT_ACCUMULATE && flags != MOE_OUT_OVERWRITE) return fail(MOE_INVALID_ARGUMENT, "bad flags");
    const int H = h->desc.hidden;
    const size_t xbytes = static_cast<size_t>(tokens) * H * 4, lbytes = static_cast<size_t>(tokens) * kRouterExperts * 4;
    const size_t cbytes = xbytes * kTopK;
    if (!aligned(x, 16) || !aligned(logits, 16) || !aligned(out, 16) || !aligned(contrib, 16) ||
        (h->desc.has_shared && !aligned(shared, 16)) || (!h->desc.has_shared && shared))
        return fail(MOE_INVALID_ARGUMENT, "x, logits, out, contributions (and shared, exactly when the layer has a "
                                          "shared expert) must be 16-byte aligned device pointers");
    if (overlap(out, xbytes, logits, lbytes) || overlap(contrib, cbytes, x, xbytes) ||
        overlap(contrib, cbytes, logits, lbytes) || overlap(contrib, cbytes, out, xbytes) ||
        (shared && (overlap(shared, xbytes, x, xbytes) || overlap(shared, xbytes, logits, lbytes) ||
                    overlap(shared, xbytes, out, xbytes) || overlap(shared, xbytes, contrib, cbytes))))
        return fail(MOE_INVALID_ARGUMENT, "trace buffers overlap an input or out");
    if (flags == MOE_OUT_OVERWRITE && overlap(out, xbytes, x, xbytes))
        return fail(MOE_INVALID_ARGUMENT, "overwrite requires out disjoint from x (accumulate may alias exactly)");
    if (flags == MOE_OUT_ACCUMULATE && overlap(out, xbytes, x, xbytes) && out != x)
        return fail(MOE_INVALID_ARGUMENT, "out may alias x only exactly");
    DeviceGuard guard(h->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    // every (token, rank) row is written by its pair; zero first so a token
    // whose routing failed (flagged) still folds defined values
    MOE_CUDA(cudaMemsetAsync(contrib, 0, cbytes, s));
    if (shared) MOE_CUDA(cudaMemsetAsync(shared, 0, xbytes, s));
    if (tokens > kChunk)
        if (const int st = launch_quantize(x, static_cast<size_t>(tokens) * H / 32, h->xq, nullptr, h->error, h->sms, s))
            return st;
    if (const int st = launch_route(h, w, x, logits, tokens, nullptr, s, nullptr, nullptr, false)) return st;
    DownSink trace;
    trace.contrib = contrib;
    trace.shared = shared;
    trace.pair_rank = h->pair_rank;
    trace.shared_expert = w->expert_count;
    if (const int st = launch_experts(h, w, nullptr, tiles_bound(tokens, h->desc.has_shared), s, nullptr, 0, &trace))
        return st;
    fold_kernel<<<std::min<size_t>((xbytes / 4 + 255) / 256, static_cast<size_t>(h->sms) * 8), 256, 0, s>>>(
        contrib, h->weights, shared, h->pair_weight + static_cast<size_t>(tokens) * kTopK, tokens, H, out,
        flags == MOE_OUT_OVERWRITE, h->error);
    return cuda_status(cudaGetLastError(), "fold_kernel");
}

int moe_quantize_q8_1(const float *x, int width, int columns, void *q8, int *error, void *stream) {
    if (width <= 0 || width > 16384 || width % 32 || columns <= 0 || columns > 65536)
        return fail(MOE_INVALID_ARGUMENT, "width must be 32..16384 and a multiple of 32; columns 1..65536");
    const size_t n = static_cast<size_t>(width) * columns;
    if (!aligned(x, 4) || !aligned(q8, 4) || !aligned(error, 4) || overlap(q8, n / 32 * 36, x, n * 4) ||
        overlap(error, 4, x, n * 4) || overlap(error, 4, q8, n / 32 * 36))
        return fail(MOE_INVALID_ARGUMENT, "null, misaligned or overlapping quantize buffers");
    int device = 0;
    MOE_CUDA(cudaGetDevice(&device));
    Q8Planar none{nullptr, nullptr};
    return launch_quantize(x, n / 32, none, static_cast<uint8_t *>(q8), error, sm_count(device),
                           static_cast<cudaStream_t>(stream));
}

int moe_q4_linear(const void *w, int rows, int k, const void *xq, int columns, float *out, int32_t *dots,
                  void *stream) {
    if (rows <= 0 || rows > 65536 || k <= 0 || k > 16384 || k % 32 || columns <= 0 || columns > 65536)
        return fail(MOE_INVALID_ARGUMENT, "bad linear shape");
    if (!aligned(w, 2) || !aligned(xq, 4) || !aligned(out, 4) || (dots && !aligned(dots, 4)))
        return fail(MOE_INVALID_ARGUMENT, "null or misaligned linear buffers");
    const size_t nb = k / 32;
    if (overlap(out, static_cast<size_t>(rows) * columns * 4, w, rows * nb * 18) ||
        overlap(out, static_cast<size_t>(rows) * columns * 4, xq, columns * nb * 36))
        return fail(MOE_INVALID_ARGUMENT, "output overlaps an input");
    int device = 0;
    MOE_CUDA(cudaGetDevice(&device));
    q4_linear_kernel<<<sm_count(device) * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t *>(w), nullptr, nullptr, rows, static_cast<int>(nb),
        static_cast<const uint8_t *>(xq), columns, out, dots);
    return cuda_status(cudaGetLastError(), "q4_linear_kernel");
}

int moe_q4_1_linear(const void *w, int rows, int k, const void *xq, int columns, float *out, int32_t *dots,
                    void *stream) {
    if (rows <= 0 || rows > 65536 || k <= 0 || k > 16384 || k % 32 || columns <= 0 || columns > 65536)
        return fail(MOE_INVALID_ARGUMENT, "bad linear shape");
    if (!aligned(w, 2) || !aligned(xq, 4) || !aligned(out, 4) || (dots && !aligned(dots, 4)))
        return fail(MOE_INVALID_ARGUMENT, "null or misaligned linear buffers");
    const size_t nb = k / 32;
    if (overlap(out, static_cast<size_t>(rows) * columns * 4, w, rows * nb * 20) ||
        overlap(out, static_cast<size_t>(rows) * columns * 4, xq, columns * nb * 36))
        return fail(MOE_INVALID_ARGUMENT, "output overlaps an input");
    int device = 0;
    MOE_CUDA(cudaGetDevice(&device));
    q4_1_linear_kernel<<<sm_count(device) * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t *>(w), nullptr, nullptr, nullptr, rows, static_cast<int>(nb),
        static_cast<const uint8_t *>(xq), columns, out, dots);
    return cuda_status(cudaGetLastError(), "q4_1_linear_kernel");
}

// ------------------------------------------------- single-expert fixture --
}  // extern "C"

struct moe_expert_s {
    moe_layer_desc desc;
    moe_weights_s *w = nullptr;
    moe_layer_s *h = nullptr;
    int max_columns;
    cudaStream_t stream = nullptr;
    cudaEvent_t begin = nullptr, end = nullptr;
    float *x = nullptr, *y = nullptr;
    uint8_t *q8 = nullptr;
    double upload_ms = 0;
};

namespace {
int expert_forward(moe_expert_s *e, int columns) {
    moe_layer_s *h = e->h;
    if (const int st = launch_quantize(e->x, static_cast<size_t>(columns) * e->desc.hidden / 32, h->xq, nullptr,
                                       h->error, h->sms, e->stream))
        return st;
    identity_route_kernel<<<(columns + 255) / 256, 256, 0, e->stream>>>(columns, kGemvTile, h->tiles, h->num_tiles,
                                                                        h->pair_token, h->pair_weight);
    MOE_CUDA(cudaGetLastError());
    MOE_CUDA(cudaMemsetAsync(e->y, 0, sizeof(float) * columns * e->desc.hidden, e->stream));
    return launch_experts(h, e->w, e->y, (columns + kGemvTile - 1) / kGemvTile, e->stream);
}
}  // namespace

extern "C" {

int moe_expert_destroy(moe_expert_t e) {
    if (!e) return MOE_OK;
    DeviceGuard guard(e->desc.device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    moe_layer_destroy(e->h);
    moe_weights_destroy(e->w);
    cudaFree(e->x);
    cudaFree(e->y);
    cudaFree(e->q8);
    if (e->begin) cudaEventDestroy(e->begin);
    if (e->end) cudaEventDestroy(e->end);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return MOE_OK;
}

int moe_expert_create(const void *gate, const void *up, const void *down, int hidden, int inter, int device,
                      int max_columns, moe_expert_t *out) {
    return moe_expert_create_typed(gate, up, down, MOE_Q4_0, hidden, inter, device, max_columns, out);
}

int moe_expert_create_typed(const void *gate, const void *up, const void *down, int down_type, int hidden, int inter,
                            int device, int max_columns, moe_expert_t *out) {
    if (!out) return fail(MOE_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    if (down_type != MOE_Q4_0 && down_type != MOE_Q4_1)
        return fail(MOE_NOT_SUPPORTED, "down matrices must be Q4_0 or Q4_1");
    if (max_columns <= 0 || max_columns > 1024) return fail(MOE_INVALID_ARGUMENT, "max_columns must be 1..1024");
    if (!gate || !up || !down) return fail(MOE_INVALID_ARGUMENT, "null expert weights");
    moe_layer_desc d{hidden, inter, kRouterExperts, kTopK, 0, device, max_columns};
    if (const int st = validate_desc(&d)) return st;
    DeviceGuard guard(device);
    MOE_CUDA(guard.status);
    auto *e = new (std::nothrow) moe_expert_s();
    if (!e) return fail(MOE_OUT_OF_MEMORY, "host allocation");
    e->desc = d;
    e->max_columns = max_columns;
    // one expert region only: the fixture never routes
    auto *w = new (std::nothrow) moe_weights_s();
    if (!w) { delete e; return fail(MOE_OUT_OF_MEMORY, "host allocation"); }
    w->desc = d;
    w->layout = make_layout(hidden, inter, down_type == MOE_Q4_1 ? kDownQ4_1 : kDownQ4_0);
    w->experts_total = 1;
    e->w = w;
    int st = cuda_status(cudaMalloc(&w->base, w->layout.bytes), "cudaMalloc");
    if (!st) st = cuda_status(cudaMalloc(&w->gate_vec, sizeof(float) * hidden), "cudaMalloc");
    if (!st) st = cuda_status(cudaMalloc(&w->staging, w->layout.bytes / 16 * 18), "cudaMalloc");
    if (!st) st = build_maps(w);
    if (!st) st = cuda_status(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "stream");
    if (!st) st = cuda_status(cudaEventCreate(&e->begin), "event");
    if (!st) st = cuda_status(cudaEventCreate(&e->end), "event");
    const size_t n = static_cast<size_t>(max_columns) * std::max(hidden, inter);
    if (!st) st = cuda_status(cudaMalloc(&e->x, n * 4), "cudaMalloc");
    if (!st) st = cuda_status(cudaMalloc(&e->y, n * 4), "cudaMalloc");
    if (!st) st = cuda_status(cudaMalloc(&e->q8, n / 32 * 36), "cudaMalloc");
    if (!st) st = moe_layer_create(&d, &e->h);
    if (!st) {
        const auto t0 = std::chrono::steady_clock::now();
        st = moe_weights_upload_expert(w, 0, gate, up, down, e->stream);
        if (!st) st = cuda_status(cudaStreamSynchronize(e->stream), "upload");   // the reference times the finished upload
        e->upload_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    }
    if (st) { moe_expert_destroy(e); return st; }
    *out = e;
    return MOE_OK;
}

int moe_expert_check_quantization(moe_expert_t e, const float *input, size_t n, const void *expected) {
    if (!e || !input || !expected) return fail(MOE_INVALID_ARGUMENT, "null argument");
    if (n == 0 || n % 32 || n > static_cast<size_t>(e->desc.hidden) * e->max_columns)
        return fail(MOE_INVALID_ARGUMENT, "GPU quantization span");
    DeviceGuard guard(e->desc.device);
    MOE_CUDA(guard.status);
    int *err = e->h->error;
    MOE_CUDA(cudaMemsetAsync(err, 0, 4, e->stream));
    MOE_CUDA(cudaMemcpyAsync(e->x, input, n * 4, cudaMemcpyHostToDevice, e->stream));
    Q8Planar none{nullptr, nullptr};
    if (const int st = launch_quantize(e->x, n / 32, none, e->q8, err, e->h->sms, e->stream)) return st;
    auto *result = new (std::nothrow) uint8_t[n / 32 * 36];
    if (!result) return fail(MOE_OUT_OF_MEMORY, "host allocation");
    int flags = 0;
    cudaError_t ce = cudaMemcpyAsync(result, e->q8, n / 32 * 36, cudaMemcpyDeviceToHost, e->stream);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(&flags, err, 4, cudaMemcpyDeviceToHost, e->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
    int st = cuda_status(ce, "check_quantization");
    if (!st && flags) st = fail(MOE_INVALID_ARGUMENT, "GPU activation not representable in Q8_1");
    if (!st && std::memcmp(result, expected, n / 32 * 36)) st = fail(MOE_NUMERIC_ERROR, "CPU/GPU Q8_1 ABI mismatch");
    delete[] result;
    return st;
}

int moe_expert_linear(moe_expert_t e, int down, int up, const void *input, int columns, float *output) {
    if (!e || !input || !output) return fail(MOE_INVALID_ARGUMENT, "null argument");
    if (columns <= 0 || columns > e->max_columns) return fail(MOE_INVALID_ARGUMENT, "GPU linear span");
    DeviceGuard guard(e->desc.device);
    MOE_CUDA(guard.status);
    const ExpertLayout &L = e->w->layout;
    const int in = down ? L.inter : L.hidden, rows = down ? L.hidden : L.inter;
    const uint8_t *ex = e->w->base;
    const size_t co = down ? L.down_codes : up ? L.up_codes : L.gate_codes;
    const size_t so = down ? L.down_scales : up ? L.up_scales : L.gate_scales;
    MOE_CUDA(cudaMemcpyAsync(e->q8, input, static_cast<size_t>(columns) * (in / 32) * 36, cudaMemcpyHostToDevice,
                             e->stream));
    if (down && L.down_type == kDownQ4_1)
        q4_1_linear_kernel<<<e->h->sms * 8, 256, 0, e->stream>>>(
            nullptr, ex + co, reinterpret_cast<const uint16_t *>(ex + so),
            reinterpret_cast<const uint16_t *>(ex + L.down_mins), rows, in / 32, e->q8, columns, e->y, nullptr);
    else
        q4_linear_kernel<<<e->h->sms * 8, 256, 0, e->stream>>>(nullptr, ex + co, reinterpret_cast<const uint16_t *>(ex + so),
                                                               rows, in / 32, e->q8, columns, e->y, nullptr);
    MOE_CUDA(cudaGetLastError());
    MOE_CUDA(cudaMemcpyAsync(output, e->y, static_cast<size_t>(columns) * rows * 4, cudaMemcpyDeviceToHost, e->stream));
    MOE_CUDA(cudaStreamSynchronize(e->stream));
    return MOE_OK;
}

int moe_expert_run(moe_expert_t e, const float *input, int columns, float *output, int repeats, double *upload_ms,
                   double *resident_ms, double *wall_ms) {
    if (!e || !input || !output) return fail(MOE_INVALID_ARGUMENT, "null argument");
    if (columns <= 0 || columns > e->max_columns || repeats <= 0 || repeats > 10000)
        return fail(MOE_INVALID_ARGUMENT, "GPU expert input/output");
    DeviceGuard guard(e->desc.device);
    MOE_CUDA(guard.status);
    const size_t n = static_cast<size_t>(columns) * e->desc.hidden;
    int *err = e->h->error;
    MOE_CUDA(cudaMemsetAsync(err, 0, 4, e->stream));
    MOE_CUDA(cudaMemcpyAsync(e->x, input, n * 4, cudaMemcpyHostToDevice, e->stream));
    if (const int st = expert_forward(e, columns)) return st;  // warm-up outside timing
    const auto t0 = std::chrono::steady_clock::now();
    MOE_CUDA(cudaEventRecord(e->begin, e->stream));
    for (int r = 0; r < repeats; ++r)
        if (const int st = expert_forward(e, columns)) return st;
    MOE_CUDA(cudaEventRecord(e->end, e->stream));
    MOE_CUDA(cudaEventSynchronize(e->end));
    float ms = 0;
    MOE_CUDA(cudaEventElapsedTime(&ms, e->begin, e->end));
    int flags = 0;
    MOE_CUDA(cudaMemcpyAsync(&flags, err, 4, cudaMemcpyDeviceToHost, e->stream));
    MOE_CUDA(cudaMemcpyAsync(output, e->y, n * 4, cudaMemcpyDeviceToHost, e->stream));
    MOE_CUDA(cudaStreamSynchronize(e->stream));
    const double wall = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (upload_ms) *upload_ms = e->upload_ms;
    if (resident_ms) *resident_ms = ms / repeats;
    if (wall_ms) *wall_ms = wall / repeats;
    if (flags) return fail(MOE_NUMERIC_ERROR, "GPU expert numeric flag");
    return MOE_OK;
}

}  // extern "C"

// ------------------------------------------------ allocation-free routing --
// moe_route_noalloc is moe_route for callers that cannot allocate device
// memory: code that enqueues its work inside CUDA stream capture (a capture
// cannot contain cudaMalloc, and an allocation made outside it would have to
// outlive the graph), and hosts whose device memory is owned by another
// allocator or a fixed arena (a serving engine, a caching allocator) and that
// therefore cannot hand this library a workspace of its own.  Its scratch is
// one file-scope device array, sized for at most kNoAllocMaxTokens tokens,
// that every GPU loading this library holds until the process exits.
namespace {

constexpr int kNoAllocMaxTokens = 1024;
constexpr int kNoAllocChunks = kNoAllocMaxTokens / kChunk;
constexpr int kNoAllocTiles = kNoAllocMaxTokens * kTopK / kGemvTile + kRouterExperts;

constexpr size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct NoAllocLayout {
    size_t masks, base, counts, offsets, pair_weight, tiles, tile_off, num_tiles, bytes;
};

constexpr NoAllocLayout noalloc_layout() {
    NoAllocLayout L{};
    size_t at = 0;
    L.masks = at;        at = align256(at + sizeof(uint32_t) * kNoAllocChunks * kRouterExperts);
    L.base = at;         at = align256(at + sizeof(int32_t) * kNoAllocChunks * kRouterExperts);
    L.counts = at;       at = align256(at + sizeof(int32_t) * kRouterExperts);
    L.offsets = at;      at = align256(at + sizeof(int32_t) * (kRouterExperts + 2));
    L.pair_weight = at;  at = align256(at + sizeof(float) * kNoAllocMaxTokens * kTopK);
    L.tiles = at;        at = align256(at + sizeof(TileRec) * kNoAllocTiles);
    L.tile_off = at;     at = align256(at + sizeof(int32_t) * kRouterExperts);
    L.num_tiles = at;    at = align256(at + 2 * sizeof(int));
    L.bytes = at;
    return L;
}

constexpr NoAllocLayout kNoAlloc = noalloc_layout();   // 326,144 bytes

// The scratch itself.  In host code this name is only a handle for
// cudaGetSymbolAddress, never a device address.
static __device__ __align__(256) unsigned char g_route_scratch[kNoAlloc.bytes];

constexpr int kNoAllocDevices = 64;
std::mutex g_noalloc_mutex;
void *g_noalloc_address[kNoAllocDevices] = {};

// Resolve the array's address on the current device once and cache it.
int noalloc_scratch(uint8_t **out) {
    int device = 0;
    MOE_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= kNoAllocDevices) return fail(MOE_NOT_SUPPORTED, "device ordinal above 63");
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_address[device]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
        if (e != cudaSuccess || !p) return cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                                                       "cudaGetSymbolAddress(route scratch)");
        g_noalloc_address[device] = p;
    }
    *out = static_cast<uint8_t *>(g_noalloc_address[device]);
    return MOE_OK;
}

}  // namespace

extern "C" int moe_route_noalloc(const float *logits, int tokens, int32_t *ids, float *weights, int32_t *offsets,
                                 int32_t *token, int32_t *rank, int *error, void *stream) {
    if (tokens < 1 || tokens > kNoAllocMaxTokens)
        return fail(MOE_INVALID_ARGUMENT, "moe_route_noalloc: tokens must be 1..1024 (size of its static scratch)");
    const size_t n = static_cast<size_t>(tokens) * kTopK;
    if (!aligned(logits, 4) || !aligned(ids, 4) || !aligned(weights, 4) || !aligned(offsets, 4) ||
        !aligned(token, 4) || !aligned(rank, 4) || !aligned(error, 4))
        return fail(MOE_INVALID_ARGUMENT, "moe_route_noalloc: null or misaligned pointer");
    const size_t lbytes = static_cast<size_t>(tokens) * kRouterExperts * 4;
    const void *outs[6] = {ids, weights, offsets, token, rank, error};
    const size_t sizes[6] = {n * 4, n * 4, (kRouterExperts + 1) * 4, n * 4, n * 4, 4};
    for (int i = 0; i < 6; ++i) {
        if (overlap(outs[i], sizes[i], logits, lbytes)) return fail(MOE_INVALID_ARGUMENT, "output overlaps logits");
        for (int j = 0; j < i; ++j)
            if (overlap(outs[i], sizes[i], outs[j], sizes[j])) return fail(MOE_INVALID_ARGUMENT, "outputs overlap");
    }
    uint8_t *sc = nullptr;
    if (const int st = noalloc_scratch(&sc)) return st;
    auto s = static_cast<cudaStream_t>(stream);
    const int chunks = (tokens + kChunk - 1) / kChunk;
    auto *masks = reinterpret_cast<uint32_t *>(sc + kNoAlloc.masks);
    auto *base = reinterpret_cast<int32_t *>(sc + kNoAlloc.base);
    auto *counts = reinterpret_cast<int32_t *>(sc + kNoAlloc.counts);
    auto *offs = reinterpret_cast<int32_t *>(sc + kNoAlloc.offsets);
    auto *pair_weight = reinterpret_cast<float *>(sc + kNoAlloc.pair_weight);
    auto *tiles = reinterpret_cast<TileRec *>(sc + kNoAlloc.tiles);
    auto *tile_off = reinterpret_cast<int32_t *>(sc + kNoAlloc.tile_off);
    auto *num_tiles = reinterpret_cast<int *>(sc + kNoAlloc.num_tiles);
    RouteParams rp;
    rp.logits = logits;
    rp.x = nullptr;
    rp.gate_vec = nullptr;
    rp.tokens = tokens;
    rp.hidden = 0;
    rp.probs = nullptr;
    rp.ids = ids;
    rp.weights = weights;
    rp.masks = masks;
    rp.pair_token = token;
    rp.pair_weight = pair_weight;
    rp.pair_rank = rank;
    rp.error = error;
    if (tokens <= kChunk) {
        SmallRouteParams sr;
        sr.r = rp;
        sr.xq = Q8Planar{nullptr, nullptr};
        sr.offsets = offs;
        sr.tiles = tiles;
        sr.tile_off = tile_off;
        sr.num_tiles = num_tiles;
        sr.max_tiles = kNoAllocTiles;
        route_small_kernel<<<1, 512, 0, s>>>(sr);
        MOE_CUDA(cudaGetLastError());
    } else {
        route_topk_kernel<<<chunks, kRouteThreads, 0, s>>>(rp);
        MOE_CUDA(cudaGetLastError());
        route_chunk_prefix_kernel<<<kRouterExperts / 32, 1024, 0, s>>>(masks, chunks, base, counts);
        MOE_CUDA(cudaGetLastError());
        ScanParams sp;
        sp.counts = counts;
        sp.tokens = tokens;
        sp.tile = kGemvTile;
        sp.has_shared = 0;
        sp.offsets = offs;
        sp.tiles = tiles;
        sp.tile_off = tile_off;
        sp.pair_token = token;
        sp.pair_weight = pair_weight;
        sp.num_tiles = num_tiles;
        sp.max_tiles = kNoAllocTiles;
        sp.error = error;
        route_scan_kernel<<<1, 512, 0, s>>>(sp);
        MOE_CUDA(cudaGetLastError());
        ScatterParams cp;
        cp.masks = masks;
        cp.base = base;
        cp.offsets = offs;
        cp.ids = ids;
        cp.weights = weights;
        cp.pair_token = token;
        cp.pair_rank = rank;
        cp.pair_weight = pair_weight;
        cp.tiles = tiles;
        cp.tile_off = tile_off;
        cp.max_tiles = kNoAllocTiles;
        route_scatter_kernel<<<dim3(chunks, kRouterExperts / 256), 256, 0, s>>>(cp);
        MOE_CUDA(cudaGetLastError());
    }
    MOE_CUDA(cudaMemcpyAsync(offsets, offs, (kRouterExperts + 1) * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
    return MOE_OK;
}

// ------------------------------------------------- expert parallelism --
// Rank-local state.  `tx` is an ordinary layer workspace for the rank's own
// tokens (quantisation, routing, shared gate); `rx` views the received slots
// as the "tokens" of the expert kernels: its x rows are the exported receive
// buffer and its output is the exported partial buffer.
struct moe_ep_s {
    moe_layer_desc desc;
    int rank = 0, world = 1, ecount = kRouterExperts, t_max = 0, slots = 0, rx_tiles = 0, rx_pairs = 0;
    bool tc = false;                 // received groups may use the tensor-core kernels
    moe_layer_s *tx = nullptr;
    moe_layer_s rx;                  // views into `exported` and `local`
    EpLayout L;
    uint8_t *exported = nullptr;     // IPC-exported arena (EpLayout)
    Arena local;                     // rx workspace + plan buffers
    EpPeers peers{};
    bool opened[kEpMaxRanks] = {};
    int32_t *pos = nullptr, *counts = nullptr;
    uint8_t *dmask = nullptr;
    uint32_t *epoch = nullptr, *blocks_done = nullptr, *quant_done = nullptr;
};

namespace {

void ep_take_rx(moe_ep_s *ep, Arena &a) {
    const int H = ep->desc.hidden, I = ep->desc.inter, S = ep->slots;
    moe_layer_s &r = ep->rx;
    const int pairs = ep->rx_pairs;
    r.mid.codes = a.take<int8_t>(static_cast<size_t>(pairs) * I);
    r.mid.scales = a.take<float2>(static_cast<size_t>(pairs) * (I / 32));
    r.masks = a.take<uint32_t>(static_cast<size_t>(S / kChunk) * kRouterExperts);
    r.base = a.take<int32_t>(static_cast<size_t>(S / kChunk) * kRouterExperts);
    r.counts = a.take<int32_t>(kRouterExperts);
    r.offsets = a.take<int32_t>(kRouterExperts + 2);
    r.pair_token = a.take<int32_t>(pairs);
    r.pair_rank = a.take<int32_t>(pairs);
    r.pair_weight = a.take<float>(pairs);
    r.tiles = a.take<TileRec>(ep->rx_tiles);
    r.tile_off = a.take<int32_t>(kRouterExperts);
    r.num_tiles = a.take<int>(2);
    r.error = a.take<int>(1);
    tc_workspace_take(r.tc, a, pairs, H, I, ep->tc);
    ep->pos = a.take<int32_t>(static_cast<size_t>(ep->t_max) * kEpMaxRanks);
    ep->dmask = a.take<uint8_t>(ep->t_max);
    ep->counts = a.take<int32_t>(kEpMaxRanks);
    ep->epoch = a.take<uint32_t>(1);
    ep->blocks_done = a.take<uint32_t>(1);
    ep->quant_done = a.take<uint32_t>(1);
}

EpParams ep_params(moe_ep_s *ep, int tokens, float *out) {
    EpParams p;
    p.peers = ep->peers;
    p.L = ep->L;
    p.rank = ep->rank;
    p.world = ep->world;
    p.ecount = ep->ecount;
    p.t_max = ep->t_max;
    p.tokens = tokens;
    p.hidden = ep->desc.hidden;
    p.ids = ep->tx->ids;
    p.weights = ep->tx->weights;
    p.xcodes = ep->tx->xq.codes;
    p.xscales = ep->tx->xq.scales;
    p.pos = ep->pos;
    p.dmask = ep->dmask;
    p.counts = ep->counts;
    p.epoch = ep->epoch;
    p.blocks_done = ep->blocks_done;
    p.out = out;
    p.error = ep->rx.error;
    return p;
}

}  // namespace

extern "C" {

int moe_ep_weights_create(const moe_layer_desc *desc, int rank, int world, moe_weights_t *out) {
    return moe_ep_weights_create_typed(desc, rank, world, MOE_Q4_0, out);
}

int moe_ep_weights_create_typed(const moe_layer_desc *desc, int rank, int world, int down_type, moe_weights_t *out) {
    if (!out) return fail(MOE_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    if (const int st = validate_desc(desc)) return st;
    if (down_type != MOE_Q4_0 && down_type != MOE_Q4_1)
        return fail(MOE_NOT_SUPPORTED, "down matrices must be Q4_0 or Q4_1");
    if (!(world == 1 || world == 2 || world == 4 || world == 8) || rank < 0 || rank >= world)
        return fail(MOE_INVALID_ARGUMENT, "world must be 1, 2, 4 or 8 and 0 <= rank < world");
    DeviceGuard guard(desc->device);
    MOE_CUDA(guard.status);
    auto *w = new (std::nothrow) moe_weights_s();
    if (!w) return fail(MOE_OUT_OF_MEMORY, "host allocation");
    w->desc = *desc;
    w->layout = make_layout(desc->hidden, desc->inter, down_type == MOE_Q4_1 ? kDownQ4_1 : kDownQ4_0);
    w->expert_count = kRouterExperts / world;
    w->expert_first = rank * w->expert_count;
    w->experts_total = w->expert_count + desc->has_shared;
    const size_t rbytes = sizeof(float) * kRouterExperts * desc->hidden;
    cudaError_t e = cudaMalloc(&w->base, w->layout.bytes * w->experts_total);
    if (e == cudaSuccess) e = cudaMalloc(&w->gate_vec, sizeof(float) * desc->hidden);
    if (e == cudaSuccess) e = cudaMalloc(&w->router, rbytes);
    if (e == cudaSuccess) e = cudaMalloc(&w->staging, w->layout.bytes / 16 * 18);
    if (e == cudaSuccess) e = cudaMemset(w->gate_vec, 0, sizeof(float) * desc->hidden);
    if (e == cudaSuccess) e = cudaMemset(w->router, 0, rbytes);
    const int st = e != cudaSuccess ? cuda_status(e, "moe_ep_weights_create") : build_maps(w);
    if (st) {
        cudaFree(w->base); cudaFree(w->gate_vec); cudaFree(w->router); cudaFree(w->staging);
        delete w;
        return st;
    }
    *out = w;
    return MOE_OK;
}

int moe_ep_create(const moe_layer_desc *desc, int rank, int world, moe_ep_t *out) {
    if (!out) return fail(MOE_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    if (const int st = validate_desc(desc)) return st;
    if (!(world == 1 || world == 2 || world == 4 || world == 8) || rank < 0 || rank >= world)
        return fail(MOE_INVALID_ARGUMENT, "world must be 1, 2, 4 or 8 and 0 <= rank < world");
    if (desc->max_tokens > 32768) return fail(MOE_INVALID_ARGUMENT, "expert-parallel max_tokens is 1..32768");
    DeviceGuard guard(desc->device);
    MOE_CUDA(guard.status);
    auto *ep = new (std::nothrow) moe_ep_s();
    if (!ep) return fail(MOE_OUT_OF_MEMORY, "host allocation");
    ep->desc = *desc;
    ep->rank = rank;
    ep->world = world;
    ep->ecount = kRouterExperts / world;
    ep->t_max = (desc->max_tokens + kChunk - 1) / kChunk * kChunk;   // slot regions of whole chunks
    ep->slots = world * ep->t_max;
    ep->tc = ep->t_max > kChunk;
    ep->rx_pairs = ep->slots * kTopK + ep->t_max;
    ep->rx_tiles = ep->rx_pairs / kGemvTile + kRouterExperts + 1 + ep->t_max / kGemvTile + 1;
    auto cleanup = [&](int st) {
        if (ep->tx) moe_layer_destroy(ep->tx);
        cudaFree(ep->exported);
        cudaFree(ep->local.base);
        delete ep;
        return st;
    };
    if (const int st = moe_layer_create(desc, &ep->tx)) return cleanup(st);
    const int H = desc->hidden, I = desc->inter;
    ep->L = make_ep_layout(H, ep->slots);
    cudaError_t e = cudaMalloc(&ep->exported, ep->L.bytes);
    if (e == cudaSuccess) e = cudaMemset(ep->exported, 0, ep->L.bytes);
    // shape stamp read back by peers before they map this arena
    const uint32_t stamp[4] = {static_cast<uint32_t>(ep->L.bytes), static_cast<uint32_t>(ep->L.bytes >> 32),
                               static_cast<uint32_t>(world), static_cast<uint32_t>(ep->t_max)};
    if (e == cudaSuccess)
        e = cudaMemcpy(ep->exported + ep->L.ctl + offsetof(EpCtl, pad), stamp, sizeof(stamp), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cleanup(cuda_status(e, "moe_ep_create"));
    for (int pass = 0; pass < 2; ++pass) {
        ep->local.used = 0;
        ep_take_rx(ep, ep->local);
        if (pass == 0) {
            const size_t bytes = ep->local.used + 256;
            e = cudaMalloc(&ep->local.base, bytes);
            if (e == cudaSuccess) e = cudaMemset(ep->local.base, 0, bytes);
            if (e != cudaSuccess) return cleanup(cuda_status(e, "moe_ep_create"));
        }
    }
    moe_layer_s &r = ep->rx;
    r.desc = *desc;
    r.desc.max_tokens = ep->slots;
    r.layout = make_layout(H, I);
    r.sms = ep->tx->sms;
    r.chunks_max = ep->slots / kChunk;
    r.pairs_max = ep->rx_pairs;
    r.tiles_max = ep->rx_tiles;
    r.xq.codes = reinterpret_cast<int8_t *>(ep->exported + ep->L.codes);
    r.xq.scales = reinterpret_cast<float2 *>(ep->exported + ep->L.scales);
    r.gu_stages = ep->tx->gu_stages;
    r.dn_stages = ep->tx->dn_stages;
    ep->peers.base[rank] = ep->exported;
    *out = ep;
    return MOE_OK;
}

int moe_ep_destroy(moe_ep_t ep) {
    if (!ep) return MOE_OK;
    DeviceGuard guard(ep->desc.device);
    cudaDeviceSynchronize();
    for (int d = 0; d < ep->world; ++d)
        if (ep->opened[d]) cudaIpcCloseMemHandle(ep->peers.base[d]);
    if (ep->tx) moe_layer_destroy(ep->tx);
    cudaFree(ep->exported);
    cudaFree(ep->local.base);
    delete ep;
    return MOE_OK;
}

int moe_ep_ipc_handle(moe_ep_t ep, void *handle) {
    if (!ep || !handle) return fail(MOE_INVALID_ARGUMENT, "null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == MOE_EP_HANDLE_BYTES, "IPC handle size");
    DeviceGuard guard(ep->desc.device);
    MOE_CUDA(guard.status);
    cudaIpcMemHandle_t h;
    MOE_CUDA(cudaIpcGetMemHandle(&h, ep->exported));
    std::memcpy(handle, &h, sizeof(h));
    return MOE_OK;
}

int moe_ep_open_peers(moe_ep_t ep, const void *handles) {
    if (!ep || !handles) return fail(MOE_INVALID_ARGUMENT, "null argument");
    DeviceGuard guard(ep->desc.device);
    MOE_CUDA(guard.status);
    for (int d = 0; d < ep->world; ++d) {
        if (d == ep->rank || ep->opened[d]) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t *>(handles) + static_cast<size_t>(d) * MOE_EP_HANDLE_BYTES, sizeof(h));
        void *ptr = nullptr;
        MOE_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        uint32_t stamp[4] = {};
        const cudaError_t e = cudaMemcpy(stamp, static_cast<uint8_t *>(ptr) + ep->L.ctl + offsetof(EpCtl, pad),
                                         sizeof(stamp), cudaMemcpyDeviceToHost);
        const uint64_t bytes = stamp[0] | (static_cast<uint64_t>(stamp[1]) << 32);
        if (e != cudaSuccess || bytes != ep->L.bytes || stamp[2] != static_cast<uint32_t>(ep->world) ||
            stamp[3] != static_cast<uint32_t>(ep->t_max)) {
            cudaIpcCloseMemHandle(ptr);
            return e != cudaSuccess ? cuda_status(e, "moe_ep_open_peers")
                                    : fail(MOE_INVALID_ARGUMENT, "a peer was created with another shape, world or max_tokens");
        }
        ep->peers.base[d] = static_cast<uint8_t *>(ptr);
        ep->opened[d] = true;
    }
    MOE_CUDA(cudaDeviceSynchronize());
    return MOE_OK;
}

int moe_ep_forward(moe_ep_t ep, moe_weights_t w, const float *x, const float *logits, int tokens, float *out,
                   int flags, void *stream) {
    if (!ep || !w) return fail(MOE_INVALID_ARGUMENT, "null handle or weights");
    for (int d = 0; d < ep->world; ++d)
        if (!ep->peers.base[d]) return fail(MOE_INVALID_ARGUMENT, "peers are not open (moe_ep_open_peers)");
    if (w->expert_count != ep->ecount || w->expert_first != ep->rank * ep->ecount ||
        std::memcmp(&w->desc, &ep->desc, offsetof(moe_layer_desc, device) + sizeof(int)) != 0)
        return fail(MOE_INVALID_ARGUMENT, "weights are not this rank's expert shard of the same layer shape");
    if (tokens < 1 || tokens > ep->desc.max_tokens) return fail(MOE_INVALID_ARGUMENT, "tokens outside 1..max_tokens");
    if (!aligned(x, 16) || !aligned(logits, 16) || !aligned(out, 16))
        return fail(MOE_INVALID_ARGUMENT, "x, logits and out must be 16-byte aligned device pointers");
    if (flags != MOE_OUT_ACCUMULATE && flags != MOE_OUT_OVERWRITE) return fail(MOE_INVALID_ARGUMENT, "bad flags");
    const int H = ep->desc.hidden;
    const size_t xbytes = static_cast<size_t>(tokens) * H * 4, lbytes = static_cast<size_t>(tokens) * kRouterExperts * 4;
    if (overlap(out, xbytes, logits, lbytes)) return fail(MOE_INVALID_ARGUMENT, "out overlaps logits");
    if (flags == MOE_OUT_OVERWRITE && overlap(out, xbytes, x, xbytes))
        return fail(MOE_INVALID_ARGUMENT, "overwrite requires out disjoint from x (accumulate may alias exactly)");
    if (flags == MOE_OUT_ACCUMULATE && overlap(out, xbytes, x, xbytes) && out != x)
        return fail(MOE_INVALID_ARGUMENT, "out may alias x only exactly");
    DeviceGuard guard(ep->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    moe_layer_s *tx = ep->tx;
    // 1. own tokens: Q8_1 (+ tensor-core constants), routing, shared gate
    if (tokens > kChunk || ep->tc)
        if (const int st = launch_quantize(x, static_cast<size_t>(tokens) * H / 32, tx->xq, nullptr, tx->error,
                                           tx->sms, s))
            return st;
    EpParams p = ep_params(ep, tokens, out);
    if (tokens <= kChunk && !ep->tc) {
        // 2-3. decode sizes: the routing launch quantises, stores every row in every
        // rank at the token's fixed slot, writes each destination's expert lists
        // and publishes the epoch
        if (const int st = launch_route(tx, w, x, logits, tokens, nullptr, s, &p, ep->quant_done)) return st;
    } else if (tokens <= 32) {
        if (const int st = launch_route(tx, w, x, logits, tokens, nullptr, s)) return st;
        // 2-3. plan and dispatch (peer stores), publish epoch + counts
        ep_plan_dispatch_small_kernel<<<1, 1024, 0, s>>>(p);
        MOE_CUDA(cudaGetLastError());
    } else {
        if (const int st = launch_route(tx, w, x, logits, tokens, nullptr, s)) return st;
        ep_plan_kernel<<<1, 1024, 0, s>>>(p);
        MOE_CUDA(cudaGetLastError());
        const int items = tokens * ep->world;
        ep_dispatch_kernel<<<std::max(1, std::min((items + 7) / 8, tx->sms * 4)), 256, 0, s>>>(p);
        MOE_CUDA(cudaGetLastError());
    }
    // 4. all sources' slots received -> group by local expert
    EpCtl *ctl = reinterpret_cast<EpCtl *>(ep->exported + ep->L.ctl);
    moe_layer_s &r = ep->rx;
    float *partial = reinterpret_cast<float *>(ep->exported + ep->L.partial);
    const float *shared_w = tx->pair_weight + static_cast<size_t>(tokens) * kTopK;
    if (ep->slots <= kEpSmallSlots && !ep->tc) {
        // decode sizes: wait, masks, scan, placement and tiles in one launch
        EpSmallGroupParams g;
        g.arena = ep->exported;
        g.L = ep->L;
        g.t_max = ep->t_max;
        g.slots = ep->slots;
        g.world = ep->world;
        g.tokens = tokens;
        g.has_shared = ep->desc.has_shared;
        g.shared_token0 = ep->rank * ep->t_max;
        g.shared_expert = ep->ecount;
        g.epoch = ep->epoch;
        g.shared_w = shared_w;
        g.offsets = r.offsets;
        g.pair_token = r.pair_token;
        g.pair_rank = r.pair_rank;
        g.pair_weight = r.pair_weight;
        g.tiles = r.tiles;
        g.num_tiles = r.num_tiles;
        g.max_tiles = r.tiles_max;
        g.error = r.error;
        ep_group_small_kernel<<<1, 512, 0, s>>>(g);
        MOE_CUDA(cudaGetLastError());
    } else {
        ep_wait_kernel<<<1, 32, 0, s>>>(ctl->recv, ep->epoch, ep->world, ep->rx.error);
        MOE_CUDA(cudaGetLastError());
        const int chunks = ep->slots / kChunk;
        EpGroupParams g{ep->exported, ep->L, ep->t_max, ep->slots, H, r.masks, partial};
        ep_masks_kernel<<<chunks, 256, 0, s>>>(g);
        MOE_CUDA(cudaGetLastError());
        route_chunk_prefix_kernel<<<kRouterExperts / 32, 1024, 0, s>>>(r.masks, chunks, r.base, r.counts);
        MOE_CUDA(cudaGetLastError());
        ScanParams sp;
        sp.counts = r.counts;
        sp.tokens = tokens;          // shared-expert pairs: the own tokens
        sp.tile = kGemvTile;
        sp.has_shared = ep->desc.has_shared;
        sp.offsets = r.offsets;
        sp.tiles = r.tiles;
        sp.tile_off = r.tile_off;
        sp.pair_token = r.pair_token;
        sp.pair_weight = r.pair_weight;
        sp.num_tiles = r.num_tiles;
        sp.max_tiles = r.tiles_max;
        sp.error = r.error;
        sp.shared_w = shared_w;
        sp.shared_token0 = ep->rank * ep->t_max;
        sp.shared_expert = ep->ecount;
        if (ep->tc && w->tc_ok) {   // above decode size: every group on the tensor-core kernels
            sp.tc_min = kRowsMinGroup;
            sp.tc_tile = kTcTile;
            sp.tc_max = r.tc.max_tiles;
            sp.tc_tiles = r.tc.tiles;
            sp.tc_num = r.tc.num_tiles;
        }
        route_scan_kernel<<<1, 512, 0, s>>>(sp);
        MOE_CUDA(cudaGetLastError());
        EpScatterParams cp{ep->exported, ep->L, r.masks, r.base, r.offsets, r.pair_token, r.pair_rank, r.pair_weight,
                           r.tiles, r.tile_off, r.tiles_max};
        ep_scatter_kernel<<<dim3(chunks, kRouterExperts / 256), 256, 0, s>>>(cp);
        MOE_CUDA(cudaGetLastError());
    }
    // expert kernels over the received slots, partial rows accumulated locally
    const bool tc = ep->tc && w->tc_ok;
    const int tc_tiles = tc ? r.tc.max_tiles : 0;
    if (const int st = launch_experts(&r, w, partial, r.tiles_max, s, nullptr, tc_tiles, nullptr, !tc)) return st;
    // 5. the combine publishes "done", waits for every peer's, then pulls the partial rows
    if (flags == MOE_OUT_OVERWRITE) MOE_CUDA(cudaMemsetAsync(out, 0, xbytes, s));
    const int cthreads = std::min(kEpCombineThreads, std::max(32, (H / 4 + 31) / 32 * 32));
    ep_combine_kernel<<<tokens, cthreads, 0, s>>>(p);
    return cuda_status(cudaGetLastError(), "ep_combine_kernel");
}

int moe_ep_forward_hidden(moe_ep_t ep, moe_weights_t w, const float *x, int tokens, float *out, int flags,
                          void *stream) {
    if (!ep || !w) return fail(MOE_INVALID_ARGUMENT, "null expert-parallel layer or weights");
    if (tokens < 1 || tokens > ep->desc.max_tokens) return fail(MOE_INVALID_ARGUMENT, "tokens outside 1..max_tokens");
    if (const int st = moe_router_logits(w, x, tokens, ep->tx->logits, stream)) return st;
    return moe_ep_forward(ep, w, x, ep->tx->logits, tokens, out, flags, stream);
}

int moe_ep_read_flags(moe_ep_t ep, int *flags, int clear, void *stream) {
    if (!ep || !flags) return fail(MOE_INVALID_ARGUMENT, "null argument");
    int a = 0, b = 0;
    if (const int st = moe_layer_read_flags(ep->tx, &a, clear, stream)) return st;
    DeviceGuard guard(ep->desc.device);
    MOE_CUDA(guard.status);
    auto s = static_cast<cudaStream_t>(stream);
    MOE_CUDA(cudaMemcpyAsync(&b, ep->rx.error, sizeof(int), cudaMemcpyDeviceToHost, s));
    if (clear) MOE_CUDA(cudaMemsetAsync(ep->rx.error, 0, sizeof(int), s));
    MOE_CUDA(cudaStreamSynchronize(s));
    *flags = a | b;
    // A timed-out wait leaves the quantising CTAs' completion count as it was
    // (late CTAs may have added to it); the stream is idle now, so rewind it.
    if (*flags & MOE_FLAG_TIMEOUT) {
        MOE_CUDA(cudaMemsetAsync(ep->quant_done, 0, sizeof(uint32_t), s));
        MOE_CUDA(cudaStreamSynchronize(s));
    }
    return MOE_OK;
}

}  // extern "C"
