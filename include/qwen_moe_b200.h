/*
 * qwen_moe_b200.h -- C ABI of the B200 routed-MoE expert FFN library
 * (libqwen_moe_b200.so, built for sm_100a).
 *
 * Conventions (mirroring the reference's borrowed-buffer launchers,
 * src/hip/session_ops.cuh:22-48, src/hip/linear.cuh:35-45):
 *  - every pointer named *_dev is caller-owned device memory on the handle's
 *    device; lifetimes and cross-stream ordering are the caller's;
 *  - every launch takes an explicit cudaStream_t (passed as void*; NULL is the
 *    legacy default stream);
 *  - invalid shapes, null or misaligned pointers and writable overlaps return
 *    MOE_INVALID_ARGUMENT before anything is enqueued; a status of MOE_OK means
 *    "enqueued", not "completed";
 *  - no call allocates device memory except the *_create / *_weights_create
 *    functions; no call synchronises except where stated; no C++ exception
 *    crosses this boundary;
 *  - numeric faults never trap: kernels OR sticky bits into a device int
 *    (MOE_FLAG_INVALID = 1 nonfinite input, MOE_FLAG_ARITHMETIC = 2 nonfinite
 *    or unrepresentable arithmetic), as the reference's session ops do.
 *
 * Q4_0 blocks are the canonical 18-byte GGML layout (half d, 16 code bytes,
 * low nibble of byte j = element j, high nibble = element j+16); Q4_1 blocks
 * the canonical 20-byte layout (half d, half m, the same 16 code bytes; value
 * d*q + m); Q8_1 blocks are the reference's 36-byte ABI (half d, half raw
 * sum, 32 int8 codes), src/quant.hpp:8-18.
 */
#ifndef QWEN_MOE_B200_H
#define QWEN_MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

enum moe_status {
    MOE_OK = 0,
    MOE_INVALID_ARGUMENT = 1, /* reference: std::invalid_argument / hipErrorInvalidValue */
    MOE_NOT_SUPPORTED = 2,    /* reference: hipErrorNotSupported */
    MOE_CUDA_ERROR = 3,       /* reference: std::runtime_error from a HIP call */
    MOE_NUMERIC_ERROR = 4,    /* a sticky numeric flag was raised */
    /* 5 is reserved (the library makes no NCCL call; expert parallelism runs
     * over CUDA IPC peer memory) */
    MOE_TIMEOUT = 6,
    MOE_OUT_OF_MEMORY = 7
};

enum moe_flags { MOE_FLAG_INVALID = 1, MOE_FLAG_ARITHMETIC = 2, MOE_FLAG_TIMEOUT = 4 /* a bounded device wait gave up */ };

/* moe_forward flags */
enum moe_forward_flags {
    MOE_OUT_ACCUMULATE = 0, /* out += layer(x): scatter-add into a residual */
    MOE_OUT_OVERWRITE = 1   /* out  = layer(x) */
};

/* Shape of one MoE layer.  Replaces the fixed constants of the reference's
 * Session (src/session.hip:40, H=2560/640) and RouteGroups (src/routes.hpp:53-55,
 * 512 experts, top-10).  Supported: hidden, inter multiples of 256 and <= 16384,
 * experts == 512, top_k == 10. */
typedef struct moe_layer_desc {
    int hidden;      /* H */
    int inter;       /* I, expert intermediate width */
    int experts;     /* routed experts (512) */
    int top_k;       /* 10 */
    int has_shared;  /* 1: one shared expert with a sigmoid scalar gate */
    int device;      /* CUDA device ordinal */
    int max_tokens;  /* capacity of one forward */
} moe_layer_desc;

/* Weight block types, numbered as the reference's TensorType (src/model.hpp:17-19). */
enum moe_tensor_type { MOE_Q4_0 = 2, MOE_Q4_1 = 3 };

typedef struct moe_layer_s *moe_layer_t;
typedef struct moe_weights_s *moe_weights_t;

const char *moe_status_string(int status);
/* Version of this library's ABI (major << 16 | minor). */
int moe_abi_version(void);

/* ---- weights: device-resident experts of one layer ------------------------
 * Storage per expert is one contiguous 1,769,472-byte region (H=2048, I=512)
 * in a planar layout: gate/up/down code bytes (16 per block, row-major
 * blocks), then gate/up/down half scales.  Byte count equals the canonical
 * Q4_0 size.  The shared expert is stored as expert index `experts`. */
int moe_weights_create(const moe_layer_desc *desc, moe_weights_t *out);
/* The same with the down matrices of type down_type (MOE_Q4_0 or MOE_Q4_1;
 * gate and up are always Q4_0).  The reference's layers 0-5 carry Q4_1 down
 * matrices (src/memory_main.hip:41-42): each block contributes
 * dot*half(d4*d8) + half(m4*s8) (src/quant.cpp:88-102).  A Q4_1-down expert
 * adds a half minimum per down block to the planar region (1,835,008 bytes
 * at H=2048, I=512).  Forwards over such weights run every expert group on
 * the dp4a kernels (no tensor-core path).  MOE_NOT_SUPPORTED for other types. */
int moe_weights_create_typed(const moe_layer_desc *desc, int down_type, moe_weights_t *out);
int moe_weights_destroy(moe_weights_t w);
/* Upload one expert from canonical host Q4_0 bytes (repacked to the planar
 * layout on the device).  Replaces the reference's expert staging
 * (src/session.hip:957-1042): all experts stay resident.  expert == experts
 * uploads the shared expert.  gate/up: [I][H/32] blocks, down: [H][I/32]
 * blocks of the weights' down type (20-byte Q4_1 blocks for MOE_Q4_1).
 * Asynchronous on `stream` like cudaMemcpyAsync: the copies and repacks are
 * enqueued and the call returns without synchronising (pageable sources are
 * read before it returns, pinned ones when the stream reaches the copy);
 * consecutive uploads into one weights object are ordered by an event on its
 * staging buffer, whatever streams they use. */
int moe_weights_upload_expert(moe_weights_t w, int expert, const void *gate_q4_0,
                              const void *up_q4_0, const void *down_q4_0, void *stream);
/* Shared expert scalar gate vector (fp32 [H]), the reference's
 * ffn_gate_inp_shexp (src/session.hip:1101, used at :1398-1402). */
int moe_weights_upload_shared_gate(moe_weights_t w, const float *gate_vec_host, void *stream);
/* Router matrix ffn_gate_inp (src/session.hip:1097) as host fp32 [512][H]
 * (row e = expert e's H weights, i.e. the GGUF tensor {H, 512} with H
 * fastest), for moe_forward_hidden / moe_router_logits.  Zero until uploaded. */
int moe_weights_upload_router(moe_weights_t w, const float *router_host, void *stream);
/* Fill every expert (and the shared expert) with the seeded synthetic Q4_0
 * generator on the device (bit-identical to the oracle's generator); Q4_1
 * down matrices take the same codes and scales plus the minimum
 * -8*d*(0.5 + u/65536) from one more 16-bit draw per block. */
int moe_weights_synthesize(moe_weights_t w, uint64_t seed, uint32_t layer, void *stream);
/* Copy one expert back as canonical bytes (host; down in the weights' down
 * type), for parity checks. */
int moe_weights_download_expert(moe_weights_t w, int expert, void *gate_q4_0, void *up_q4_0,
                                void *down_q4_0, void *stream);
/* Bytes of one expert's planar region with Q4_0 down matrices. */
size_t moe_weights_expert_bytes(const moe_layer_desc *desc);

/* ---- layer workspace and forward ----------------------------------------- */
int moe_layer_create(const moe_layer_desc *desc, moe_layer_t *out);
int moe_layer_destroy(moe_layer_t h);

/* Whole routed-MoE FFN for T tokens, replacing the body of the reference's
 * Layer::ffn (src/session.hip:1412-1556) from the router probabilities on:
 * softmax over router logits, top-10 + renormalised weights, GPU grouping,
 * Q8_1 quantisation of x, grouped gate/up + fused SiLU*up + Q8_1
 * requantisation, down projection, router-weighted scatter-add of every
 * routed expert and of the sigmoid-gated shared expert into out.
 * x_dev fp32 [T][H]; logits_dev fp32 [T][experts]; out_dev fp32 [T][H].
 * No host synchronisation: the call is capturable in a CUDA graph. */
int moe_forward(moe_layer_t h, moe_weights_t w, const float *x_dev, const float *logits_dev,
                int tokens, float *out_dev, int flags, void *stream);

/* moe_forward from the hidden state: the router logits x * W_router^T are
 * computed on the device (fp32, into the layer's workspace) and routed with
 * no host round trip -- the reference's router.apply + router_softmax +
 * probability D2H + host select_routes (src/session.hip:1420-1433) as one
 * device sequence.  Requires moe_weights_upload_router. */
int moe_forward_hidden(moe_layer_t h, moe_weights_t w, const float *x_dev, int tokens, float *out_dev,
                       int flags, void *stream);
/* Router logits tap: logits_dev fp32 [T][512] = x_dev [T][H] times the
 * uploaded router matrix (fp32 products and sums on the CUDA cores; the
 * reference uses a dense BLAS GEMM, so agreement is to fp32 rounding). */
int moe_router_logits(moe_weights_t w, const float *x_dev, int tokens, float *logits_dev, void *stream);

/* moe_forward with three caller-created CUDA events recorded on `stream`:
 * events[0] before the gate/up kernel, events[1] between gate/up and down,
 * events[2] after the down kernel -- the timing tap bench.py uses to measure
 * the expert kernels' own durations on their launching stream. */
int moe_forward_profiled(moe_layer_t h, moe_weights_t w, const float *x_dev, const float *logits_dev,
                         int tokens, float *out_dev, int flags, void *stream, void *const *events);

/* Deterministic trace mode of moe_forward, for bitwise debugging against
 * the reference's grouped path (moe_scatter + routed_fold +
 * shared_sigmoid_add, src/hip/session_ops.hip:305-391, called from
 * src/session.hip:1412-1556).  Every routed pair's unweighted down output is
 * stored at contrib_dev[token][rank][H] (the reference's [T][10][H]
 * contribution layout), the shared expert's at shared_dev[token][H] (NULL
 * exactly when the layer has no shared expert); then, per element, the
 * reference's operation order over those buffers: value = sum over ranks
 * 0..9 of weight*contribution (ten separately rounded multiply/adds from 0;
 * 0 on any non-finite operand), then value + sigmoid(gate)*shared (0 on any
 * non-finite operand); out = value (MOE_OUT_OVERWRITE) or out + value
 * (MOE_OUT_ACCUMULATE).  No atomics: bit-identical from run to run.  Every
 * expert group runs on the dp4a kernels (no tensor-core path), so this is a
 * debugging mode, not the fast path.  contrib_dev: T*10*H floats; shared_dev:
 * T*H floats; both caller-owned, 16-byte aligned, disjoint from x, logits
 * and out. */
int moe_forward_contributions(moe_layer_t h, moe_weights_t w, const float *x_dev, const float *logits_dev,
                              int tokens, float *contrib_dev, float *shared_dev, float *out_dev, int flags,
                              void *stream);

/* Routing only (parity tap for src/hip/session_ops.hip:401-434 router_softmax,
 * src/session.hip:666-687 select_routes and src/routes.cpp:59-115 grouping).
 * Outputs (device, any may be NULL): probs fp32 [T][experts], ids int32
 * [T][top_k], weights fp32 [T][top_k], offsets int32 [experts+1], and the
 * sorted assignment list as token/rank int32 [T*top_k]. */
int moe_route(moe_layer_t h, const float *logits_dev, int tokens, float *probs_dev,
              int32_t *ids_dev, float *weights_dev, int32_t *offsets_dev, int32_t *token_dev,
              int32_t *rank_dev, void *stream);

/* Routing that allocates nothing: the same results as moe_route (ids,
 * weights, offsets [experts+1], sorted token/rank [T*top_k], all device
 * memory owned by the caller; sticky bits ORed into the caller-zeroed
 * *error_dev) for callers that cannot allocate device memory -- work enqueued
 * inside CUDA stream capture, or hosts whose device memory belongs to another
 * allocator.  It has no counterpart in the reference.  Its scratch is one
 * static device array of 326,144 bytes, held by every GPU that loads the
 * library until the process exits, which limits tokens to 1..1024 (larger
 * counts return MOE_INVALID_ARGUMENT).  The first call on a device resolves
 * that array's address on the current device (cudaGetSymbolAddress); make
 * that first call before any stream capture.  The address is kept per
 * device ordinal for the life of the process, so resetting a device
 * (cudaDeviceReset) after that first call is not supported.  Every call shares
 * the array: calls whose GPU work overlaps (other streams, other threads) race. */
int moe_route_noalloc(const float *logits_dev, int tokens, int32_t *ids_dev, float *weights_dev,
                      int32_t *offsets_dev, int32_t *token_dev, int32_t *rank_dev, int *error_dev,
                      void *stream);

/* Read (and optionally clear) the sticky numeric flags of a layer.  This is
 * the only call here that synchronises (on `stream`). */
int moe_layer_read_flags(moe_layer_t h, int *flags_host, int clear, void *stream);

/* ---- expert parallelism over peer memory ----------------------------------
 * One process per GPU, `world` in {1, 2, 4, 8} ranks of one node with peer
 * access (NVLink / NVSwitch).  Rank r owns routed experts
 * [r*512/world, (r+1)*512/world) plus a replica of the shared expert, and its
 * own tokens.  Replaces the single-device expert loop of the reference
 * (src/session.hip:957-1071 Experts::run/run_chunk) with the expert-sharded
 * plan of its multi-GPU design: dispatch of Q8_1 rows to the owning ranks,
 * local grouped expert kernels, combine of pre-reduced partial rows into the
 * owner's residual.  Transport is peer stores/loads inside this library's own
 * kernels on CUDA IPC mappings (no NCCL); every wait on a peer is bounded and
 * raises MOE_FLAG_TIMEOUT instead of hanging.  All ranks must call
 * moe_ep_forward the same number of times, in the same order. */
typedef struct moe_ep_s *moe_ep_t;
enum { MOE_EP_HANDLE_BYTES = 64 };

/* Expert-shard weights of rank `rank`: 512/world routed experts (local index
 * i is global expert rank*512/world + i) and the shared expert at local index
 * 512/world.  Upload, synthesis (same bits as the global experts) and
 * download work as for moe_weights_t with local indices. */
int moe_ep_weights_create(const moe_layer_desc *desc, int rank, int world, moe_weights_t *out);
/* The same with down matrices of type down_type (see moe_weights_create_typed). */
int moe_ep_weights_create_typed(const moe_layer_desc *desc, int rank, int world, int down_type,
                                moe_weights_t *out);
/* Workspace of one rank; desc->max_tokens is the per-rank token capacity. */
int moe_ep_create(const moe_layer_desc *desc, int rank, int world, moe_ep_t *out);
int moe_ep_destroy(moe_ep_t ep);
/* The rank's exportable buffer as an opaque MOE_EP_HANDLE_BYTES-byte handle
 * (cudaIpcGetMemHandle) for the caller to exchange (e.g. all-gather). */
int moe_ep_ipc_handle(moe_ep_t ep, void *handle_host);
/* Map every peer's buffer from the world * MOE_EP_HANDLE_BYTES handles in
 * rank order (the own entry is ignored).  Synchronises the device. */
int moe_ep_open_peers(moe_ep_t ep, const void *handles_host);
/* Expert-parallel forward of this rank's T tokens (same contract as
 * moe_forward for x, logits and out).  Capturable in a CUDA graph once the
 * peers are open. */
int moe_ep_forward(moe_ep_t ep, moe_weights_t w, const float *x_dev, const float *logits_dev, int tokens,
                   float *out_dev, int flags, void *stream);
/* moe_ep_forward from the hidden state (router logits computed on the
 * device from the shard weights' router matrix, as moe_forward_hidden). */
int moe_ep_forward_hidden(moe_ep_t ep, moe_weights_t w, const float *x_dev, int tokens, float *out_dev,
                          int flags, void *stream);
/* Sticky flags of the rank (MOE_FLAG_TIMEOUT included); synchronises `stream`.
 * After a reported timeout it also rewinds the rank's internal completion
 * counters, so the next forward starts clean. */
int moe_ep_read_flags(moe_ep_t ep, int *flags_host, int clear, void *stream);

/* ---- kernels exposed for parity taps ------------------------------------- */
/* fp32 [columns][width] -> canonical Q8_1 [columns][width/32] (36-byte blocks).
 * Same contract as the reference's launch_quantize_q8_1
 * (src/hip/linear.cuh:89-108): failing blocks are written as zero and set
 * sticky bits in *error_dev (caller-zeroed). */
int moe_quantize_q8_1(const float *x_dev, int width, int columns, void *q8_dev, int *error_dev,
                      void *stream);
/* Per-block dot tap of the forward's own expert kernels (the parity tap
 * moe_debug_block_dots; the reference checks its Session producer kernels
 * against its CPU expert the same way, src/cpu_expert_shadow.hip:333-341).
 * Runs moe_forward with MOE_OUT_OVERWRITE into out_dev, through the kernels a
 * forward of this size uses (streaming dp4a kernels at decode sizes, the
 * tensor-core kernels above), and records for the pairs of `expert` (0..511,
 * or 512 for the shared expert), in the grouped pair order, numbered from the
 * expert's first pair:
 *   gate_dots, up_dots  int32 [max_pairs][I][H/32]  uncentred sum(q*x) per block,
 *   down_dots           int32 [max_pairs][H][I/32]  against the middle Q8_1 the
 *                                                  gate/up kernel produced,
 *   mid_codes           int8  [max_pairs][I]        that middle's codes,
 *   mid_ds              uint32 [max_pairs][I/32]    its half d | half s << 16.
 * Pairs beyond max_pairs are not recorded. */
int moe_debug_block_dots(moe_layer_t h, moe_weights_t w, const float *x_dev, const float *logits_dev, int tokens,
                         int expert, int max_pairs, int32_t *gate_dots, int32_t *up_dots, int32_t *down_dots,
                         int8_t *mid_codes, uint32_t *mid_ds, float *out_dev, void *stream);
/* The exponential of the gate/up kernels' SiLU over a range of inputs:
 * out_dev[i] = exp of the float whose bit pattern is first_bits + i (i < count,
 * no wrap past 0xffffffff), computed as the expert kernels compute it: exp in
 * double precision rounded once to float, then the build's table of the C
 * library's expf corrections.  The parity tap for the SiLU, whose reference is
 * the C library's expf in the reference's CPU expert
 * (src/cpu_expert.cpp:248-259). */
int moe_debug_expf(uint32_t first_bits, uint32_t count, float *out_dev, void *stream);
/* Q4_0 x Q8_1 linear: out[c][r] = sum_b d4*(dot*d8 - 8*s8) for canonical
 * Q4_0 weights [rows][K/32] and canonical Q8_1 input [columns][K/32].
 * Replaces launch_quantized_linear{,_short,_tiled} (src/hip/linear.hip:445-490).
 * When dots_dev is non-NULL the per-block int32 dots are also written
 * ([columns][rows][K/32]), the bit-exact parity tap. */
int moe_q4_linear(const void *w_q4_0_dev, int rows, int k, const void *x_q8_dev, int columns,
                  float *out_dev, int32_t *dots_dev, void *stream);
/* Q4_1 x Q8_1 linear on canonical 20-byte Q4_1 weights [rows][K/32]:
 * out[c][r] = sum over ascending b of the block terms
 * acc + fma(dot, half(d4*d8), half(m4*s8)) -- the contract of the
 * reference's Q4_1 down projection (src/quant.cpp:88-102,
 * src/hip/linear.hip:204-211, src/cpu_expert.cpp:194-205).  dots_dev as for
 * moe_q4_linear (the uncentred sum of code*activation per block). */
int moe_q4_1_linear(const void *w_q4_1_dev, int rows, int k, const void *x_q8_dev, int columns,
                    float *out_dev, int32_t *dots_dev, void *stream);

/* ---- single-expert fixture API (src/gpu_expert.hpp:7-21) ---------------- */
typedef struct moe_expert_s *moe_expert_t;
int moe_expert_create(const void *gate_q4_0, const void *up_q4_0, const void *down_q4_0,
                      int hidden, int inter, int device, int max_columns, moe_expert_t *out);
/* GpuExpert with a down matrix of type down_type (MOE_Q4_0 or MOE_Q4_1), as
 * the reference's native expert shapes use (Q4_0 gate/up, Q4_1 down). */
int moe_expert_create_typed(const void *gate_q4_0, const void *up_q4_0, const void *down, int down_type,
                            int hidden, int inter, int device, int max_columns, moe_expert_t *out);
int moe_expert_destroy(moe_expert_t e);
/* Host fp32 [n] -> compare the GPU Q8_1 bytes with `expected` (host Q8_1);
 * MOE_INVALID_ARGUMENT when the input is not representable, MOE_NUMERIC_ERROR
 * when the bytes differ (GpuExpert::check_quantization). */
int moe_expert_check_quantization(moe_expert_t e, const float *input, size_t n,
                                  const void *expected_q8);
/* One projection of host Q8_1 input (GpuExpert::linear): down selects the
 * down matrix, else up selects up, else gate.  Output host fp32 [columns][rows]. */
int moe_expert_linear(moe_expert_t e, int down, int up, const void *input_q8, int columns,
                      float *output);
/* Resident float -> Q8 -> gate/up -> SiLU*up -> Q8 -> down, host fp32 in/out
 * [columns][hidden]; timings in milliseconds (GpuExpert::run). */
int moe_expert_run(moe_expert_t e, const float *input, int columns, float *output, int repeats,
                   double *upload_ms, double *resident_ms, double *wall_ms);

/* ---- route grouping on the host (src/routes.hpp:28-65) ------------------- */
typedef struct moe_route_groups_s *moe_route_groups_t;
/* bound 0: capacity 1..1024, bound 1: capacity 1..16384 */
int moe_route_groups_create(int token_capacity, int bound, moe_route_groups_t *out);
int moe_route_groups_destroy(moe_route_groups_t g);
int moe_route_groups_prepare(moe_route_groups_t g, const int32_t *ids, const float *weights,
                             size_t n, int tokens);
/* 16-byte records {int token, int rank, int expert, float weight}. */
size_t moe_route_groups_assignments(moe_route_groups_t g, void *out, size_t capacity);
int moe_route_groups_counts(moe_route_groups_t g, int32_t *out512);
/* Message of the last rejected create/prepare on this thread. */
const char *moe_route_groups_message(void);
const char *moe_last_error_message(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif
