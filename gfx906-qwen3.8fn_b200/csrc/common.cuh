// common.cuh -- shared device helpers for the sm_100a routed-MoE kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qwen_moe_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library is written for sm_100a (Blackwell) only"
#endif

namespace qmoe {

constexpr int kTopK = 10;
constexpr int kRouterExperts = 512;
constexpr int kFlagInvalid = MOE_FLAG_INVALID;
constexpr int kFlagArithmetic = MOE_FLAG_ARITHMETIC;

// Planar Q8 activations used between kernels: int8 codes [rows][K] and per
// block (d, s) decoded to fp32 [rows][K/32] -- the same information as the
// canonical 36-byte Q8_1 blocks, rearranged so codes load as aligned 16-byte
// vectors.
struct Q8Planar {
    int8_t *codes;
    float2 *scales;
};

constexpr int kGemvTile = 4;     // pairs per work tile

// Work tile: up to kGemvTile consecutive pairs (one expert) of the sorted
// assignment list, with their tokens and router weights inline so a kernel
// needs a single 80-byte load per tile.
struct __align__(16) TileRec {
    int e, p0, n, pad;
    int tok[kGemvTile];
    float w[kGemvTile];
};
static_assert(sizeof(TileRec) % 16 == 0, "tile record is whole 16-byte vectors");

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Unsigned-byte x signed-byte 4-way dot product accumulate (dp4a.u32.s32).
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Uncentred u4 x s8 dot of one 32-element block: 16 code bytes as a uint4
// (byte j: low nibble element j, high nibble element j+16) against 32 int8
// activation codes as two int4 (elements 0..15, 16..31).  Exact in int32.
__device__ __forceinline__ int block_dot(const uint4 w, const int4 xlo, const int4 xhi) {
    int acc = 0;
    acc = dp4a_us(w.x & 0x0f0f0f0fu, xlo.x, acc);
    acc = dp4a_us(w.y & 0x0f0f0f0fu, xlo.y, acc);
    acc = dp4a_us(w.z & 0x0f0f0f0fu, xlo.z, acc);
    acc = dp4a_us(w.w & 0x0f0f0f0fu, xlo.w, acc);
    acc = dp4a_us((w.x >> 4) & 0x0f0f0f0fu, xhi.x, acc);
    acc = dp4a_us((w.y >> 4) & 0x0f0f0f0fu, xhi.y, acc);
    acc = dp4a_us((w.z >> 4) & 0x0f0f0f0fu, xhi.z, acc);
    acc = dp4a_us((w.w >> 4) & 0x0f0f0f0fu, xhi.w, acc);
    return acc;
}

// Exact int -> float for |v| < 2^22: the integer added to the bit pattern of
// 1.5 * 2^23 lands in the mantissa, and subtracting 1.5 * 2^23 is exact.
// (An integer add and a float add instead of the quarter-rate I2F.)
__device__ __forceinline__ float small_int_to_float(int v) {
    return __int_as_float(v + 0x4b400000) - 12582912.0f;
}

// One block's contribution with the reference's Q4_0 correction
// d4*(dot*d8 - 8*s8) (src/quant.cpp:88-102), as two FMAs.  |dot| <= 32*15*128.
__device__ __forceinline__ float block_term(int dot, float d4, float d8, float s8x8, float acc) {
    return fmaf(d4, fmaf(small_int_to_float(dot), d8, -s8x8), acc);
}

// Packed pairs of fp32 (Blackwell f32x2 arithmetic), low word = first element.
__device__ __forceinline__ uint64_t pk2(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ uint64_t pkf2(float lo, float hi) { return pk2(__float_as_uint(lo), __float_as_uint(hi)); }
__device__ __forceinline__ void upk2(uint64_t v, float &lo, float &hi) {
    uint32_t a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(a), "=r"(b) : "l"(v));
    lo = __uint_as_float(a);
    hi = __uint_as_float(b);
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// Both elements rounded to half (RNE) and back to fp32.
__device__ __forceinline__ uint64_t round_half2(uint64_t v) {
    float a, b;
    upk2(v, a, b);
    const float2 f = __half22float2(__floats2half2_rn(a, b));
    return pkf2(f.x, f.y);
}
// block_term for two weight rows against the same activation block, as
// packed f32x2 operations with the scalar form's per-element rounding (the
// results are bit-identical to two block_term calls).
__device__ __forceinline__ uint64_t block_term2(int dot0, int dot1, uint64_t d4, uint64_t d8, uint64_t neg_s8x8,
                                                uint64_t acc) {
    const uint64_t bias = pkf2(-12582912.0f, -12582912.0f);
    const uint64_t f = add2(pk2(static_cast<uint32_t>(dot0 + 0x4b400000), static_cast<uint32_t>(dot1 + 0x4b400000)),
                            bias);
    return fma2(d4, fma2(f, d8, neg_s8x8), acc);
}

// Block dot as two independent dp4a chains.  High nibbles are masked in place
// (byte values 16*q) and the chain is shifted once: each partial is a multiple
// of 16 and |partial| <= 16*240*128 < 2^31, so the result equals block_dot.
__device__ __forceinline__ int block_dot2(const uint4 w, const int4 xlo, const int4 xhi) {
    int a = dp4a_us(w.x & 0x0f0f0f0fu, xlo.x, 0);
    int b = dp4a_us(w.x & 0xf0f0f0f0u, xhi.x, 0);
    a = dp4a_us(w.y & 0x0f0f0f0fu, xlo.y, a);
    b = dp4a_us(w.y & 0xf0f0f0f0u, xhi.y, b);
    a = dp4a_us(w.z & 0x0f0f0f0fu, xlo.z, a);
    b = dp4a_us(w.z & 0xf0f0f0f0u, xhi.z, b);
    a = dp4a_us(w.w & 0x0f0f0f0fu, xlo.w, a);
    b = dp4a_us(w.w & 0xf0f0f0f0u, xhi.w, b);
    return a + (b >> 4);
}

// The two 16-element fragment dots of one block in the reference's MMVQ
// order (src/cpu_expert.cpp:156-213): fragment 0 = elements 0..7 and
// 16..23 (code bytes 0..7), fragment 1 = elements 8..15 and 24..31 (bytes
// 8..15).  Uncentred u4 x s8, exact in int32; f0 + f1 == block_dot.
__device__ __forceinline__ void frag_dots(const uint4 w, const int4 xlo, const int4 xhi, int &f0, int &f1) {
    f0 = dp4a_us(w.x & 0x0f0f0f0fu, xlo.x, 0);
    f0 = dp4a_us(w.y & 0x0f0f0f0fu, xlo.y, f0);
    f0 = dp4a_us((w.x >> 4) & 0x0f0f0f0fu, xhi.x, f0);
    f0 = dp4a_us((w.y >> 4) & 0x0f0f0f0fu, xhi.y, f0);
    f1 = dp4a_us(w.z & 0x0f0f0f0fu, xlo.z, 0);
    f1 = dp4a_us(w.w & 0x0f0f0f0fu, xlo.w, f1);
    f1 = dp4a_us((w.z >> 4) & 0x0f0f0f0fu, xhi.z, f1);
    f1 = dp4a_us((w.w >> 4) & 0x0f0f0f0fu, xhi.w, f1);
}

// The reference's Q4_0 x Q8_1 reduction order (MMVQ: src/hip/linear.hip:197-281,
// restated on the CPU by matrix_gpu_order, src/cpu_expert.cpp:156-213): block b
// fragment f accumulates into lane 2*(b % 64) + f as
//   lane = fma(d4, fma(float(dot_f), d8, -4*s8), lane)   (lanes start at +0),
// then lane[i] += lane[i + 64] for i < 64, then an XOR butterfly with masks
// 1, 2, ..., 32 over the 64 lanes.  With lane pairs (beta, beta + 32) of
// blocks packed as (fragment 0, fragment 1) f32x2 accumulators a0 (blocks
// b % 64 == beta) and a1 (b % 64 == beta + 32), the value of the first two
// levels is this leaf; the remaining levels are an ascending butterfly over
// beta (warp_tree_sum when lane = beta).
__device__ __forceinline__ uint64_t mmvq_term2(uint64_t dots, uint64_t d4, uint64_t d8, uint64_t m4, uint64_t acc) {
    return fma2(d4, fma2(dots, d8, m4), acc);
}
__device__ __forceinline__ float mmvq_leaf(uint64_t a0, uint64_t a1) {
    float x0, y0, x1, y1;
    upk2(a0, x0, y0);
    upk2(a1, x1, y1);
    return __fadd_rn(__fadd_rn(x0, x1), __fadd_rn(y0, y1));
}
__device__ __forceinline__ float warp_tree_sum(float v) {
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}
// warp_tree_sum of V values at once (V a power of two <= 32), bit-identical
// to V separate calls: recursive halving over masks 1 .. V/2 (at the level of
// mask m a lane keeps the values whose index bit matches its lane bit and
// sends the others, so every total is summed over the same lane pairs in the
// same order), then a plain butterfly over the remaining masks; V - 1 + 5 -
// log2(V) shuffles instead of 5 V.  On return lane l holds the total of
// value l % V.
template <int V>
__device__ __forceinline__ float warp_tree_sum_n(float (&v)[V], int lane) {
#pragma unroll
    for (int m = 1, n = V; m < V; m <<= 1, n >>= 1) {
        const bool hi = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = hi ? v[2 * i] : v[2 * i + 1];
            const float keep = hi ? v[2 * i + 1] : v[2 * i];
            v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, m));
        }
    }
    float t = v[0];
#pragma unroll
    for (int m = V; m < 32; m <<= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, m));
    return t;
}

// The C library's expf, bit for bit: the reference's CPU SiLU computes
// g / (1 + expf(-g)) (src/cpu_expert.cpp:248-259), and a middle Q8_1 that is
// to equal the reference's byte for byte needs the same exp.  The device
// takes the double-precision exponential rounded once to float and corrects
// the inputs where the C library's expf rounds differently (0.008 % of the
// floats in [-104, 89], listed at build time by csrc/expf_table.c), looked up
// in a hash table of (x bits, expf bits) pairs in buckets of four (one
// 32-byte sector per bucket), probing bucket after bucket; empty entries
// hold key 0xffffffff (a NaN pattern, never a key).  With 2^18 buckets for
// ~170 k corrections a lookup reads one bucket in all but ~0.5 % of cases.
// The table is filled once per device before any kernel of this library
// runs (expf_table_upload).
constexpr int kExpfBucketsLog2 = 18;
constexpr int kExpfBucket = 4;                         // entries per bucket
constexpr uint32_t kExpfEmpty = 0xffffffffu;
constexpr int kExpfMaxProbe = 64;                      // buckets
static __device__ uint4 g_expf_fix[(1u << kExpfBucketsLog2) * kExpfBucket / 2];   // 2 entries per uint4

__host__ __device__ __forceinline__ uint32_t expf_fix_bucket(uint32_t key) {
    return (key * 2654435761u) >> (32 - kExpfBucketsLog2);
}
// Look key up in bucket b (entries e0 = {k0, v0, k1, v1}, e1 = {k2, v2, k3, v3}):
// 1 found (value in *v), 0 absent (the bucket has an empty entry), -1 the
// bucket is full without it (continue with the next bucket).
__device__ __forceinline__ int expf_fix_match(uint4 e0, uint4 e1, uint32_t key, uint32_t *v) {
    if (e0.x == key) { *v = e0.y; return 1; }
    if (e0.z == key) { *v = e0.w; return 1; }
    if (e1.x == key) { *v = e1.y; return 1; }
    if (e1.z == key) { *v = e1.w; return 1; }
    return (e0.x == kExpfEmpty || e0.z == kExpfEmpty || e1.x == kExpfEmpty || e1.z == kExpfEmpty) ? 0 : -1;
}
// N exponentials at once: the N first-bucket loads are in flight together.
template <int N>
__device__ __forceinline__ void expf_ref_n(const float (&x)[N], float (&y)[N]) {
    uint32_t k[N], b[N];
    uint4 e0[N], e1[N];
#pragma unroll
    for (int j = 0; j < N; ++j) {
        k[j] = __float_as_uint(x[j]);
        b[j] = expf_fix_bucket(k[j]);
        e0[j] = g_expf_fix[2 * b[j]];
        e1[j] = g_expf_fix[2 * b[j] + 1];
    }
#pragma unroll
    for (int j = 0; j < N; ++j) y[j] = __double2float_rn(exp(static_cast<double>(x[j])));
#pragma unroll
    for (int j = 0; j < N; ++j) {
        uint32_t v = 0;
        int r = expf_fix_match(e0[j], e1[j], k[j], &v);
        for (int i = 1; r < 0 && i < kExpfMaxProbe; ++i) {   // rare: the first bucket is full
            const uint32_t bb = (b[j] + i) & ((1u << kExpfBucketsLog2) - 1);
            r = expf_fix_match(g_expf_fix[2 * bb], g_expf_fix[2 * bb + 1], k[j], &v);
        }
        if (r > 0) y[j] = __uint_as_float(v);
    }
}
__device__ __forceinline__ float expf_ref(float x) {
    const float xs[1] = {x};
    float ys[1];
    expf_ref_n<1>(xs, ys);
    return ys[0];
}

__device__ __forceinline__ void report(int flags, int *error) {
    if (flags) atomicOr(error, flags);
}

__device__ __forceinline__ float operand(float x, int &flags) {
    if (!isfinite(x)) { flags |= kFlagInvalid; return 0.0f; }
    return x;
}
__device__ __forceinline__ float arithmetic(float x, int &flags) {
    if (!isfinite(x)) { flags |= kFlagArithmetic; return 0.0f; }
    return x;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

// Quantise one 32-value block held one value per lane (lane = element).
// Byte-identical to the reference's quantize_q8 (src/quant.cpp:275-325) for
// valid blocks; invalid blocks yield zero and sticky flags, like
// src/hip/linear.hip:99-150.  The raw sum uses the XOR butterfly 1,2,4,8,16.
struct Q8Lane {
    int8_t code;
    uint16_t d, s;   // meaningful on every lane
    int flags;       // block flags, identical on every lane
};

__device__ __forceinline__ Q8Lane quantize_lane(float x) {
    int bad = !isfinite(x);
    if (bad) x = 0.0f;
    float amax = fabsf(x);
    float sum = x;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        bad |= __shfl_xor_sync(0xffffffffu, bad, m);
        sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, m));
    }
    const float d = __fdiv_rn(amax, 127.0f);
    const uint16_t hd = f2h(d), hs = f2h(sum);
    const bool representable = isfinite(sum) && (hs & 0x7c00u) != 0x7c00u &&
                               (hd & 0x7c00u) != 0x7c00u && (amax == 0.0f || d > 0.0f);
    const float code = (!bad && representable && amax != 0.0f) ? roundf(__fdiv_rn(x, d)) : 0.0f;
    int bad_code = !isfinite(code) || code < -127.0f || code > 127.0f;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) bad_code |= __shfl_xor_sync(0xffffffffu, bad_code, m);
    const bool valid = !bad && representable && !bad_code;
    Q8Lane q;
    q.code = valid ? static_cast<int8_t>(code) : int8_t(0);
    q.d = (valid && amax != 0.0f) ? hd : uint16_t(0);
    q.s = (valid && amax != 0.0f) ? hs : uint16_t(0);
    q.flags = (bad ? kFlagInvalid : 0) | ((representable && !bad_code) ? 0 : kFlagArithmetic);
    return q;
}

}  // namespace qmoe
