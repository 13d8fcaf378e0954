/*
 * moe_oracle.c -- CPU restatement of the reference's routed-MoE expert FFN path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product links, loads or calls this
 * file: it is the checker used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py.  It is pinned against the reference's own
 * C++ code (built from the reference sources into oracle/_ref/ by
 * oracle/build_ref.py) and against golden vectors in tests/golden/.
 *
 * Every function names the reference file:line whose behaviour it restates
 * (paths relative to the reference project root).  Compile with
 * -ffp-contract=off: every multiply/add below is a separately rounded IEEE
 * operation unless written as fmaf(), exactly as the reference requires.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#if defined(__FAST_MATH__)
#error "the oracle requires strict IEEE arithmetic"
#endif

#define O_EXPORT __attribute__((visibility("default")))

typedef struct { uint16_t d; uint16_t s; int8_t qs[32]; } o_q8_1;   /* src/quant.hpp:17 */
typedef struct { uint16_t d; uint8_t qs[16]; } o_q4_0;               /* src/quant.hpp:8  */
typedef struct { uint16_t d, m; uint8_t qs[16]; } o_q4_1;            /* src/quant.hpp:9  */
_Static_assert(sizeof(o_q8_1) == 36, "Q8_1 ABI is 36 bytes");
_Static_assert(sizeof(o_q4_0) == 18, "Q4_0 ABI is 18 bytes");
_Static_assert(sizeof(o_q4_1) == 20, "Q4_1 ABI is 20 bytes");
enum { O_Q4_0 = 2, O_Q4_1 = 3 };   /* TensorType values, src/model.hpp:17-19 */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---------------------------------------------------------------------------
 * IEEE binary16 <-> binary32.  Same results as src/quant.cpp:211-260
 * (half_to_float / float_to_half, RNE, NaN quieting keeps the payload).
 * ------------------------------------------------------------------------- */
O_EXPORT float o_half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 31u) return u2f(sign | 0x7f800000u | (m << 13) | (m ? 0x00400000u : 0u));
    float v = e == 0u ? ldexpf((float)m, -24) : ldexpf((float)(m | 1024u), (int)e - 25);
    return sign ? -v : v;
}

O_EXPORT uint16_t o_float_to_half(float f) {
    const uint32_t bits = f2u(f);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const uint32_t x = bits & 0x7fffffffu;
    if (x > 0x7f800000u) return (uint16_t)(sign | 0x7c00u | 0x0200u | ((x & 0x007fffffu) >> 13));
    if (x >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);          /* >= 65520 rounds to inf */
    if (x >= 0x38800000u) {                                            /* normal half */
        const uint32_t r = x + 0x0fffu + ((x >> 13) & 1u);
        return (uint16_t)(sign | ((r - 0x38000000u) >> 13));
    }
    if (x < 0x33000000u) return (uint16_t)sign;                        /* below 2^-25 */
    const uint32_t e = x >> 23, m = (x & 0x007fffffu) | 0x00800000u;
    const uint32_t shift = 126u - e;                                   /* 14..24 */
    const uint32_t t = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    return (uint16_t)(sign | (t + (rem > half || (rem == half && (t & 1u)))));
}

/* ---------------------------------------------------------------------------
 * Q8_1 activation quantisation, one 32-value block.
 * Bytes of valid blocks follow src/quant.cpp:275-325 (amax/127 scale, codes
 * roundf(x/d) with the FP32 scale, half(d), half(raw sum) with the XOR
 * butterfly 1,2,4,8,16).  Invalid blocks follow the GPU launcher contract of
 * src/hip/linear.hip:99-150 / linear.cuh:99-108: the block is written as all
 * zero and sticky bits are returned (1 = nonfinite input, 2 = scale/sum/code
 * not representable).
 * ------------------------------------------------------------------------- */
O_EXPORT int o_quantize_block(const float *in, o_q8_1 *out) {
    float x[32], sums[32];
    int bad = 0;
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) {
        x[i] = in[i];
        if (!isfinite(x[i])) { bad = 1; x[i] = 0.0f; }
        const float a = fabsf(x[i]);
        amax = a > amax ? a : amax;
        sums[i] = x[i];
    }
    for (int mask = 1; mask < 32; mask <<= 1) {
        float next[32];
        for (int l = 0; l < 32; ++l) next[l] = sums[l] + sums[l ^ mask];
        memcpy(sums, next, sizeof(next));
    }
    const float d = amax / 127.0f, sum = sums[0];
    const uint16_t hd = o_float_to_half(d), hs = o_float_to_half(sum);
    const int representable = isfinite(sum) && (hs & 0x7c00u) != 0x7c00u &&
                              (hd & 0x7c00u) != 0x7c00u && (amax == 0.0f || d > 0.0f);
    int bad_code = 0;
    float code[32];
    for (int i = 0; i < 32; ++i) {
        code[i] = (!bad && representable && amax != 0.0f) ? roundf(x[i] / d) : 0.0f;
        if (!isfinite(code[i]) || code[i] < -127.0f || code[i] > 127.0f) bad_code = 1;
    }
    const int valid = !bad && representable && !bad_code;
    memset(out, 0, sizeof(*out));
    if (valid && amax != 0.0f) {
        out->d = hd;
        out->s = hs;
        for (int i = 0; i < 32; ++i) out->qs[i] = (int8_t)code[i];
    }
    return (bad ? 1 : 0) | ((representable && !bad_code) ? 0 : 2);
}

/* quantize n values (n % 32 == 0); returns the OR of all block flags. */
O_EXPORT int o_quantize_q8_1(const float *in, size_t n, o_q8_1 *out) {
    int flags = 0;
    for (size_t b = 0; b < n / 32; ++b) flags |= o_quantize_block(in + 32 * b, out + b);
    return flags;
}

/* ---------------------------------------------------------------------------
 * Uncentred u4 x s8 block dot: low nibble of byte j pairs with qs[j], high
 * nibble with qs[j+16].  src/quant.cpp:48-55 (integer_dot_scalar).
 * ------------------------------------------------------------------------- */
O_EXPORT int o_block_dot(const uint8_t *codes16, const int8_t *qs32) {
    int sum = 0;
    for (int j = 0; j < 16; ++j) {
        sum += (int)(codes16[j] & 15u) * (int)qs32[j];
        sum += (int)(codes16[j] >> 4) * (int)qs32[j + 16];
    }
    return sum;
}

/* All per-block int32 dots of a Q4_0 matrix against Q8_1 columns:
 * dots[(c*rows + r)*blocks + b].  Canonical 18-byte row-major blocks. */
O_EXPORT void o_block_dots(const uint8_t *w, const o_q8_1 *x, int rows, int blocks,
                           int columns, int32_t *dots) {
    for (int c = 0; c < columns; ++c)
        for (int r = 0; r < rows; ++r)
            for (int b = 0; b < blocks; ++b) {
                const uint8_t *blk = w + ((size_t)r * blocks + b) * 18;
                dots[((size_t)c * rows + r) * blocks + b] =
                    o_block_dot(blk + 2, x[(size_t)c * blocks + b].qs);
            }
}

/* Serial full-block matrix product: sum_b d4*(dot*d8 - 8*s8), ascending b,
 * separately rounded.  src/quant.cpp:141-170 (matmul<false, Q4_0>).
 * out[c*rows + r]. */
O_EXPORT void o_matrix_serial(const uint8_t *w, const o_q8_1 *x, int rows, int blocks,
                              int columns, float *out) {
    for (int c = 0; c < columns; ++c)
        for (int r = 0; r < rows; ++r) {
            float acc = 0.0f;
            for (int b = 0; b < blocks; ++b) {
                const uint8_t *blk = w + ((size_t)r * blocks + b) * 18;
                uint16_t hd; memcpy(&hd, blk, 2);
                const o_q8_1 *a = &x[(size_t)c * blocks + b];
                const float d4 = o_half_to_float(hd), d8 = o_half_to_float(a->d),
                            s8 = o_half_to_float(a->s);
                const int dot = o_block_dot(blk + 2, a->qs);
                acc = acc + d4 * ((float)dot * d8 - 8.0f * s8);
            }
            out[(size_t)c * rows + r] = acc;
        }
}

/* Reference GPU (MMVQ) order: lane tid = 2*(b%64)+f holds fragment f
 * (bytes 8f..8f+7, both nibbles); acc = fma(d4, fma(dot, d8, -4*s8), acc);
 * lanes 64..127 merge into 0..63, then an XOR butterfly 1..32.
 * src/cpu_expert.cpp:156-213 (matrix_gpu_order<Q4_0>),
 * src/hip/linear.hip:197-281 (accumulate32 / matrix32). */
O_EXPORT void o_matrix_mmvq(const uint8_t *w, const o_q8_1 *x, int rows, int blocks,
                            int columns, float *out) {
    for (int c = 0; c < columns; ++c)
        for (int r = 0; r < rows; ++r) {
            float lane[128];
            for (int i = 0; i < 128; ++i) lane[i] = 0.0f;
            for (int b = 0; b < blocks; ++b) {
                const uint8_t *blk = w + ((size_t)r * blocks + b) * 18;
                uint16_t hd; memcpy(&hd, blk, 2);
                const o_q8_1 *a = &x[(size_t)c * blocks + b];
                const float d4 = o_half_to_float(hd), d8 = o_half_to_float(a->d),
                            s8 = o_half_to_float(a->s);
                for (int f = 0; f < 2; ++f) {
                    int dot = 0;
                    for (int j = 8 * f; j < 8 * f + 8; ++j) {
                        dot += (int)(blk[2 + j] & 15u) * (int)a->qs[j];
                        dot += (int)(blk[2 + j] >> 4) * (int)a->qs[j + 16];
                    }
                    float *acc = &lane[2 * (b % 64) + f];
                    *acc = fmaf(d4, fmaf((float)dot, d8, -4.0f * s8), *acc);
                }
            }
            for (int i = 0; i < 64; ++i) lane[i] = lane[i] + lane[i + 64];
            for (int mask = 1; mask < 64; mask <<= 1) {
                float next[64];
                for (int i = 0; i < 64; ++i) next[i] = lane[i] + lane[i ^ mask];
                memcpy(lane, next, sizeof(next));
            }
            out[(size_t)c * rows + r] = lane[0];
        }
}

/* ---------------------------------------------------------------------------
 * Q4_1 (20-byte blocks: half d, half m, 16 code bytes; value d*q + m).
 * Block term: float(dot)*half(d4*d8) + half(m4*s8), both products rounded to
 * half RNE (src/quant.cpp:88-102 scaled_dot<Q4_1>).
 * ------------------------------------------------------------------------- */
static inline float o_half_round(float v) { return o_half_to_float(o_float_to_half(v)); }

/* Per-block int32 dots of a Q4_1 matrix (uncentred sum of code*activation). */
O_EXPORT void o_block_dots_q4_1(const uint8_t *w, const o_q8_1 *x, int rows, int blocks, int columns,
                                int32_t *dots) {
    for (int c = 0; c < columns; ++c)
        for (int r = 0; r < rows; ++r)
            for (int b = 0; b < blocks; ++b) {
                const uint8_t *blk = w + ((size_t)r * blocks + b) * 20;
                dots[((size_t)c * rows + r) * blocks + b] = o_block_dot(blk + 4, x[(size_t)c * blocks + b].qs);
            }
}

/* Serial product, src/quant.cpp:141-170 (matmul<false, Q4_1>): per block
 * t = float(dot)*dd; t = t + ms; acc = acc + t (separately rounded). */
O_EXPORT void o_matrix_serial_q4_1(const uint8_t *w, const o_q8_1 *x, int rows, int blocks, int columns,
                                   float *out) {
    for (int c = 0; c < columns; ++c)
        for (int r = 0; r < rows; ++r) {
            float acc = 0.0f;
            for (int b = 0; b < blocks; ++b) {
                const uint8_t *blk = w + ((size_t)r * blocks + b) * 20;
                uint16_t hd, hm; memcpy(&hd, blk, 2); memcpy(&hm, blk + 2, 2);
                const o_q8_1 *a = &x[(size_t)c * blocks + b];
                const float dd = o_half_round(o_half_to_float(hd) * o_half_to_float(a->d));
                const float ms = o_half_round(o_half_to_float(hm) * o_half_to_float(a->s));
                const float t = (float)o_block_dot(blk + 4, a->qs) * dd;
                acc = acc + (t + ms);
            }
            out[(size_t)c * rows + r] = acc;
        }
}

/* MMVQ order for Q4_1, src/cpu_expert.cpp:156-213 (matrix_gpu_order<Q4_1>)
 * and src/hip/linear.hip:197-211: lane 2*(b%64)+f accumulates
 * acc + fma(float(dot_f), dd, ms*0.5) for fragment f (bytes 8f..8f+7, both
 * nibbles); then the same 128 -> 64 merge and XOR butterfly as Q4_0. */
O_EXPORT void o_matrix_mmvq_q4_1(const uint8_t *w, const o_q8_1 *x, int rows, int blocks, int columns,
                                 float *out) {
    for (int c = 0; c < columns; ++c)
        for (int r = 0; r < rows; ++r) {
            float lane[128];
            for (int i = 0; i < 128; ++i) lane[i] = 0.0f;
            for (int b = 0; b < blocks; ++b) {
                const uint8_t *blk = w + ((size_t)r * blocks + b) * 20;
                uint16_t hd, hm; memcpy(&hd, blk, 2); memcpy(&hm, blk + 2, 2);
                const o_q8_1 *a = &x[(size_t)c * blocks + b];
                const float dd = o_half_round(o_half_to_float(hd) * o_half_to_float(a->d));
                const float ms = o_half_round(o_half_to_float(hm) * o_half_to_float(a->s));
                for (int f = 0; f < 2; ++f) {
                    int dot = 0;
                    for (int j = 8 * f; j < 8 * f + 8; ++j) {
                        dot += (int)(blk[4 + j] & 15u) * (int)a->qs[j];
                        dot += (int)(blk[4 + j] >> 4) * (int)a->qs[j + 16];
                    }
                    float *acc = &lane[2 * (b % 64) + f];
                    *acc = *acc + fmaf((float)dot, dd, ms * 0.5f);
                }
            }
            for (int i = 0; i < 64; ++i) lane[i] = lane[i] + lane[i + 64];
            for (int mask = 1; mask < 64; mask <<= 1) {
                float next[64];
                for (int i = 0; i < 64; ++i) next[i] = lane[i] + lane[i ^ mask];
                memcpy(lane, next, sizeof(next));
            }
            out[(size_t)c * rows + r] = lane[0];
        }
}

/* ---------------------------------------------------------------------------
 * Whole expert for `columns` tokens: gate/up in MMVQ order, host-libm SiLU
 * g/(1+expf(-g)) * u, requantise the middle, down in MMVQ order.
 * src/cpu_expert.cpp:216-272 (execute, whole stage), shape-generic.
 * Returns sticky flags (1 nonfinite, 2 arithmetic / not representable).
 * gate/up: [inter][hidden/32] blocks; down: [hidden][inter/32] blocks.
 * xq: [columns][hidden/32]; out: [columns][hidden]; scratch >= columns*(3*inter)
 * floats and mq >= columns*inter/32 blocks.
 * ------------------------------------------------------------------------- */
O_EXPORT int o_expert_whole_typed(const uint8_t *gate, const uint8_t *up, const uint8_t *down, int down_type,
                                  int hidden, int inter, const o_q8_1 *xq, int columns,
                                  float *out, float *scratch, o_q8_1 *mq);
O_EXPORT int o_expert_whole(const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                            int hidden, int inter, const o_q8_1 *xq, int columns,
                            float *out, float *scratch, o_q8_1 *mq) {
    return o_expert_whole_typed(gate, up, down, O_Q4_0, hidden, inter, xq, columns, out, scratch, mq);
}

/* As o_expert_whole with a Q4_0 (2) or Q4_1 (3) down matrix
 * (src/cpu_expert.cpp:216-228 picks matrix_gpu_order by the down type). */
O_EXPORT int o_expert_whole_typed(const uint8_t *gate, const uint8_t *up, const uint8_t *down, int down_type,
                                  int hidden, int inter, const o_q8_1 *xq, int columns,
                                  float *out, float *scratch, o_q8_1 *mq) {
    float *g = scratch, *u = scratch + (size_t)columns * inter, *mid = u + (size_t)columns * inter;
    o_matrix_mmvq(gate, xq, inter, hidden / 32, columns, g);
    o_matrix_mmvq(up, xq, inter, hidden / 32, columns, u);
    int flags = 0;
    for (size_t i = 0; i < (size_t)columns * inter; ++i) {
        float gv = g[i], uv = u[i];
        int f = 0;
        if (!isfinite(gv)) { f |= 1; gv = 0.0f; }
        if (!isfinite(uv)) { f |= 1; uv = 0.0f; }
        float act = gv / (1.0f + expf(-gv));
        if (!isfinite(act)) { f |= 2; act = 0.0f; }
        float v = act * uv;
        if (!isfinite(v)) { f |= 2; v = 0.0f; }
        mid[i] = f ? 0.0f : v;
        flags |= f;
    }
    flags |= o_quantize_q8_1(mid, (size_t)columns * inter, mq);
    if (down_type == O_Q4_1) o_matrix_mmvq_q4_1(down, mq, hidden, inter / 32, columns, out);
    else o_matrix_mmvq(down, mq, hidden, inter / 32, columns, out);
    return flags;
}

/* ---------------------------------------------------------------------------
 * Specified exponential used by the router softmax on both sides of the
 * parity check (the GPU kernel implements the identical operation sequence).
 * Method: Cody-Waite reduction x = n*ln2 + r with ln2 split into a short high
 * part (exact products) and a low correction, |r| <= ln2/2, then the degree-7
 * Taylor polynomial of e^r (coefficients 1/k!) in Horner form with fmaf, and
 * an exact power-of-two scaling in two steps so results down to the
 * subnormal range are formed by exact multiplications.  Inputs below -104
 * return +0; inputs above 88.8 return +inf.  Error <= 2 ulp against expf.
 * ------------------------------------------------------------------------- */
O_EXPORT float o_route_exp(float x) {
    if (!(x == x)) return x;
    if (x < -104.0f) return 0.0f;
    if (x > 88.8f) return INFINITY;
    const float log2e = 1.44269502f;
    const float ln2_hi = 0.693145751953125f;      /* 0x3f317200: 16 significant bits */
    const float ln2_lo = 1.42860677e-06f;         /* ln2 - ln2_hi */
    const float n = rintf(x * log2e);
    float r = fmaf(-n, ln2_hi, x);
    r = fmaf(-n, ln2_lo, r);
    float p = 1.98412701e-04f;                    /* 1/5040 */
    p = fmaf(p, r, 1.38888892e-03f);              /* 1/720  */
    p = fmaf(p, r, 8.33333377e-03f);              /* 1/120  */
    p = fmaf(p, r, 4.16666679e-02f);              /* 1/24   */
    p = fmaf(p, r, 1.66666672e-01f);              /* 1/6    */
    p = fmaf(p, r, 5.00000000e-01f);              /* 1/2    */
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int k = (int)n;
    /* scale by 2^k in two exact steps: 2^(k/2) * 2^(k - k/2) */
    const int k1 = k / 2, k2 = k - k1;
    const float s1 = u2f((uint32_t)(127 + k1) << 23), s2 = u2f((uint32_t)(127 + k2) << 23);
    return (p * s1) * s2;
}

/* ---------------------------------------------------------------------------
 * Router softmax over 512 logits per token.
 * src/hip/session_ops.hip:401-434 (router_softmax): logical width-32 group,
 * lane l owns logits l+32k (k = 0..15); row max; w = exp(x - max); per-lane
 * ascending 16-term sum from +0; XOR butterfly 1,2,4,8,16; inverse = 1/total;
 * p = w * inverse.  A nonfinite input or arithmetic result zeroes the whole
 * row and sets sticky bits (1 input, 2 arithmetic).  The exponential is
 * o_route_exp (see above).
 * ------------------------------------------------------------------------- */
O_EXPORT int o_router_softmax(const float *logits, int tokens, float *probs) {
    int all = 0;
    for (int t = 0; t < tokens; ++t) {
        const float *row = logits + (size_t)t * 512;
        float *p = probs + (size_t)t * 512;
        int flags = 0;
        float x[512], w[512], lane_total[32];
        float mx = -INFINITY;
        for (int i = 0; i < 512; ++i) {
            x[i] = row[i];
            if (!isfinite(x[i])) { flags |= 1; x[i] = 0.0f; }
            mx = x[i] > mx ? x[i] : mx;
        }
        for (int l = 0; l < 32; ++l) {
            float total = 0.0f;
            for (int k = 0; k < 16; ++k) {
                const int i = l + 32 * k;
                float sh = x[i] - mx;
                if (!isfinite(sh)) { flags |= 2; sh = 0.0f; }
                float e = o_route_exp(sh);
                if (!isfinite(e)) { flags |= 2; e = 0.0f; }
                w[i] = e;
                total = total + e;
                if (!isfinite(total)) { flags |= 2; total = 0.0f; }
            }
            lane_total[l] = total;
        }
        for (int mask = 1; mask < 32; mask <<= 1) {
            float next[32];
            for (int l = 0; l < 32; ++l) next[l] = lane_total[l] + lane_total[l ^ mask];
            memcpy(lane_total, next, sizeof(next));
        }
        float total = lane_total[0];
        if (!isfinite(total)) { flags |= 2; total = 0.0f; }
        if (!(total > 0.0f)) flags |= 2;
        float inv = 0.0f;
        if (total > 0.0f) {
            inv = 1.0f / total;
            if (!isfinite(inv)) { flags |= 2; inv = 0.0f; }
        }
        for (int i = 0; i < 512; ++i) {
            float v = w[i] * inv;
            if (!isfinite(v)) { flags |= 2; v = 0.0f; }
            w[i] = v;
        }
        /* the whole row's flags decide, as after the reference's cross-lane OR */
        for (int i = 0; i < 512; ++i) p[i] = flags ? 0.0f : w[i];
        all |= flags;
    }
    return all;
}

/* ---------------------------------------------------------------------------
 * Top-10 selection and renormalisation.  src/session.hip:666-687
 * (select_routes): order by (prob desc, id asc); buckets[id%32] += prob in
 * rank order; XOR butterfly 1..16 over the 32 buckets; denominator =
 * max(bucket0, 1/16384); weight = prob * (1/denominator).
 * Returns 0, or -1 when the denominator is not a positive finite value (the
 * reference throws).
 * ------------------------------------------------------------------------- */
O_EXPORT int o_select_routes(const float *probs, int tokens, int32_t *ids, float *weights) {
    for (int t = 0; t < tokens; ++t) {
        const float *row = probs + (size_t)t * 512;
        int taken[512];
        memset(taken, 0, sizeof(taken));
        int order[10];
        for (int k = 0; k < 10; ++k) {
            int best = -1;
            for (int i = 0; i < 512; ++i) {
                if (taken[i]) continue;
                if (best < 0 || row[i] > row[best]) best = i;   /* ties keep the lower id */
            }
            taken[best] = 1;
            order[k] = best;
        }
        float buckets[32];
        for (int l = 0; l < 32; ++l) buckets[l] = 0.0f;
        for (int k = 0; k < 10; ++k) buckets[order[k] % 32] += row[order[k]];
        for (int d = 1; d < 32; d <<= 1) {
            float prev[32];
            memcpy(prev, buckets, sizeof(prev));
            for (int l = 0; l < 32; ++l) buckets[l] = prev[l] + prev[l ^ d];
        }
        const float floor_v = 1.0f / 16384.0f;
        const float den = buckets[0] > floor_v ? buckets[0] : floor_v;
        if (!(den > 0.0f) || !isfinite(den)) return -1;
        const float inv = 1.0f / den;
        for (int k = 0; k < 10; ++k) {
            ids[t * 10 + k] = order[k];
            weights[t * 10 + k] = row[order[k]] * inv;
        }
    }
    return 0;
}

/* ---------------------------------------------------------------------------
 * Stable grouping.  src/routes.cpp:59-115 (RouteGroups::prepare):
 * histogram over experts, exclusive scan, scatter in (token, rank) order.
 * Outputs: counts[experts], offsets[experts+1], and for every sorted position
 * p: token[p], rank[p], expert[p], weight bits[p].  No validation here (the
 * callers validate); ids must be in [0, experts).
 * ------------------------------------------------------------------------- */
O_EXPORT void o_route_groups(const int32_t *ids, const float *weights, int tokens, int top_k,
                             int experts, int32_t *counts, int32_t *offsets, int32_t *tok,
                             int32_t *rank, int32_t *expert, float *weight) {
    for (int e = 0; e < experts; ++e) counts[e] = 0;
    for (int i = 0; i < tokens * top_k; ++i) ++counts[ids[i]];
    offsets[0] = 0;
    for (int e = 0; e < experts; ++e) offsets[e + 1] = offsets[e] + counts[e];
    int cursor[4096];
    for (int e = 0; e < experts && e < 4096; ++e) cursor[e] = offsets[e];
    for (int t = 0; t < tokens; ++t)
        for (int r = 0; r < top_k; ++r) {
            const int i = t * top_k + r, e = ids[i], p = cursor[e]++;
            tok[p] = t; rank[p] = r; expert[p] = e; weight[p] = weights[i];
        }
}

/* ---------------------------------------------------------------------------
 * Router-weighted rank-order fold.  src/hip/session_ops.hip:307-324
 * (routed_fold) / :292-303 (scaled_add): value = +0; for rank 0..9:
 * value = value + w*contribution, MUL and ADD separately rounded.
 * contrib [tokens][10][hidden] (unweighted), weights [tokens][10].
 * ------------------------------------------------------------------------- */
O_EXPORT void o_routed_fold(const float *contrib, const float *weights, int tokens, int hidden,
                            float *out) {
    for (int t = 0; t < tokens; ++t)
        for (int h = 0; h < hidden; ++h) {
            float v = 0.0f;
            for (int r = 0; r < 10; ++r) {
                const float c = weights[t * 10 + r] * contrib[((size_t)t * 10 + r) * hidden + h];
                v = v + c;
            }
            out[(size_t)t * hidden + h] = v;
        }
}

/* Shared expert gate: raw = sum_h x[h]*w[h] (ascending, separately rounded;
 * the reference computes it with a dense BLAS dot, src/session.hip:1398-1402),
 * then out += (1/(1+expf(-raw))) * shared, src/hip/session_ops.hip:376-391. */
O_EXPORT void o_shared_add(const float *x, const float *gate_vec, const float *shared, int tokens,
                           int hidden, float *out) {
    for (int t = 0; t < tokens; ++t) {
        float raw = 0.0f;
        for (int h = 0; h < hidden; ++h) raw = raw + x[(size_t)t * hidden + h] * gate_vec[h];
        const float scale = 1.0f / (1.0f + expf(-raw));
        for (int h = 0; h < hidden; ++h) {
            const float c = scale * shared[(size_t)t * hidden + h];
            out[(size_t)t * hidden + h] = out[(size_t)t * hidden + h] + c;
        }
    }
}

/* ---------------------------------------------------------------------------
 * Seeded synthetic Q4_0 weights (the generator the GPU side reproduces bit
 * for bit).  Per 32-element block: 16 uniformly random code bytes, and a
 * scale d = half(M * 6.6073582e-08) where M is the largest |S - 131070| over
 * 32 Irwin-Hall(4) draws S of 16-bit uniforms: an integer-exact stand-in for
 * max|w|/8 with w ~ N(0, 0.02).  Counter based: word j of block i is
 * mix64(base + (i << 6) + j), base = mix64(seed ^ mix64(stream + golden)),
 * stream = layer << 32 | expert << 8 | matrix.
 * ------------------------------------------------------------------------- */
static inline uint64_t o_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

O_EXPORT uint64_t o_synth_base(uint64_t seed, uint32_t layer, uint32_t expert, uint32_t matrix) {
    const uint64_t stream = ((uint64_t)layer << 32) | ((uint64_t)expert << 8) | (uint64_t)matrix;
    return o_mix64(seed ^ o_mix64(stream + 0x9e3779b97f4a7c15ull));
}

O_EXPORT void o_synth_q4_0(uint64_t seed, uint32_t layer, uint32_t expert, uint32_t matrix,
                           size_t nblocks, uint8_t *out) {
    const uint64_t base = o_synth_base(seed, layer, expert, matrix);
    for (size_t i = 0; i < nblocks; ++i) {
        uint8_t *blk = out + i * 18;
        const uint64_t c0 = o_mix64(base + (i << 6) + 0), c1 = o_mix64(base + (i << 6) + 1);
        for (int j = 0; j < 8; ++j) {
            blk[2 + j] = (uint8_t)(c0 >> (8 * j));
            blk[10 + j] = (uint8_t)(c1 >> (8 * j));
        }
        uint32_t m = 0;
        for (int j = 2; j < 34; ++j) {
            const uint64_t r = o_mix64(base + (i << 6) + (uint64_t)j);
            const uint32_t s = (uint32_t)(r & 0xffffu) + (uint32_t)((r >> 16) & 0xffffu) +
                               (uint32_t)((r >> 32) & 0xffffu) + (uint32_t)(r >> 48);
            const uint32_t dev = s >= 131070u ? s - 131070u : 131070u - s;
            m = dev > m ? dev : m;
        }
        const uint16_t d = o_float_to_half((float)m * 6.6073582e-08f);
        memcpy(blk, &d, 2);
    }
}

/* Q4_1 version of the generator (for Q4_1 down matrices): the same codes
 * and scale d as o_synth_q4_0, plus the minimum m = half(-8*d*(0.5 + u/65536))
 * with u the low 16 bits of draw 34 of the block. */
O_EXPORT void o_synth_q4_1(uint64_t seed, uint32_t layer, uint32_t expert, uint32_t matrix,
                           size_t nblocks, uint8_t *out) {
    const uint64_t base = o_synth_base(seed, layer, expert, matrix);
    uint8_t q40[18];
    for (size_t i = 0; i < nblocks; ++i) {
        /* one Q4_0 block of the same stream position */
        const uint64_t c0 = o_mix64(base + (i << 6) + 0), c1 = o_mix64(base + (i << 6) + 1);
        for (int j = 0; j < 8; ++j) {
            q40[2 + j] = (uint8_t)(c0 >> (8 * j));
            q40[10 + j] = (uint8_t)(c1 >> (8 * j));
        }
        uint32_t mx = 0;
        for (int j = 2; j < 34; ++j) {
            const uint64_t r = o_mix64(base + (i << 6) + (uint64_t)j);
            const uint32_t s = (uint32_t)(r & 0xffffu) + (uint32_t)((r >> 16) & 0xffffu) +
                               (uint32_t)((r >> 32) & 0xffffu) + (uint32_t)(r >> 48);
            const uint32_t dev = s >= 131070u ? s - 131070u : 131070u - s;
            mx = dev > mx ? dev : mx;
        }
        const uint16_t d = o_float_to_half((float)mx * 6.6073582e-08f);
        const uint64_t r = o_mix64(base + (i << 6) + 34);
        const float f = 0.5f + (float)(uint32_t)(r & 0xffffu) * (1.0f / 65536.0f);
        const uint16_t m = o_float_to_half((-8.0f * o_half_to_float(d)) * f);
        uint8_t *blk = out + i * 20;
        memcpy(blk, &d, 2);
        memcpy(blk + 2, &m, 2);
        memcpy(blk + 4, q40 + 2, 16);
    }
}

/* ---------------------------------------------------------------------------
 * The reference test fixture's Q4_0 weights (tests/cpu_expert_test.cpp:227-246):
 * block i has scale (2 + (i*7 + state) % 11)/2048, negated when
 * (i + state) % 3 == 0, stored as half, then 16 code bytes from a 32-bit
 * xorshift (13, 17, 5) whose state carries across blocks.
 * ------------------------------------------------------------------------- */
O_EXPORT void o_fixture_xorshift_q4_0(uint32_t seed, size_t nblocks, uint8_t *out) {
    for (size_t i = 0; i < nblocks; ++i) {
        const float scale = (float)(2 + (i * 7 + seed) % 11) / 2048.0f;
        const uint16_t d = o_float_to_half((i + seed) % 3 == 0 ? -scale : scale);
        memcpy(out + i * 18, &d, 2);
        for (int j = 0; j < 16; ++j) {
            seed ^= seed << 13;
            seed ^= seed >> 17;
            seed ^= seed << 5;
            out[i * 18 + 2 + j] = (uint8_t)(seed & 255u);
        }
    }
}

/* The same fixture for Q4_1 matrices (tests/cpu_expert_test.cpp:219-241):
 * 20-byte blocks with the same scale and codes and the minimum
 * half(-7.5 * scale) of the unsigned scale. */
O_EXPORT void o_fixture_xorshift_q4_1(uint32_t seed, size_t nblocks, uint8_t *out) {
    for (size_t i = 0; i < nblocks; ++i) {
        const float scale = (float)(2 + (i * 7 + seed) % 11) / 2048.0f;
        const uint16_t d = o_float_to_half((i + seed) % 3 == 0 ? -scale : scale);
        const uint16_t m = o_float_to_half(-7.5f * scale);
        memcpy(out + i * 20, &d, 2);
        memcpy(out + i * 20 + 2, &m, 2);
        for (int j = 0; j < 16; ++j) {
            seed ^= seed << 13;
            seed ^= seed >> 17;
            seed ^= seed << 5;
            out[i * 20 + 4 + j] = (uint8_t)(seed & 255u);
        }
    }
}

/* Exhaustive check of an expf implementation against the C library's expf,
 * the exponential of the reference CPU expert's SiLU (src/cpu_expert.cpp:248-259,
 * the same call as o_expert_whole above): the number of i < count where y[i]
 * differs in bits from expf of the float with bit pattern first + i (two NaNs
 * compare equal); *first_bad receives the first such input's bits. */
O_EXPORT int64_t o_expf_mismatches(const float *y, uint32_t first, uint32_t count, uint32_t *first_bad) {
    int64_t bad = 0;
    for (uint32_t i = 0; i < count; ++i) {
        const uint32_t xb = first + i;
        float x, want;
        memcpy(&x, &xb, 4);
        want = expf(x);
        uint32_t a, b;
        memcpy(&a, &want, 4);
        memcpy(&b, &y[i], 4);
        if (a != b && !(want != want && y[i] != y[i])) {
            if (bad == 0 && first_bad) *first_bad = xb;
            ++bad;
        }
    }
    return bad;
}
