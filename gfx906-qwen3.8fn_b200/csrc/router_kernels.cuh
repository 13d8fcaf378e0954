// router_kernels.cuh -- router logits on the device:
//   logits[t][e] = sum_h x[t][h] * W[e][h]   (fp32, W = ffn_gate_inp as [512][H])
// The reference applies ffn_gate_inp (an F32 [H x 512] tensor) with a dense
// BLAS GEMM and copies the probabilities to the host every layer
// (src/session.hip:561-590 Matrix::apply, :1420-1426).  Here the logits stay
// on the device and feed the routing kernels directly.  The products stay
// fp32 on the CUDA cores: a TF32 tensor-core GEMM would move logits by ~1e-3
// relative and flip near-tie routes.
#pragma once
#include "common.cuh"

namespace qmoe {

constexpr int kRouterGemvTokens = 32;   // T <= 32: one warp per expert, all tokens at once
constexpr int kRouterGemvWarps = 4;

// Decode sizes: warp = expert; the expert's weight row streams once (lane
// strided float4), every token's activation row is read through L1/L2.
__global__ void __launch_bounds__(32 * kRouterGemvWarps)
router_gemv_kernel(const float *x, const float *W, float *logits, int T, int H) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * kRouterGemvWarps + warp;
    if (e >= kRouterExperts) return;
    const float4 *wr = reinterpret_cast<const float4 *>(W + static_cast<size_t>(e) * H);
    float acc[kRouterGemvTokens];
#pragma unroll
    for (int t = 0; t < kRouterGemvTokens; ++t) acc[t] = 0.0f;
    for (int h = lane; h < H / 4; h += 32) {
        const float4 wv = __ldg(wr + h);
#pragma unroll
        for (int t = 0; t < kRouterGemvTokens; ++t)
            if (t < T) {
                const float4 xv = __ldg(reinterpret_cast<const float4 *>(x + static_cast<size_t>(t) * H) + h);
                acc[t] = fmaf(xv.x, wv.x, acc[t]);
                acc[t] = fmaf(xv.y, wv.y, acc[t]);
                acc[t] = fmaf(xv.z, wv.z, acc[t]);
                acc[t] = fmaf(xv.w, wv.w, acc[t]);
            }
    }
#pragma unroll
    for (int t = 0; t < kRouterGemvTokens; ++t)
        if (t < T) {
            const float v = warp_sum(acc[t]);
            if (lane == 0) logits[static_cast<size_t>(t) * kRouterExperts + e] = v;
        }
}

// Larger T: 64 tokens x 64 experts per CTA, K chunks of 16 staged in shared
// memory, 16 x 16 threads with 4 x 4 outputs each.
constexpr int kRouterTile = 64;
constexpr int kRouterK = 16;

__global__ void __launch_bounds__(256) router_gemm_kernel(const float *x, const float *W, float *logits, int T, int H) {
    __shared__ float xs[kRouterK][kRouterTile + 4];
    __shared__ float ws[kRouterK][kRouterTile + 4];
    const int t0 = blockIdx.y * kRouterTile, e0 = blockIdx.x * kRouterTile;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int lr = threadIdx.x >> 2, lc = (threadIdx.x & 3) * 4;   // loader: row, first k of a float4
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < H; k0 += kRouterK) {
        const int t = t0 + lr;
        const float4 xv = t < T ? __ldg(reinterpret_cast<const float4 *>(x + static_cast<size_t>(t) * H + k0 + lc))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 wv = __ldg(reinterpret_cast<const float4 *>(W + static_cast<size_t>(e0 + lr) * H + k0 + lc));
        xs[lc + 0][lr] = xv.x; xs[lc + 1][lr] = xv.y; xs[lc + 2][lr] = xv.z; xs[lc + 3][lr] = xv.w;
        ws[lc + 0][lr] = wv.x; ws[lc + 1][lr] = wv.y; ws[lc + 2][lr] = wv.z; ws[lc + 3][lr] = wv.w;
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kRouterK; ++k) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) { a[i] = xs[k][ty * 4 + i]; b[i] = ws[k][tx * 4 + i]; }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + ty * 4 + i;
        if (t < T)
            *reinterpret_cast<float4 *>(logits + static_cast<size_t>(t) * kRouterExperts + e0 + tx * 4) =
                make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    }
}

}  // namespace qmoe
