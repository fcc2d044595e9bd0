// The projections of the host half on the GPU: matvec (numerics/fp.py:25-62,
// ops/project.py:22-55) -- fp16-rounded operands, fp32 products and fp32
// sums -- as a hand-written kernel.
//
// y[t][o] = sum_i w16[o][i] * x16[t][i] (+ bias[o]). The weights are held as
// fp16 (the rounding the reference applies at load time, weights.py:70-109),
// the inputs are rounded to fp16 here (the reference's x16). A product of two
// fp16 values is exact in fp32 (11 + 11 significant bits), so each fused
// multiply-add rounds only the sum, as numpy's float32 accumulation does; the
// order of the sums differs from numpy's, which the parity tests bound by the
// float32 rounding of the result.
//
// Decode multiplies one token (or a few) by a weight matrix that does not
// stay in L2 across layers: the bound is reading the fp16 weights once. One
// warp per output row reads the row in 16-byte pieces (8 weights a lane,
// coalesced), each piece serving up to TT tokens whose fp16 inputs sit in
// shared memory; a warp-shuffle tree adds the lanes' partial sums.
#pragma once

#include <cuda_fp16.h>

namespace ins {

constexpr int PROJ_TT = 8;          // tokens per pass over the weights
constexpr int PROJ_WARPS = 8;

__global__ void __launch_bounds__(PROJ_WARPS * 32) k_project(int n, int in_dim, int out_dim,
                                                             const __half *__restrict__ w,
                                                             const float *__restrict__ x,
                                                             const float *__restrict__ bias,
                                                             float *__restrict__ y) {
    extern __shared__ __align__(16) __half xs[];       // [PROJ_TT][in_dim]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int t0 = 0; t0 < n; t0 += PROJ_TT) {
        const int tt = min(PROJ_TT, n - t0);
        __syncthreads();
        for (int i = threadIdx.x; i < PROJ_TT * in_dim; i += blockDim.x) {
            const int t = i / in_dim, c = i - t * in_dim;
            xs[i] = __float2half_rn(t < tt ? x[(int64_t)(t0 + t) * in_dim + c] : 0.0f);
        }
        __syncthreads();
        for (int o = blockIdx.x * PROJ_WARPS + warp; o < out_dim; o += gridDim.x * PROJ_WARPS) {
            const __half *wr = w + (int64_t)o * in_dim;
            float acc[PROJ_TT];
#pragma unroll
            for (int t = 0; t < PROJ_TT; ++t) acc[t] = 0.0f;
            for (int c = lane * 8; c < in_dim; c += 256) {
                const uint4 wv = __ldg(reinterpret_cast<const uint4 *>(wr + c));
                const __half2 *wh = reinterpret_cast<const __half2 *>(&wv);
                float wf[8];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 f = __half22float2(wh[k]);
                    wf[2 * k] = f.x;
                    wf[2 * k + 1] = f.y;
                }
#pragma unroll
                for (int t = 0; t < PROJ_TT; ++t) {
                    if (t >= tt) break;
                    const uint4 xv = *reinterpret_cast<const uint4 *>(xs + t * in_dim + c);
                    const __half2 *xh = reinterpret_cast<const __half2 *>(&xv);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 f = __half22float2(xh[k]);
                        acc[t] = fmaf(wf[2 * k], f.x, acc[t]);
                        acc[t] = fmaf(wf[2 * k + 1], f.y, acc[t]);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < PROJ_TT; ++t) {
                float v = acc[t];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(FULL, v, off);
                acc[t] = v;
            }
            if (lane < tt) {
                float v = acc[0];
#pragma unroll
                for (int t = 1; t < PROJ_TT; ++t) v = lane == t ? acc[t] : v;
                y[(int64_t)(t0 + lane) * out_dim + o] = bias ? v + bias[o] : v;
            }
        }
    }
}

}  // namespace ins
