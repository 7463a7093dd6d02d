// cta_mv.cuh - CTA-wide matrix-vector products in the reference's order of operations
// (coopVecMatMulAddNV as modelled by the oracle: fp32 products and sums rounded
// separately, summed in k order, bias added last, one rounding to fp16).
#pragma once
#include "common.cuh"

namespace prism {

// Y[t][r] = h( sum_k W[r][k] * X[t][k] + b[r] ),  t < TT, r < N.
// X: smem [TT][ldx] (float or __half), Y: smem [TT][ldy] float.  CTA-wide; each
// thread owns output rows r = tid, tid + blockDim, ...  Where every weight row starts 16- or
// 8-byte aligned, the weights come eight or four per load (the products are still summed one k at
// a time, in k order, so the result is the same).
template <int TT, typename XT>
__device__ void cta_mv(const __half* __restrict__ W, int ldw, const __half* __restrict__ b, int N, int K,
                       const XT* Xs, int ldx, float* Ys, int ldy) {
    const uintptr_t align = reinterpret_cast<uintptr_t>(W) | ((uintptr_t)ldw * 2);
    const bool vec8 = (align & 15) == 0 && (K & 7) == 0;
    const bool vec = (align & 7) == 0 && (K & 3) == 0;
    for (int r = threadIdx.x; r < N; r += blockDim.x) {
        float acc[TT];
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[t] = 0.0f;
        const __half* wr = W + (size_t)r * ldw;
        if (vec8) {
            // (four loads in flight: each thread streams its own row, so a lone load per iteration
            // waits the whole L2 latency)
#pragma unroll 4
            for (int k = 0; k < K; k += 8) {
                const uint4 w8 = __ldg(reinterpret_cast<const uint4*>(wr + k));
                const float wv[8] = {lo_h2f(w8.x), hi_h2f(w8.x), lo_h2f(w8.y), hi_h2f(w8.y),
                                     lo_h2f(w8.z), hi_h2f(w8.z), lo_h2f(w8.w), hi_h2f(w8.w)};
#pragma unroll
                for (int j = 0; j < 8; ++j)
#pragma unroll
                    for (int t = 0; t < TT; ++t)
                        acc[t] = __fadd_rn(acc[t], __fmul_rn(wv[j], (float)Xs[t * ldx + k + j]));
            }
        } else if (vec) {
#pragma unroll 4
            for (int k = 0; k < K; k += 4) {
                const uint2 w4 = __ldg(reinterpret_cast<const uint2*>(wr + k));
                const float wv[4] = {lo_h2f(w4.x), hi_h2f(w4.x), lo_h2f(w4.y), hi_h2f(w4.y)};
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int t = 0; t < TT; ++t)
                        acc[t] = __fadd_rn(acc[t], __fmul_rn(wv[j], (float)Xs[t * ldx + k + j]));
            }
        } else {
            for (int k = 0; k < K; ++k) {
                const float w = __half2float(wr[k]);
#pragma unroll
                for (int t = 0; t < TT; ++t) acc[t] = __fadd_rn(acc[t], __fmul_rn(w, (float)Xs[t * ldx + k]));
            }
        }
        const float bias = __half2float(b[r]);
#pragma unroll
        for (int t = 0; t < TT; ++t) Ys[t * ldy + r] = rh(__fadd_rn(acc[t], bias));
    }
}

}  // namespace prism
