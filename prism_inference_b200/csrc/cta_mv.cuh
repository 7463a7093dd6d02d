// cta_mv.cuh - CTA-wide matrix-vector products in the reference's order of operations
// (coopVecMatMulAddNV as modelled by the oracle: fp32 products and sums rounded
// separately, summed in k order, bias added last, one rounding to fp16).
#pragma once
#include "common.cuh"

namespace prism {

// Y[t][r] = h( sum_k W[r][k] * X[t][k] + b[r] ),  t < TT, r < N.
// X: smem [TT][ldx] (float or __half), Y: smem [TT][ldy] float.  CTA-wide; each
// thread owns output rows r = tid, tid + blockDim, ...
template <int TT, typename XT>
__device__ void cta_mv(const __half* __restrict__ W, int ldw, const __half* __restrict__ b, int N, int K,
                       const XT* Xs, int ldx, float* Ys, int ldy) {
    for (int r = threadIdx.x; r < N; r += blockDim.x) {
        float acc[TT];
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[t] = 0.0f;
        const __half* wr = W + (size_t)r * ldw;
        for (int k = 0; k < K; ++k) {
            const float w = __half2float(wr[k]);
#pragma unroll
            for (int t = 0; t < TT; ++t) acc[t] = __fadd_rn(acc[t], __fmul_rn(w, (float)Xs[t * ldx + k]));
        }
        const float bias = __half2float(b[r]);
#pragma unroll
        for (int t = 0; t < TT; ++t) Ys[t * ldy + r] = rh(__fadd_rn(acc[t], bias));
    }
}

}  // namespace prism
