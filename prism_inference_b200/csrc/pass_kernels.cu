// pass_kernels.cu - the per-pass drop-in kernels: one launch per reference
// vkCmdDispatch, operating on the caller's weight blob / feature arena / aux arena
// exactly as the GLSL does (element offsets, HWC fp16, masked stores).
//
// These run on the CUDA cores with the reference's order of operations: every
// coopVecMatMulAddNV is an fp32 dot product summed in k order with separately
// rounded multiplies and adds, plus the bias, rounded once to fp16.  They read the
// blob at any 2-byte alignment (the reference layout puts experts on 8-byte
// boundaries).  The batched fast path (stack.cu with attn_tc.cu, expert_tc.cu, tc_ffn.cu) uses
// tcgen05 tensor-core tiles instead.
#include <algorithm>

#include "common.cuh"
#include "cta_mv.cuh"
#include "pass_kernels.cuh"

namespace prism {

// ---- windowed attention: split2_qkv_attn_d256.comp.glsl:24-79 ------------------
// One CTA per 8x8 window, 256 threads.  Shared memory: X fp32 [64][D], Q/K/V fp16
// [64][D] each, attention output fp16 [64][D], scratch fp32 [32][D].
template <int D>
__global__ void __launch_bounds__(256) attn_window_kernel(AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* Xs = reinterpret_cast<float*>(smem);                 // [64][D]
    __half* Qs = reinterpret_cast<__half*>(Xs + 64 * D);        // [64][D]
    __half* Ks = Qs + 64 * D;
    __half* Vs = Ks + 64 * D;
    __half* Ao = Vs + 64 * D;                                   // [64][D]
    float* Ys = reinterpret_cast<float*>(Ao + 64 * D);          // [32][D]

    const int wi = blockIdx.x;
    const int wx = (a.W + 7) / 8;
    const int wy = wi / wx, wxx = wi % wx;
    const __half* xin = a.x + (size_t)blockIdx.y * a.frame_stride;
    // :25-37 gather; invalid slots are zero
    for (int i = threadIdx.x; i < 64 * D; i += blockDim.x) {
        const int li = i / D, c = i % D;
        const int gy = wy * 8 + li / 8, gx = wxx * 8 + li % 8;
        const bool valid = gy < a.H && gx < a.W;
        Xs[i] = valid ? __half2float(xin[(size_t)(gy * a.W + gx) * D + c]) : 0.0f;
    }
    __syncthreads();
    // :40-51 Q, K, V in two halves of 32 tokens
    __half* dst3[3] = {Qs, Ks, Vs};
    for (int m = 0; m < 3; ++m) {
        for (int half = 0; half < 2; ++half) {
            cta_mv<32>(a.weights + a.qkv_w + (size_t)m * D * D, D, a.weights + a.qkv_b + m * D, D, D,
                       Xs + half * 32 * D, D, Ys, D);
            __syncthreads();
            for (int i = threadIdx.x; i < 32 * D; i += blockDim.x) dst3[m][half * 32 * D + i] = __float2half_rn(Ys[i]);
            __syncthreads();
        }
    }
    // :53-69 attention, per (token, head), keys = first min(64, n_tokens) slots
    const int H = D / 32;
    const int wt = a.n_tokens < 64 ? a.n_tokens : 64;
    for (int pair = threadIdx.x; pair < 64 * H; pair += blockDim.x) {
        const int i = pair / H, h = pair % H, ch = h * 32;
        float q[32], sc[64], rr[32];
#pragma unroll
        for (int d = 0; d < 32; ++d) q[d] = __half2float(Qs[i * D + ch + d]);
        float mx = -1e9f;
        for (int j = 0; j < wt; ++j) {
            float s = 0.0f;
#pragma unroll
            for (int d = 0; d < 32; ++d) s = __fadd_rn(s, __fmul_rn(q[d], __half2float(Ks[j * D + ch + d])));
            s = __fmul_rn(s, a.scale);
            sc[j] = s;
            if (s > mx) mx = s;
        }
        float se = 0.0f;
#pragma unroll
        for (int d = 0; d < 32; ++d) rr[d] = 0.0f;
        for (int j = 0; j < wt; ++j) {
            const float w = expf(__fsub_rn(sc[j], mx));
            se = __fadd_rn(se, w);
#pragma unroll
            for (int d = 0; d < 32; ++d) rr[d] = __fadd_rn(rr[d], __fmul_rn(w, __half2float(Vs[j * D + ch + d])));
        }
        const float iv = __frcp_rn(fmaxf(se, 1e-6f));
#pragma unroll
        for (int d = 0; d < 32; ++d) Ao[i * D + ch + d] = __float2half_rn(__fmul_rn(rr[d], iv));
    }
    __syncthreads();
    // :71-78 out-projection, fp16 residual add, masked store
    __half* yout = a.y + (size_t)blockIdx.y * a.frame_stride;
    for (int half = 0; half < 2; ++half) {
        cta_mv<32>(a.weights + a.out_w, D, a.weights + a.out_b, D, D, Ao + half * 32 * D, D, Ys, D);
        __syncthreads();
        for (int i = threadIdx.x; i < 32 * D; i += blockDim.x) {
            const int li = half * 32 + i / D, c = i % D;
            const int gy = wy * 8 + li / 8, gx = wxx * 8 + li % 8;
            if (gy < a.H && gx < a.W)
                yout[(size_t)(gy * a.W + gx) * D + c] = __float2half_rn(__fadd_rn(Ys[i], Xs[li * D + c]));
        }
        __syncthreads();
    }
}

// ---- router: moe_router.comp.glsl:24-52 with the N-wide logits of
// moe_ffn_16exp.comp.glsl:27-34.  One CTA per 32 tokens.
template <int D>
__global__ void __launch_bounds__(256) router_kernel(RouterArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* Xs = reinterpret_cast<float*>(smem);  // [32][D]
    float* Ls = Xs + 32 * D;                     // [32][N]
    const int t0 = blockIdx.x * 32;
    const int nt = min(32, a.n_tokens - t0);
    for (int i = threadIdx.x; i < 32 * D; i += blockDim.x) {
        const int t = i / D;
        Xs[i] = t < nt ? __half2float(a.x[(size_t)(t0 + t) * D + (i % D)]) : 0.0f;
    }
    __syncthreads();
    cta_mv<32>(a.weights + a.router_w, D, a.weights + a.router_b, a.n_experts, D, Xs, D, Ls, a.n_experts);
    __syncthreads();
    if (threadIdx.x < nt) {
        const float* l = Ls + threadIdx.x * a.n_experts;
        int best = 0;
        float bv = l[0];
        for (int e = 1; e < a.n_experts; ++e)
            if (l[e] > bv) {  // strict '>': first maximum wins (:44)
                bv = l[e];
                best = e;
            }
        a.assign[t0 + threadIdx.x] = best;
        atomicAdd(&a.counts[best], 1);
    }
}

// ---- expert FFN with skip: moe_expert_skip.comp.glsl:25-54 (one dispatch per expert; tokens of
// other experts return early, :30).  Every CTA scans the assignments and ranks this expert's
// tokens in token order (warp ballots, a running count per 256-token chunk); CTA b computes tiles
// b, b + gridDim.x, ... of kExpertTile of them.  A dispatch thus reads the expert's weights once per
// kExpertTile of its tokens, not once per window of the arena, and spreads an expert's ~T/E tokens
// over T/E/kExpertTile SMs (a dispatch is a latency: 4-token tiles measured faster than 8); the
// arithmetic of every token is that of the shader (cta_mv rows are independent), so the outputs do
// not depend on the tiling.
constexpr int kExpertTile = 4;
template <int D>
__global__ void __launch_bounds__(256) expert_kernel(ExpertArgs a, int tiles_per_cta) {
    constexpr int TT = kExpertTile;
    extern __shared__ __align__(16) unsigned char smem[];
    float* Xs = reinterpret_cast<float*>(smem);            // [TT][D]
    float* Hs = Xs + TT * D;                               // [TT][D]
    float* Rs = Hs + TT * D;                               // [TT][D]
    int* list = reinterpret_cast<int*>(Rs + TT * D);       // [tiles_per_cta][TT]: this CTA's tokens
    __shared__ int wcount[8];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int G = gridDim.x;
    int n = 0;  // the expert's tokens before the current chunk (the same in every thread)
    for (int t0 = 0; t0 < a.n_tokens; t0 += 256) {
        const int t = t0 + tid;
        const bool mine = t < a.n_tokens && a.assign[t] == a.expert_id;  // :30
        const unsigned bal = __ballot_sync(0xffffffffu, mine);
        if (lane == 0) wcount[w] = __popc(bal);
        __syncthreads();
        int before = n, in_chunk = 0;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            before += v < w ? wcount[v] : 0;
            in_chunk += wcount[v];
        }
        if (mine) {
            const int r = before + __popc(bal & ((1u << lane) - 1u));
            const int tile = r / TT;
            if (tile % G == (int)blockIdx.x && tile / G < tiles_per_cta) list[(tile / G) * TT + r % TT] = t;
        }
        n += in_chunk;
        __syncthreads();  // wcount is rewritten by the next chunk; list is complete after the loop
    }
    for (int k = 0; (int)blockIdx.x + k * G < (n + TT - 1) / TT && k < tiles_per_cta; ++k) {
        const int tile = blockIdx.x + k * G;
        const int nt = min(TT, n - tile * TT);
        const int* tok = list + k * TT;
        for (int i = tid; i < TT * D; i += blockDim.x) {
            const int t = i / D;
            Xs[i] = t < nt ? __half2float(a.x[(size_t)tok[t] * D + (i % D)]) : 0.0f;
        }
        __syncthreads();
        cta_mv<TT>(a.weights + a.w1, D, a.weights + a.b1, D, D, Xs, D, Hs, D);
        __syncthreads();
        for (int i = tid; i < TT * D; i += blockDim.x) Hs[i] = rh(gelu_exact(Hs[i]));
        __syncthreads();
        cta_mv<TT>(a.weights + a.w2, D, a.weights + a.b2, D, D, Hs, D, Rs, D);
        __syncthreads();
        for (int i = tid; i < nt * D; i += blockDim.x) {
            const int t = i / D, c = i % D;
            a.y[(size_t)tok[t] * D + c] = __float2half_rn(__fadd_rn(Rs[i], Xs[i]));  // :52
        }
        __syncthreads();  // Xs / Rs are rewritten by the next tile
    }
}

// ---- adapters: pw_project_128to256 (ReLU) / pw_project_256to128 -------------------
template <int K, int N, bool RELU>
__global__ void __launch_bounds__(256) proj_kernel(ProjArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* Xs = reinterpret_cast<float*>(smem);  // [32][K]
    float* Ys = Xs + 32 * K;                     // [32][N]
    const int t0 = blockIdx.x * 32;
    const int nt = min(32, a.n_tokens - t0);
    for (int i = threadIdx.x; i < 32 * K; i += blockDim.x) {
        const int t = i / K;
        Xs[i] = t < nt ? __half2float(a.x[(size_t)(t0 + t) * K + (i % K)]) : 0.0f;
    }
    __syncthreads();
    cta_mv<32>(a.weights + a.w, K, a.weights + a.b, N, K, Xs, K, Ys, N);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * N; i += blockDim.x) {
        float v = Ys[i];
        if (RELU) v = v < 0.0f ? 0.0f : v;
        a.y[(size_t)t0 * N + i] = __float2half_rn(v);
    }
}

// ---- dense FFN of attention_windowed{,_d256}.comp.glsl, in place on the block's
// output rows (which hold the attention result y):
//   acc = sum_c (fp16 accumulate) MV(W2[:, chunk c], b2, gelu_h(MV(W1[chunk c], b1[c], y)))
//   out = h(acc - (n_chunks - 1) * b2 + y)
template <int D>
__global__ void __launch_bounds__(256) dense_ffn_kernel(DenseFfnArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* Xs = reinterpret_cast<float*>(smem);  // [32][D]
    float* Acc = Xs + 32 * D;                    // [32][D]
    float* Oc = Acc + 32 * D;                    // [32][D]
    float* Hs = Oc + 32 * D;                     // [32][chunk]
    const int t0 = blockIdx.x * 32;
    const int nt = min(32, a.n_tokens - t0);
    __half* io = a.io;
    for (int i = threadIdx.x; i < 32 * D; i += blockDim.x) {
        const int t = i / D;
        Xs[i] = t < nt ? __half2float(io[(size_t)(t0 + t) * D + (i % D)]) : 0.0f;
        Acc[i] = 0.0f;
    }
    __syncthreads();
    const int nch = a.hidden / a.chunk;
    for (int c = 0; c < nch; ++c) {
        cta_mv<32>(a.weights + a.w1 + (size_t)c * a.chunk * D, D, a.weights + a.b1 + c * a.chunk, a.chunk, D, Xs,
                   D, Hs, a.chunk);
        __syncthreads();
        for (int i = threadIdx.x; i < 32 * a.chunk; i += blockDim.x) Hs[i] = rh(gelu_exact(Hs[i]));
        __syncthreads();
        cta_mv<32>(a.weights + a.w2 + c * a.chunk, a.hidden, a.weights + a.b2, D, a.chunk, Hs, a.chunk, Oc, D);
        __syncthreads();
        for (int i = threadIdx.x; i < 32 * D; i += blockDim.x) Acc[i] = rh(__fadd_rn(Acc[i], Oc[i]));
        __syncthreads();
    }
    const float corr = (float)(nch - 1);
    for (int i = threadIdx.x; i < nt * D; i += blockDim.x) {
        const float b2 = __half2float(a.weights[a.b2 + (i % D)]);
        const float v = __fadd_rn(__fsub_rn(Acc[i], __fmul_rn(corr, b2)), Xs[i]);
        io[(size_t)t0 * D + i] = __float2half_rn(v);
    }
}

// ---- launchers ------------------------------------------------------------------
template <typename K>
static cudaError_t set_smem(K kernel, size_t bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

cudaError_t launch_attn_window(const AttnArgs& a, int dim, int frames, cudaStream_t s) {
    const dim3 nwin(((a.W + 7) / 8) * ((a.H + 7) / 8), frames);
    if (dim == 256) {
        const size_t sm = 64 * 256 * 4 + 4 * 64 * 256 * 2 + 32 * 256 * 4;
        cudaError_t e = set_smem(attn_window_kernel<256>, sm);
        if (e != cudaSuccess) return e;
        attn_window_kernel<256><<<nwin, 256, sm, s>>>(a);
    } else {
        const size_t sm = 64 * 128 * 4 + 4 * 64 * 128 * 2 + 32 * 128 * 4;
        cudaError_t e = set_smem(attn_window_kernel<128>, sm);
        if (e != cudaSuccess) return e;
        attn_window_kernel<128><<<nwin, 256, sm, s>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t launch_router(const RouterArgs& a, int dim, cudaStream_t s) {
    const int grid = (a.n_tokens + 31) / 32;
    const size_t sm = (size_t)32 * dim * 4 + (size_t)32 * a.n_experts * 4;
    if (grid == 0) return cudaSuccess;
    if (dim == 256) {
        cudaError_t e = set_smem(router_kernel<256>, sm);
        if (e != cudaSuccess) return e;
        router_kernel<256><<<grid, 256, sm, s>>>(a);
    } else {
        cudaError_t e = set_smem(router_kernel<128>, sm);
        if (e != cudaSuccess) return e;
        router_kernel<128><<<grid, 256, sm, s>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t launch_expert(const ExpertArgs& a, int dim, cudaStream_t s) {
    // tiles if every token went to this expert; one CTA per SM-ish, more when a CTA's token list
    // (tiles_per_cta x kExpertTile ints beside the three [kExpertTile][dim] fp32 tiles) would not fit
    const int tiles = (a.n_tokens + kExpertTile - 1) / kExpertTile;
    if (tiles == 0) return cudaSuccess;
    const int grid = std::max(std::min(tiles, 148), (tiles + 4095) / 4096);
    const int tiles_per_cta = (tiles + grid - 1) / grid;
    const size_t sm = (size_t)3 * kExpertTile * dim * 4 + (size_t)tiles_per_cta * kExpertTile * 4;
    if (dim == 256) {
        cudaError_t e = set_smem(expert_kernel<256>, sm);
        if (e != cudaSuccess) return e;
        expert_kernel<256><<<grid, 256, sm, s>>>(a, tiles_per_cta);
    } else {
        cudaError_t e = set_smem(expert_kernel<128>, sm);
        if (e != cudaSuccess) return e;
        expert_kernel<128><<<grid, 256, sm, s>>>(a, tiles_per_cta);
    }
    return cudaGetLastError();
}

cudaError_t launch_proj(const ProjArgs& a, bool up, cudaStream_t s) {
    const int grid = (a.n_tokens + 31) / 32;
    const size_t sm = (size_t)32 * (128 + 256) * 4;
    if (grid == 0) return cudaSuccess;
    if (up) {
        cudaError_t e = set_smem(proj_kernel<128, 256, true>, sm);
        if (e != cudaSuccess) return e;
        proj_kernel<128, 256, true><<<grid, 256, sm, s>>>(a);
    } else {
        cudaError_t e = set_smem(proj_kernel<256, 128, false>, sm);
        if (e != cudaSuccess) return e;
        proj_kernel<256, 128, false><<<grid, 256, sm, s>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t launch_dense_ffn(const DenseFfnArgs& a, int dim, cudaStream_t s) {
    const int grid = (a.n_tokens + 31) / 32;
    const size_t sm = (size_t)3 * 32 * dim * 4 + (size_t)32 * a.chunk * 4;
    if (grid == 0) return cudaSuccess;
    if (dim == 256) {
        cudaError_t e = set_smem(dense_ffn_kernel<256>, sm);
        if (e != cudaSuccess) return e;
        dense_ffn_kernel<256><<<grid, 256, sm, s>>>(a);
    } else {
        cudaError_t e = set_smem(dense_ffn_kernel<128>, sm);
        if (e != cudaSuccess) return e;
        dense_ffn_kernel<128><<<grid, 256, sm, s>>>(a);
    }
    return cudaGetLastError();
}

}  // namespace prism
