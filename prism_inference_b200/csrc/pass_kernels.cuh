// pass_kernels.cuh - argument blocks and launchers of the per-pass drop-in kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace prism {

// Pointers already include the reference's element offsets.
struct AttnArgs {
    const __half* weights;
    const __half* x;       // frame 0 input  [T][D]
    __half* y;             // frame 0 output [T][D]
    int64_t frame_stride;  // elements between frames (grid.y = frames)
    int qkv_w, qkv_b, out_w, out_b;
    int W, H, n_tokens;    // n_tokens: the push constant (keys = min(64, n_tokens))
    float scale;
};
struct RouterArgs {
    const __half* weights;
    const __half* x;       // [n_tokens][D]
    int32_t* assign;       // [n_tokens]
    int32_t* counts;       // [n_experts], atomically incremented
    int router_w, router_b, n_experts, n_tokens;
};
struct ExpertArgs {
    const __half* weights;
    const __half* x;
    __half* y;
    const int32_t* assign;
    int w1, b1, w2, b2, expert_id, n_tokens;
};
struct ProjArgs {
    const __half* weights;
    const __half* x;
    __half* y;
    int w, b, n_tokens;
};
struct DenseFfnArgs {
    const __half* weights;
    __half* io;            // [n_tokens][D], attention output in, block output out
    int w1, b1, w2, b2, hidden, chunk, n_tokens;
};

cudaError_t launch_attn_window(const AttnArgs& a, int dim, int frames, cudaStream_t s);
cudaError_t launch_router(const RouterArgs& a, int dim, cudaStream_t s);
cudaError_t launch_expert(const ExpertArgs& a, int dim, cudaStream_t s);
cudaError_t launch_proj(const ProjArgs& a, bool up, cudaStream_t s);
cudaError_t launch_dense_ffn(const DenseFfnArgs& a, int dim, cudaStream_t s);

}  // namespace prism
