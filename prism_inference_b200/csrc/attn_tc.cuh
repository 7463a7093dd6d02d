// attn_tc.cuh - arguments of the fused tcgen05 windowed-attention (+ router) kernel.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace prism {

struct AttnTcArgs {
    int W, H, frames;        // frame geometry; tokens are HWC, frames consecutive
    int n_keys;              // keys per window = min(64, n_tokens)
    int n_experts;           // 0: no router (dense block)
    int n_experts_pad;       // router N rounded up to a multiple of 16 (<= 256)
    float scale;             // 1/sqrt(32)
    const float* bqkv;       // [8][96] head-major q|k|v biases (fp32 copies of the fp16 blob)
    const float* bo;         // [256]
    const float* br;         // [n_experts_pad]
    int32_t* assign;         // [frames * W * H] expert of every token
    int32_t* counts;         // [n_experts] += tokens routed
    uint32_t* err;
};

// Maps: x / y  4-D fp16 (C=256, X=W, Y=H, F=frames), box {64, 8, 8, 1}, 128B swizzle
//       wqkv  2-D [768][256] head-major rows (q|k|v of head h at rows 96h..96h+95), box {64, 96}
//       wo    2-D [256][256], box {64, 128};  wr 2-D [npad][256], box {64, min(128, npad)}
cudaError_t launch_attn_tc(const AttnTcArgs& a, const CUtensorMap& x, const CUtensorMap& y, const CUtensorMap& wqkv,
                           const CUtensorMap& wo, const CUtensorMap& wr, int grid, cudaStream_t s);
int attn_tc_smem_bytes();

}  // namespace prism
