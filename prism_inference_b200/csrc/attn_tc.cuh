// attn_tc.cuh - arguments of the fused tcgen05 windowed-attention (+ router) kernel.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace prism {

struct AttnTcArgs {
    int W, H, frames;        // frame geometry; tokens are HWC, frames consecutive
    int n_keys;              // keys per window = min(64, n_tokens)
    int n_experts;           // 0: no router (dense block); MoE blocks are dim 256
    int n_experts_pad;       // router N rounded up to a multiple of 16 (<= 256)
    float scale;             // 1/sqrt(32)
    const float* bqkv;       // [D/32][96] head-major q|k|v biases (fp32 copies of the fp16 blob)
    const float* bo;         // [D]
    const float* br;         // [n_experts_pad]
    int32_t* assign;         // [frames * W * H] expert of every token
    int32_t* counts;         // [n_experts] += tokens routed
    // Bucket permutation (nullable): token t routed to expert e goes to perm_b[e * perm_stride + k],
    // k = the value counts[e] had before this token (so counts doubles as the bucket cursor), and
    // the grouped expert kernel reads its tiles straight from the buckets; null: the CTA
    // histograms are added to counts and the route kernel builds the permutation.
    int32_t* perm_b;
    int perm_stride;         // bucket capacity, >= the tokens of the forward
    uint32_t* err;
};

// dim = D, the model width: 256 (MoE / dense "Standard" blocks) or 128 (dense "Baseline").
// Maps: x / y  4-D fp16 (C=D, X=W, Y=H, F=frames), box {64, 8, 8, 1}, 128B swizzle
//       wqkv  3-D K-block-major [D/64][3D][64] (q|k|v of head h at rows 96h..96h+95), box {64, 96, D/64}
//       wo    2-D [D][D], box {64, D};  wr 3-D K-block-major [4][npad][64], box {64, min(96, npad), 4}
cudaError_t launch_attn_tc(int dim, const AttnTcArgs& a, const CUtensorMap& x, const CUtensorMap& y,
                           const CUtensorMap& wqkv, const CUtensorMap& wo, const CUtensorMap& wr, int grid,
                           cudaStream_t s);
int attn_tc_smem_bytes(int dim);

// The same block at D = 256 with every tile's heads split over a cluster of two CTAs (the
// latency path for forwards of few tiles): 2 * n_tiles CTAs, one tile per cluster; same maps.
cudaError_t launch_attn_pair(const AttnTcArgs& a, const CUtensorMap& x, const CUtensorMap& y, const CUtensorMap& wqkv,
                             const CUtensorMap& wo, const CUtensorMap& wr, int n_tiles, cudaStream_t s);
int attn_pair_smem_bytes();

}  // namespace prism
