// tc_ffn.cuh - argument block of the tcgen05 row-tile GEMM-chain kernel.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace prism {

// Modes of the row-tile GEMM chain.
enum FfnMode : int {
    FFN_EXPERT = 0,     // gathered rows of one expert: x + W2 gelu(W1 x + b1) + b2, scattered back
    FFN_PROJ_UP = 1,    // relu(W x + b), 128 -> 256
    FFN_PROJ_DOWN = 2,  // W x + b, 256 -> 128
    FFN_DENSE = 3,      // dense FFN of width NCH*HID, fp16 accumulation of NCH chunk outputs
    FFN_DENSE_UNSPLIT = 4  // dense FFN of width NCH*HID as ONE product: GEMM2 accumulates over every
                           // chunk's H in fp32, rounded once (attention_windowed.comp.glsl:151-170)
};

// One tile of the grouped expert GEMM: rows perm[start .. start+rows) of expert e.
struct ExpertTile {
    int expert, start, rows, pad;
};

struct FfnArgs {
    const __half* x;           // input rows [n_rows][KIN] fp16
    __half* y;                 // output rows [n_rows][NOUT] fp16 (may alias x only row-wise in place)
    const int32_t* perm;       // FFN_EXPERT: sorted row -> token
    const ExpertTile* tiles;   // FFN_EXPERT: tile list
    const int32_t* n_tiles;    // FFN_EXPERT: device tile count
    int n_rows;                // rows of x (expert mode: of the gather map), other modes: rows to process
    const float* b1;           // fp32 biases [experts][HID*NCH]
    const float* b2;           // fp32 biases [experts][NOUT]
    uint32_t* err;             // device error word
    int32_t* route_counts;     // FFN_EXPERT: the router's counts and the scatter cursors, cleared by
    int32_t* route_cursor;     //   the expert kernel for the next MoE block (nullable)
    int n_route;               // FFN_EXPERT: entries of route_counts / route_cursor
    // FFN_EXPERT with tiles == nullptr: bucket routing.  Expert e's rows are the tokens
    // perm[e * perm_stride + k], k < route_counts[e] (written by the router, attn_tc.cuh); every
    // CTA derives the tile list from the counts itself, and the last CTA to read them clears them
    // (route_done counts the CTAs that have read; it is zero between launches).
    int perm_stride;
    uint32_t* route_done;
    int32_t* counts_out;       // optional copy of the counts (bucket routing)
};

// Grouped expert FFN (expert_tc.cu): w1, w2 = 2-D [E*256][256] maps with box {64, 256}; the token
// rows are gathered from a.x with cp.async; a.n_rows = rows of a.x.
cudaError_t launch_ffn_expert256(const FfnArgs& a, const CUtensorMap& w1, const CUtensorMap& w2, int grid,
                                 cudaStream_t s);
cudaError_t launch_ffn_dense256(const FfnArgs& a, const CUtensorMap& x, const CUtensorMap& w1, const CUtensorMap& w2,
                                int n_chunks, int grid, cudaStream_t s);
// Dense FFN of a dim-128 block (x: [rows][128], w1: [hidden][128] map with box {64, chunk rows},
// w2: [128][hidden] map with box {64, 128}).  chunk == hidden: one product (the d128 shader);
// chunk 128 or 256 < hidden: fp16 accumulation of chunk outputs (the d256 shader's rule).
// Supported: hidden == chunk == 128; hidden == chunk, a multiple of 256; chunk 128 or 256
// dividing hidden.  Returns cudaErrorInvalidValue for other shapes.
cudaError_t launch_ffn_dense128(const FfnArgs& a, const CUtensorMap& x, const CUtensorMap& w1, const CUtensorMap& w2,
                                int hidden, int chunk, int grid, cudaStream_t s);
// Row count of the W1 tensor-map box launch_ffn_dense128 expects for (hidden, chunk), 0 if unsupported.
int ffn_dense128_w1_box(int hidden, int chunk);
cudaError_t launch_ffn_proj_up(const FfnArgs& a, const CUtensorMap& x, const CUtensorMap& w, int grid,
                               cudaStream_t s);
cudaError_t launch_ffn_proj_down(const FfnArgs& a, const CUtensorMap& x, const CUtensorMap& w, int grid,
                                 cudaStream_t s);

}  // namespace prism
