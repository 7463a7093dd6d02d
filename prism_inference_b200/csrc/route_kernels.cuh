// route_kernels.cuh - counts -> segment offsets, tile list, token permutation.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace prism {

struct ExpertTile;

struct RoutePlanArgs {
    int32_t* counts;       // [n_experts] tokens per expert (reset to 0 on exit)
    int32_t* counts_out;   // optional copy of the counts (nullable)
    int32_t* offsets;      // [n_experts] first sorted row of each expert
    int32_t* cursor;       // [n_experts] scatter cursors (set to 0)
    ExpertTile* tiles;     // [max_tiles]
    int32_t* n_tiles;      // device tile count
    int n_experts, n_tokens;
    uint32_t* err;
};
struct RouteScatterArgs {
    const int32_t* assign;  // [n_tokens] expert of each token
    const int32_t* offsets;
    int32_t* cursor;
    int32_t* perm;          // [n_tokens] sorted row -> token
    int n_experts, n_tokens;
    uint32_t* err;
};

cudaError_t launch_route(const RoutePlanArgs& p, const RouteScatterArgs& s, cudaStream_t st);

}  // namespace prism
